"""DiLoCo outer step, compression and replica drop / rejoin on gloo CPU ranks.

Failures are injected on the host (a rank stops heart-beating and skips an
outer step); no GPU is involved."""

import time

import pytest
import torch

from tests.dist_utils import run_ranks


def _shards(rank, n=1000):
    g = torch.Generator().manual_seed(0)  # replicas start from the same weights
    return [torch.randn(n, generator=g), torch.randn(37, 3, generator=g)]


def _outer_math(rank, world, quant, comm="collective"):
    from llm_research_b200.parallel.diloco import DiLoCo, DiLoCoConfig, make_diloco_groups

    _, rg, ranks, _ = make_diloco_groups(world)
    shards = _shards(rank)
    dl = DiLoCo(shards, rg, ranks, DiLoCoConfig(inner_steps=2, quantize_bits=quant, comm=comm))
    # CPU ranks have no multicast or peer memory: "nvls" falls back to the collective path
    assert dl.comm == "collective"
    anchor0 = dl.anchor.clone()
    for s in shards:  # "inner training": each replica drifts differently
        s.add_(0.01 * (rank + 1))
    assert not dl.step()
    assert dl.step()  # outer step after inner_steps=2
    return anchor0, torch.cat([s.reshape(-1) for s in shards]), dl.anchor[: dl.numel].clone()


@pytest.mark.parametrize("quant,comm", [(0, "collective"), (4, "collective"), (0, "nvls")])
def test_diloco_nesterov_outer_step(quant, comm):
    world = 3
    res = run_ranks(_outer_math, world, quant, comm)
    anchor0 = res[0][0][: res[0][2].numel()]
    for r in range(world):
        torch.testing.assert_close(res[r][0][: res[r][2].numel()], anchor0)  # same start on every replica
        torch.testing.assert_close(res[r][2], res[0][2])                    # same result on every replica
        torch.testing.assert_close(res[r][1], res[0][2])                    # local weights reset to anchor
    delta = -0.01 * torch.tensor([1.0, 2.0, 3.0]).mean()  # anchor - local, averaged
    m = delta  # momentum starts at zero
    want = anchor0 - 0.7 * (delta + 0.9 * m)
    tol = 1e-6 if quant == 0 else 2e-3
    torch.testing.assert_close(res[0][2], want.expand_as(res[0][2]) if want.dim() == 0 else want, atol=tol, rtol=0)


def _drop_rejoin(rank, world):
    import torch.distributed as dist

    from llm_research_b200.parallel.diloco import DiLoCo, DiLoCoConfig, make_diloco_groups
    from llm_research_b200.parallel.fault import FaultInjector, HeartbeatMonitor, default_store

    _, rg, ranks, _ = make_diloco_groups(world)
    mon = HeartbeatMonitor(interval_s=0.05, timeout_s=0.6).start()
    inj = FaultInjector("2:1:hang")
    shards = _shards(rank, 256)
    dl = DiLoCo(shards, rg, ranks, DiLoCoConfig(inner_steps=1, comm="collective", max_island_failures=1),
                monitor=mon)
    store = default_store()
    log = []
    # outer step 1: everybody
    shards[0].add_(0.1 * (rank + 1))
    dl.step()
    log.append(list(dl.members))
    if inj.check(1, mon) == "leave":  # rank 2 "hangs": stops beating, skips outer step 2
        store.wait(["diloco/roster/0/2"])
        store.set("test/rank2_back", "1")
        dl.rejoin()
        log.append(list(dl.members))
    else:
        time.sleep(1.0)  # let rank 2's heartbeat go stale
        shards[0].add_(0.1)
        dl.step()  # outer step 2 without rank 2
        log.append(list(dl.members))
        store.wait(["test/rank2_back"])
        time.sleep(0.2)
        shards[0].add_(0.1)
        dl.step()  # outer step 3: rank 2 rejoins
        log.append(list(dl.members))
    mon.stop()
    store.set(f"test/done/{rank}", "1")
    store.wait([f"test/done/{r}" for r in range(world)])
    return log, dl.anchor[: dl.numel].clone(), torch.cat([s.reshape(-1) for s in shards])


def test_diloco_replica_drop_and_rejoin():
    res = run_ranks(_drop_rejoin, 3)
    assert res[0][0] == [[0, 1, 2], [0, 1], [0, 1, 2]]
    assert res[1][0] == res[0][0]
    assert res[2][0] == [[0, 1, 2], [0, 1, 2]]
    for r in range(3):
        torch.testing.assert_close(res[r][1], res[0][1])   # all replicas agree after the rejoin
        torch.testing.assert_close(res[r][2], res[0][1])


def test_fault_injector_modes():
    from llm_research_b200.parallel.fault import FaultInjector

    inj = FaultInjector("0:3:raise,1:2:leave", rank=0)
    assert inj.check(1) is None
    with pytest.raises(RuntimeError):
        inj.check(3)
    assert FaultInjector("0:3:raise,1:2:leave", rank=1).check(2) == "leave"
