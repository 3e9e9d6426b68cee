"""NVSwitch multicast (NVLS) collectives on 2+ GPUs (one NCCL rank per GPU)
against NCCL: the multimem all-reduce, the FSDP reduce-scatter / all-gather
kernels, the training engine with ``comm="nvls"`` and DiLoCo's fused outer step.

Skipped when fewer than two GPUs are visible or the node offers no multicast."""

import pytest
import torch

from tests.dist_utils import run_ranks

pytestmark = pytest.mark.gpu

needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs at least two GPUs")


def _multicast_or_none(rank):
    from llm_research_b200.parallel.nvls import MulticastHeap, NVLSUnavailable

    try:
        return MulticastHeap(1 << 26, device=torch.device("cuda", rank))
    except NVLSUnavailable:
        return None


def _collectives(rank, world):
    import torch.distributed as dist

    from llm_research_b200._ext import native
    from llm_research_b200.parallel.nvls import NVLSAllReduce

    C = native()
    dev = torch.device("cuda", rank)
    heap = _multicast_or_none(rank)
    if heap is None:
        return {"skip": True}
    out = {"skip": False}
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    # all-reduce, fp32 and bf16, three epochs on the same buffers (flag reuse);
    # the size is not a multiple of world * 16 bytes, so the last slice is ragged
    for dtype, tol in ((torch.float32, 1e-6), (torch.bfloat16, 2e-2)):
        ar = NVLSAllReduce(40000 + 8 * 13, dtype=dtype, heap=heap)
        errs = []
        for _ in range(3):
            x = torch.randn(ar.numel, device=dev, generator=g).to(dtype)
            ref = x.float().clone()
            dist.all_reduce(ref)
            ar.tensor().copy_(x)
            got = ar.run(scale=0.5).float()
            torch.cuda.synchronize(dev)
            errs.append(((got - 0.5 * ref).norm() / ref.norm()).item())
        out[f"ar_{dtype}"] = (max(errs), tol)
    # reduce-scatter (stage + reduce) and the broadcast all-gather
    shard = 4096 + 8 * 37
    stage_off = heap.alloc(world * shard * 2)
    flag_off = heap.alloc(16 * world)
    ag_off = heap.alloc(world * shard * 2)
    stage = heap.view(stage_off, (world * shard,), torch.bfloat16)
    flags = heap.view(flag_off, (4 * world,), torch.int32)
    ready, consumed, agfree, agready = (flags[i * world:(i + 1) * world] for i in range(4))
    counters = torch.zeros(4, dtype=torch.int32, device=dev)
    errs = []
    for epoch in (1, 2, 3):
        src = torch.randn(world * shard, device=dev, generator=g)
        ref = torch.empty(shard, device=dev)
        dist.reduce_scatter_tensor(ref, src.clone(), op=dist.ReduceOp.AVG)
        dst = torch.zeros(shard, device=dev)
        sumsq = torch.zeros((), device=dev)
        C.nvls_rs_stage(src, stage, consumed, heap.bases, flag_off, rank, world, epoch, counters[0:1], heap.err)
        C.nvls_rs_reduce(heap.mc(stage_off), dst, 1.0 / world, False, ready, heap.bases, flag_off + 4 * world, rank,
                         world, epoch, sumsq, counters[1:2], heap.err)
        torch.cuda.synchronize(dev)
        errs.append(((dst - ref).norm() / ref.norm()).item())
        assert float(src.abs().max()) == 0.0
        out[f"sumsq{epoch}"] = (float(sumsq), float(dst.pow(2).sum()))
    out["rs_rel_err"] = max(errs)
    master = torch.randn(shard, device=dev, generator=g)
    gathered = heap.view(ag_off, (world * shard,), torch.bfloat16)
    for epoch in (1, 2):
        master.add_(1.0)
        C.nvls_ag_publish(master, heap.mc(ag_off), agfree, heap.bases, flag_off + 8 * world, flag_off + 12 * world,
                          rank, world, epoch, counters[2:3], heap.err)
        C.nvls_wait(agready, world, epoch, heap.err)
        ref = torch.empty(world * shard, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(ref, master.to(torch.bfloat16))
        torch.cuda.synchronize(dev)
        out[f"ag_equal{epoch}"] = bool(torch.equal(gathered, ref))
    heap.check()
    heap.close()
    return out


@needs2
def test_nvls_collectives_match_nccl():
    world = min(torch.cuda.device_count(), 4)
    res = run_ranks(_collectives, world, backend="nccl")
    if res[0]["skip"]:
        pytest.skip("no NVSwitch multicast on this node")
    for r in res:
        for key in ("ar_torch.float32", "ar_torch.bfloat16"):
            err, tol = r[key]
            assert err < tol, (key, err)
        assert r["rs_rel_err"] < 1e-2, r
        for e in (1, 2, 3):
            a, b = r[f"sumsq{e}"]
            assert abs(a - b) <= 1e-3 * b
        assert r["ag_equal1"] and r["ag_equal2"]


def _engine_steps(rank, world, comm):
    import torch.distributed as dist

    from genesis.model import HLRT, HLRTConfig
    from llm_research_b200.parallel.fsdp import FlatShardEngine

    torch.manual_seed(0)
    cfg = HLRTConfig(vocab_size=512, d_model=128, tier1_num_layers=2, tier1_num_heads=2, tier1_d_ff=256,
                     gate1_chunk_size=16, num_latent_vectors=4, latent_pool_num_heads=2,
                     tier2_d_model=128, tier2_num_layers=1, tier2_num_heads=2, tier2_d_ff=256,
                     tier3_d_model=128, tier3_num_layers=1, tier3_num_heads=2, tier3_d_ff=256)
    dev = torch.device("cuda", rank)
    model = HLRT(cfg).to(dev)
    eng = FlatShardEngine(model, comm=comm)
    if eng.comm != comm:
        return {"skip": True}
    opt = eng.make_optimizer(torch.optim.AdamW, {"lr": 1e-3})
    g = torch.Generator().manual_seed(rank)
    losses = []
    for step in range(3):
        for micro in range(2):  # gradient accumulation: the reduce-scatter runs on the second
            eng.set_sync(micro == 1)
            ids = torch.randint(0, 512, (2, 64), generator=g).to(dev)
            out = eng(ids)
            loss = torch.nn.functional.cross_entropy(out["logits"][:, :-1].float().reshape(-1, 512),
                                                     ids[:, 1:].reshape(-1))
            loss.backward()
        eng.clip_grad_norm_(1.0)
        opt.step()
        opt.zero_grad()
        t = loss.detach().clone()
        dist.all_reduce(t)
        losses.append(float(t) / world)
    full = eng.full_state_dict()
    if eng.heap is not None:
        eng.heap.check()
    eng.close()
    return {"skip": False, "losses": losses, "params": {k: v for k, v in list(full.items())[:6]}}


@needs2
def test_engine_nvls_matches_nccl():
    a = run_ranks(_engine_steps, 2, "nccl", backend="nccl")
    b = run_ranks(_engine_steps, 2, "nvls", backend="nccl")
    if b[0]["skip"]:
        pytest.skip("no NVSwitch multicast on this node")
    for la, lb in zip(a[0]["losses"], b[0]["losses"]):
        assert abs(la - lb) < 2e-2 * abs(la), (a[0]["losses"], b[0]["losses"])
    for k in a[0]["params"]:
        torch.testing.assert_close(a[0]["params"][k], b[0]["params"][k], atol=5e-3, rtol=5e-2)


def _diloco(rank, world, comm, nesterov):
    from llm_research_b200.parallel.diloco import DiLoCo, DiLoCoConfig, make_diloco_groups

    dev = torch.device("cuda", rank)
    _, rg, ranks, _ = make_diloco_groups(world)
    g = torch.Generator(device=dev).manual_seed(0)
    shards = [torch.randn(5000, device=dev, generator=g), torch.randn(300, 7, device=dev, generator=g)]
    dl = DiLoCo(shards, rg, ranks, DiLoCoConfig(inner_steps=1, comm=comm, nesterov=nesterov))
    if dl.comm != comm:
        dl.close()
        return None
    for step in range(3):
        for s in shards:
            s.add_(0.01 * (rank + 1) * (step + 1))
        dl.step()
    out = dl.anchor[: dl.numel].cpu().clone()
    dl.close()
    return out


@needs2
@pytest.mark.parametrize("nesterov", [True, False])
def test_diloco_nvls_outer_step_matches_collective(nesterov):
    world = min(torch.cuda.device_count(), 4)
    a = run_ranks(_diloco, world, "collective", nesterov, backend="nccl")
    b = run_ranks(_diloco, world, "nvls", nesterov, backend="nccl")
    if b[0] is None:
        pytest.skip("no NVSwitch multicast on this node")
    for r in range(world):
        torch.testing.assert_close(b[r], a[r], atol=1e-5, rtol=1e-5)
