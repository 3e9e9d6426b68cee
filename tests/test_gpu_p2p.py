"""Symmetric-memory collectives on 2+ GPUs (one NCCL rank per GPU) against NCCL.

Skipped when fewer than two GPUs are visible."""

import pytest
import torch

from tests.dist_utils import run_ranks

pytestmark = pytest.mark.gpu

needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs at least two GPUs")


def _collectives(rank, world):
    import torch.distributed as dist

    from llm_research_b200._ext import native
    from llm_research_b200.parallel.symm import SymmetricHeap

    C = native()
    dev = torch.device("cuda", rank)
    shard = 4096 + 8 * 37
    heap = SymmetricHeap(1 << 24, device=dev)
    recv_off = heap.alloc(world * shard * 2)
    ready_off = heap.alloc(4 * world)
    consumed_off = heap.alloc(4)
    ag_off = heap.alloc(shard * 2)
    agready_off = heap.alloc(4)
    recv = heap.view(recv_off, (world * shard,), torch.bfloat16)
    ready = heap.view(ready_off, (world,), torch.int32)
    consumed = heap.view(consumed_off, (1,), torch.int32)
    agready = heap.view(agready_off, (1,), torch.int32)
    counters = torch.zeros(4, dtype=torch.int32, device=dev)
    out = {}
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    errs = []
    for epoch in (1, 2, 3):  # slot reuse across epochs
        src = torch.randn(world * shard, device=dev, generator=g)
        ref = torch.empty(shard, device=dev)
        dist.reduce_scatter_tensor(ref, src.clone(), op=dist.ReduceOp.AVG)
        dst = torch.zeros(shard, device=dev)
        sumsq = torch.zeros((), device=dev)
        C.p2p_rs_push(src, heap.bases, recv_off, ready_off, consumed_off, rank, world, shard, epoch,
                      counters[0:1], heap.err)
        C.p2p_rs_reduce(recv, dst, world, 1.0 / world, False, ready, consumed, epoch, sumsq, counters[1:2], heap.err)
        torch.cuda.synchronize(dev)
        errs.append(((dst - ref).norm() / ref.norm()).item())
        assert float(src.abs().max()) == 0.0
        out[f"sumsq{epoch}"] = (float(sumsq), float(dst.pow(2).sum()))
    out["rs_rel_err"] = max(errs)
    master = torch.randn(shard, device=dev, generator=g)
    shard_view = heap.view(ag_off, (shard,), torch.bfloat16)
    full = torch.empty(world * shard, dtype=torch.bfloat16, device=dev)
    for epoch in (1, 2):
        master.add_(1.0)
        C.p2p_ag_publish(master, shard_view, agready, epoch, counters[2:3])
        C.p2p_pull(full, heap.bases, ag_off, agready_off, world, epoch, heap.err)
        ref = torch.empty(world * shard, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(ref, master.to(torch.bfloat16))
        torch.cuda.synchronize(dev)
        out[f"ag_equal{epoch}"] = bool(torch.equal(full, ref))
    heap.check()
    heap.close()
    return out


@needs2
def test_p2p_reduce_scatter_and_all_gather_match_nccl():
    world = min(torch.cuda.device_count(), 4)
    res = run_ranks(_collectives, world, backend="nccl")
    for r in res:
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
    assert eng.comm == comm
    opt = eng.make_optimizer(torch.optim.AdamW, {"lr": 1e-3})
    g = torch.Generator().manual_seed(rank)
    losses = []
    for step in range(3):
        ids = torch.randint(0, 512, (2, 64), generator=g).to(dev)
        out = eng(ids)
        loss = torch.nn.functional.cross_entropy(out["logits"][:, :-1].float().reshape(-1, 512), ids[:, 1:].reshape(-1))
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
    return losses, {k: v for k, v in list(full.items())[:4]}


@needs2
def test_engine_p2p_matches_nccl():
    a = run_ranks(_engine_steps, 2, "nccl", backend="nccl")
    b = run_ranks(_engine_steps, 2, "p2p", backend="nccl")
    for la, lb in zip(a[0][0], b[0][0]):
        assert abs(la - lb) < 2e-2 * abs(la), (a[0][0], b[0][0])
    for k in a[0][1]:
        torch.testing.assert_close(a[0][1][k], b[0][1][k], atol=5e-3, rtol=5e-2)


def _diloco(rank, world, comm):
    from llm_research_b200.parallel.diloco import DiLoCo, DiLoCoConfig, make_diloco_groups

    dev = torch.device("cuda", rank)
    _, rg, ranks, _ = make_diloco_groups(world)
    g = torch.Generator(device=dev).manual_seed(0)
    shards = [torch.randn(5000, device=dev, generator=g), torch.randn(300, 7, device=dev, generator=g)]
    dl = DiLoCo(shards, rg, ranks, DiLoCoConfig(inner_steps=1, comm=comm))
    assert dl.comm == comm
    for step in range(3):
        for s in shards:
            s.add_(0.01 * (rank + 1) * (step + 1))
        dl.step()
    out = dl.anchor[: dl.numel].cpu().clone()
    dl.close()
    return out


@needs2
def test_diloco_p2p_outer_step_matches_collective():
    world = min(torch.cuda.device_count(), 4)
    a = run_ranks(_diloco, world, "collective", backend="nccl")
    b = run_ranks(_diloco, world, "p2p", backend="nccl")
    for r in range(world):
        torch.testing.assert_close(a[r], a[0])
        torch.testing.assert_close(b[r], a[r], atol=1e-5, rtol=1e-5)


def _dmuon_steps(rank, world, dmuon_comm):
    """Three MuonAdamWHybrid steps through the engine with the distributed-Muon
    exchange on symmetric memory (P2P pulls) or on NCCL all-to-alls."""
    import os

    import torch.distributed as dist

    os.environ["LRB_DMUON_COMM"] = dmuon_comm
    from genesis.model import HLRT, HLRTConfig
    from llm_research_b200.parallel.fsdp import FlatShardEngine
    from olympus.optim import MuonAdamWHybrid

    torch.manual_seed(0)
    cfg = HLRTConfig(vocab_size=512, d_model=128, tier1_num_layers=2, tier1_num_heads=2, tier1_d_ff=256,
                     gate1_chunk_size=16, num_latent_vectors=4, latent_pool_num_heads=2,
                     tier2_d_model=128, tier2_num_layers=1, tier2_num_heads=2, tier2_d_ff=256,
                     tier3_d_model=128, tier3_num_layers=1, tier3_num_heads=2, tier3_d_ff=256)
    dev = torch.device("cuda", rank)
    eng = FlatShardEngine(HLRT(cfg).to(dev), comm="nccl")
    opt = eng.make_optimizer(MuonAdamWHybrid, {"lr_muon": 0.02, "lr_adamw": 1e-3, "momentum": 0.95,
                                               "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay_muon": 0.0,
                                               "weight_decay_adamw": 0.01, "ns_steps": 5,
                                               "muon_max_aspect_ratio": 8.0})
    assert (opt.p2p is not None) == (dmuon_comm == "p2p")
    g = torch.Generator().manual_seed(rank)
    for _ in range(3):
        ids = torch.randint(0, 512, (2, 64), generator=g).to(dev)
        out = eng(ids)
        loss = torch.nn.functional.cross_entropy(out["logits"][:, :-1].float().reshape(-1, 512), ids[:, 1:].reshape(-1))
        loss.backward()
        opt.step()
        opt.zero_grad()
    full = eng.full_state_dict()
    if opt.p2p is not None:
        opt.p2p.heap.check()
        opt.p2p.close()
    torch.cuda.synchronize()
    dist.barrier()
    return {k: v for k, v in full.items() if v.dim() == 2}


@needs2
def test_distributed_muon_p2p_exchange_matches_nccl():
    a = run_ranks(_dmuon_steps, 2, "nccl", backend="nccl")
    b = run_ranks(_dmuon_steps, 2, "p2p", backend="nccl")
    assert a[0].keys() == b[0].keys() and len(a[0]) > 4
    for k in a[0]:
        torch.testing.assert_close(b[0][k], a[0][k], atol=2e-3, rtol=2e-2, msg=k)
