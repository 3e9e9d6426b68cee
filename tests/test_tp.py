"""Tensor-parallel linear layers: gloo CPU ranks (collective fallback) and, on
2+ GPUs, the fused ag_gemm / gemm_rs kernels, against an unsharded layer."""

import pytest
import torch

from tests.dist_utils import run_ranks


def _tp_case(rank, world, fused):
    import torch.distributed as dist

    from llm_research_b200.parallel.tp import ColumnParallelLinear, RowParallelLinear, TPComm, shard_linear_weight

    dev = torch.device("cuda", rank) if fused else torch.device("cpu")
    dt = torch.bfloat16 if fused else torch.float32
    T, d, h = 512, 256, 512
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, d, generator=g).to(dev, dt)
    w1 = (torch.randn(h, d, generator=g) * 0.05).to(dev, dt)
    w2 = (torch.randn(d, h, generator=g) * 0.05).to(dev, dt)
    dy = torch.randn(T, d, generator=g).to(dev, dt)
    comm = TPComm(None, max_tokens=T, max_width=max(d, h), device=dev) if fused else None
    col = ColumnParallelLinear(d, h, comm=comm, device=dev, dtype=dt)
    row = RowParallelLinear(h, d, comm=comm, device=dev, dtype=dt)
    with torch.no_grad():
        col.weight.copy_(shard_linear_weight(w1, None, 0))
        row.weight.copy_(shard_linear_weight(w2, None, 1))
    xs = x.chunk(world)[rank].clone().requires_grad_()
    res = x.chunk(world)[rank].clone()
    hmid = torch.nn.functional.gelu(col(xs).float()).to(dt)
    y = row(hmid, residual=res)
    y.backward(dy.chunk(world)[rank])
    out = {"y": y.detach().float().cpu(), "dx": xs.grad.float().cpu(), "dw1": col.weight.grad.float().cpu(),
           "dw2": row.weight.grad.float().cpu()}
    if comm is not None:
        comm.heap.check()
        comm.close()
    return out


def _reference(world):
    T, d, h = 512, 256, 512
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, d, generator=g)
    w1 = torch.randn(h, d, generator=g) * 0.05
    w2 = torch.randn(d, h, generator=g) * 0.05
    dy = torch.randn(T, d, generator=g)
    x.requires_grad_()
    w1.requires_grad_()
    w2.requires_grad_()
    y = torch.nn.functional.gelu(x @ w1.t()) @ w2.t() + x.detach()
    y.backward(dy)
    return y.detach(), x.grad, w1.grad, w2.grad


def _check(res, world, tol):
    y, dx, dw1, dw2 = _reference(world)
    for r, o in enumerate(res):
        torch.testing.assert_close(o["y"], y.chunk(world)[r], atol=tol, rtol=tol)
        torch.testing.assert_close(o["dx"], dx.chunk(world)[r], atol=tol, rtol=tol)
        torch.testing.assert_close(o["dw1"], dw1.chunk(world, 0)[r], atol=tol * 4, rtol=tol)
        torch.testing.assert_close(o["dw2"], dw2.chunk(world, 1)[r], atol=tol * 4, rtol=tol)


def test_tp_layers_collective_fallback_cpu():
    _check(run_ranks(_tp_case, 2, False), 2, 1e-4)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_layers_fused_kernels_gpu():
    _check(run_ranks(_tp_case, 2, True, backend="nccl"), 2, 5e-2)


def _hlrt_tp_case(rank, world, fused, memory=False, labels=False):
    """HLRT with a tensor + sequence parallel Tier 1 against the same weights unsharded."""
    import torch.distributed as dist

    from genesis.model.hlrt import HLRT
    from llm_research_b200.models.presets import build_hlrt_config
    from llm_research_b200.parallel.tp import TPComm, tensor_parallel

    dev = torch.device("cuda", rank) if fused else torch.device("cpu")
    cfg = build_hlrt_config("toy")
    cfg.gate_loss_weight = 0.0
    if memory:  # memory reads between the sequence-parallel blocks
        cfg.tier1_memory_every = 1
        cfg.memory_slots = 512
        cfg.memory_top_k = 4
    torch.manual_seed(0)
    full = HLRT(cfg).to(dev)
    comm = TPComm(None, max_tokens=256, max_width=512, device=dev) if fused else None
    with tensor_parallel(dist.group.WORLD, comm):
        tp = HLRT(cfg).to(dev)
    fp = dict(full.named_parameters())
    with torch.no_grad():
        for name, p in tp.named_parameters():
            src = fp[name]
            dim = getattr(p, "_lrb_tp", None)
            p.copy_(src if dim is None else src.chunk(world, dim=dim)[rank])
        fb = dict(full.named_buffers())
        for name, b in tp.named_buffers():
            b.copy_(fb[name])
    dt = torch.bfloat16 if fused else torch.float32
    full.to(dt)
    tp.to(dt)
    ids = torch.randint(0, cfg.vocab_size, (2, 128), generator=torch.Generator().manual_seed(1)).to(dev)
    if labels:  # fused head + loss: vocabulary-parallel over the TP group
        assert tp._vocab_parallel_group is not None and full._vocab_parallel_group is None
        tgt = torch.cat([ids[:, 1:], ids.new_full((2, 1), -100)], dim=1)
        out_f = full(ids, labels=tgt)["lm_loss"]
        out_t = tp(ids, labels=tgt)["lm_loss"]
        out_f.backward()
        out_t.backward()
    else:
        out_f = full(ids)["logits"]
        out_t = tp(ids)["logits"]
        gl = torch.randn(out_f.shape, generator=torch.Generator().manual_seed(2)).to(dev, dt)
        (out_f.float() * gl.float()).sum().backward()
        (out_t.float() * gl.float()).sum().backward()
    res = {"logits": (out_f.float().cpu(), out_t.float().cpu()), "grads": {}}
    for name, p in tp.named_parameters():
        if p.grad is None:
            continue
        g_full = fp[name].grad
        dim = getattr(p, "_lrb_tp", None)
        ref = g_full if dim is None else g_full.chunk(world, dim=dim)[rank]
        res["grads"][name] = (ref.float().cpu(), p.grad.float().cpu())
    if comm is not None:
        comm.heap.check()
        comm.close()
    return res


@pytest.mark.parametrize("memory", [False, True])
def test_hlrt_tensor_parallel_tier1_matches_unsharded_cpu(memory):
    for res in run_ranks(_hlrt_tp_case, 2, False, memory):
        ref, got = res["logits"]
        torch.testing.assert_close(got, ref, atol=1e-4, rtol=1e-4)
        assert any("q_proj" in n for n in res["grads"]) and any("attn_norm" in n for n in res["grads"])
        for name, (r, g) in res["grads"].items():
            torch.testing.assert_close(g, r, atol=1e-4, rtol=1e-3, msg=name)


def test_hlrt_tensor_parallel_vocab_parallel_loss_cpu():
    for res in run_ranks(_hlrt_tp_case, 2, False, False, True):
        ref, got = res["logits"]
        torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)
        assert any("embeddings" in n for n in res["grads"])
        for name, (r, g) in res["grads"].items():
            torch.testing.assert_close(g, r, atol=1e-4, rtol=1e-3, msg=name)


def _vocab_ce_case(rank, world, V, ignore=-100):
    import torch.distributed as dist

    from llm_research_b200.ops.loss import linear_cross_entropy, vocab_parallel_linear_cross_entropy

    g = torch.Generator().manual_seed(3)
    h = torch.randn(50, 16, generator=g)
    w = torch.randn(V, 16, generator=g) * 0.5
    t = torch.randint(0, V, (50,), generator=g)
    t[::7] = ignore
    out = {}
    for name, fn in (("full", lambda a, b: linear_cross_entropy(a, b, t, ignore_index=ignore, chunk=16)),
                     ("vp", lambda a, b: vocab_parallel_linear_cross_entropy(a, b, t, dist.group.WORLD,
                                                                             ignore_index=ignore, chunk=16))):
        a, b = h.clone().requires_grad_(), w.clone().requires_grad_()
        loss = fn(a, b)
        (loss * 1.5).backward()
        out[name] = (loss.detach(), a.grad, b.grad)
    return out


@pytest.mark.parametrize("V", [40, 37])
def test_vocab_parallel_linear_cross_entropy_cpu(V):
    for res in run_ranks(_vocab_ce_case, 2, V):
        for r, g in zip(res["full"], res["vp"]):
            torch.testing.assert_close(g, r, atol=1e-5, rtol=1e-5)


def test_vocab_parallel_linear_cross_entropy_ignore_minus_one_cpu():
    """ignore_index=-1 must not collide with the marker of rows owned by another shard."""
    for res in run_ranks(_vocab_ce_case, 2, 40, -1):
        for r, g in zip(res["full"], res["vp"]):
            torch.testing.assert_close(g, r, atol=1e-5, rtol=1e-5)


def test_vocab_parallel_linear_cross_entropy_empty_shard_cpu():
    """V=5 over 4 ranks: ceil(5/4)=2 rows per rank, so the last rank owns none."""
    for res in run_ranks(_vocab_ce_case, 4, 5):
        for r, g in zip(res["full"], res["vp"]):
            torch.testing.assert_close(g, r, atol=1e-5, rtol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("labels", [False, True])
def test_hlrt_tensor_parallel_tier1_fused_kernels(labels):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    for res in run_ranks(_hlrt_tp_case, 2, True, False, labels, backend="nccl"):
        ref, got = res["logits"]
        assert ((got - ref).norm() / ref.norm()).item() < 2e-2
        for name, (r, g) in res["grads"].items():
            rel = ((g - r).norm() / (r.norm() + 1e-6)).item()
            assert rel < 5e-2, (name, rel)


def _fsdp_tp_train(rank, world, fused_loss=False):
    """FSDP x2 (dp) + TP x2 on 4 gloo ranks, Muon hybrid + clipping, two steps;
    ``fused_loss``: the head + loss run vocabulary-parallel over the TP group."""
    import torch.distributed as dist

    from genesis.training.train_phase1_bootstrap import ntp_objective
    from llm_research_b200.parallel.tp import tensor_parallel
    from olympus.core.training_orchestrator import ModelConfig, ObjectiveConfig
    from olympus.distributed.distributed_orchestrator import DistributedTrainingOrchestrator
    from olympus.distributed.fsdp_wrapper import FSDPConfig
    from olympus.optim import MuonAdamWHybrid
    from tests.test_engine import _data, _toy_model

    tp = 2
    tp_groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
    dp_groups = [dist.new_group([0, 2]), dist.new_group([1, 3])]
    tpg, dpg = tp_groups[rank // tp], dp_groups[rank % tp]
    full = _toy_model()
    with tensor_parallel(tpg):
        model = _toy_model()
    fp = dict(full.named_parameters())
    with torch.no_grad():
        for name, p in model.named_parameters():
            dim = getattr(p, "_lrb_tp", None)
            p.copy_(fp[name] if dim is None else fp[name].chunk(tp, dim=dim)[rank % tp])
    opt = MuonAdamWHybrid(model.parameters(), lr_muon=0.02, lr_adamw=1e-3, weight_decay_muon=0.01)
    orch = DistributedTrainingOrchestrator(
        fsdp_config=FSDPConfig(mixed_precision="fp32", activation_checkpointing=False, process_group=dpg, tp_group=tpg),
        device=torch.device("cpu"))
    orch.add_model(ModelConfig("hlrt", model, opt, max_grad_norm=1.0))
    orch.add_objective(ObjectiveConfig("ntp", ntp_objective))
    data = _data()
    d = rank // tp
    for _ in range(2):
        orch.step({"input_ids": data[2 * d: 2 * d + 2], "fused_lm_loss": fused_loss})
    sd = orch._models["hlrt"].model.full_state_dict()
    return {k: (v, getattr(dict(model.named_parameters())[k], "_lrb_tp", None)) for k, v in sd.items()}


@pytest.mark.parametrize("fused_loss", [False, True])
def test_fsdp_plus_tensor_parallel_matches_single_process(fused_loss):
    from tests.test_engine import _data, _toy_model, _train

    single, _ = _train(_toy_model(), [_data()], engine=False, steps=2)
    res = run_ranks(_fsdp_tp_train, 4, fused_loss)
    for rank, sd in enumerate(res):
        for k, (v, dim) in sd.items():
            ref = single[k] if dim is None else single[k].chunk(2, dim=dim)[rank % 2]
            torch.testing.assert_close(v, ref, atol=5e-5, rtol=1e-4, msg=f"rank {rank} {k}")


def _tp_rows_and_nvfp4_case(rank, world, use_comm):
    """The heap's P2P row all-gather / reduce-scatter against NCCL, then an NVFP4
    column + row layer pair (P2P collectives around the block-scaled GEMMs)."""
    import torch.distributed as dist

    from llm_research_b200.ops.linear import linear_precision
    from llm_research_b200.parallel.tp import ColumnParallelLinear, RowParallelLinear, TPComm, shard_linear_weight

    dev = torch.device("cuda", rank)
    T, d, h = 512, 256, 512
    comm = TPComm(None, max_tokens=T, max_width=max(d, h), device=dev) if use_comm else None
    out = {}
    if comm is not None:
        g = torch.Generator(device=dev).manual_seed(10 + rank)
        for e in range(3):  # slot and flag reuse
            xs = torch.randn(T // world, d, device=dev, generator=g).to(torch.bfloat16)
            ref = torch.empty(T, d, dtype=torch.bfloat16, device=dev)
            dist.all_gather_into_tensor(ref, xs)
            out[f"ag{e}"] = bool(torch.equal(comm.all_gather(xs), ref))
            y = torch.randn(T, h, device=dev, generator=g).to(torch.bfloat16)
            res = torch.randn(T // world, h, device=dev, generator=g).to(torch.bfloat16)
            ref = torch.empty(T // world, h, device=dev)
            dist.reduce_scatter_tensor(ref, y.float())
            got = comm.reduce_scatter(y, res).float()
            out[f"rs{e}"] = ((got - ref - res.float()).norm() / ref.norm()).item()
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, d, generator=g).to(dev, torch.bfloat16)
    w1 = (torch.randn(h, d, generator=g) * 0.05).to(dev, torch.bfloat16)
    w2 = (torch.randn(d, h, generator=g) * 0.05).to(dev, torch.bfloat16)
    dy = torch.randn(T, d, generator=g).to(dev, torch.bfloat16)
    col = ColumnParallelLinear(d, h, comm=comm, device=dev, dtype=torch.bfloat16)
    row = RowParallelLinear(h, d, comm=comm, device=dev, dtype=torch.bfloat16)
    with torch.no_grad():
        col.weight.copy_(shard_linear_weight(w1, None, 0))
        row.weight.copy_(shard_linear_weight(w2, None, 1))
    xs = x.chunk(world)[rank].clone().requires_grad_()
    with linear_precision("nvfp4"):
        y = row(torch.relu(col(xs)), residual=x.chunk(world)[rank].clone())
        y.backward(dy.chunk(world)[rank])
    out.update(y=y.detach().float().cpu(), dx=xs.grad.float().cpu(), dw1=col.weight.grad.float().cpu(),
               dw2=row.weight.grad.float().cpu())
    if comm is not None:
        comm.heap.check()
        comm.close()
    return out


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_p2p_rows_and_nvfp4_layers_gpu():
    a = run_ranks(_tp_rows_and_nvfp4_case, 2, True, backend="nccl")
    b = run_ranks(_tp_rows_and_nvfp4_case, 2, False, backend="nccl")
    for r in range(2):
        for e in range(3):
            assert a[r][f"ag{e}"], (r, e)
            assert a[r][f"rs{e}"] < 1e-2, (r, e, a[r][f"rs{e}"])
        # same NVFP4 GEMMs (and stochastic-rounding draws) around P2P or NCCL collectives
        for k in ("y", "dx", "dw1", "dw2"):
            torch.testing.assert_close(a[r][k], b[r][k], atol=3e-2, rtol=3e-2, msg=k)
