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
