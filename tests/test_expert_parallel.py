"""Expert-parallel MoE against a single-process statement of the same math
(gloo CPU ranks: all_to_all path; 2 GPUs: the P2P push / pull kernels)."""

import math

import pytest
import torch
import torch.nn.functional as F

from tests.dist_utils import run_ranks

E, K, D, FF, T = 8, 2, 64, 128, 96


def _full_weights():
    g = torch.Generator().manual_seed(0)
    return (torch.randn(E, D, generator=g) * 0.5, torch.randn(E, 2 * FF, D, generator=g) * 0.05,
            torch.randn(E, D, FF, generator=g) * 0.05)


def _reference(x, router_w, w_ug, w_dn):
    logits = x @ router_w.t()
    probs = torch.softmax(logits, -1)
    w, idx = probs.topk(K, dim=-1)
    w = w / w.sum(-1, keepdim=True)
    cap = math.ceil(1.25 * x.shape[0] * K / E)
    flat = idx.reshape(-1)
    oh = F.one_hot(flat, E)
    keep = ((oh.cumsum(0) * oh).sum(-1) - 1 < cap).view(x.shape[0], K)
    y = torch.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(K):
            if keep[t, j]:
                e = int(idx[t, j])
                gu = w_ug[e] @ x[t]
                h = gu[:FF] * F.silu(gu[FF:])
                y[t] += w[t, j] * (w_dn[e] @ h)
    return y


def _case(rank, world, fused):
    from llm_research_b200.parallel.expert_parallel import EPComm, ExpertParallelMoE

    dev = torch.device("cuda", rank) if fused else torch.device("cpu")
    dt = torch.bfloat16 if fused else torch.float32
    rw, wug, wdn = _full_weights()
    epl = E // world
    comm = EPComm(None, max_tokens=T, top_k=K, d=D, experts_per_rank=epl, capacity_factor=1.25, device=dev) if fused else None
    moe = ExpertParallelMoE(D, FF, E, top_k=K, capacity_factor=1.25, shared_expert=False, comm=comm, device=dev, dtype=dt)
    with torch.no_grad():
        moe.router.weight.copy_(rw)
        moe.w_up_gate.copy_(wug[rank * epl:(rank + 1) * epl])
        moe.w_down.copy_(wdn[rank * epl:(rank + 1) * epl])
    g = torch.Generator().manual_seed(10 + rank)
    x = torch.randn(T, D, generator=g).to(dev, dt).requires_grad_()
    y = moe(x)
    y.float().pow(2).sum().backward()
    out = {"x": x.detach().float().cpu(), "y": y.detach().float().cpu(), "gx": x.grad.float().cpu(),
           "gug": moe.w_up_gate.grad.float().cpu()}
    if comm is not None:
        comm.heap.check()
        comm.close()
    return out


def _check(res, world, tol):
    rw, wug, wdn = _full_weights()
    wug = wug.clone().requires_grad_()
    loss = 0.0
    ys = []
    xs = []
    for r in range(world):
        x = res[r]["x"].clone().requires_grad_()
        y = _reference(x, rw, wug, wdn)
        loss = loss + y.pow(2).sum()
        ys.append(y)
        xs.append(x)
    loss.backward()
    epl = E // world
    for r in range(world):
        torch.testing.assert_close(res[r]["y"], ys[r].detach(), atol=tol, rtol=tol)
        torch.testing.assert_close(res[r]["gx"], xs[r].grad, atol=tol * 4, rtol=tol * 4)
        torch.testing.assert_close(res[r]["gug"], wug.grad[r * epl:(r + 1) * epl], atol=tol * 8, rtol=tol * 4)


def test_expert_parallel_collective_cpu():
    _check(run_ranks(_case, 2, False), 2, 1e-4)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_p2p_kernels_gpu():
    _check(run_ranks(_case, 2, True, backend="nccl"), 2, 5e-2)
