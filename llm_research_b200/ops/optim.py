"""Optimizer kernels: Muon prologue/epilogue, batched Newton-Schulz, multi-tensor AdamW.

Muon prologue, per 2-D parameter (``olympus/optim/muon_adamw_hybrid.py:118-136``):
``p *= 1 - lr*wd``; ``buf = mu*buf + g``; ``u = g + mu*buf``; ``||g||_F``.
All matrices of a group are handled by one launch; ``u`` is written in the
Newton-Schulz compute dtype.

Newton-Schulz: ``X = G / (||G||_F + eps)`` then ``steps`` times
``A = X X^T; X = a X + (b A + c A A) X`` on the wide orientation (rows <= cols),
``(a, b, c) = (3.4445, -4.7750, 2.0315)``.  Batched over a leading dimension.

Muon epilogue: ``p -= lr * ||g|| / (||o|| + 1e-8) * o``.

AdamW (bias-corrected, decoupled decay) over a list of tensors in one launch
per chunk of tensors: ``p *= 1 - lr*wd; m = b1 m + (1-b1) g;
v = b2 v + (1-b2) g^2; p -= lr * (m/bc1) / (sqrt(v/bc2) + eps)``.
"""

from __future__ import annotations

from typing import List, Sequence, Tuple

import torch

from llm_research_b200._ext import native

NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315


@torch.no_grad()
def muon_prologue(
    params: Sequence[torch.Tensor],
    grads: Sequence[torch.Tensor],
    bufs: Sequence[torch.Tensor],
    lr: float,
    momentum: float,
    weight_decay: float,
    out_dtype: torch.dtype | None = None,
) -> Tuple[List[torch.Tensor], torch.Tensor]:
    if not params:
        return [], torch.zeros(0)
    if not params[0].is_cuda:
        outs, norms = [], []
        for p, g, b in zip(params, grads, bufs):
            if weight_decay != 0.0:
                p.mul_(1.0 - lr * weight_decay)
            b.mul_(momentum).add_(g)
            outs.append(g + momentum * b)
            norms.append(g.norm())
        return outs, torch.stack(norms)
    dt = torch.bfloat16 if out_dtype is None else out_dtype
    outs = [torch.empty(p.shape, dtype=dt, device=p.device) for p in params]
    gnorm = native().muon_prologue(list(params), list(grads), list(bufs), outs, float(lr), float(momentum), float(weight_decay))
    return outs, gnorm


@torch.no_grad()
def muon_prologue_into(params, grads, bufs, outs, lr: float, momentum: float, weight_decay: float) -> torch.Tensor:
    """Like :func:`muon_prologue` but writes the Nesterov directions into ``outs``."""
    if not params:
        return torch.zeros(0)
    if not params[0].is_cuda:
        norms = []
        for p, g, b, o in zip(params, grads, bufs, outs):
            if weight_decay != 0.0:
                p.mul_(1.0 - lr * weight_decay)
            b.mul_(momentum).add_(g)
            o.copy_(g + momentum * b)
            norms.append(g.norm())
        return torch.stack(norms)
    return native().muon_prologue(list(params), list(grads), list(bufs), list(outs), float(lr), float(momentum), float(weight_decay))


@torch.no_grad()
def axpy_list(xs, ys, alpha: float) -> None:
    """``x += alpha * y`` for every pair (``y`` may have a narrower dtype)."""
    if not xs:
        return
    if not xs[0].is_cuda:
        for x, y in zip(xs, ys):
            x.add_(y.to(x.dtype), alpha=alpha)
        return
    native().axpy_list(list(xs), list(ys), float(alpha))


@torch.no_grad()
def muon_epilogue(params: Sequence[torch.Tensor], orth: Sequence[torch.Tensor], gnorms: torch.Tensor, lr: float) -> None:
    if not params:
        return
    if not params[0].is_cuda:
        for i, (p, o) in enumerate(zip(params, orth)):
            scale = gnorms[i] / (o.norm() + 1e-8)
            p.add_(o.to(p.dtype) * scale, alpha=-lr)
        return
    native().muon_epilogue(list(params), [o.contiguous() for o in orth], gnorms, float(lr))


@torch.no_grad()
def newton_schulz(G: torch.Tensor, steps: int = 5, eps: float = 1e-7, compute_dtype: torch.dtype | None = None) -> torch.Tensor:
    squeeze = G.dim() == 2
    X = G.unsqueeze(0) if squeeze else G
    transposed = X.shape[-2] > X.shape[-1]
    if transposed:
        X = X.transpose(-1, -2)
    if compute_dtype is None:
        compute_dtype = torch.bfloat16 if G.is_cuda else torch.float32
    norms = X.float().flatten(1).norm(dim=1).view(-1, 1, 1)
    X = (X.float() / (norms + eps)).to(compute_dtype)
    if G.is_cuda:
        X = native().newton_schulz(X.contiguous(), int(steps), NS_A, NS_B, NS_C)
    else:
        for _ in range(steps):
            A = X @ X.transpose(-1, -2)
            Bm = NS_B * A + NS_C * (A @ A)
            X = NS_A * X + Bm @ X
    if transposed:
        X = X.transpose(-1, -2)
    X = X.to(G.dtype)
    return X.squeeze(0) if squeeze else X


@torch.no_grad()
def adamw_step(
    params: Sequence[torch.Tensor],
    grads: Sequence[torch.Tensor],
    exp_avgs: Sequence[torch.Tensor],
    exp_avg_sqs: Sequence[torch.Tensor],
    steps: Sequence[int],
    lr: float,
    beta1: float,
    beta2: float,
    eps: float,
    weight_decay: float,
) -> None:
    if not params:
        return
    if not params[0].is_cuda:
        for p, g, m, v, t in zip(params, grads, exp_avgs, exp_avg_sqs, steps):
            if weight_decay != 0.0:
                p.mul_(1.0 - lr * weight_decay)
            m.mul_(beta1).add_(g, alpha=1.0 - beta1)
            v.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
            denom = (v / (1.0 - beta2 ** t)).sqrt().add_(eps)
            p.addcdiv_(m / (1.0 - beta1 ** t), denom, value=-lr)
        return
    bc1 = [1.0 - beta1 ** t for t in steps]
    bc2 = [1.0 - beta2 ** t for t in steps]
    native().adamw_step(list(params), list(grads), list(exp_avgs), list(exp_avg_sqs), bc1, bc2,
                        float(lr), float(beta1), float(beta2), float(eps), float(weight_decay))
