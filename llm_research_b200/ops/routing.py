"""Routing and escalation primitives.

* :func:`softmax_topk` -- fp32 softmax over experts, top-k (ties to the lower
  index), renormalised weights ``w / (sum w + 1e-9)``; returns
  ``(weights fp32, indices int64, probs fp32)``
  (``olympus/kernels/fused_gate_route.py:36-46``).  Differentiable in
  ``weights`` and ``probs``.
* :func:`route_slots` -- for routed assignments ``idx (T, k)`` in (token, k)
  order: the capacity slot of each (its rank among earlier assignments to the
  same expert, ``-1`` at or over ``cap``; ``cap < 0`` keeps all), its owner
  rank and local expert under ``experts_per_rank``, and the per-expert counts
  -- one device kernel, no host read (the capacity rule of
  ``genesis/model/moe.py`` and of the expert-parallel dispatch).
* :func:`chunk_mean_pool` -- ``(B, S, D) -> (B, S/c, D)`` mean over chunks of
  ``c`` tokens, fp32 accumulation.
* :func:`compact_chunks` -- pack the selected chunk ids of every row of a bool
  ``(B, C)`` mask to the front: returns ``ids (B, N)`` (unused slots hold
  ``C``), ``valid (B, N)`` and ``N = max(max row count, 1)``.  One kernel does
  the per-row prefix sum and scatter; ``N`` is the only host read.
* :func:`compact_chunks_fixed` -- the same packing at the fixed width ``C``
  (every chunk could be selected), with the row counts and ``N`` left on the
  device: no host read, so the escalation path never stalls the launch queue.
"""

from __future__ import annotations

from typing import Tuple

import torch
import torch.nn.functional as F

from llm_research_b200._ext import native


def _softmax_topk_ref(logits: torch.Tensor, k: int):
    probs = F.softmax(logits, dim=-1, dtype=torch.float32)
    w, idx = torch.topk(probs, k, dim=-1)
    w = w / (w.sum(dim=-1, keepdim=True) + 1e-9)
    return w, idx, probs


class _SoftmaxTopkFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, k):
        w, idx, probs = native().softmax_topk_fwd(logits, int(k))
        ctx.save_for_backward(probs, idx)
        ctx.mark_non_differentiable(idx)
        return w, idx, probs

    @staticmethod
    def backward(ctx, dw, _didx, dprobs):
        probs, idx = ctx.saved_tensors
        sel = probs.gather(1, idx)
        denom = sel.sum(-1, keepdim=True) + 1e-9
        dw = torch.zeros_like(sel) if dw is None else dw.float()
        dsel = (dw - (dw * sel / denom).sum(-1, keepdim=True)) / denom
        dp = torch.zeros_like(probs).scatter_add_(1, idx, dsel)
        if dprobs is not None:
            dp = dp + dprobs.float()
        dlogits = probs * (dp - (probs * dp).sum(-1, keepdim=True))
        return dlogits, None


def softmax_topk(logits: torch.Tensor, top_k: int):
    if not logits.is_cuda:
        return _softmax_topk_ref(logits, top_k)
    w, idx, probs = _SoftmaxTopkFn.apply(logits.contiguous(), top_k)
    return w, idx, probs


def route_slots(idx: torch.Tensor, num_experts: int, experts_per_rank: int | None = None, cap: int = -1):
    """``(dest, local_expert, slot, counts)``, int32: see the module docstring."""
    epl = num_experts if experts_per_rank is None else int(experts_per_rank)
    if idx.is_cuda:
        return native().route_slots(idx.contiguous().long(), int(num_experts), epl, int(cap))
    flat = idx.reshape(-1).long()
    onehot = F.one_hot(flat, num_experts)
    pos = (onehot.cumsum(0) * onehot).sum(-1) - 1
    slot = pos if cap < 0 else torch.where(pos < cap, pos, torch.full_like(pos, -1))
    return ((flat // epl).int(), (flat % epl).int(), slot.int(), onehot.sum(0).int())


class _ChunkPoolFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, c):
        ctx.shape = x.shape
        ctx.c = c
        return native().chunk_mean_pool_fwd(x, int(c))

    @staticmethod
    def backward(ctx, g):
        B, S, D = ctx.shape
        c = ctx.c
        dx = (g.unsqueeze(2).expand(B, S // c, c, D) / c).reshape(B, S, D)
        return dx.contiguous(), None


def chunk_mean_pool(x: torch.Tensor, chunk_size: int) -> torch.Tensor:
    B, S, D = x.shape
    if not x.is_cuda:
        return x.view(B, S // chunk_size, chunk_size, D).mean(dim=2)
    return _ChunkPoolFn.apply(x.contiguous(), chunk_size)


def compact_chunks(mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, int]:
    B, C = mask.shape
    if mask.is_cuda:
        ids, counts = native().compact_chunks(mask.contiguous())
        n = max(int(counts.max()), 1)
        ids = ids[:, :n]
    else:
        counts = mask.sum(-1)
        n = max(int(counts.max()), 1) if B > 0 else 1
        rank = torch.cumsum(mask.to(torch.int64), dim=1) - 1
        pos = torch.where(mask, rank, torch.full_like(rank, n))
        ids = torch.full((B, n + 1), C, dtype=torch.long, device=mask.device)
        ids.scatter_(1, pos, torch.arange(C, device=mask.device).expand(B, C).contiguous())
        ids = ids[:, :n]
    valid = torch.arange(n, device=mask.device)[None, :] < counts[:, None]
    return ids, valid, n


def compact_chunks_fixed(mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """``(ids (B, C), valid (B, C), counts (B,), n (0-d))`` for a bool ``(B, C)`` mask:
    selected chunk ids packed to the front in ascending order, unused slots ``C``;
    ``n = max(max row count, 1)`` as a device scalar (the reference's slot count)."""
    B, C = mask.shape
    if mask.is_cuda:
        ids, counts = native().compact_chunks(mask.contiguous())
        ids = ids[:, :C]
    else:
        counts = mask.sum(-1)
        rank = torch.cumsum(mask.to(torch.int64), dim=1) - 1
        pos = torch.where(mask, rank, torch.full_like(rank, C))
        ids = torch.full((B, C + 1), C, dtype=torch.long, device=mask.device)
        ids.scatter_(1, pos, torch.arange(C, device=mask.device).expand(B, C).contiguous())
        ids = ids[:, :C]
    counts = counts.to(torch.int64)
    valid = torch.arange(C, device=mask.device)[None, :] < counts[:, None]
    n = counts.max().clamp_min(1) if B > 0 else torch.ones((), dtype=torch.int64, device=mask.device)
    return ids.to(torch.long), valid, counts, n
