"""Top-k memory read (PHMA semantic memory).

``topk_memory_read(q, keys, values, k)``: cosine similarity of each query
against every key, keep the ``k`` best (ties -> lower index), softmax over
their similarities and return the weighted sum of their values
(``genesis/memory/semantic_memory.py:83-134``).

CUDA: the similarity matrix is one tensor-core GEMM of the normalised
operands; selection, softmax and the value gather are one fused kernel
(``csrc/kernels/memory.cu``, one warp per query).  Differentiable with
respect to the queries (and keys) through the similarity matrix.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from llm_research_b200._ext import native


class _TopkGather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, sim, values, k):
        out, idx, w = native().topk_softmax_gather(sim.contiguous(), values.contiguous(), int(k))
        ctx.save_for_backward(values, idx, w)
        ctx.n = sim.shape[1]
        return out

    @staticmethod
    def backward(ctx, g):
        values, idx, w = ctx.saved_tensors
        Q, k = idx.shape
        dsim = torch.zeros(Q, ctx.n, device=g.device, dtype=torch.float32)
        step = max(1, (1 << 26) // max(1, k * values.shape[1]))
        for s in range(0, Q, step):
            sl = slice(s, s + step)
            dw = torch.einsum("qd,qkd->qk", g[sl].float(), values[idx[sl]].float())
            ds = w[sl] * (dw - (w[sl] * dw).sum(-1, keepdim=True))
            dsim[sl].scatter_(1, idx[sl], ds)
        return dsim, None, None


def topk_memory_read(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, k: int) -> torch.Tensor:
    sim = F.normalize(q.float(), dim=-1) @ F.normalize(keys.float(), dim=-1).t()
    if not q.is_cuda:
        top, idx = sim.topk(k, dim=-1)
        w = F.softmax(top, dim=-1)
        return (w.unsqueeze(-1) * values[idx].float()).sum(1)
    return _TopkGather.apply(sim, values, k)


# ---------------------------------------------------------------- fused bank read
TOPK_FUSED = 32


class _BankRead(torch.autograd.Function):
    """Top-32 read of a large bank without the (queries x slots) matrix: tcgen05
    similarity tiles with a streaming per-row top-32 (``memory_topk_candidates``,
    one candidate list per bank slice), a merge of the slices, then the softmax /
    value-gather kernel.  Gradient: to the queries only (the bank is memory state)."""

    @staticmethod
    def forward(ctx, qn, keys_n, values):
        C = native()
        T = qn.shape[0]
        cs, ci = C.memory_topk_candidates(qn.contiguous(), keys_n, 0)
        if cs.shape[0] > 1:
            cand_s = cs.permute(1, 0, 2).reshape(T, -1)
            cand_i = ci.permute(1, 0, 2).reshape(T, -1)
            top, pos = cand_s.topk(TOPK_FUSED, dim=1)
            idx = cand_i.gather(1, pos)
        else:
            top, idx = cs[0], ci[0]
        out, w = C.topk_gather_fwd(top.contiguous(), idx.contiguous(), values)
        ctx.save_for_backward(w, idx, values, keys_n)
        ctx.mark_non_differentiable(idx)
        return out, idx

    @staticmethod
    def backward(ctx, g, _gidx):
        w, idx, values, keys_n = ctx.saved_tensors
        dq = native().topk_gather_bwd(g.contiguous(), w, idx, values, keys_n)
        return dq.to(values.dtype), None, None


def bank_read(q: torch.Tensor, keys_n: torch.Tensor, values: torch.Tensor, k: int = TOPK_FUSED):
    """Cosine top-k read of a memory bank whose keys are already L2-normalised.

    ``q`` (T, Dk), ``keys_n`` (N, Dk), ``values`` (N, Dv).  Returns ``(out (T, Dv),
    idx (T, k))``: the softmax over the k best similarities weights the k values.
    CUDA + bf16 + k == 32: the fused kernels; otherwise the explicit matrix (the oracle)."""
    qn = F.normalize(q.float(), dim=-1)
    if (q.is_cuda and k == TOPK_FUSED and keys_n.dtype == torch.bfloat16 and values.dtype == torch.bfloat16
            and q.shape[-1] % 64 == 0 and values.shape[-1] % 256 == 0):
        out, idx = _BankRead.apply(qn.to(torch.bfloat16), keys_n, values)
        return out, idx
    sim = qn @ keys_n.float().t()
    top, idx = sim.topk(min(k, keys_n.shape[0]), dim=-1)
    w = F.softmax(top, dim=-1)
    return (w.unsqueeze(-1) * values[idx].float()).sum(1).to(values.dtype), idx
