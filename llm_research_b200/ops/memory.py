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
