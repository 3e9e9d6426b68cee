"""Flash attention with native grouped-query heads.

``q (B, Sq, H, D)``, ``k, v (B, Skv, Hkv, D)`` with ``H % Hkv == 0``; query
head ``h`` reads K/V head ``h // (H / Hkv)``.  With ``causal`` the mask is
aligned to the end of the key sequence: query ``i`` sees keys
``j <= i + (Skv - Sq)`` (prefill and cached decode alike, as in
``genesis/model/attention.py:176-187``).  Softmax in fp32 with scale
``1/sqrt(D)``.  Output ``(B, Sq, H, D)`` in the input dtype; the row
log-sum-exp is kept for the backward pass (and is the hook for
sequence-parallel merging).

Forward: bf16 with head_dim 128 runs the tcgen05/TMEM kernel
(``csrc/kernels/attention_sm100.cu``); other head dims and fp16 run the
``mma.sync`` kernel (``csrc/kernels/attention.cu``); the backward follows
the same split (``csrc/kernels/attention_bwd_sm100.cu`` for bf16 / 128).
``LRB_ATTN_SM100=0`` disables the tcgen05 forward and ``LRB_ATTN_BWD_SM100=0``
the tcgen05 backward; ``LRB_ATTN_FWD_ONE_TILE=1`` selects the earlier
one-Q-tile-per-CTA forward instead of the two-tile ping-pong kernel (for A/B
comparisons).
"""

from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from llm_research_b200._ext import native


def _reference(q, k, v, causal: bool, scale: float) -> torch.Tensor:
    B, Sq, H, D = q.shape
    Skv, Hkv = k.shape[1], k.shape[2]
    g = H // Hkv
    qh = q.transpose(1, 2).float()
    kh = k.transpose(1, 2).float().repeat_interleave(g, dim=1)
    vh = v.transpose(1, 2).float().repeat_interleave(g, dim=1)
    s = torch.matmul(qh, kh.transpose(-1, -2)) * scale
    if causal:
        mask = torch.ones(Sq, Skv, dtype=torch.bool, device=q.device).triu(Skv - Sq + 1)
        s = s.masked_fill(mask, float("-inf"))
    p = F.softmax(s, dim=-1)
    return torch.matmul(p, vh).transpose(1, 2).to(q.dtype)


_USE_SM100 = os.environ.get("LRB_ATTN_SM100", "1") != "0"
_USE_SM100_BWD = os.environ.get("LRB_ATTN_BWD_SM100", "1") != "0"


def _forward(q, k, v, causal: bool, scale: float):
    C = native()
    if _USE_SM100 and C.attn_sm100_supported(q, k, v):
        return C.attn_fwd_sm100(q, k, v, bool(causal), float(scale))  # tcgen05 / TMEM kernel
    return C.attn_fwd(q, k, v, bool(causal), float(scale))          # mma.sync kernel, any head dim


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        out, lse = _forward(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal = causal
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        C = native()
        dout = dout.contiguous()
        sm100 = _USE_SM100_BWD and C.attn_sm100_supported(q, k, v) and C.attn_sm100_supported(dout, k, v)
        dq, dk, dv = C.attn_bwd(dout, q, k, v, out, lse, ctx.causal, ctx.scale, sm100)
        return dq, dk, dv, None, None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True, scale: float | None = None) -> torch.Tensor:
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    if not q.is_cuda:
        return _reference(q, k, v, causal, scale)
    return _FlashAttnFn.apply(q, k, v, causal, scale)
