"""Split the fused QKV projection into q, k, v and apply RoPE to q and k.

Input ``qkv``: ``(B, S, (H + 2*Hkv) * D)`` laid out ``[q heads | k heads | v heads]``.
Outputs, all contiguous: ``q (B, S, H, D)``, ``k (B, S, Hkv, D)``, ``v (B, S, Hkv, D)``.
Rotation at absolute position ``p = offset + s`` (rotate-half convention of
``genesis/model/rotary.py:74-99``): for ``i < D/2`` with angle ``p * inv_freq[i]``
``out[i] = x[i] cos - x[i + D/2] sin``, ``out[i + D/2] = x[i + D/2] cos + x[i] sin``.
The tables are read in fp32.  Backward applies the inverse rotation.
"""

from __future__ import annotations

import torch

from llm_research_b200._ext import native


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    xf = x.float()
    rot = torch.cat([-xf[..., h:], xf[..., :h]], dim=-1)
    return (xf * cos + rot * sin).to(x.dtype)


class _RopeQKVFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos, sin, H, Hkv, D, offset):
        q, k, v = native().rope_qkv_fwd(qkv, cos, sin, H, Hkv, D, offset)
        ctx.save_for_backward(cos, sin)
        ctx.meta = (H, Hkv, D, offset)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin = ctx.saved_tensors
        H, Hkv, D, offset = ctx.meta
        dqkv = native().rope_qkv_bwd(dq.contiguous(), dk.contiguous(), dv.contiguous(), cos, sin, H, Hkv, D, offset)
        return dqkv, None, None, None, None, None, None


def rope_qkv(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, H: int, Hkv: int, D: int, offset: int = 0):
    B, S, _ = qkv.shape
    if not qkv.is_cuda:
        q, k, v = qkv.split([H * D, Hkv * D, Hkv * D], dim=-1)
        c = cos[offset:offset + S].float()[None, :, None, :]
        s = sin[offset:offset + S].float()[None, :, None, :]
        q = _rotate(q.reshape(B, S, H, D), c, s)
        k = _rotate(k.reshape(B, S, Hkv, D), c, s)
        return q, k, v.reshape(B, S, Hkv, D)
    return _RopeQKVFn.apply(qkv.contiguous(), cos.float().contiguous(), sin.float().contiguous(), H, Hkv, D, int(offset))
