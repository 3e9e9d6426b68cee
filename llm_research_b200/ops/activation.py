"""SwiGLU gating on the output of the fused ``[W1; W_gate]`` projection.

``gu[..., :F]`` is the value (``W1 x``) and ``gu[..., F:]`` the gate
pre-activation (``W_gate x``) -- the order in which ``SwiGLUFFN`` registers
its weights, so the fused weight is a zero-copy view in the engine's flat
buffer.  ``h = silu(gate) * value`` computed in fp32, rounded once.
Backward: ``d_gate = dh * value * s * (1 + gate * (1 - s))`` with
``s = sigmoid(gate)``; ``d_value = dh * silu(gate)``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from llm_research_b200._ext import native


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        return native().swiglu_fwd(gu)

    @staticmethod
    def backward(ctx, dh):
        (gu,) = ctx.saved_tensors
        return native().swiglu_bwd(dh.contiguous(), gu)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    if not gu.is_cuda:
        u, g = gu.chunk(2, dim=-1)
        return (F.silu(g.float()) * u.float()).to(gu.dtype)
    return _SwiGLUFn.apply(gu.contiguous())
