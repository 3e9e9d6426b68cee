"""SwiGLU gating on the output of the fused ``[W_gate; W1]`` projection.

``gu[..., :F]`` is the gate pre-activation and ``gu[..., F:]`` the value;
``h = silu(gate) * value`` computed in fp32, rounded once.
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
        g, u = gu.chunk(2, dim=-1)
        return (F.silu(g.float()) * u.float()).to(gu.dtype)
    return _SwiGLUFn.apply(gu.contiguous())
