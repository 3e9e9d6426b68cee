"""Quantised linear layer API (``olympus/kernels/fp4_matmul.py:298-360``).

``fp4_matmul(x, w, b, act_group_size, weight_group_size)`` computes
``qdq(x) @ qdq(w)^T + b`` with the reference's INT4 fake quantisation and a
straight-through backward (``dx = dy w``, ``dw = dy^T x``).  Quantisation
groups are applied exactly as specified for every group size; the reference
kernel applies a single scale group per 64-wide K tile
(``fp4_matmul.py:141-142``), which is wrong for groups smaller than 64.

:class:`FP4Linear` wraps an ``nn.Linear``.  For real 4-bit training use
``mode="nvfp4"``: E2M1 weights/activations with e4m3 block scales
(``llm_research_b200.ops.nvfp4``), same straight-through backward.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from olympus.kernels.fp4_quantize import quantize_dequantize


class _FP4MatmulFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, ag, wg):
        out = F.linear(quantize_dequantize(x, ag).to(x.dtype), quantize_dequantize(weight, wg).to(x.dtype),
                       None if bias is None else bias.to(x.dtype))
        ctx.save_for_backward(x, weight, bias)
        return out

    @staticmethod
    def backward(ctx, g):
        x, w, b = ctx.saved_tensors
        gx = g.matmul(w.to(g.dtype)) if ctx.needs_input_grad[0] else None
        gw = g.reshape(-1, g.shape[-1]).t().matmul(x.reshape(-1, x.shape[-1]).to(g.dtype)).to(w.dtype) \
            if ctx.needs_input_grad[1] else None
        gb = g.reshape(-1, g.shape[-1]).sum(0).to(b.dtype) if (b is not None and ctx.needs_input_grad[2]) else None
        return gx, gw, gb, None, None


def _fp4_matmul_pt(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                   act_group_size: int = -1, weight_group_size: int = -1) -> torch.Tensor:
    """Plain-PyTorch fake-quantised linear (``fp4_matmul.py:37-57``):
    ``qdq(x) @ qdq(w)^T + b`` with straight-through gradients to x, w and b."""
    from olympus.kernels.fp4_quantize import _dequantize_pt, _quantize_pt

    def qdq(t, g):
        q, s = _quantize_pt(t.detach(), g)
        return t + (_dequantize_pt(q, s, g).to(t.dtype) - t).detach()

    return F.linear(qdq(x, act_group_size), qdq(weight, weight_group_size), bias)


def _nvfp4_linear(x, weight, bias):
    from llm_research_b200.ops.nvfp4 import nvfp4_linear

    return nvfp4_linear(x, weight, bias)


def fp4_matmul(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
               act_group_size: int = -1, weight_group_size: int = -1, mode: str = "int4") -> torch.Tensor:
    if mode == "nvfp4":
        return _nvfp4_linear(x, weight, bias)
    return _FP4MatmulFn.apply(x, weight, bias, act_group_size, weight_group_size)


class FP4Linear(nn.Module):
    def __init__(self, linear: nn.Linear, act_group_size: int = -1, weight_group_size: int = -1,
                 mode: str = "int4") -> None:
        super().__init__()
        self.linear = linear
        self.act_group_size = act_group_size
        self.weight_group_size = weight_group_size
        self.mode = mode

    @property
    def weight(self) -> torch.Tensor:
        return self.linear.weight

    @property
    def bias(self) -> torch.Tensor | None:
        return self.linear.bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return fp4_matmul(x, self.linear.weight, self.linear.bias, self.act_group_size, self.weight_group_size,
                          mode=self.mode)
