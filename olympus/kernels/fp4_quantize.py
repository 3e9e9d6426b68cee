"""INT4 absmax quantisation API (``olympus/kernels/fp4_quantize.py:275-344``).

Despite the module name, the reference's format is symmetric INT4: values in
``[-8, 7]`` stored one per int8, per-row (``group_size=-1``) or per-group fp32
scales ``max(absmax/7, 1e-10)``.  This module keeps that API and semantics
(the sm_100a kernels in ``llm_research_b200.ops.quant`` on CUDA); the real
E2M1 NVFP4 format used for FP4 training lives in
``llm_research_b200.ops.nvfp4_quantize``.
"""

from __future__ import annotations

import torch

from llm_research_b200.ops.quant import (INT4_MAX, INT4_MIN, SCALE_EPS, _resolve_group, int4_dequantize,
                                         int4_dequantize_torch, int4_quantize, int4_quantize_torch)

__all__ = ["quantize", "dequantize", "quantize_dequantize", "INT4_MIN", "INT4_MAX", "SCALE_EPS", "_resolve_group_size"]

_resolve_group_size = _resolve_group
# The reference exposes HAS_TRITON for its Triton path; this framework has none.
HAS_TRITON = False


def _quantize_pt(x: torch.Tensor, group_size: int = -1):
    """Plain-PyTorch quantiser on any device (``fp4_quantize.py:38-62``):
    ``(q int8 (..., D), scales fp32 (..., ceil(D / g)))``."""
    D = x.shape[-1]
    q, s = int4_quantize_torch(x.reshape(-1, D), group_size)
    return q.reshape(x.shape), s.reshape(*x.shape[:-1], s.shape[-1])


def _dequantize_pt(q: torch.Tensor, scales: torch.Tensor, group_size: int = -1, orig_D: int | None = None):
    """Plain-PyTorch dequantiser (``fp4_quantize.py:65-83``); ``orig_D`` trims
    a padded last dimension."""
    D = q.shape[-1] if orig_D is None else orig_D
    q2 = q.reshape(-1, q.shape[-1])[:, :D]
    out = int4_dequantize_torch(q2.contiguous(), scales.reshape(-1, scales.shape[-1]).float(), group_size)
    return out.reshape(*q.shape[:-1], D)


def quantize(x: torch.Tensor, group_size: int = -1):
    D = x.shape[-1]
    q, s = int4_quantize(x.reshape(-1, D), group_size)
    return q.reshape(x.shape), s.reshape(*x.shape[:-1], s.shape[-1])


def dequantize(q: torch.Tensor, scales: torch.Tensor, group_size: int = -1) -> torch.Tensor:
    D = q.shape[-1]
    out = int4_dequantize(q.reshape(-1, D), scales.reshape(-1, scales.shape[-1]), group_size)
    return out.reshape(q.shape)


class _QDQ(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group_size):
        q, s = quantize(x, group_size)
        return dequantize(q, s, group_size).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        return g, None  # straight-through estimator


def quantize_dequantize(x: torch.Tensor, group_size: int = -1) -> torch.Tensor:
    return _QDQ.apply(x, group_size)
