"""Zero-copy concatenation of weight matrices along their output dimension.

The attention and FFN blocks run one GEMM against ``[Wq; Wk; Wv]`` and
``[W1; W_gate]``.  When the pieces are adjacent in memory -- which the flat
parameter engine guarantees, since it lays parameters out in registration
order -- the concatenation is a view of the first piece's storage; the
backward splits the gradient back into the pieces.  Otherwise it falls back
to ``torch.cat``.
"""

from __future__ import annotations

from typing import Sequence

import torch


def _adjacent(ws: Sequence[torch.Tensor]) -> bool:
    first = ws[0]
    if not all(w.is_contiguous() and w.dtype == first.dtype and w.device == first.device and w.dim() == 2
               and w.shape[1] == first.shape[1] for w in ws):
        return False
    st = first.untyped_storage().data_ptr()
    nxt = first.data_ptr() + first.numel() * first.element_size()
    for w in ws[1:]:
        if w.untyped_storage().data_ptr() != st or w.data_ptr() != nxt:
            return False
        nxt = w.data_ptr() + w.numel() * w.element_size()
    return True


class _CatRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, *ws):
        ctx.rows = [w.shape[0] for w in ws]
        if _adjacent(ws):
            first = ws[0]
            return first.as_strided((sum(ctx.rows), first.shape[1]), (first.shape[1], 1))
        return torch.cat(ws, dim=0)

    @staticmethod
    def backward(ctx, g):
        return tuple(g.split(ctx.rows, dim=0))


def cat_rows(*ws: torch.Tensor) -> torch.Tensor:
    """``torch.cat(ws, 0)`` for 2-D weights, without a copy when they are adjacent."""
    if len(ws) == 1:
        return ws[0]
    if not any(w.requires_grad for w in ws):
        return ws[0].as_strided((sum(w.shape[0] for w in ws), ws[0].shape[1]), (ws[0].shape[1], 1)) \
            if _adjacent(ws) else torch.cat(ws, 0)
    return _CatRows.apply(*ws)


# ------------------------------------------------------------ linear precision
# The model's projections call ``project``; the process-wide precision decides
# whether it is a bf16 GEMM or an NVFP4 block-scaled training GEMM.
import contextlib
import itertools

import torch.nn.functional as F

_PRECISION = "bf16"
_SEEDS = itertools.count(1)


def set_linear_precision(precision: str) -> None:
    """``"bf16"`` (default) or ``"nvfp4"``."""
    global _PRECISION
    if precision not in ("bf16", "nvfp4"):
        raise ValueError(f"unknown linear precision {precision!r}")
    _PRECISION = precision


def get_linear_precision() -> str:
    return _PRECISION


@contextlib.contextmanager
def linear_precision(precision: str):
    old = _PRECISION
    set_linear_precision(precision)
    try:
        yield
    finally:
        set_linear_precision(old)


class _NVFP4LinearFn(torch.autograd.Function):
    """y = x W^T with NVFP4 operands (E2M1, e4m3 per 16 elements, fp32 per tensor).

    Forward rounds to nearest and quantises ``x`` and ``W`` once each, in both
    orientations (one pass per tensor): the row-wise copies feed the forward GEMM,
    the transposed copies are what the backward needs (``W^T`` for dX, ``X^T`` for
    dW), so only FP4 operands are kept for backward.  The backward quantises dY
    (row-wise and transposed, one pass) with stochastic rounding so the gradient
    is unbiased in expectation.  All three GEMMs run on the tcgen05 block-scaled
    kernel."""

    @staticmethod
    def forward(ctx, x2d, w):
        from llm_research_b200.ops.quant import matmul_nvfp4, nvfp4_quantize_dual

        need_dx, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        xr, xc, _ = nvfp4_quantize_dual(x2d, colwise=need_dw)
        wr, wc, _ = nvfp4_quantize_dual(w, colwise=need_dx)
        ctx.xc, ctx.wc = xc, wc
        return matmul_nvfp4(xr, wr)

    @staticmethod
    def backward(ctx, dy):
        from llm_research_b200.ops.quant import matmul_nvfp4, nvfp4_quantize_dual

        need_dx, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        seed = next(_SEEDS)
        dyr, dyc, _ = nvfp4_quantize_dual(dy.contiguous(), rowwise=need_dx, colwise=need_dw, stochastic=True,
                                          seed=seed)
        dx = matmul_nvfp4(dyr, ctx.wc) if need_dx else None
        dw = matmul_nvfp4(dyc, ctx.xc) if need_dw else None
        ctx.xc = ctx.wc = None
        return dx, dw


def _fp4_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    T = x.numel() // x.shape[-1]
    return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and w.shape[1] % 256 == 0
            and w.shape[0] % 256 == 0 and T % 256 == 0)


def project(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear`` under the current linear precision (NVFP4 where the shapes allow it:
    K, N and the token count multiples of 256; bf16 otherwise)."""
    if _PRECISION == "nvfp4" and _fp4_ok(x, w):
        y = _NVFP4LinearFn.apply(x.reshape(-1, x.shape[-1]), w).view(*x.shape[:-1], w.shape[0])
        return y + b if b is not None else y
    return F.linear(x, w, b)
