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
    """``torch.cat(ws, 0)`` for 2-D weights, without a copy when they are adjacent.
    When the pieces' fp32 gradient accumulators (``_lrb_acc``) are adjacent too,
    the result carries their concatenation as its own accumulator view."""
    if len(ws) == 1:
        return ws[0]
    if not any(w.requires_grad for w in ws):
        return ws[0].as_strided((sum(w.shape[0] for w in ws), ws[0].shape[1]), (ws[0].shape[1], 1)) \
            if _adjacent(ws) else torch.cat(ws, 0)
    out = _CatRows.apply(*ws)
    accs = [getattr(w, "_lrb_acc", None) for w in ws]
    if all(a is not None for a in accs) and _adjacent(accs):
        out._lrb_acc = accs[0].as_strided((out.shape[0], out.shape[1]), (out.shape[1], 1))
    return out


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


# ------------------------------------------------ direct gradient accumulation
# A weight handed to the model by the sharding engine carries ``_lrb_acc``: the
# fp32 gradient-accumulator view its gradient belongs to.  The pair kernel's
# wgrad then adds ``dY^T x`` straight into it (fp32 epilogue) and the backward
# returns ACCUMULATED -- an all-zero gradient, a broadcast view of one zero
# scalar -- for the weight; the engine's gradient sink recognises that storage
# and only does its bookkeeping.  Anything autograd sums with the marker is a
# real gradient again (the marker is zero), so tied or reused weights stay exact.
_ZEROS: dict = {}


def accumulated_marker(like: torch.Tensor) -> torch.Tensor:
    key = (like.device, like.dtype)
    z = _ZEROS.get(key)
    if z is None:
        z = _ZEROS[key] = torch.zeros((), dtype=like.dtype, device=like.device)
    return z.expand(like.shape)


def is_accumulated_marker(g: torch.Tensor) -> bool:
    z = _ZEROS.get((g.device, g.dtype))
    return z is not None and g.untyped_storage().data_ptr() == z.untyped_storage().data_ptr()


_DIRECT_ACC = True


def set_direct_grad_accumulation(on: bool) -> None:
    """Switch the direct fp32 wgrad accumulation on (default) or off (dW is then
    returned in the weight's dtype and the engine adds it)."""
    global _DIRECT_ACC
    _DIRECT_ACC = bool(on)


def _acc_of(w: torch.Tensor):
    if not _DIRECT_ACC:
        return None
    acc = getattr(w, "_lrb_acc", None)
    if acc is None or acc.shape != w.shape or acc.dtype != torch.float32 or acc.stride(-1) != 1:
        return None
    return acc


class _PairLinearFn(torch.autograd.Function):
    """y = x W^T with all three GEMMs on the CTA-pair tcgen05 kernel, each operand
    read where it lies: forward (x, W K-major), dgrad dY W (W MN-major), wgrad
    dY^T x (dY and x MN-major) -- accumulated in fp32 into the weight's gradient
    buffer when the engine provides one."""

    @staticmethod
    def forward(ctx, x2d, w, acc):
        from llm_research_b200.ops.gemm import linear_fwd

        ctx.save_for_backward(x2d, w)
        ctx.acc = acc
        return linear_fwd(x2d, w)

    @staticmethod
    def backward(ctx, dy):
        from llm_research_b200.ops.gemm import linear_dgrad, linear_wgrad

        x2d, w = ctx.saved_tensors
        dy = _rows(dy)
        dx = linear_dgrad(dy, w) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            if ctx.acc is not None:
                linear_wgrad(dy, x2d, out=ctx.acc, accumulate=True)
                dw = accumulated_marker(w)
            else:
                dw = linear_wgrad(dy, x2d)
        ctx.acc = None
        return dx, dw, None


class _PairLinearResidualFn(torch.autograd.Function):
    """y = r + x W^T with the residual added in the forward GEMM's epilogue (the
    pair kernel's axpby mode reads r by TMA): no separate add over the
    activations.  Backward: dr = dY, and the linear's dgrad / wgrad."""

    @staticmethod
    def forward(ctx, x2d, w, acc, r2d):
        from llm_research_b200._ext import native

        ctx.save_for_backward(x2d, w)
        ctx.acc = acc
        y = torch.empty(x2d.shape[0], w.shape[0], dtype=x2d.dtype, device=x2d.device)
        native().gemm_pair_axpby(x2d, w, False, y, r2d, 1.0, 1.0)
        return y

    @staticmethod
    def backward(ctx, dy):
        dx, dw, _ = _PairLinearFn.backward(ctx, dy)
        return dx, dw, None, dy


def project_residual(x: torch.Tensor, w: torch.Tensor, r: torch.Tensor) -> torch.Tensor:
    """``r + project(x, w)``: on the pair kernel with the residual added in the GEMM
    epilogue where it applies (bf16 precision, 16-bit CUDA operands of one dtype,
    aligned rows), else the separate add."""
    if (_PRECISION == "bf16" and x.numel() > 0 and _pair_ok(x, w) and r.dtype == x.dtype and r.is_cuda
            and r.shape == (*x.shape[:-1], w.shape[0])):
        r2d = _rows(r.reshape(-1, w.shape[0]))
        x2d = _rows(x.reshape(-1, x.shape[-1]))
        acc = _acc_of(w) if torch.is_grad_enabled() and w.requires_grad else None
        return _PairLinearResidualFn.apply(x2d, w, acc, r2d).view(r.shape)
    return r + project(x, w)


def _aligned_rows(t: torch.Tensor) -> bool:
    return t.dim() == 2 and t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0


def _rows(t: torch.Tensor) -> torch.Tensor:
    """``t`` as a 2-D matrix with unit column stride and a 16-byte aligned row pitch."""
    return t if _aligned_rows(t) else t.contiguous()


def _pair_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    """Shapes the pair kernel takes: 16-bit CUDA operands of one dtype, the weight's
    row pitch and both of its dimensions multiples of 8 elements (its rows are the
    K-major B of the forward, its columns the MN-major B of dgrad; the output
    width is the MN-major A pitch of wgrad)."""
    return (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype and w.dim() == 2
            and w.shape[0] % 8 == 0 and w.shape[1] % 8 == 0 and _aligned_rows(w) and x.shape[-1] == w.shape[1])


def linear_bf16(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` over the last dimension of ``x`` on the pair kernel (no bias)."""
    x2d = _rows(x.reshape(-1, x.shape[-1]))
    acc = _acc_of(w) if torch.is_grad_enabled() and w.requires_grad else None
    return _PairLinearFn.apply(x2d, w, acc).view(*x.shape[:-1], w.shape[0])


def dense(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear`` in the input precision whatever the linear precision (the output
    head stays bf16 under NVFP4 training): the pair kernel where it applies."""
    if x.numel() > 0 and _pair_ok(x, w):
        y = linear_bf16(x, w)
        return y + b if b is not None else y
    return F.linear(x, w, b)


def _fp4_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    T = x.numel() // x.shape[-1]
    return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and w.shape[1] % 256 == 0
            and w.shape[0] % 256 == 0 and T % 256 == 0)


def project(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear`` under the current linear precision: NVFP4 block-scaled GEMMs where
    the shapes allow it (K, N and the token count multiples of 256), otherwise the
    bf16/fp16 CTA-pair kernel on CUDA (K and N multiples of 8); PyTorch for CPU
    tensors, fp32 and the remaining shapes."""
    if _PRECISION == "nvfp4" and _fp4_ok(x, w):
        y = _NVFP4LinearFn.apply(x.reshape(-1, x.shape[-1]), w).view(*x.shape[:-1], w.shape[0])
        return y + b if b is not None else y
    if x.numel() > 0 and _pair_ok(x, w):
        y = linear_bf16(x, w)
        return y + b if b is not None else y
    return F.linear(x, w, b)


# ------------------------------------------------------------ grouped experts
class _GroupedSwiGLUFn(torch.autograd.Function):
    """``y_e = (silu(x_e W_gate,e^T) * x_e W_up,e^T) W_down,e^T`` for every expert e at
    once: the four GEMMs of forward and backward that involve weights, and the
    two activation GEMMs, are batched CTA-pair launches over the expert dimension
    (equal row counts per expert: the capacity-padded dispatch buffer)."""

    @staticmethod
    def forward(ctx, x_e, w_ug, w_down):
        from llm_research_b200.ops.activation import swiglu
        from llm_research_b200.ops.gemm import gemm

        gu = gemm(x_e, w_ug)                       # (E, R, 2F) = [up | gate]
        h = swiglu(gu)                             # (E, R, F)
        ctx.save_for_backward(x_e, w_ug, w_down, gu, h)
        return gemm(h, w_down)                     # (E, R, d)

    @staticmethod
    def backward(ctx, dy):
        from llm_research_b200._ext import native
        from llm_research_b200.ops.gemm import gemm

        x_e, w_ug, w_down, gu, h = ctx.saved_tensors
        dy = dy.contiguous()
        dh = gemm(dy, w_down, b_mn=True)           # dY W_down         (E, R, F)
        dw_down = gemm(dy, h, a_mn=True, b_mn=True)  # dY^T h          (E, d, F)
        dgu = native().swiglu_bwd(dh, gu)          # (E, R, 2F)
        dx = gemm(dgu, w_ug, b_mn=True) if ctx.needs_input_grad[0] else None  # dGU W_ug  (E, R, d)
        dw_ug = gemm(dgu, x_e, a_mn=True, b_mn=True)  # dGU^T x_e      (E, 2F, d)
        return dx, dw_ug, dw_down


def grouped_swiglu(x_e: torch.Tensor, w_ug: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """SwiGLU experts over capacity-padded rows: ``x_e (E, R, d)``, ``w_ug (E, 2F, d)``
    (``[up; gate]`` rows), ``w_down (E, d, F)`` -> ``(E, R, d)``."""
    from llm_research_b200.ops.activation import swiglu

    E, R, d = x_e.shape
    F2 = w_ug.shape[1]
    ok = (x_e.is_cuda and x_e.dtype in (torch.bfloat16, torch.float16) and w_ug.dtype == x_e.dtype
          and w_down.dtype == x_e.dtype and d % 8 == 0 and F2 % 16 == 0 and R % 8 == 0 and R > 0)
    if ok:
        return _GroupedSwiGLUFn.apply(x_e.contiguous(), w_ug.contiguous(), w_down.contiguous())
    gu = torch.bmm(x_e, w_ug.transpose(1, 2))
    h = swiglu(gu.reshape(-1, F2)).view(E, R, -1)
    return torch.bmm(h, w_down.transpose(1, 2))


# ------------------------------------------------------- fused SwiGLU up/gate
class _SwiGLUUpFn(torch.autograd.Function):
    """``h = silu(x W_gate^T) * (x W1^T)`` with both projections and the gating in
    one CTA-pair launch (``gemm_pair_swiglu``); ``gu = [u | g]`` is kept for the
    backward: ``dgu = swiglu_bwd(dh, gu)``, ``dx = dgu [W1; W_gate]``,
    ``[dW1; dW_gate] = dgu^T x`` (added straight into the engine's fp32 buffer
    when the two weights' accumulators are adjacent)."""

    @staticmethod
    def forward(ctx, x2d, w1, wg, acc):
        from llm_research_b200._ext import native

        F = w1.shape[0]
        gu = torch.empty(x2d.shape[0], 2 * F, dtype=x2d.dtype, device=x2d.device)
        h = torch.empty(x2d.shape[0], F, dtype=x2d.dtype, device=x2d.device)
        native().gemm_pair_swiglu(x2d, w1, wg, gu, h)
        ctx.save_for_backward(x2d, w1, wg, gu)
        ctx.acc = acc
        return h

    @staticmethod
    def backward(ctx, dh):
        from llm_research_b200._ext import native
        from llm_research_b200.ops.gemm import linear_dgrad, linear_wgrad

        x2d, w1, wg, gu = ctx.saved_tensors
        dgu = native().swiglu_bwd(_rows(dh), gu)
        w = w1.as_strided((2 * w1.shape[0], w1.shape[1]), (w1.shape[1], 1)) if _adjacent([w1, wg]) \
            else torch.cat([w1, wg], 0)
        dx = linear_dgrad(dgu, w) if ctx.needs_input_grad[0] else None
        dw1 = dwg = None
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            if ctx.acc is not None:
                linear_wgrad(dgu, x2d, out=ctx.acc, accumulate=True)
                dw1, dwg = accumulated_marker(w1), accumulated_marker(wg)
            else:
                dw = linear_wgrad(dgu, x2d)
                dw1, dwg = dw[: w1.shape[0]], dw[w1.shape[0]:]
        ctx.acc = None
        return dx, dw1, dwg, None


def swiglu_up(x: torch.Tensor, w1: torch.Tensor, wg: torch.Tensor) -> torch.Tensor:
    """``silu(x W_gate^T) * (x W1^T)`` over the last dimension of ``x`` (bf16 CUDA,
    shapes the pair kernel takes), or None when the fused path does not apply."""
    if not (_PRECISION == "bf16" and x.is_cuda and x.dtype == torch.bfloat16 and x.numel() > 0
            and _pair_ok(x, w1) and _pair_ok(x, wg) and w1.shape == wg.shape):
        return None
    x2d = _rows(x.reshape(-1, x.shape[-1]))
    acc = None
    if torch.is_grad_enabled() and (w1.requires_grad or wg.requires_grad) and _DIRECT_ACC:
        a1, ag = getattr(w1, "_lrb_acc", None), getattr(wg, "_lrb_acc", None)
        if a1 is not None and ag is not None and _adjacent([a1, ag]):
            acc = a1.as_strided((2 * a1.shape[0], a1.shape[1]), (a1.shape[1], 1))
    h = _SwiGLUUpFn.apply(x2d, w1, wg, acc)
    return h.view(*x.shape[:-1], w1.shape[0])


# ---------------------------------------------------- whole SwiGLU FFN, fused
class _SwiGLUFFNFn(torch.autograd.Function):
    """y = [r +] silu(x Wg^T) * (x W1^T) W2^T as one autograd node, so the backward
    can run the down projection's dgrad and the SwiGLU backward as one launch
    (``gemm_pair_swiglu_bwd``: dh = dY W2 never reaches memory).  Forward: the
    up/gate GEMM with the SwiGLU epilogue, then the down GEMM (with the residual
    in its epilogue when given).  Backward: dgu (fused), dW2 = dY^T h,
    dx = dgu [W1; Wg], [dW1; dWg] = dgu^T x, dr = dY; weight gradients go straight
    into the engine's fp32 accumulators when it provides them."""

    @staticmethod
    def forward(ctx, x2d, w1, wg, w2, r2d, acc_ug, acc_2):
        from llm_research_b200._ext import native
        from llm_research_b200.ops.gemm import linear_fwd

        F = w1.shape[0]
        gu = torch.empty(x2d.shape[0], 2 * F, dtype=x2d.dtype, device=x2d.device)
        h = torch.empty(x2d.shape[0], F, dtype=x2d.dtype, device=x2d.device)
        native().gemm_pair_swiglu(x2d, w1, wg, gu, h)
        if r2d is not None:
            y = torch.empty(x2d.shape[0], w2.shape[0], dtype=x2d.dtype, device=x2d.device)
            native().gemm_pair_axpby(h, w2, False, y, r2d, 1.0, 1.0)
        else:
            y = linear_fwd(h, w2)
        ctx.save_for_backward(x2d, w1, wg, w2, gu, h)
        ctx.accs = (acc_ug, acc_2)
        ctx.has_r = r2d is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        from llm_research_b200._ext import native
        from llm_research_b200.ops.gemm import linear_dgrad, linear_wgrad

        x2d, w1, wg, w2, gu, h = ctx.saved_tensors
        acc_ug, acc_2 = ctx.accs
        dy = _rows(dy)
        dgu = torch.empty_like(gu)
        native().gemm_pair_swiglu_bwd(dy, w2, gu, dgu)
        dw2 = None
        if ctx.needs_input_grad[3]:
            if acc_2 is not None:
                linear_wgrad(dy, h, out=acc_2, accumulate=True)
                dw2 = accumulated_marker(w2)
            else:
                dw2 = linear_wgrad(dy, h)
        w = w1.as_strided((2 * w1.shape[0], w1.shape[1]), (w1.shape[1], 1)) if _adjacent([w1, wg]) \
            else torch.cat([w1, wg], 0)
        dx = linear_dgrad(dgu, w) if ctx.needs_input_grad[0] else None
        dw1 = dwg = None
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            if acc_ug is not None:
                linear_wgrad(dgu, x2d, out=acc_ug, accumulate=True)
                dw1, dwg = accumulated_marker(w1), accumulated_marker(wg)
            else:
                dw = linear_wgrad(dgu, x2d)
                dw1, dwg = dw[: w1.shape[0]], dw[w1.shape[0]:]
        ctx.accs = None
        return dx, dw1, dwg, dw2, (dy if ctx.has_r else None), None, None


def swiglu_ffn(x: torch.Tensor, w1: torch.Tensor, wg: torch.Tensor, w2: torch.Tensor,
               residual: torch.Tensor | None = None):
    """``[residual +] W2(silu(x Wg^T) * (x W1^T))`` over the last dimension of ``x`` as
    one fused node (see ``_SwiGLUFFNFn``), or None when it does not apply (bf16
    CUDA and the pair kernel's shapes)."""
    if not (_PRECISION == "bf16" and x.is_cuda and x.dtype == torch.bfloat16 and x.numel() > 0
            and _pair_ok(x, w1) and _pair_ok(x, wg) and w1.shape == wg.shape and w2.dtype == x.dtype
            and w2.dim() == 2 and w2.shape[1] == w1.shape[0] and w2.shape[0] % 8 == 0 and _aligned_rows(w2)):
        return None
    if residual is not None and not (residual.is_cuda and residual.dtype == x.dtype
                                     and residual.shape == (*x.shape[:-1], w2.shape[0])):
        return None
    x2d = _rows(x.reshape(-1, x.shape[-1]))
    r2d = None if residual is None else _rows(residual.reshape(-1, w2.shape[0]))
    acc_ug = acc_2 = None
    if torch.is_grad_enabled() and _DIRECT_ACC:
        a1, ag = getattr(w1, "_lrb_acc", None), getattr(wg, "_lrb_acc", None)
        if (w1.requires_grad or wg.requires_grad) and a1 is not None and ag is not None and _adjacent([a1, ag]):
            acc_ug = a1.as_strided((2 * a1.shape[0], a1.shape[1]), (a1.shape[1], 1))
        if w2.requires_grad:
            acc_2 = _acc_of(w2)
    y = _SwiGLUFFNFn.apply(x2d, w1, wg, w2, r2d, acc_ug, acc_2)
    return y.view(*x.shape[:-1], w2.shape[0])


# ------------------------------------------------------------ fused QKV + RoPE
_TABLES_T: dict = {}


def _columns_major(cos: torch.Tensor, sin: torch.Tensor):
    """``(128, positions)`` contiguous copies of the RoPE tables, as the fused
    QKV epilogue reads them (a warp's 32 consecutive positions of one column are
    one coalesced line).  Cached per table storage, shape and version (the
    tables of a model are built once and reused every step); an entry holds its
    source tensors, so their storage cannot be freed and reused under the key."""
    key = (cos.data_ptr(), cos._version, sin.data_ptr(), sin._version, tuple(cos.shape), cos.device)
    hit = _TABLES_T.get(key)
    if hit is None:
        if len(_TABLES_T) >= 8:
            _TABLES_T.clear()
        hit = (cos, sin, cos.t().contiguous(), sin.t().contiguous())
        _TABLES_T[key] = hit
    return hit[2], hit[3]


class _QKVRopeFn(torch.autograd.Function):
    """``qkv = x W^T`` with RoPE applied to the query and key heads in the GEMM
    epilogue (one launch, no separate rotation pass); q, k, v are returned as
    strided views of ``qkv``.  Backward: the inverse rotation packs ``dq, dk, dv``
    back into ``dqkv`` (one pass), then the linear's dgrad / wgrad."""

    @staticmethod
    def forward(ctx, x2d, w, acc, cos, sin, H, Hkv, D, B, S, offset):
        from llm_research_b200._ext import native

        out = torch.empty(x2d.shape[0], w.shape[0], dtype=x2d.dtype, device=x2d.device)
        cos_t, sin_t = _columns_major(cos, sin)
        native().gemm_pair_rope(x2d, w, out, cos_t, sin_t, S, offset, (H + Hkv) * D)
        ctx.save_for_backward(x2d, w, cos, sin)
        ctx.acc, ctx.meta = acc, (H, Hkv, D, B, S, offset)
        v4 = out.view(B, S, H + 2 * Hkv, D)
        return v4[:, :, :H], v4[:, :, H:H + Hkv], v4[:, :, H + Hkv:]

    @staticmethod
    def backward(ctx, dq, dk, dv):
        from llm_research_b200._ext import native
        from llm_research_b200.ops.gemm import linear_dgrad, linear_wgrad

        x2d, w, cos, sin = ctx.saved_tensors
        H, Hkv, D, B, S, offset = ctx.meta
        dqkv = native().rope_qkv_bwd(dq.contiguous(), dk.contiguous(), dv.contiguous(), cos, sin, H, Hkv, D, offset)
        dqkv = dqkv.view(B * S, -1)
        dx = linear_dgrad(dqkv, w) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            if ctx.acc is not None:
                linear_wgrad(dqkv, x2d, out=ctx.acc, accumulate=True)
                dw = accumulated_marker(w)
            else:
                dw = linear_wgrad(dqkv, x2d)
        ctx.acc = None
        return dx, dw, None, None, None, None, None, None, None, None, None


def qkv_rope(x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, H: int, Hkv: int, D: int,
             offset: int = 0):
    """``(q, k, v)`` of ``(B, S, heads, D)`` for ``x (B, S, d)`` and the fused weight
    ``w ((H + 2 Hkv) D, d)``, RoPE on q and k, or None when the fused path does not
    apply (head_dim 128, bf16 CUDA, the pair kernel's shapes, tables covering
    the positions)."""
    B, S, _ = x.shape
    N = (H + 2 * Hkv) * D
    if not (_PRECISION == "bf16" and x.is_cuda and x.dtype == torch.bfloat16 and D == 128 and N % 256 == 0
            and w.shape[0] == N and _pair_ok(x, w) and B * S > 0 and cos.shape[0] >= offset + S):
        return None
    x2d = _rows(x.reshape(-1, x.shape[-1]))
    acc = _acc_of(w) if torch.is_grad_enabled() and w.requires_grad else None
    return _QKVRopeFn.apply(x2d, w, acc, cos.float().contiguous(), sin.float().contiguous(), H, Hkv, D, B, S,
                            int(offset))
