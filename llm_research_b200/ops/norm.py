"""RMSNorm, optionally fused with the residual add that precedes it.

Math (matches ``genesis/model/rmsnorm.py:34-49`` of the reference):
``r = rsqrt(mean(x^2) + eps)`` in fp32, ``n = cast(x * r, x.dtype)``,
``y = n * weight`` (rounded to the output dtype).
Backward: ``dn = dy * w``; ``dx = r * (dn - xhat * mean(dn * xhat))`` with
``xhat = x * r``; ``dw = sum_rows(dy * n)``.
"""

from __future__ import annotations

import torch

from llm_research_b200._ext import native


def _ref_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    n = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps)).type_as(x)
    return n * w


def _out_dtype(x: torch.Tensor, w: torch.Tensor) -> torch.dtype:
    return torch.promote_types(x.dtype, w.dtype)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, residual):
        C = native()
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        r2 = residual.reshape(-1, shape[-1]) if residual is not None else None
        y, rstd, s = C.rmsnorm_fwd(x2, w, float(eps), r2, _out_dtype(x, w))
        src = s if s is not None else x2
        ctx.save_for_backward(src, w, rstd)
        ctx.has_res = residual is not None
        ctx.shape = shape
        y = y.view(*shape[:-1], y.shape[-1])
        if s is None:
            return y, None
        return y, s.view(shape)

    @staticmethod
    def backward(ctx, dy, ds):
        src, w, rstd = ctx.saved_tensors
        C = native()
        d = src.shape[-1]
        dy2 = dy.reshape(-1, d).contiguous()
        ds2 = ds.reshape(-1, d).contiguous() if (ds is not None and ctx.has_res) else None
        dx, dw = C.rmsnorm_bwd(dy2, src, w, rstd, ds2)
        dx = dx.view(ctx.shape)
        dw = dw.to(w.dtype)
        if ctx.has_res:
            return dx, dw, None, dx
        return dx, dw, None, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if not x.is_cuda:
        return _ref_norm(x, weight, eps)
    if x.stride(-1) != 1:
        x = x.contiguous()
    return _RMSNormFn.apply(x, weight, eps, None)[0]


def rms_norm_residual(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6):
    """Return ``(norm(x + residual) * weight, x + residual)``."""
    if not x.is_cuda:
        s = residual + x
        return _ref_norm(s, weight, eps), s
    return _RMSNormFn.apply(x.contiguous(), weight, eps, residual.contiguous())
