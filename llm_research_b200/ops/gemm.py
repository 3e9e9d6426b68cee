"""tcgen05 GEMMs: ``C = alpha * A @ B^T`` and ``C += alpha * A @ B^T`` (fp32 C).

Both operands K-major (row-major ``A (M, K)``, ``B (N, K)``: the nn.Linear
weight layout), bf16 or fp16, fp32 accumulation in tensor memory; see
``csrc/kernels/gemm_sm100.cu`` for the pipeline.  Requirements: unit column
stride, 16-byte aligned base and row stride (``K % 8 == 0`` for packed rows).
"""

from __future__ import annotations

import torch

from llm_research_b200._ext import native


def matmul_tn(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype | None = None, alpha: float = 1.0) -> torch.Tensor:
    out_dtype = a.dtype if out_dtype is None else out_dtype
    if not a.is_cuda:
        return (alpha * (a.float() @ b.float().t())).to(out_dtype)
    return native().gemm_tn(a, b, out_dtype, float(alpha))


def matmul_tn_accumulate(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, alpha: float = 1.0) -> torch.Tensor:
    if not a.is_cuda:
        c.add_(alpha * (a.float() @ b.float().t()))
        return c
    native().gemm_tn_accumulate(a, b, c, float(alpha))
    return c


def sm100_error(device: int = 0) -> int:
    """Read and clear the error word of the tcgen05 kernels (0 = no timeout recorded)."""
    return int(native().sm100_error(int(device)))


# ------------------------------------------------------------- grouped linear
def _grouped_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.shape[1] % 8 == 0
            and x.shape[2] % 8 == 0 and w.shape[1] % 8 == 0)


class _GroupedLinearFn(torch.autograd.Function):
    """``y[e] = x[e] w[e]^T`` for ``x (E, rows, K)``, ``w (E, N, K)`` on the batched
    tcgen05 GEMM: forward K-major x K-major; dX = dY w with w read MN-major; dW =
    dY^T x with x read MN-major (dY^T is the one transposed copy)."""

    @staticmethod
    def forward(ctx, x, w):
        C = native()
        x, w = x.contiguous(), w.contiguous()
        y = torch.empty(x.shape[0], x.shape[1], w.shape[1], device=x.device, dtype=x.dtype)
        C.gemm_batched(x, w, False, y, None, 1.0, 0.0)
        ctx.save_for_backward(x, w)
        return y

    @staticmethod
    def backward(ctx, dy):
        C = native()
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty_like(x)
            C.gemm_batched(dy, w, True, dx, None, 1.0, 0.0)
        if ctx.needs_input_grad[1]:
            dw = torch.empty_like(w)
            C.gemm_batched(dy.transpose(1, 2).contiguous(), x, True, dw, None, 1.0, 0.0)
        return dx, dw


def grouped_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Batched ``x @ w.transpose(1, 2)`` (equal-shape groups, e.g. one rank's experts)."""
    if _grouped_ok(x, w):
        return _GroupedLinearFn.apply(x, w)
    return torch.bmm(x, w.to(x.dtype).transpose(1, 2))
