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
