"""tcgen05 GEMMs.

``matmul_tn`` / ``matmul_tn_accumulate``: ``C = alpha * A @ B^T`` and
``C += alpha * A @ B^T`` on the one-CTA kernel (``csrc/kernels/gemm_sm100.cu``;
the TP fused kernels share its pipeline).

``gemm``: the CTA-pair kernel (``csrc/kernels/gemm_pair_sm100.cu``) with either
operand K-major or MN-major, which the model's linears use for all three of
their GEMMs:

* ``linear_fwd(x, w)``         ``x @ w.T``   (x (T, K), w (N, K))
* ``linear_dgrad(dy, w)``      ``dy @ w``    (dy (T, N), w (N, K))
* ``linear_wgrad(dy, x)``      ``dy.T @ x``  (dy (T, N), x (T, K)); with ``out``
  fp32 and ``accumulate=True`` it adds into ``out`` (gradient accumulation).

Operands: bf16 or fp16, unit column stride, 16-byte aligned base and row
pitch.  CPU tensors take the plain PyTorch path (fp32 math).
"""

from __future__ import annotations

from typing import Optional

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


def gemm(a: torch.Tensor, b: torch.Tensor, a_mn: bool = False, b_mn: bool = False,
         out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
         accumulate: bool = False, alpha: float = 1.0) -> torch.Tensor:
    """``C = alpha * op(A) op(B)^T`` (``+=`` into an fp32 ``out`` with ``accumulate``).

    ``op(A)`` is ``a`` (M, K), or ``a.T`` when ``a_mn`` (``a`` stored (K, M));
    ``op(B)^T`` is ``b.T`` for ``b`` (N, K), or ``b`` when ``b_mn`` (``b`` stored
    (K, N)).  With a leading batch dimension on ``a``, ``b`` (and ``out``) every
    batch entry is one GEMM of the same shape, all in one launch."""
    M = a.shape[-1] if a_mn else a.shape[-2]
    N = b.shape[-1] if b_mn else b.shape[-2]
    if out is None:
        if accumulate:
            raise ValueError("accumulate needs an output tensor")
        out = torch.empty(*a.shape[:-2], M, N, dtype=out_dtype or a.dtype, device=a.device)
    if not a.is_cuda:
        av = a.float().transpose(-1, -2) if a_mn else a.float()
        bv = b.float() if b_mn else b.float().transpose(-1, -2)
        r = alpha * (av @ bv)
        if accumulate:
            out.add_(r.to(out.dtype))
        else:
            out.copy_(r)
        return out
    native().gemm_pair(a, b, bool(a_mn), bool(b_mn), out, bool(accumulate), float(alpha))
    return out


def linear_fwd(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    return gemm(x, w, False, False, out=out)


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    return gemm(dy, w, False, True, out=out)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                 accumulate: bool = False) -> torch.Tensor:
    return gemm(dy, x, True, True, out=out, accumulate=accumulate)


def gemm_pair_error(device: int = 0) -> int:
    """Read and clear the error word of the CTA-pair GEMM (0 = no timeout recorded)."""
    return int(native().gemm_pair_error(int(device)))


def sm100_error(device: int = 0) -> int:
    """Read and clear the error word of the tcgen05 kernels (0 = no timeout recorded)."""
    return int(native().sm100_error(int(device)))
