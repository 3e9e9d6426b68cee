"""Quantisation formats.

INT4 absmax (reference compatibility, ``olympus/kernels/fp4_quantize.py:38-83``):
per row or per group of ``group_size`` elements along the last dim,
``scale = max(absmax / 7, 1e-10)``, ``q = clamp(round(x / scale), -8, 7)`` stored
as int8 (one value per byte), fp32 scales.  ``round`` is round-half-to-even,
the PyTorch fallback's rounding.

NVFP4 (the training format of the FP4 configs): E2M1 values
``{0, 0.5, 1, 1.5, 2, 3, 4, 6}`` with sign, 16-element blocks along the last
dim, one e4m3 scale per block and one fp32 scale per tensor:
``s_t = amax(x) / (6 * 448)``, ``s_b = e4m3(amax(block) / (6 * s_t))``,
``q = rne_e2m1(x / (s_b * s_t))``; dequantised ``q * s_b * s_t``.  Two values
per byte, element ``2i`` in the low nibble.  ``stochastic=True`` rounds
``x / (s_b s_t)`` to one of its two neighbouring grid points with probability
proportional to proximity (unbiased), as used for gradients.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from llm_research_b200._ext import native

INT4_MIN, INT4_MAX, SCALE_EPS = -8, 7, 1e-10
E2M1_GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
FP4_MAX, E4M3_MAX = 6.0, 448.0


def _resolve_group(group_size: int, D: int) -> int:
    return D if group_size <= 0 or group_size > D else group_size


def int4_quantize(x2d: torch.Tensor, group_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    M, D = x2d.shape
    g = _resolve_group(group_size, D)
    if x2d.is_cuda:
        return native().int4_quantize(x2d.contiguous(), g)
    return int4_quantize_torch(x2d, g)


def int4_quantize_torch(x2d: torch.Tensor, group_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """The same quantiser in plain PyTorch on any device (the oracle of the kernel)."""
    M, D = x2d.shape
    g = _resolve_group(group_size, D)
    ng = (D + g - 1) // g
    xp = F.pad(x2d, (0, ng * g - D)).view(M, ng, g).float()
    scale = (xp.abs().amax(-1, keepdim=True) / INT4_MAX).clamp(min=SCALE_EPS)
    q = (xp / scale).round().clamp(INT4_MIN, INT4_MAX).to(torch.int8).view(M, ng * g)[:, :D]
    return q.contiguous(), scale.squeeze(-1)


def int4_dequantize(q2d: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    M, D = q2d.shape
    g = _resolve_group(group_size, D)
    if q2d.is_cuda:
        return native().int4_dequantize(q2d.contiguous(), scales.contiguous().float(), g)
    return int4_dequantize_torch(q2d, scales, g)


def int4_dequantize_torch(q2d: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    M, D = q2d.shape
    g = _resolve_group(group_size, D)
    ng = scales.shape[1]
    qp = F.pad(q2d, (0, ng * g - D)).view(M, ng, g).float()
    return (qp * scales[:, :, None]).view(M, ng * g)[:, :D]


def _rne_e2m1(a: torch.Tensor) -> torch.Tensor:
    """Round non-negative values to the nearest E2M1 magnitude, ties to even."""
    grid = E2M1_GRID.to(a.device)
    a = a.clamp(max=FP4_MAX)
    # index of the largest grid point <= a
    lo = torch.bucketize(a, grid, right=True) - 1
    lo = lo.clamp(0, 7)
    hi = (lo + 1).clamp(max=7)
    glo, ghi = grid[lo], grid[hi]
    d_lo, d_hi = a - glo, ghi - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0) & (hi != lo))
    return torch.where(pick_hi, hi, lo)


def nvfp4_quantize(x2d: torch.Tensor, stochastic: bool = False, seed: int = 0):
    """Return ``(packed uint8 (M, K/2), block scales e4m3 (M, K/16), tensor scale fp32 ())``."""
    M, K = x2d.shape
    assert K % 16 == 0, "NVFP4 needs the last dim to be a multiple of 16"
    if x2d.is_cuda:
        return native().nvfp4_quantize(x2d.contiguous(), bool(stochastic), int(seed))
    xf = x2d.float()
    amax = xf.abs().max()
    s_t = (amax / (FP4_MAX * E4M3_MAX)).clamp(min=1e-12)
    blk = xf.view(M, K // 16, 16)
    s_b = (blk.abs().amax(-1) / (FP4_MAX * s_t)).clamp(max=E4M3_MAX).to(torch.float8_e4m3fn)
    denom = (s_b.float() * s_t).clamp(min=1e-30)[:, :, None]
    y = blk * (1.0 / denom)  # one reciprocal per block, as the kernels do
    mag = y.abs()
    if stochastic:
        gen = torch.Generator(device="cpu").manual_seed(seed)
        grid = E2M1_GRID
        lo = (torch.bucketize(mag.clamp(max=FP4_MAX), grid, right=True) - 1).clamp(0, 7)
        hi = (lo + 1).clamp(max=7)
        span = (grid[hi] - grid[lo]).clamp(min=1e-12)
        p_hi = ((mag.clamp(max=FP4_MAX) - grid[lo]) / span).clamp(0, 1)
        code = torch.where(torch.rand(mag.shape, generator=gen) < p_hi, hi, lo)
    else:
        code = _rne_e2m1(mag)
    code = code | ((y < 0) & (code > 0)).to(code.dtype) * 8
    code = code.view(M, K).to(torch.uint8)
    packed = code[:, 0::2] | (code[:, 1::2] << 4)
    return packed.contiguous(), s_b, s_t


def nvfp4_dequantize(packed: torch.Tensor, s_b: torch.Tensor, s_t: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    M, K2 = packed.shape
    K = K2 * 2
    if packed.is_cuda:
        return native().nvfp4_dequantize(packed.contiguous(), s_b.contiguous(), s_t.float().reshape(()), dtype)
    lo = (packed & 0xF).long()
    hi = (packed >> 4).long()
    code = torch.stack([lo, hi], dim=-1).view(M, K)
    mag = E2M1_GRID[code & 7]
    val = torch.where(code >= 8, -mag, mag)
    val = val.view(M, K // 16, 16) * s_b.float()[:, :, None] * s_t.float()
    return val.view(M, K).to(dtype)


# ---------------------------------------------------------------- NVFP4 GEMM
def nvfp4_swizzle_scales(s_b: torch.Tensor) -> torch.Tensor:
    """Row-major block scales ``(M, K/16)`` (e4m3) -> the tensor-core atom layout
    used by :func:`matmul_nvfp4`: ``(ceil(M/128), K/64, 512)`` bytes where the
    scale of (row m, k-block j) in a 128 x 64 block sits at byte
    ``16*(m % 32) + 4*(m // 32) + j``.  Rows past M are zero."""
    M, KB = s_b.shape
    assert KB % 4 == 0, "K must be a multiple of 64"
    mb = -(-M // 128)
    raw = s_b.view(torch.uint8) if s_b.dtype != torch.uint8 else s_b
    if mb * 128 != M:
        raw = torch.cat([raw, raw.new_zeros(mb * 128 - M, KB)])
    # (mb, q=4, r=32, kb=KB/4, j=4) -> (mb, kb, r, q, j)
    return raw.view(mb, 4, 32, KB // 4, 4).permute(0, 3, 2, 1, 4).contiguous().view(mb, KB // 4, 512)


def nvfp4_unswizzle_scales(atoms: torch.Tensor, M: int) -> torch.Tensor:
    """Inverse of :func:`nvfp4_swizzle_scales`: atoms -> row-major ``(M, K/16)`` e4m3."""
    mb, kb, _ = atoms.shape
    raw = atoms.view(mb, kb, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(mb * 128, kb * 4)[:M]
    return raw.contiguous().view(torch.float8_e4m3fn)


def nvfp4_quantize_dual(x2d: torch.Tensor, amax: Optional[torch.Tensor] = None, rowwise: bool = True,
                        colwise: bool = True, stochastic: bool = False, seed: int = 0):
    """Quantise ``x`` (M, K) and/or ``x^T`` to NVFP4 in one pass, scales already in the
    tensor-core atom layout: ``(row, col, tensor_scale)`` where ``row`` / ``col`` are
    :class:`NVFP4Tensor` (or None) for ``x`` (blocks along K) and ``x^T`` (blocks along M).
    Both share the per-tensor scale (one amax; ``amax`` may be passed in). M, K multiples
    of 128. On CPU: :func:`nvfp4_quantize` of ``x`` and of ``x.t()`` (the oracle; stochastic
    rounding draws from torch's generator there)."""
    if x2d.is_cuda:
        pr, ar, pc, ac, st = native().nvfp4_quantize_dual(x2d.contiguous(), amax, rowwise, colwise, stochastic, int(seed))
        row = NVFP4Tensor.from_atoms(pr, ar, st) if rowwise else None
        col = NVFP4Tensor.from_atoms(pc, ac, st) if colwise else None
        return row, col, st
    row = NVFP4Tensor(*nvfp4_quantize(x2d, stochastic, seed)) if rowwise else None
    col = NVFP4Tensor(*nvfp4_quantize(x2d.t().contiguous(), stochastic, seed + 1)) if colwise else None
    return row, col, (row or col).tensor_scale


class NVFP4Tensor:
    """A 2-D tensor quantised to NVFP4 for :func:`matmul_nvfp4` (rows = M or N, K-major).
    ``scales`` (row-major e4m3) may be None when only the atom layout is known."""

    def __init__(self, packed: torch.Tensor, scales: Optional[torch.Tensor], tensor_scale: torch.Tensor,
                 atoms: Optional[torch.Tensor] = None) -> None:
        self.packed, self.scales, self.tensor_scale = packed, scales, tensor_scale.float().reshape(())
        self.atoms = nvfp4_swizzle_scales(scales) if atoms is None else atoms

    @classmethod
    def from_atoms(cls, packed: torch.Tensor, atoms: torch.Tensor, tensor_scale: torch.Tensor) -> "NVFP4Tensor":
        return cls(packed, None, tensor_scale, atoms)

    @classmethod
    def quantize(cls, x2d: torch.Tensor, stochastic: bool = False, seed: int = 0) -> "NVFP4Tensor":
        return cls(*nvfp4_quantize(x2d, stochastic, seed))

    def dequantize(self, dtype=torch.float32) -> torch.Tensor:
        scales = self.scales if self.scales is not None else nvfp4_unswizzle_scales(self.atoms, self.packed.shape[0])
        return nvfp4_dequantize(self.packed, scales, self.tensor_scale, dtype)

    @property
    def shape(self):
        return (self.packed.shape[0], self.packed.shape[1] * 2)


def matmul_nvfp4(a: NVFP4Tensor, b: NVFP4Tensor) -> torch.Tensor:
    """``a @ b.T`` in bf16 with tcgen05 block-scaled FP4 MMAs (fp32 accumulation).
    K must be a multiple of 256.  On CPU: dequantise and multiply (the oracle)."""
    if a.packed.is_cuda:
        return native().gemm_nvfp4(a.packed, a.atoms, a.tensor_scale, b.packed, b.atoms, b.tensor_scale)
    return (a.dequantize() @ b.dequantize().t()).to(torch.bfloat16)
