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
