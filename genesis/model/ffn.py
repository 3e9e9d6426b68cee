"""SwiGLU feed-forward network (``genesis/model/ffn.py:15-66``).

``FFN(x) = W2( silu(W_gate x) * (W1 x) )``; ``d_ff`` defaults to
``ceil(8/3 * d_model / 256) * 256``.  On B200 the two up projections are one
GEMM against ``[W1; W_gate]`` and the gating runs in one fused kernel
(``llm_research_b200.ops.swiglu``).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200 import ops
from llm_research_b200.ops.linear import cat_rows, project


def default_ffn_dim(d_model: int) -> int:
    d_ff = int(8 / 3 * d_model)
    return ((d_ff + 255) // 256) * 256


class SwiGLUFFN(nn.Module):
    def __init__(self, d_model: int, d_ff: int | None = None, dropout: float = 0.0, bias: bool = False) -> None:
        super().__init__()
        d_ff = default_ffn_dim(d_model) if d_ff is None else d_ff
        self.d_ff = d_ff
        self.w1 = nn.Linear(d_model, d_ff, bias=bias)
        self.w_gate = nn.Linear(d_model, d_ff, bias=bias)
        self.w2 = nn.Linear(d_ff, d_model, bias=bias)
        self.dropout = nn.Dropout(dropout) if dropout > 0.0 else nn.Identity()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = cat_rows(self.w1.weight, self.w_gate.weight)
        b = None
        if self.w1.bias is not None:
            b = torch.cat([self.w1.bias, self.w_gate.bias], 0)
        gu = project(x, w, b)  # [..., up | gate]
        h = ops.swiglu(gu)
        return project(self.dropout(h), self.w2.weight, self.w2.bias)
