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
from llm_research_b200.ops.linear import cat_rows, project, project_residual, swiglu_ffn, swiglu_up


def default_ffn_dim(d_model: int) -> int:
    d_ff = int(8 / 3 * d_model)
    return ((d_ff + 255) // 256) * 256


class SwiGLUFFN(nn.Module):
    def __init__(self, d_model: int, d_ff: int | None = None, dropout: float = 0.0, bias: bool = False) -> None:
        super().__init__()
        d_ff = default_ffn_dim(d_model) if d_ff is None else d_ff
        self.d_ff = d_ff
        from llm_research_b200.parallel.tp import current_tensor_parallel, mark_tp

        self.tp = tp = current_tensor_parallel()
        nt = 1 if tp is None else torch.distributed.get_world_size(tp[0])
        assert d_ff % nt == 0 and (tp is None or not bias), "tensor parallelism: d_ff % tp == 0, no biases"
        # Under tensor parallelism: this rank's d_ff/tp columns of the hidden layer.
        self.w1 = nn.Linear(d_model, d_ff // nt, bias=bias)
        self.w_gate = nn.Linear(d_model, d_ff // nt, bias=bias)
        self.w2 = nn.Linear(d_ff // nt, d_model, bias=bias)
        if tp is not None:
            mark_tp(self.w1.weight, 0)
            mark_tp(self.w_gate.weight, 0)
            mark_tp(self.w2.weight, 1)
        self.dropout = nn.Dropout(dropout) if dropout > 0.0 else nn.Identity()

    def forward_tp(self, x_shard: torch.Tensor) -> torch.Tensor:
        """``(B*S/tp, d)`` sequence shard -> all-gather->GEMM (up|gate, this rank's
        columns) -> SwiGLU -> GEMM->reduce-scatter (down) -> ``(B*S/tp, d)``."""
        from llm_research_b200.parallel.tp import column_parallel, row_parallel

        group, comm = self.tp
        gu = column_parallel(x_shard, cat_rows(self.w1.weight, self.w_gate.weight), group, comm)
        h = ops.swiglu(gu)
        return row_parallel(self.dropout(h), self.w2.weight, group, comm)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``FFN(x)``, or ``residual + FFN(x)`` with the addition folded into the down
        projection's GEMM epilogue when ``residual`` is given."""
        if self.w1.bias is None and self.w2.bias is None and not isinstance(self.dropout, nn.Dropout):
            # one autograd node: up/gate + SwiGLU in one launch, the down projection
            # (+ residual in its epilogue), and a backward whose down-projection
            # dgrad runs the SwiGLU backward in its epilogue
            y = swiglu_ffn(x, self.w1.weight, self.w_gate.weight, self.w2.weight, residual)
            if y is not None:
                return y
        if self.w1.bias is None and not isinstance(self.dropout, nn.Dropout):
            h = swiglu_up(x, self.w1.weight, self.w_gate.weight)  # one launch: both projections + gating
            if h is not None:
                if residual is not None and self.w2.bias is None:
                    return project_residual(h, self.w2.weight, residual)
                y = project(h, self.w2.weight, self.w2.bias)
                return y if residual is None else residual + y
        w = cat_rows(self.w1.weight, self.w_gate.weight)
        b = None
        if self.w1.bias is not None:
            b = torch.cat([self.w1.bias, self.w_gate.bias], 0)
        gu = project(x, w, b)  # [..., up | gate]
        h = ops.swiglu(gu)
        y = project(self.dropout(h), self.w2.weight, self.w2.bias)
        return y if residual is None else residual + y
