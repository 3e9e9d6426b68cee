"""Mixture-of-experts SwiGLU FFN (``genesis/model/moe.py:17-109``).

``y[n] = sum_k w[n,k] * expert_{idx[n,k]}(x[n])``.  The reference loops over
``(k, expert)`` with boolean masks (one host sync each).  Here tokens are
grouped by expert with one sort and each expert runs once on its contiguous
slice (one host read of the per-expert counts per layer).

``capacity_factor``: the reference stores it without using it.  With
``enforce_capacity=True`` each expert keeps at most
``ceil(capacity_factor * N * top_k / E)`` assignments (lowest token index
first) and drops the rest, which is the capacity rule the expert-parallel
path (``llm_research_b200.parallel.expert_parallel``) uses.  On CUDA (16-bit,
bias- and dropout-free experts) that path runs on device kernels only: the
routing kernel's capacity slots, per-expert row blocks, the experts as batched
CTA-pair GEMMs, and a weighted gather back -- no host read.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from genesis.model.ffn import SwiGLUFFN
from genesis.model.moe_router import ExpertRouter
from llm_research_b200 import ops
from olympus.core.compute_router import grouped_expert_apply


def capacity_mask(indices: torch.Tensor, num_experts: int, capacity: int) -> torch.Tensor:
    """Bool ``(N, k)``: True where the assignment fits in its expert's capacity.

    Assignments are ranked per expert in (token, k) order (``ops.route_slots``:
    one device kernel on CUDA).
    """
    _, _, slot, _ = ops.route_slots(indices, num_experts, num_experts, capacity)
    return (slot >= 0).reshape(indices.shape)


class MoEFFN(nn.Module):
    def __init__(
        self,
        d_model: int,
        d_ff: int | None = None,
        num_experts: int = 8,
        top_k: int = 2,
        capacity_factor: float = 1.25,
        dropout: float = 0.0,
        jitter_noise: float = 0.0,
        enforce_capacity: bool = False,
        num_shared_experts: int = 0,
    ) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_experts = num_experts
        self.top_k = top_k
        self.capacity_factor = capacity_factor
        self.enforce_capacity = enforce_capacity
        self.router = ExpertRouter(d_model=d_model, num_experts=num_experts, top_k=top_k, jitter_noise=jitter_noise)
        self.experts = nn.ModuleList([SwiGLUFFN(d_model=d_model, d_ff=d_ff, dropout=dropout) for _ in range(num_experts)])
        # always-on experts added to every token (DeepSeek-style shared experts); none in the reference
        self.shared_experts = nn.ModuleList([SwiGLUFFN(d_model=d_model, d_ff=d_ff, dropout=dropout)
                                             for _ in range(num_shared_experts)])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        w, idx, _ = self.router(xf)
        if self.enforce_capacity:
            cap = math.ceil(self.capacity_factor * xf.shape[0] * self.top_k / self.num_experts)
            if self._device_path_ok(xf):
                out = self._capacity_forward(xf, w, idx, cap)
                for e in self.shared_experts:
                    out = out + e(xf)
                return out.to(x.dtype).reshape(shape)
            w = w * capacity_mask(idx, self.num_experts, cap).to(w.dtype)
        out = grouped_expert_apply(xf, idx, w, self.experts, self.num_experts)
        for e in self.shared_experts:
            out = out + e(xf)
        return out.to(x.dtype).reshape(shape)

    def _device_path_ok(self, xf: torch.Tensor) -> bool:
        e0 = self.experts[0]
        return (xf.is_cuda and xf.dtype in (torch.bfloat16, torch.float16) and e0.w1.bias is None
                and not isinstance(e0.dropout, nn.Dropout) and e0.w1.weight.dtype == xf.dtype)

    def _capacity_forward(self, xf: torch.Tensor, w: torch.Tensor, idx: torch.Tensor, cap: int) -> torch.Tensor:
        """The capacity rule with no host read: the routing kernel ranks the
        assignments per expert; kept rows are copied into per-expert blocks of
        ``R = cap`` rounded up to 8 rows (the rest stay zero), the experts run as
        batched CTA-pair GEMMs (``grouped_swiglu``), and each token sums its kept
        rows with its routing weights.  Dropped assignments go to a spare row
        that no expert reads."""
        from llm_research_b200.ops.linear import grouped_swiglu

        N, d = xf.shape
        E, k = self.num_experts, self.top_k
        R = (cap + 7) // 8 * 8
        _, le, slot, _ = ops.route_slots(idx, E, E, cap)
        keep = slot >= 0
        spare = E * R
        pos = torch.where(keep, le.long() * R + slot.long(), torch.full_like(slot, spare, dtype=torch.long))
        tok = torch.arange(N * k, device=xf.device) // k
        x_e = xf.new_zeros(spare + 1, d).index_copy(0, pos, xf.index_select(0, tok))
        w_ug = torch.stack([torch.cat([e.w1.weight, e.w_gate.weight], 0) for e in self.experts])
        w_dn = torch.stack([e.w2.weight for e in self.experts])
        y_e = grouped_swiglu(x_e[:spare].view(E, R, d), w_ug, w_dn).reshape(spare, d)
        y_e = torch.cat([y_e, y_e.new_zeros(1, d)], 0)
        rows = y_e.index_select(0, pos).view(N, k, d)
        wk = (w.reshape(N, k) * keep.view(N, k).to(w.dtype)).to(rows.dtype)
        return (rows * wk.unsqueeze(-1)).sum(1)

    def load_balance_loss(self) -> torch.Tensor:
        return self.router.load_balance_loss()
