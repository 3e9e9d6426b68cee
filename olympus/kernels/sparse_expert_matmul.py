"""Sorted expert dispatch (``olympus/kernels/sparse_expert_matmul.py:26-164``).

``sparse_expert_matmul(x, idx, w, experts, E, k)`` =
``sum_k w[n,k] * experts[idx[n,k]](x[n])``: one stable sort groups the
``N*k`` assignments by expert, each expert runs once on a contiguous slice,
the weighted outputs are scattered back with one ``index_add``.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from olympus.core.compute_router import grouped_expert_apply


def _naive_expert_dispatch(x, expert_indices, expert_weights, experts, num_experts, top_k):
    out = torch.zeros_like(x)
    for k in range(top_k):
        for e in range(num_experts):
            m = expert_indices[:, k] == e
            if m.any():
                out[m] += expert_weights[m, k:k + 1] * experts[e](x[m])
    return out


def sparse_expert_matmul(x: torch.Tensor, expert_indices: torch.Tensor, expert_weights: torch.Tensor,
                         experts: nn.ModuleList, num_experts: int, top_k: int) -> torch.Tensor:
    return grouped_expert_apply(x, expert_indices[:, :top_k], expert_weights[:, :top_k], experts, num_experts).to(x.dtype)


def _sorted_expert_dispatch(x, expert_indices, expert_weights, experts, num_experts, top_k):
    """The sorted dispatch itself (``sparse_expert_matmul.py:26-99``): one stable
    sort by expert, one contiguous slice per expert, one ``index_add`` back."""
    return grouped_expert_apply(x, expert_indices[:, :top_k], expert_weights[:, :top_k], experts, num_experts).to(x.dtype)
