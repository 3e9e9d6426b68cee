"""Chunk gating + expert routing API (``olympus/kernels/fused_gate_route.py:279-386``).

``chunk_mean_pool`` and ``softmax_topk`` run as sm_100a kernels on CUDA
(``llm_research_b200.ops.routing``); ``fused_gate_route`` composes them with
the gate MLP and the router projection exactly like the reference.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200._ext import available as _native_available
from llm_research_b200.ops.routing import _softmax_topk_ref, chunk_mean_pool, softmax_topk

# The reference exposes HAS_TRITON; this framework has no Triton path.
HAS_TRITON = False
HAS_NATIVE = _native_available()


def _chunk_mean_pool_pt(x: torch.Tensor, chunk_size: int) -> torch.Tensor:
    """Plain-PyTorch chunk mean (``fused_gate_route.py:30-34``), the kernel's oracle."""
    B, S, D = x.shape
    return x.view(B, S // chunk_size, chunk_size, D).mean(dim=2)


def _softmax_topk_pt(logits: torch.Tensor, top_k: int):
    """Plain-PyTorch softmax + top-k + renormalisation (``fused_gate_route.py:37-47``)."""
    return _softmax_topk_ref(logits, top_k)


def fused_gate_route(
    x: torch.Tensor,
    gate_mlp: nn.Module,
    router_gate: nn.Linear,
    chunk_size: int = 32,
    threshold: float = 0.5,
    top_k: int = 2,
    jitter_noise: float = 0.0,
    training: bool = True,
):
    B, S, D = x.shape
    pad = (-S) % chunk_size
    if pad:
        x = F.pad(x, (0, 0, 0, pad))
    scores = torch.sigmoid(gate_mlp(chunk_mean_pool(x, chunk_size)).squeeze(-1))
    mask = scores if training else scores >= threshold
    xf = x.reshape(-1, D)
    if training and jitter_noise > 0.0:
        xf = xf * torch.empty_like(xf).uniform_(1.0 - jitter_noise, 1.0 + jitter_noise)
    w, idx, probs = softmax_topk(router_gate(xf), top_k)
    return mask, scores, w.type_as(x), idx, probs
