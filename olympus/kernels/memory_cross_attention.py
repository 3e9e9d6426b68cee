"""Cross-attention from hidden states to a memory bank
(``olympus/kernels/memory_cross_attention.py:120-194``).

Projects the query ``(B, Sq, d)`` and the bank ``(M, dm)`` or ``(B, M, dm)``,
attends without a causal mask, projects back.  Without a mask the attention
is the flash-attention kernel (non-causal); an optional ``(B, M)`` bool mask
(True = valid slot) uses an explicit masked softmax.  The top-k PHMA read
(only the k best slots per query) is :func:`llm_research_b200.ops.memory.topk_memory_attention`.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200 import ops

HAS_TRITON = False
HAS_SDPA = True


def _expand_mask_pt(mask: torch.Tensor) -> torch.Tensor:
    """``(B, M)`` bool -> ``(B, 1, 1, M)`` additive fp32 bias (0 or -inf)."""
    return torch.where(mask[:, None, None, :], 0.0, float("-inf"))


def _manual_cross_attention(q, k, v, attn_mask, scale, dropout_p, training):
    w = torch.matmul(q, k.transpose(-2, -1)) * scale
    if attn_mask is not None:
        w = w + attn_mask
    w = F.softmax(w, dim=-1, dtype=torch.float32).type_as(q)
    w = F.dropout(w, p=dropout_p, training=training)
    return torch.matmul(w, v)


def memory_cross_attention(
    query: torch.Tensor,
    memory_keys: torch.Tensor,
    memory_values: torch.Tensor,
    q_proj: nn.Linear,
    k_proj: nn.Linear,
    v_proj: nn.Linear,
    o_proj: nn.Linear,
    num_heads: int,
    memory_mask: Optional[torch.Tensor] = None,
    dropout_p: float = 0.0,
    training: bool = True,
) -> torch.Tensor:
    B, Sq, d = query.shape
    if memory_keys.dim() == 2:
        memory_keys = memory_keys.unsqueeze(0).expand(B, -1, -1)
    if memory_values.dim() == 2:
        memory_values = memory_values.unsqueeze(0).expand(B, -1, -1)
    M = memory_keys.shape[1]
    hd = d // num_heads
    q = q_proj(query).view(B, Sq, num_heads, hd)
    k = k_proj(memory_keys).view(B, M, num_heads, hd)
    v = v_proj(memory_values).view(B, M, num_heads, hd)
    drop = dropout_p if training else 0.0
    if memory_mask is None and drop == 0.0 and hd in (16, 32, 64, 96, 128) and q.dtype != torch.float32 or (
            memory_mask is None and drop == 0.0 and not q.is_cuda):
        out = ops.attention(q, k, v, causal=False)
    else:
        mask = _expand_mask_pt(memory_mask).to(q.dtype) if memory_mask is not None else None
        out = _manual_cross_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), mask,
                                      1.0 / math.sqrt(hd), drop, training).transpose(1, 2)
    return o_proj(out.reshape(B, Sq, d))
