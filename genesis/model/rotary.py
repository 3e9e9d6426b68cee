"""Rotary position embeddings (``genesis/model/rotary.py:15-99``).

``inv_freq[i] = base^(-2i/dim)``; tables ``cos/sin`` of shape ``(seq, dim)``
hold each frequency twice (rotate-half convention) and are non-persistent
buffers, rebuilt when a longer sequence is requested.
``apply_rotary_emb(x, cos, sin) = x * cos + rotate_half(x) * sin`` with
``rotate_half([x1, x2]) = [-x2, x1]``.
"""

from __future__ import annotations

import torch
import torch.nn as nn


class RotaryEmbedding(nn.Module):
    def __init__(self, dim: int, max_seq_len: int = 8192, base: float = 10000.0) -> None:
        super().__init__()
        assert dim % 2 == 0, "RoPE dimension must be even."
        self.dim = dim
        self.max_seq_len = max_seq_len
        self.base = base
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        self._build_cache(max_seq_len)

    def _build_cache(self, seq_len: int) -> None:
        self.max_seq_len = seq_len
        pos = torch.arange(seq_len, dtype=torch.float32, device=self.inv_freq.device)
        ang = torch.outer(pos, self.inv_freq.float())
        ang = torch.cat([ang, ang], dim=-1)
        self.register_buffer("cos_cached", ang.cos().to(self.inv_freq.dtype), persistent=False)
        self.register_buffer("sin_cached", ang.sin().to(self.inv_freq.dtype), persistent=False)

    def forward(self, seq_len: int):
        if seq_len > self.max_seq_len:
            self._build_cache(seq_len)
        return self.cos_cached[:seq_len], self.sin_cached[:seq_len]


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate ``x`` of shape ``(B, H, S, D)`` with tables of shape ``(S, D)``."""
    return x * cos[None, None] + _rotate_half(x) * sin[None, None]
