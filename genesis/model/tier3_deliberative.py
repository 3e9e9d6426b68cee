"""Tier 3: weight-shared recurrent transformer (``genesis/model/tier3_deliberative.py:21-188``).

``h = input_proj(x)``; ``recurrence_steps`` times: ``h += step_embedding[t]``,
run all layers, ``h += input_proj(x)`` (the cross-step residual); then
``final_norm`` and ``output_proj`` back to the Tier-2 width.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from genesis.model.rmsnorm import RMSNorm
from genesis.model.rotary import RotaryEmbedding
from genesis.model.tier1_token_processor import TransformerBlock


class Tier3TransformerBlock(TransformerBlock):
    def forward(self, x, cos, sin, attention_mask=None, **_):  # type: ignore[override]
        return super().forward(x, cos, sin, attention_mask=attention_mask)


class Tier3DeliberativeReasoner(nn.Module):
    def __init__(
        self,
        num_layers: int,
        input_dim: int,
        d_model: int,
        num_heads: int,
        d_ff: int | None = None,
        num_kv_heads: int | None = None,
        dropout: float = 0.0,
        use_flash_attention: bool = True,
        max_seq_len: int = 1024,
        rope_base: float = 10000.0,
        norm_eps: float = 1e-6,
        recurrence_steps: int = 4,
    ) -> None:
        super().__init__()
        self.input_dim = input_dim
        self.d_model = d_model
        self.recurrence_steps = recurrence_steps
        self.input_proj = nn.Linear(input_dim, d_model, bias=False)
        self.output_proj = nn.Linear(d_model, input_dim, bias=False)
        self.rotary_emb = RotaryEmbedding(dim=d_model // num_heads, max_seq_len=max_seq_len, base=rope_base)
        self.layers = nn.ModuleList([
            Tier3TransformerBlock(
                d_model=d_model, num_heads=num_heads, d_ff=d_ff, num_kv_heads=num_kv_heads,
                dropout=dropout, use_flash_attention=use_flash_attention, norm_eps=norm_eps,
            )
            for _ in range(num_layers)
        ])
        self.final_norm = RMSNorm(d_model, eps=norm_eps)
        self.step_embedding = nn.Parameter(torch.randn(recurrence_steps, d_model) * 0.02)

    def forward(self, x: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, N, L, _ = x.shape
        h = self.input_proj(x.reshape(B, N * L, self.input_dim))
        cos, sin = self.rotary_emb(h.shape[1])
        residual = h
        for t in range(self.recurrence_steps):
            h = h + self.step_embedding[t]
            for layer in self.layers:
                h = layer(h, cos, sin, attention_mask=attention_mask)
            h = h + residual
        return self.output_proj(self.final_norm(h)).view(B, N, L, self.input_dim)
