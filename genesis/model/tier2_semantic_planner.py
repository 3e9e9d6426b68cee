"""Tier 2: transformer over the flattened latents, optionally MoE
(``genesis/model/tier2_semantic_planner.py:22-204``)."""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from genesis.model.ffn import SwiGLUFFN
from genesis.model.moe import MoEFFN
from genesis.model.rmsnorm import RMSNorm
from genesis.model.rotary import RotaryEmbedding
from genesis.model.tier1_token_processor import TransformerBlock


class Tier2TransformerBlock(TransformerBlock):
    def __init__(
        self,
        d_model: int,
        num_heads: int,
        d_ff: int | None = None,
        num_kv_heads: int | None = None,
        dropout: float = 0.0,
        use_flash_attention: bool = True,
        norm_eps: float = 1e-6,
        moe_num_experts: int | None = None,
        moe_top_k: int = 2,
    ) -> None:
        self._moe_cfg = (moe_num_experts, moe_top_k)
        super().__init__(d_model, num_heads, d_ff, num_kv_heads, dropout, use_flash_attention, norm_eps)
        self.is_moe = isinstance(self.ffn, MoEFFN)

    def _make_ffn(self, d_model: int, d_ff: int | None, dropout: float) -> nn.Module:
        n_exp, top_k = self._moe_cfg
        if n_exp is not None and n_exp > 1:
            return MoEFFN(d_model=d_model, d_ff=d_ff, num_experts=n_exp, top_k=top_k, dropout=dropout)
        return SwiGLUFFN(d_model=d_model, d_ff=d_ff, dropout=dropout)

    def forward(self, x, cos, sin, attention_mask=None, **_):  # type: ignore[override]
        return super().forward(x, cos, sin, attention_mask=attention_mask)

    def load_balance_loss(self) -> torch.Tensor:
        return self.ffn.load_balance_loss() if self.is_moe else torch.tensor(0.0)


class Tier2SemanticPlanner(nn.Module):
    def __init__(
        self,
        num_layers: int,
        d_model: int,
        num_heads: int,
        d_ff: int | None = None,
        num_kv_heads: int | None = None,
        dropout: float = 0.0,
        use_flash_attention: bool = True,
        max_seq_len: int = 2048,
        rope_base: float = 10000.0,
        norm_eps: float = 1e-6,
        moe_num_experts: int | None = None,
        moe_top_k: int = 2,
    ) -> None:
        super().__init__()
        self.d_model = d_model
        self.rotary_emb = RotaryEmbedding(dim=d_model // num_heads, max_seq_len=max_seq_len, base=rope_base)
        self.layers = nn.ModuleList([
            Tier2TransformerBlock(
                d_model=d_model, num_heads=num_heads, d_ff=d_ff, num_kv_heads=num_kv_heads, dropout=dropout,
                use_flash_attention=use_flash_attention, norm_eps=norm_eps,
                moe_num_experts=moe_num_experts, moe_top_k=moe_top_k,
            )
            for _ in range(num_layers)
        ])
        self.final_norm = RMSNorm(d_model, eps=norm_eps)

    def forward(self, latent_vectors: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, N, L, D = latent_vectors.shape
        x = latent_vectors.reshape(B, N * L, D)
        cos, sin = self.rotary_emb(N * L)
        for layer in self.layers:
            x = layer(x, cos, sin, attention_mask=attention_mask)
        return self.final_norm(x).view(B, N, L, D)

    def load_balance_loss(self) -> torch.Tensor:
        total = torch.tensor(0.0)
        for layer in self.layers:
            lb = layer.load_balance_loss()
            total = total.to(lb.device) + lb
        return total
