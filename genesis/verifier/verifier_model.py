"""Verifier encoder (``genesis/verifier/verifier_model.py:21-176``).

A narrower, shallower copy of the Tier-1 stack that shares the generator's
vocabulary: embeddings → ``num_layers`` TransformerBlocks (RoPE, causal
attention, SwiGLU) → RMSNorm → masked mean pool → ``tanh(Linear)``.
Returns ``{"hidden_states": (B, S, d), "pooled_output": (B, d)}``.

Without a padding mask the blocks run the fused flash-attention path; with one,
the mask becomes an additive ``(B, 1, 1, S)`` bias (``finfo.min`` on pads) and
attention takes the masked path.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn as nn

from genesis.model.embeddings import SharedEmbeddings
from genesis.model.rmsnorm import RMSNorm
from genesis.model.rotary import RotaryEmbedding
from genesis.model.tier1_token_processor import TransformerBlock


class VerifierModel(nn.Module):
    def __init__(self, vocab_size: int = 32000, d_model: int = 512, num_layers: int = 8, num_heads: int = 8,
                 d_ff: int = 2048, max_seq_len: int = 4096, dropout: float = 0.0, norm_eps: float = 1e-6,
                 rope_base: float = 10000.0) -> None:
        super().__init__()
        self.d_model = d_model
        self.vocab_size = vocab_size
        self.num_layers = num_layers
        self.embeddings = SharedEmbeddings(vocab_size=vocab_size, d_model=d_model, dropout=dropout)
        self.rotary_emb = RotaryEmbedding(dim=d_model // num_heads, max_seq_len=max_seq_len, base=rope_base)
        self.layers = nn.ModuleList([
            TransformerBlock(d_model=d_model, num_heads=num_heads, d_ff=d_ff, dropout=dropout,
                             use_flash_attention=True, norm_eps=norm_eps)
            for _ in range(num_layers)
        ])
        self.final_norm = RMSNorm(d_model, eps=norm_eps)
        self.pool_proj = nn.Linear(d_model, d_model)
        nn.init.xavier_uniform_(self.pool_proj.weight)
        nn.init.zeros_(self.pool_proj.bias)

    @staticmethod
    def _mean_pool(hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if attention_mask is None:
            return hidden_states.mean(dim=1)
        m = attention_mask.unsqueeze(-1).to(hidden_states.dtype)
        return (hidden_states * m).sum(dim=1) / m.sum(dim=1).clamp(min=1.0)

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
        x = self.embeddings(input_ids)
        cos, sin = self.rotary_emb(x.size(1))
        bias = None
        if attention_mask is not None:
            bias = (1.0 - attention_mask.to(x.dtype))[:, None, None, :] * torch.finfo(x.dtype).min
        for layer in self.layers:
            x = layer(x, cos, sin, attention_mask=bias)
        hidden = self.final_norm(x)
        pooled = torch.tanh(self.pool_proj(self._mean_pool(hidden, attention_mask)))
        return {"hidden_states": hidden, "pooled_output": pooled}
