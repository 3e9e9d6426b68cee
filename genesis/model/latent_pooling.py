"""Cross-attention pooling of escalated chunks into learned latents
(``genesis/model/latent_pooling.py:17-173``).

For every chunk selected by the gate (``mask > 0.5`` in training, the bool
mask in evaluation) ``num_latent_vectors`` learned queries attend over the
chunk's ``chunk_size`` projected tokens; output ``(B, N, L, d2)`` with ``N`` the
largest per-sample count of escalated chunks, escalated chunks packed to the
front in ascending chunk order and the padding slots zeroed.

Differences in execution (same result):
  * the packing is done on the device with a prefix sum over the mask
    (``llm_research_b200.ops.compact_chunks``); the reference loops over the
    batch in Python.  One host read of ``N`` remains, since it sets a shape;
  * the query projection of the learned queries is computed once and
    broadcast instead of once per (batch, chunk);
  * ``input_proj`` is applied after the gather (it is per-token and bias free,
    so it commutes with the gather and touches only escalated tokens).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200 import ops


class LatentPooling(nn.Module):
    def __init__(
        self,
        input_dim: int,
        output_dim: int,
        num_latent_vectors: int = 8,
        num_heads: int = 4,
        chunk_size: int = 32,
        dropout: float = 0.0,
    ) -> None:
        super().__init__()
        assert output_dim % num_heads == 0, "output_dim must be divisible by num_heads"
        self.input_dim = input_dim
        self.output_dim = output_dim
        self.num_latent_vectors = num_latent_vectors
        self.num_heads = num_heads
        self.chunk_size = chunk_size
        self.head_dim = output_dim // num_heads
        self.learned_queries = nn.Parameter(torch.randn(num_latent_vectors, output_dim) * 0.02)
        self.input_proj = nn.Linear(input_dim, output_dim, bias=False)
        self.q_proj = nn.Linear(output_dim, output_dim, bias=False)
        self.k_proj = nn.Linear(output_dim, output_dim, bias=False)
        self.v_proj = nn.Linear(output_dim, output_dim, bias=False)
        self.o_proj = nn.Linear(output_dim, output_dim, bias=False)
        self.dropout_p = dropout
        self.norm = nn.LayerNorm(output_dim)

    def forward(self, x: torch.Tensor, chunk_mask: torch.Tensor) -> torch.Tensor:
        x, C, sel = self._chunks(x, chunk_mask)
        idx, valid, n_max = ops.compact_chunks(sel)  # (B, N) chunk ids (C = padding), (B, N) bool
        return self._pool(x, C, idx, valid, n_max)

    def forward_fixed(self, x: torch.Tensor, chunk_mask: torch.Tensor):
        """The same pooling into all ``C`` chunk slots (no host read of the slot
        count): returns ``(out (B, C, L, d2), n)`` where the first ``n`` slots (a
        device scalar) are exactly ``forward``'s output and the rest are zero."""
        x, C, sel = self._chunks(x, chunk_mask)
        idx, valid, _, n = ops.compact_chunks_fixed(sel)
        return self._pool(x, C, idx, valid, C), n

    def _chunks(self, x: torch.Tensor, chunk_mask: torch.Tensor):
        S = x.shape[1]
        cs = self.chunk_size
        pad = (-S) % cs
        if pad:
            x = F.pad(x, (0, 0, 0, pad))
        sel = chunk_mask if chunk_mask.dtype == torch.bool else chunk_mask > 0.5
        return x, x.shape[1] // cs, sel

    def _pool(self, x: torch.Tensor, C: int, idx: torch.Tensor, valid: torch.Tensor, n_max: int) -> torch.Tensor:
        B = x.shape[0]
        cs = self.chunk_size
        chunks = x.view(B, C, cs, self.input_dim)
        chunks = torch.cat([chunks, chunks.new_zeros(B, 1, cs, self.input_dim)], dim=1)
        gathered = chunks[torch.arange(B, device=x.device)[:, None], idx]  # (B, N, cs, d1)
        kv = self.input_proj(gathered).reshape(B * n_max, cs, self.output_dim)

        L, H, hd = self.num_latent_vectors, self.num_heads, self.head_dim
        q = self.q_proj(self.learned_queries).view(1, L, H, hd).transpose(1, 2)  # (1, H, L, hd)
        k = self.k_proj(kv).view(B * n_max, cs, H, hd).transpose(1, 2)
        v = self.v_proj(kv).view(B * n_max, cs, H, hd).transpose(1, 2)
        scores = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(hd))
        probs = F.softmax(scores, dim=-1, dtype=torch.float32).type_as(q)
        probs = F.dropout(probs, p=self.dropout_p, training=self.training)
        out = torch.matmul(probs, v).transpose(1, 2).reshape(B * n_max, L, self.output_dim)
        out = self.norm(self.o_proj(out)).view(B, n_max, L, self.output_dim)
        return out * valid[:, :, None, None].to(out.dtype)
