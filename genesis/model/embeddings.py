"""Token embeddings shared with the output head (``genesis/model/embeddings.py:13-56``)."""

from __future__ import annotations

import torch
import torch.nn as nn


class SharedEmbeddings(nn.Module):
    def __init__(self, vocab_size: int, d_model: int, dropout: float = 0.0, padding_idx: int | None = None) -> None:
        super().__init__()
        self.d_model = d_model
        self.embedding = nn.Embedding(vocab_size, d_model, padding_idx=padding_idx)
        self.dropout = nn.Dropout(dropout) if dropout > 0.0 else nn.Identity()

    @property
    def weight(self) -> torch.Tensor:
        return self.embedding.weight

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.dropout(self.embedding(input_ids))
