"""Memory-mapped reader for packed token blocks (``olympus/data/packed_dataset.py:25-68``).

Directory layout written by the ``genesis-pack`` tool: ``meta.json`` plus
``{train,val}_input_ids.bin``, raw little-endian uint32, ``n_blocks x block_size``.
Items are ``{"input_ids": int64 tensor (block_size,)}``.

:class:`SyntheticTokenDataset` produces the same items from a seeded uniform
distribution, for benchmarks and tests that must not touch the file system.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Dict

import numpy as np
import torch
from torch.utils.data import Dataset


class PackedDataset(Dataset):
    def __init__(self, data_dir: str | Path, split: str = "train") -> None:
        data_dir = Path(data_dir)
        with open(data_dir / "meta.json") as f:
            self.meta = json.load(f)
        self.block_size: int = int(self.meta["block_size"])
        if split not in ("train", "val"):
            raise ValueError(f"split must be 'train' or 'val', got {split!r}")
        self.n_blocks = int(self.meta["train_blocks" if split == "train" else "val_blocks"])
        self.data = np.memmap(data_dir / f"{split}_input_ids.bin", dtype="<u4", mode="r",
                              shape=(self.n_blocks, self.block_size))

    def __len__(self) -> int:
        return self.n_blocks

    def __getitem__(self, idx: int) -> Dict[str, torch.Tensor]:
        return {"input_ids": torch.from_numpy(np.asarray(self.data[idx], dtype=np.int64))}

    def __repr__(self) -> str:
        return f"PackedDataset(blocks={self.n_blocks}, block_size={self.block_size}, tokens={self.n_blocks * self.block_size:,})"


class SyntheticTokenDataset(Dataset):
    """``n_blocks`` sequences of ``block_size`` ids uniform in ``[0, vocab_size)``."""

    def __init__(self, n_blocks: int, block_size: int, vocab_size: int, seed: int = 0) -> None:
        g = torch.Generator().manual_seed(seed)
        self.data = torch.randint(0, vocab_size, (n_blocks, block_size), generator=g, dtype=torch.int64)
        self.block_size = block_size

    def __len__(self) -> int:
        return self.data.shape[0]

    def __getitem__(self, idx: int) -> Dict[str, torch.Tensor]:
        return {"input_ids": self.data[idx]}
