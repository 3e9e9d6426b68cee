"""Per-layer key/value cache for incremental decoding (``genesis/inference/kv_cache.py:16-121``).

Same interface as the reference (``LayerKVCache.update`` returns the full
``(B, Hkv, S, D)`` key/value, ``KVCache[i]``, ``seq_len``, ``clear``,
``estimate_memory``), but storage is a preallocated buffer grown by
doubling, and new positions are written in place.  The reference
concatenates on every token, which copies the whole cache each step
(quadratic traffic over a generation).  The returned tensors are views of
the buffer; the attention kernel reads them with their strides.
"""

from __future__ import annotations

from typing import Optional

import torch


class LayerKVCache:
    def __init__(self, initial_capacity: int = 256) -> None:
        self._k: Optional[torch.Tensor] = None
        self._v: Optional[torch.Tensor] = None
        self._len = 0
        self._initial = initial_capacity

    @property
    def key(self) -> Optional[torch.Tensor]:
        return None if self._k is None else self._k[:, :, : self._len]

    @property
    def value(self) -> Optional[torch.Tensor]:
        return None if self._v is None else self._v[:, :, : self._len]

    @property
    def seq_len(self) -> int:
        return self._len

    def _grow(self, need: int, like: torch.Tensor) -> None:
        cap = 0 if self._k is None else self._k.shape[2]
        if need <= cap:
            return
        new_cap = max(need, 2 * cap, self._initial)
        B, H, _, D = like.shape
        k = like.new_empty(B, H, new_cap, D)
        v = like.new_empty(B, H, new_cap, D)
        if self._k is not None and self._len:
            k[:, :, : self._len].copy_(self._k[:, :, : self._len])
            v[:, :, : self._len].copy_(self._v[:, :, : self._len])
        self._k, self._v = k, v

    def update(self, new_k: torch.Tensor, new_v: torch.Tensor):
        s = new_k.shape[2]
        if self._k is not None and (self._k.shape[0] != new_k.shape[0] or self._k.dtype != new_k.dtype):
            self.clear()
        self._grow(self._len + s, new_k)
        self._k[:, :, self._len: self._len + s].copy_(new_k)
        self._v[:, :, self._len: self._len + s].copy_(new_v)
        self._len += s
        return self.key, self.value

    def clear(self) -> None:
        self._k = self._v = None
        self._len = 0


class KVCache:
    def __init__(self, num_layers: int) -> None:
        self.layers = [LayerKVCache() for _ in range(num_layers)]

    def __getitem__(self, idx: int) -> LayerKVCache:
        return self.layers[idx]

    def __len__(self) -> int:
        return len(self.layers)

    @property
    def seq_len(self) -> int:
        return self.layers[0].seq_len if self.layers else 0

    def clear(self) -> None:
        for layer in self.layers:
            layer.clear()

    @staticmethod
    def estimate_memory(num_layers: int, num_kv_heads: int, head_dim: int, max_seq_len: int, batch_size: int = 1,
                        dtype: torch.dtype = torch.float16) -> int:
        elem = torch.tensor([], dtype=dtype).element_size()
        return 2 * num_layers * batch_size * num_kv_heads * max_seq_len * head_dim * elem
