"""CUDA-graph decoding for HLRT (an extension: the reference decodes eagerly,
``genesis/inference/generator.py:26-315``).

A decode step is one token through Tier 1, the cached plan vector and the
head: a few hundred small kernels whose launch cost exceeds their run time.
:class:`GraphDecoder` makes the step shape-static -- a fixed-capacity K/V
buffer per layer, the write position and the valid-slot mask on the device,
RoPE rows gathered at that position -- captures it once into a CUDA graph and
replays it for every later token.  The prompt is prefilled by the ordinary
cached forward and copied into the static buffers.

``StaticKVCache`` has the ``KVCache`` indexing interface (``cache[i]``,
``len(cache)``, ``seq_len``); its layers are marked ``is_static`` so that
attention takes the device-position path.  Without CUDA (or with
``use_graph=False``) the same static step runs eagerly.
"""

from __future__ import annotations

from typing import Optional

import torch

from genesis.inference.kv_cache import KVCache


class _StaticLayer:
    is_static = True

    def __init__(self, owner: "StaticKVCache", k: torch.Tensor, v: torch.Tensor) -> None:
        self.owner, self.k, self.v = owner, k, v

    @property
    def pos(self) -> torch.Tensor:
        return self.owner.pos

    @property
    def valid(self) -> torch.Tensor:
        return self.owner.valid

    def write(self, k: torch.Tensor, v: torch.Tensor):
        """Store one position (``k``/``v``: ``(B, 1, Hkv, D)``) at the device-side position."""
        self.k.index_copy_(1, self.owner.pos, k.to(self.k.dtype))
        self.v.index_copy_(1, self.owner.pos, v.to(self.v.dtype))
        return self.k, self.v


class StaticKVCache:
    def __init__(self, num_layers: int, batch: int, capacity: int, num_kv_heads: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device) -> None:
        self.capacity = capacity
        shape = (batch, capacity, num_kv_heads, head_dim)
        self.layers = [_StaticLayer(self, torch.zeros(shape, dtype=dtype, device=device),
                                    torch.zeros(shape, dtype=dtype, device=device)) for _ in range(num_layers)]
        self.pos = torch.zeros(1, dtype=torch.long, device=device)
        self._slots = torch.arange(capacity, device=device)
        self.valid = torch.zeros(capacity, dtype=torch.bool, device=device)

    def __getitem__(self, i: int) -> _StaticLayer:
        return self.layers[i]

    def __len__(self) -> int:
        return len(self.layers)

    @property
    def seq_len(self) -> int:
        return int(self.pos)

    def begin_step(self) -> None:
        torch.le(self._slots, self.pos, out=self.valid)

    def end_step(self) -> None:
        self.pos.add_(1)

    @torch.no_grad()
    def load(self, cache: KVCache) -> None:
        """Copy a prefilled dynamic cache (``(B, Hkv, S, D)`` per layer) into the buffers."""
        S = cache.seq_len
        assert S < self.capacity, "prompt longer than the decode capacity"
        for dst, src in zip(self.layers, [cache[i] for i in range(len(cache))]):
            dst.k[:, :S].copy_(src.key.transpose(1, 2))
            dst.v[:, :S].copy_(src.value.transpose(1, 2))
        self.pos.fill_(S)


class GraphDecoder:
    """Prefill + per-token decode of ``model`` for ``batch`` sequences of up to ``capacity`` tokens."""

    def __init__(self, model, batch: int, capacity: int, use_graph: Optional[bool] = None) -> None:
        c = model.config
        p = model.embeddings.weight
        self.model, self.batch, self.capacity = model, batch, capacity
        heads = c.tier1_num_heads
        self.cache = StaticKVCache(c.tier1_num_layers, batch, capacity, c.tier1_num_kv_heads or heads,
                                   c.d_model // heads, p.dtype, p.device)
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=p.device)
        self.logits: Optional[torch.Tensor] = None
        self.use_graph = (p.is_cuda if use_graph is None else use_graph) and p.is_cuda
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor) -> torch.Tensor:
        cache = KVCache(self.model.config.tier1_num_layers)
        out = self.model(input_ids, kv_cache=cache, position_offset=0)
        self.cache.load(cache)
        return out["logits"][:, -1, :]

    def _step(self) -> None:
        self.cache.begin_step()
        # position_offset only sizes the RoPE tables; the position itself is on the device
        out = self.model(self.ids, kv_cache=self.cache, position_offset=self.capacity - 1)
        self.logits = out["logits"][:, -1, :]
        self.cache.end_step()

    @torch.no_grad()
    def step(self, tok: torch.Tensor) -> torch.Tensor:
        """Feed one token per sequence; returns the next-token logits ``(B, vocab)`` (a
        buffer that the next call overwrites)."""
        self.ids.copy_(tok.view(self.batch, 1))
        if not self.use_graph:
            self._step()
            return self.logits
        if self.graph is None:
            self._capture()
        self.graph.replay()
        return self.logits

    def _capture(self) -> None:
        pos0 = self.cache.pos.clone()
        side = torch.cuda.Stream(device=self.ids.device)
        side.wait_stream(torch.cuda.current_stream(self.ids.device))
        with torch.cuda.stream(side):
            self._step()  # warm-up: builds RoPE tables, selects kernels, sets kernel attributes
        torch.cuda.current_stream(self.ids.device).wait_stream(side)
        self.cache.pos.copy_(pos0)  # the warm-up's write is redone by the first replay
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step()
        self.graph = g
