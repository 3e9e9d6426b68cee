"""Autoregressive generation with HLRT (``genesis/inference/generator.py:26-315``).

Prefill runs the full hierarchy with a Tier-1 KV cache; every decode step
feeds one token, which takes HLRT's single-token path (Tier 1 + cached plan
vector).  On a GPU the decode steps replay one captured CUDA graph
(``genesis.inference.graph_decode``).  ``use_kv_cache=False`` recomputes the whole sequence every step
(the reference's uncached mode).  Gate-threshold overrides in
:class:`GenerationConfig` are applied to the model's gates for the duration of
the call (the reference records them but never applies them).
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Dict, Iterator

import torch

from genesis.inference.cascade_router import CascadeRouter
from genesis.inference.kv_cache import KVCache
from genesis.inference.sampling import SamplingConfig, sample
from genesis.model.hlrt import HLRT, HLRTConfig


@dataclass
class GenerationConfig:
    max_new_tokens: int = 256
    sampling: SamplingConfig = None  # type: ignore[assignment]
    eos_token_id: int | None = None
    pad_token_id: int | None = None
    use_kv_cache: bool = True
    gate1_threshold: float | None = None
    gate2_threshold: float | None = None

    def __post_init__(self) -> None:
        if self.sampling is None:
            self.sampling = SamplingConfig()


class Generator:
    """``cuda_graph``: decode through :class:`GraphDecoder` (one captured CUDA graph
    replayed per token) when the model is on a GPU -- the default; ``False`` keeps
    the eager cached decode."""

    def __init__(self, model: HLRT, cuda_graph: bool | None = None) -> None:
        self.model = model
        self.config = model.config
        self.cuda_graph = cuda_graph

    def _graph_decoder(self, input_ids: torch.Tensor, cfg: "GenerationConfig"):
        on_gpu = input_ids.is_cuda and self.model.embeddings.weight.is_cuda
        if not cfg.use_kv_cache or not on_gpu or self.cuda_graph is False:
            return None
        from genesis.inference.graph_decode import GraphDecoder

        B, S = input_ids.shape
        return GraphDecoder(self.model, B, S + cfg.max_new_tokens + 1)

    @contextlib.contextmanager
    def _thresholds(self, cfg: GenerationConfig):
        g1, g2 = self.model.gate1.threshold, self.model.gate2.threshold
        if cfg.gate1_threshold is not None:
            self.model.gate1.threshold = cfg.gate1_threshold
        if cfg.gate2_threshold is not None:
            self.model.gate2.threshold = cfg.gate2_threshold
        try:
            yield
        finally:
            self.model.gate1.threshold, self.model.gate2.threshold = g1, g2

    def _forward(self, ids, cache, offset):
        out = self.model(ids, return_tier_activations=True, kv_cache=cache, position_offset=offset)
        acts = out.get("tier_activations", {})
        return out["logits"][:, -1, :], "tier2" in acts, "tier3" in acts

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, config: GenerationConfig | None = None) -> Dict[str, object]:
        cfg = config or GenerationConfig()
        self.model.eval()
        B, S = input_ids.shape
        router = CascadeRouter(cfg.gate1_threshold, cfg.gate2_threshold)
        graph = self._graph_decoder(input_ids, cfg)
        cache = KVCache(self.config.tier1_num_layers) if cfg.use_kv_cache and graph is None else None
        with self._thresholds(cfg):
            if graph is not None:
                cache_out = KVCache(self.config.tier1_num_layers)
                logits, t2, t3 = self._forward(input_ids, cache_out, 0)
                graph.cache.load(cache_out)
                del cache_out
            else:
                logits, t2, t3 = self._forward(input_ids, cache, 0)
            router.record(S, t2, t3)
            tok = sample(logits, cfg.sampling)
            new = [tok]
            seq = torch.cat([input_ids, tok[:, None]], dim=1)
            for step in range(1, cfg.max_new_tokens):
                if cfg.eos_token_id is not None and bool((tok == cfg.eos_token_id).all()):
                    break
                if graph is not None:  # single-token path: Tier 1 + cached plan, no upper tiers
                    logits, t2, t3 = graph.step(tok), False, False
                elif cache is not None:
                    logits, t2, t3 = self._forward(tok[:, None], cache, S + step - 1)
                else:
                    logits, t2, t3 = self._forward(seq, None, 0)
                router.record(1, t2, t3)
                tok = sample(logits, cfg.sampling, torch.stack(new, dim=1))
                new.append(tok)
                seq = torch.cat([seq, tok[:, None]], dim=1)
        return {"token_ids": seq, "new_token_ids": torch.stack(new, dim=1), "cascade_stats": router.stats}

    @torch.no_grad()
    def generate_streaming(self, input_ids: torch.Tensor, config: GenerationConfig | None = None) -> Iterator[int]:
        cfg = config or GenerationConfig()
        self.model.eval()
        B, S = input_ids.shape
        assert B == 1, "Streaming generation only supports batch_size=1"
        router = CascadeRouter(cfg.gate1_threshold, cfg.gate2_threshold)
        cache = KVCache(self.config.tier1_num_layers) if cfg.use_kv_cache else None
        with self._thresholds(cfg):
            logits, t2, t3 = self._forward(input_ids, cache, 0)
            router.record(S, t2, t3)
            tok = sample(logits, cfg.sampling)
            ids = [int(tok)]
            yield ids[-1]
            if cfg.eos_token_id is not None and ids[-1] == cfg.eos_token_id:
                return
            seq = torch.cat([input_ids, tok.view(1, 1)], dim=1)
            for step in range(1, cfg.max_new_tokens):
                if cache is not None:
                    logits, t2, t3 = self._forward(tok.view(1, 1), cache, S + step - 1)
                else:
                    logits, t2, t3 = self._forward(seq, None, 0)
                router.record(1, t2, t3)
                tok = sample(logits, cfg.sampling, torch.tensor([ids], device=input_ids.device))
                ids.append(int(tok))
                seq = torch.cat([seq, tok.view(1, 1)], dim=1)
                yield ids[-1]
                if cfg.eos_token_id is not None and ids[-1] == cfg.eos_token_id:
                    break

    @staticmethod
    def estimate_memory(config: HLRTConfig, max_seq_len: int, batch_size: int = 1,
                        dtype: torch.dtype = torch.float16) -> Dict[str, int]:
        elem = torch.tensor([], dtype=dtype).element_size()

        def tier(layers: int, d: int) -> int:
            return layers * (4 * d * d + 3 * d * int(8 / 3 * d))

        params = (tier(config.tier1_num_layers, config.d_model) + tier(config.tier2_num_layers, config.tier2_d_model)
                  + tier(config.tier3_num_layers, config.tier3_d_model) + config.vocab_size * config.d_model)
        kv = KVCache.estimate_memory(config.tier1_num_layers, config.tier1_num_kv_heads or config.tier1_num_heads,
                                     config.d_model // config.tier1_num_heads, max_seq_len, batch_size, dtype)
        acts = config.tier1_num_layers * batch_size * max_seq_len * config.d_model * elem
        return {"model_weights": params * elem, "kv_cache": kv, "activations": acts, "total": params * elem + kv + acts}
