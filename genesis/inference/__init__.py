"""GENESIS inference: generation, KV caching, sampling and cascade routing."""
from genesis.inference.cascade_router import CascadeRouter, CascadeStats
from genesis.inference.generator import GenerationConfig, Generator
from genesis.inference.kv_cache import KVCache, LayerKVCache
from genesis.inference.sampling import SamplingConfig, sample

__all__ = ["CascadeRouter", "CascadeStats", "GenerationConfig", "Generator", "KVCache", "LayerKVCache",
           "SamplingConfig", "sample"]
