"""Data pipeline: tokenizer, packed datasets, curriculum, batching, quality filter, flywheel buffer."""
from olympus.data.tokenizer import TokenizerWrapper, SPECIAL_TOKENS
from olympus.data.quality_filter import QualityFilter
from olympus.data.curriculum import Curriculum, PhaseConfig
from olympus.data.flywheel_buffer import FlywheelBuffer, TraceEntry
from olympus.data.memory_aware_batcher import MemoryAwareBatcher
from olympus.data.packed_dataset import PackedDataset, SyntheticTokenDataset

__all__ = [
    "TokenizerWrapper", "SPECIAL_TOKENS", "QualityFilter", "Curriculum", "PhaseConfig", "FlywheelBuffer",
    "TraceEntry", "MemoryAwareBatcher", "PackedDataset", "SyntheticTokenDataset",
]
