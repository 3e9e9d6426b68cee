"""Data pipeline: tokenizer, packed datasets, curriculum, batching, quality filter, flywheel buffer."""
from olympus.data.tokenizer import TokenizerWrapper, SPECIAL_TOKENS
from olympus.data.packed_dataset import PackedDataset, SyntheticTokenDataset

__all__ = ["TokenizerWrapper", "SPECIAL_TOKENS", "PackedDataset", "SyntheticTokenDataset"]
