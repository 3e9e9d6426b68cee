"""GENESIS: the HLRT model family, PHMA memory, ACT-V verifier, training pipelines and inference."""
