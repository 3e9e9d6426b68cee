"""Tokenizer front-end (``olympus/data/tokenizer.py:15-230``).

Backends, tried in order for ``backend="tiktoken"``: tiktoken ``cl100k_base``
(vocabulary ``n_vocab + 10`` special ids), sentencepiece (needs a model path),
then a byte-level fallback.  ``backend="char"`` selects the fallback directly.

The ten special tokens (pad, bos, eos, reason_start/end, memory_read/write,
tier_escalate, trace_start/end) get ids ``base + i`` for the BPE backends and
``256 + i`` for the byte fallback, whose other ids are ``ord(ch) % 256``.
"""

from __future__ import annotations

import os

import logging
from typing import Dict, List, Optional

logger = logging.getLogger(__name__)

SPECIAL_TOKENS: Dict[str, str] = {
    "pad": "<|pad|>",
    "bos": "<|bos|>",
    "eos": "<|eos|>",
    "reason_start": "<|reason_start|>",
    "reason_end": "<|reason_end|>",
    "memory_read": "<|memory_read|>",
    "memory_write": "<|memory_write|>",
    "tier_escalate": "<|tier_escalate|>",
    "trace_start": "<|trace_start|>",
    "trace_end": "<|trace_end|>",
}


class _CharLevelBackend:
    BASE = 256

    def __init__(self, vocab_size: int = 100287) -> None:
        self._vocab_size = vocab_size
        self._special_to_id = {tok: self.BASE + i for i, tok in enumerate(SPECIAL_TOKENS.values())}
        self._id_to_special = {v: k for k, v in self._special_to_id.items()}
        # longest first so that no special token shadows a longer one
        self._specials = sorted(self._special_to_id, key=len, reverse=True)

    @property
    def vocab_size(self) -> int:
        return self._vocab_size

    def encode(self, text: str) -> List[int]:
        ids: List[int] = []
        i, n = 0, len(text)
        while i < n:
            if text[i] == "<":
                hit = next((t for t in self._specials if text.startswith(t, i)), None)
                if hit is not None:
                    ids.append(self._special_to_id[hit])
                    i += len(hit)
                    continue
            ids.append(ord(text[i]) % 256)
            i += 1
        return ids

    def decode(self, ids: List[int]) -> str:
        out = []
        for t in ids:
            t = int(t)
            if t in self._id_to_special:
                out.append(self._id_to_special[t])
            elif 0 <= t < 256:
                out.append(chr(t))
            else:
                out.append(f"<unk_{t}>")
        return "".join(out)

    def special_token_id(self, name: str) -> Optional[int]:
        tok = SPECIAL_TOKENS.get(name)
        return None if tok is None else self._special_to_id.get(tok)


class _LocalTiktoken:
    """The subset of ``tiktoken.Encoding`` the wrapper uses, over :class:`olympus.data.bpe.BytePairEncoder`."""

    def __init__(self, enc) -> None:
        self._enc = enc
        self.n_vocab = enc.n_vocab

    def encode_ordinary(self, text: str):
        return self._enc.encode_ordinary(text)

    def encode(self, text: str, **_):
        return self._enc.encode_ordinary(text)

    def decode(self, ids):
        return self._enc.decode(ids)


class TokenizerWrapper:
    def __init__(self, backend: str = "tiktoken", vocab_size: int = 100287, sp_model_path: Optional[str] = None) -> None:
        self._backend_name = "none"
        self._tiktoken_enc = None
        self._sp_processor = None
        self._char_backend: Optional[_CharLevelBackend] = None
        self._vocab_size = vocab_size
        if backend in ("tiktoken", "auto"):
            try:
                import tiktoken  # type: ignore

                self._tiktoken_enc = tiktoken.get_encoding("cl100k_base")
                self._vocab_size = self._tiktoken_enc.n_vocab + len(SPECIAL_TOKENS)
                self._backend_name = "tiktoken"
            except Exception:
                path = os.environ.get("LRB_TIKTOKEN_FILE")
                if path and os.path.exists(path):  # local cl100k_base.tiktoken, no tiktoken package
                    from olympus.data.bpe import BytePairEncoder

                    self._tiktoken_enc = _LocalTiktoken(BytePairEncoder.from_file(path))
                    self._vocab_size = self._tiktoken_enc.n_vocab + len(SPECIAL_TOKENS)
                    self._backend_name = "tiktoken"
                else:
                    logger.info("tiktoken cl100k_base unavailable; trying sentencepiece")
        if self._backend_name == "none" and backend in ("sentencepiece", "tiktoken", "auto") and sp_model_path:
            try:
                import sentencepiece as spm  # type: ignore

                self._sp_processor = spm.SentencePieceProcessor()
                self._sp_processor.Load(sp_model_path)
                self._vocab_size = self._sp_processor.GetPieceSize() + len(SPECIAL_TOKENS)
                self._backend_name = "sentencepiece"
            except Exception:
                logger.info("sentencepiece unavailable; using the byte fallback")
        if self._backend_name == "none":
            self._char_backend = _CharLevelBackend(vocab_size)
            self._vocab_size = vocab_size
            self._backend_name = "char"
        if self._backend_name == "tiktoken":
            base = self._tiktoken_enc.n_vocab
            self._special_ids = {name: base + i for i, name in enumerate(SPECIAL_TOKENS)}
        elif self._backend_name == "sentencepiece":
            base = self._sp_processor.GetPieceSize()
            self._special_ids = {name: base + i for i, name in enumerate(SPECIAL_TOKENS)}
        else:
            self._special_ids = {n: self._char_backend.special_token_id(n) for n in SPECIAL_TOKENS}

    def encode(self, text: str, return_tensors: Optional[str] = None, **_):
        if self._backend_name == "tiktoken":
            ids = self._tiktoken_enc.encode(text, allowed_special="all")
        elif self._backend_name == "sentencepiece":
            ids = self._sp_processor.Encode(text)
        else:
            ids = self._char_backend.encode(text)
        if return_tensors == "pt":  # HF-style call used by the GRPO/flywheel trainers
            import torch

            return torch.tensor([ids], dtype=torch.long)
        return ids

    def decode(self, ids, skip_special_tokens: bool = False, **_) -> str:
        if hasattr(ids, "tolist"):
            ids = ids.tolist()
        if ids and isinstance(ids[0], list):
            ids = ids[0]
        if self._backend_name == "tiktoken":
            base = self._tiktoken_enc.n_vocab
            return self._tiktoken_enc.decode([i for i in ids if i < base])
        if self._backend_name == "sentencepiece":
            base = self._sp_processor.GetPieceSize()
            return self._sp_processor.Decode([i for i in ids if i < base])
        if skip_special_tokens:
            ids = [i for i in ids if i not in self._special_ids.values()]
        return self._char_backend.decode(ids)

    @property
    def vocab_size(self) -> int:
        return self._vocab_size

    @property
    def backend_name(self) -> str:
        return self._backend_name

    @property
    def pad_id(self) -> int:
        return self._special_ids["pad"]

    @property
    def bos_id(self) -> int:
        return self._special_ids["bos"]

    @property
    def eos_id(self) -> int:
        return self._special_ids["eos"]

    # HF-style aliases used by the RL trainers
    @property
    def eos_token_id(self) -> int:
        return self.eos_id

    @property
    def pad_token_id(self) -> int:
        return self.pad_id

    def special_token_id(self, name: str) -> Optional[int]:
        return self._special_ids.get(name)

    def special_token_ids(self) -> Dict[str, int]:
        return dict(self._special_ids)

    def __repr__(self) -> str:
        return f"TokenizerWrapper(backend={self._backend_name!r}, vocab_size={self._vocab_size})"
