"""Byte-level BPE with a ``.tiktoken`` rank table (cl100k_base format).

Pure-Python statement of the algorithm that ``csrc/tools/genesis_pack.cpp``
implements natively: pre-tokenise with the cl100k pattern, then, for each
piece not in the table, repeatedly merge the adjacent pair whose
concatenation has the lowest rank (leftmost on ties).  It is the oracle for
the native packer's tests and the ``tiktoken`` backend of
:class:`~olympus.data.tokenizer.TokenizerWrapper` when the ``tiktoken``
package is absent but a rank file is available (``LRB_TIKTOKEN_FILE``).
"""

from __future__ import annotations

import base64
from typing import Dict, Iterable, List

import regex

CL100K_PATTERN = (r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"""
                  r"""|\s*[\r\n]+|\s+(?!\S)|\s+""")


def load_tiktoken_ranks(path: str) -> Dict[bytes, int]:
    ranks: Dict[bytes, int] = {}
    with open(path, "rb") as f:
        for line in f:
            if line.strip():
                tok, rank = line.split()
                ranks[base64.b64decode(tok)] = int(rank)
    return ranks


def save_tiktoken_ranks(ranks: Dict[bytes, int], path: str) -> None:
    with open(path, "wb") as f:
        for tok, rank in sorted(ranks.items(), key=lambda kv: kv[1]):
            f.write(base64.b64encode(tok) + b" " + str(rank).encode() + b"\n")


def byte_pair_merge(piece: bytes, ranks: Dict[bytes, int]) -> List[int]:
    parts = [piece[i:i + 1] for i in range(len(piece))]
    while len(parts) > 1:
        best, at = None, -1
        for i in range(len(parts) - 1):
            r = ranks.get(parts[i] + parts[i + 1])
            if r is not None and (best is None or r < best):
                best, at = r, i
        if best is None:
            break
        parts[at:at + 2] = [parts[at] + parts[at + 1]]
    return [ranks[p] for p in parts]


class BytePairEncoder:
    def __init__(self, ranks: Dict[bytes, int], pattern: str = CL100K_PATTERN) -> None:
        self.ranks = ranks
        self.decoder = {v: k for k, v in ranks.items()}
        self.pattern = regex.compile(pattern)
        self._cache: Dict[bytes, List[int]] = {}

    @classmethod
    def from_file(cls, path: str) -> "BytePairEncoder":
        return cls(load_tiktoken_ranks(path))

    def pieces(self, text: str) -> List[str]:
        return self.pattern.findall(text)

    def encode_ordinary(self, text: str) -> List[int]:
        out: List[int] = []
        for piece in self.pieces(text):
            b = piece.encode("utf-8")
            r = self.ranks.get(b)
            if r is not None:
                out.append(r)
                continue
            ids = self._cache.get(b)
            if ids is None:
                ids = byte_pair_merge(b, self.ranks)
                if len(self._cache) < 1 << 16:
                    self._cache[b] = ids
            out.extend(ids)
        return out

    def decode_bytes(self, ids: Iterable[int]) -> bytes:
        return b"".join(self.decoder[i] for i in ids)

    def decode(self, ids: Iterable[int]) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")

    @property
    def n_vocab(self) -> int:
        return max(self.ranks.values()) + 1
