"""Topic-coherent batching by greedy TF-IDF clustering
(``olympus/data/memory_aware_batcher.py:19-208``).

Documents are lower-cased and whitespace-tokenised; the ``max_vocab`` most
document-frequent terms get ``idf = ln((n+1)/(df+1)) + 1``; rows are
L2-normalised ``tf * idf``.  Batches grow from a random seed by repeatedly
adding the remaining document most similar to the (normalised) batch
centroid, until the batch is full or the best similarity drops below
``similarity_threshold``.  Fewer than ``min_docs_for_clustering`` documents
are batched randomly.

The vectors are a dense ``(docs, vocab)`` matrix and every greedy step is one
matrix-vector product over the remaining documents, instead of a Python loop
over sparse dictionaries.
"""

from __future__ import annotations

import logging
import math
import random
from collections import Counter
from typing import List

import torch

logger = logging.getLogger(__name__)


class MemoryAwareBatcher:
    def __init__(self, max_vocab: int = 10_000, min_docs_for_clustering: int = 8, similarity_threshold: float = 0.05) -> None:
        self.max_vocab = max_vocab
        self.min_docs_for_clustering = min_docs_for_clustering
        self.similarity_threshold = similarity_threshold

    @staticmethod
    def _tokenize(text: str) -> List[str]:
        return text.lower().split()

    def _tfidf_matrix(self, documents: List[str]) -> torch.Tensor:
        toks = [self._tokenize(d) for d in documents]
        df: Counter = Counter()
        for t in toks:
            df.update(set(t))
        vocab = [w for w, _ in df.most_common(self.max_vocab)] if len(df) > self.max_vocab else list(df)
        index = {w: i for i, w in enumerate(vocab)}
        n = len(documents)
        idf = torch.tensor([math.log((n + 1) / (df[w] + 1)) + 1.0 for w in vocab], dtype=torch.float64)
        mat = torch.zeros(n, max(len(vocab), 1), dtype=torch.float64)
        for r, t in enumerate(toks):
            total = len(t) or 1
            for w, c in Counter(t).items():
                j = index.get(w)
                if j is not None:
                    mat[r, j] = c / total * idf[j]
        norms = mat.norm(dim=1, keepdim=True)
        return mat / torch.where(norms > 0, norms, torch.ones_like(norms))

    def create_batches(self, documents: List[str], batch_size: int) -> List[List[str]]:
        if not documents:
            return []
        if batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if len(documents) < self.min_docs_for_clustering:
            return self._random_batches(documents, batch_size)
        try:
            return self._clustered_batches(documents, batch_size)
        except Exception as exc:  # pragma: no cover - defensive, mirrors the reference
            logger.warning("Clustering failed (%s), falling back to random batching", exc)
            return self._random_batches(documents, batch_size)

    def _random_batches(self, documents: List[str], batch_size: int) -> List[List[str]]:
        docs = list(documents)
        random.shuffle(docs)
        return [docs[i: i + batch_size] for i in range(0, len(docs), batch_size)]

    def _clustered_batches(self, documents: List[str], batch_size: int) -> List[List[str]]:
        X = self._tfidf_matrix(documents)
        alive = torch.ones(len(documents), dtype=torch.bool)
        batches: List[List[str]] = []
        while bool(alive.any()):
            seed = random.choice(alive.nonzero().flatten().tolist())
            alive[seed] = False
            members = [seed]
            total = X[seed].clone()
            while len(members) < batch_size and bool(alive.any()):
                c = total / len(members)
                c = c / (c.norm() if c.norm() > 0 else 1.0)
                sims = torch.where(alive, X @ c, torch.full((len(documents),), -1.0, dtype=X.dtype))
                best = int(sims.argmax())
                if float(sims[best]) < self.similarity_threshold:
                    break
                alive[best] = False
                members.append(best)
                total += X[best]
            batches.append([documents[i] for i in members])
        return batches
