"""Heuristic text quality score in [0, 1] (``olympus/data/quality_filter.py:17-212``).

Five surface features, weighted (weights renormalised to sum to 1):

* ``avg_word_length`` (0.20): Gaussian around 5.5 characters, sigma 2.5;
* ``unique_word_ratio`` (0.25): type/token ratio, penalised below 0.1 and above 0.95;
* ``has_punctuation`` (0.15): sentence enders per 15 words (70 %) and commas per 20 words (30 %);
* ``line_length_variance`` (0.15): coefficient of variation of line lengths
  (single line 0.6, < 0.05 -> 0.4, > 2 -> 0.3, else 0.5 + 0.5 min(cv, 1));
* ``special_char_ratio`` (0.25): share of characters outside ASCII letters,
  digits, whitespace and punctuation (< 1 % -> 1, < 5 % -> 0.8, < 15 % -> 0.5).

Texts with fewer than ``min_words`` words score ``0.3 * words / min_words``.
The feature definitions and constants are the reference's, so scores (and
therefore filtered corpora) are identical.
"""

from __future__ import annotations

import math
import string
from typing import Dict, List, Optional

_ALLOWED = frozenset(string.ascii_letters + string.digits + string.whitespace + string.punctuation)


def _gauss_word_length(words: List[str]) -> float:
    if not words:
        return 0.0
    mean = sum(map(len, words)) / len(words)
    return math.exp(-0.5 * ((mean - 5.5) / 2.5) ** 2)


def _type_token(words: List[str]) -> float:
    if not words:
        return 0.0
    r = len({w.lower() for w in words}) / len(words)
    if r < 0.1:
        return r / 0.1 * 0.3
    if r > 0.95:
        return max(0.5, 1.0 - (r - 0.95) / 0.05)
    return min(1.0, r / 0.6)


def _punctuation(text: str) -> float:
    n = len(text.split())
    if n == 0:
        return 0.0
    enders = sum(text.count(c) for c in ".!?")
    return 0.7 * min(1.0, enders / max(1, n / 15)) + 0.3 * min(1.0, text.count(",") / max(1, n / 20))


def _line_spread(text: str) -> float:
    lines = text.split("\n")
    if len(lines) < 2:
        return 0.6
    lens = [len(l) for l in lines if l.strip()]
    if not lens:
        return 0.0
    mean = sum(lens) / len(lens)
    if mean == 0:
        return 0.0
    cv = math.sqrt(sum((x - mean) ** 2 for x in lens) / len(lens)) / (mean + 1e-8)
    if cv < 0.05:
        return 0.4
    if cv > 2.0:
        return 0.3
    return min(1.0, 0.5 + 0.5 * min(cv, 1.0))


def _special(text: str) -> float:
    if not text:
        return 0.0
    r = sum(1 for c in text if c not in _ALLOWED) / len(text)
    if r < 0.01:
        return 1.0
    if r < 0.05:
        return 0.8
    if r < 0.15:
        return 0.5
    return max(0.0, 1.0 - r)


class QualityFilter:
    DEFAULT_WEIGHTS: Dict[str, float] = {
        "avg_word_length": 0.20,
        "unique_word_ratio": 0.25,
        "has_punctuation": 0.15,
        "line_length_variance": 0.15,
        "special_char_ratio": 0.25,
    }

    def __init__(self, min_words: int = 10, weights: Optional[Dict[str, float]] = None) -> None:
        self.min_words = min_words
        w = dict(weights or self.DEFAULT_WEIGHTS)
        tot = sum(w.values())
        self.weights = {k: v / tot for k, v in w.items()} if tot > 0 else w

    _score_avg_word_length = staticmethod(_gauss_word_length)
    _score_unique_word_ratio = staticmethod(_type_token)
    _score_has_punctuation = staticmethod(_punctuation)
    _score_line_length_variance = staticmethod(_line_spread)
    _score_special_char_ratio = staticmethod(_special)

    def _features(self, text: str, words: List[str]) -> Dict[str, float]:
        return {
            "avg_word_length": _gauss_word_length(words),
            "unique_word_ratio": _type_token(words),
            "has_punctuation": _punctuation(text),
            "line_length_variance": _line_spread(text),
            "special_char_ratio": _special(text),
        }

    def score(self, text: str) -> float:
        words = text.split()
        if len(words) < self.min_words:
            return max(0.0, len(words) / self.min_words * 0.3)
        feats = self._features(text, words)
        return max(0.0, min(1.0, sum(w * feats.get(k, 0.0) for k, w in self.weights.items())))

    def score_detailed(self, text: str) -> Dict[str, float]:
        feats = self._features(text, text.split())
        feats["total"] = max(0.0, min(1.0, sum(self.weights.get(k, 0.0) * v for k, v in feats.items())))
        return feats

    def filter(self, texts: List[str], threshold: float = 0.7) -> List[str]:
        return [t for t in texts if self.score(t) >= threshold]

    def filter_with_scores(self, texts: List[str], threshold: float = 0.7):
        out = []
        for t in texts:
            s = self.score(t)
            if s >= threshold:
                out.append((t, s))
        return out
