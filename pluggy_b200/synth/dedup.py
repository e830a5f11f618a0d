"""Near-duplicate filter: exact hash, MinHash candidates, exact Jaccard check.

Parity: reference ``pluggy/synth/dedup.py:42-67`` (word 13-gram shingles, Jaccard
threshold 0.8). Signatures here are a true MinHash: ``k`` universal hash functions
``(a x + b) mod p`` (p = 2^31 - 1) over 32-bit shingle fingerprints, computed with numpy in one
vectorised pass per document. A document whose signature shares any value with an
earlier one is compared by exact Jaccard of the shingle sets, so the index never
produces a false positive; with 8 hashes and threshold 0.8 the chance to miss a
true near-duplicate is below 0.2^8.
"""

from __future__ import annotations

import hashlib
import re

import numpy as np

_P = np.uint64((1 << 31) - 1)  # Mersenne prime modulus: a * x stays below 2^63
_WORD = re.compile(r"\w+")


def _fp(s: str) -> int:
    return int.from_bytes(hashlib.blake2b(s.encode(), digest_size=4).digest(), "little")


def shingles(text: str, n: int) -> set[int]:
    w = _WORD.findall(text.lower())
    if len(w) < n:
        return {_fp(" ".join(w))}
    return {_fp(" ".join(w[i:i + n])) for i in range(len(w) - n + 1)}


class Deduper:
    def __init__(self, ngram: int = 13, threshold: float = 0.8, num_hashes: int = 8, seed: int = 1):
        self.ngram, self.threshold = ngram, threshold
        rng = np.random.default_rng(seed)
        self.a = rng.integers(1, (1 << 31) - 1, size=num_hashes, dtype=np.uint64)
        self.b = rng.integers(0, (1 << 31) - 1, size=num_hashes, dtype=np.uint64)
        self.exact: set[bytes] = set()
        self.sets: list[set[int]] = []
        self.index: dict[tuple[int, int], list[int]] = {}

    def _signature(self, sh: set[int]) -> list[int]:
        x = np.fromiter(sh, dtype=np.uint64, count=len(sh))
        return [int(((a * x + b) % _P).min()) for a, b in zip(self.a, self.b)]

    def is_duplicate(self, text: str) -> bool:
        """Whether ``text`` near-duplicates a document seen before; records it if not."""
        key = hashlib.blake2b(" ".join(text.lower().split()).encode(), digest_size=16).digest()
        if key in self.exact:
            return True
        sh = shingles(text, self.ngram)
        sig = self._signature(sh)
        seen: set[int] = set()
        for i, v in enumerate(sig):
            for d in self.index.get((i, v), ()):
                if d in seen:
                    continue
                seen.add(d)
                other = self.sets[d]
                inter = len(sh & other)
                if inter / (len(sh) + len(other) - inter) >= self.threshold:
                    return True
        self.exact.add(key)
        d = len(self.sets)
        self.sets.append(sh)
        for i, v in enumerate(sig):
            self.index.setdefault((i, v), []).append(d)
        return False
