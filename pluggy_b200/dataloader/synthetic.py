"""Synthetic packed token source: Zipf-distributed ids with EOS separators.

The benchmark configs ask for "packed sequences of Zipf(s=1.1)-distributed token
ids over the vocab, with EOS separators placed every U[512,4096] tokens". This
source produces exactly that, deterministically and resumably:

* row ``i`` of dp shard ``r`` is generated from a Philox-style counter RNG keyed
  on ``(seed, r, i)``, so any row can be regenerated from its index alone;
* ``state_dict()`` is just the next row index, so a ``StatefulDataLoader`` over
  it resumes exactly (the same invariant the reference's HF stream provides);
* token ids: rank ``k`` (1-based) has probability ``k^-s / H(V, s)``; rank ``k``
  maps to id ``k - 1``, except that the EOS id is never sampled as content;
* document boundaries: the gap between two EOS tokens is drawn from
  ``U[min_doc, max_doc]``; a document may continue across rows (packed stream).

``kind="uniform"`` draws ids uniformly from ``[0, vocab_size)`` with no EOS (the
CPU/gloo plumbing config).
"""

from __future__ import annotations

import numpy as np
import torch
from torch.utils.data import IterableDataset


class ZipfTable:
    """Inverse-CDF sampler for a bounded Zipf law over ``vocab_size`` ranks."""

    def __init__(self, vocab_size: int, s: float = 1.1):
        ranks = np.arange(1, vocab_size + 1, dtype=np.float64)
        p = ranks ** (-s)
        self.cdf = np.cumsum(p / p.sum())
        self.cdf[-1] = 1.0

    def sample(self, rng: np.random.Generator, n: int) -> np.ndarray:
        return np.searchsorted(self.cdf, rng.random(n), side="right").astype(np.int64)


class SyntheticZipfRows(IterableDataset):
    """Infinite stream of ``{"input_ids": [seq_len]}`` rows for one dp shard."""

    def __init__(self, vocab_size: int, seq_len: int, eos_id: int | None = None, seed: int = 0,
                 dp_rank: int = 0, zipf_s: float = 1.1, min_doc: int = 512, max_doc: int = 4096,
                 kind: str = "zipf"):
        if kind not in ("zipf", "uniform"):
            raise ValueError(f"synthetic kind must be 'zipf' or 'uniform', got {kind!r}")
        self.kind = kind
        self.vocab_size = vocab_size
        self.seq_len = seq_len
        self.eos_id = vocab_size - 1 if eos_id is None else eos_id
        self.seed = seed
        self.dp_rank = dp_rank
        self.zipf_s = zipf_s
        self.min_doc, self.max_doc = min_doc, max_doc
        self._table = None
        self._next = 0

    def _rng(self, row: int) -> np.random.Generator:
        return np.random.Generator(np.random.Philox(key=[self.seed, (self.dp_rank << 40) | row]))

    def row(self, i: int) -> np.ndarray:
        if self.kind == "uniform":  # ids uniform over the vocab, no document structure
            return self._rng(i).integers(0, self.vocab_size, self.seq_len, dtype=np.int64)
        if self._table is None:
            self._table = ZipfTable(self.vocab_size, self.zipf_s)
        rng = self._rng(i)
        ids = self._table.sample(rng, self.seq_len)
        ids[ids == self.eos_id] = 0
        # EOS positions: a random phase into the current document, then U[min,max] gaps
        pos = int(rng.integers(0, self.max_doc))
        while True:
            pos += int(rng.integers(self.min_doc, self.max_doc + 1))
            if pos >= self.seq_len + self.max_doc:
                break
            p = pos - self.max_doc
            if 0 <= p < self.seq_len:
                ids[p] = self.eos_id
        return ids

    def __iter__(self):
        info = torch.utils.data.get_worker_info()
        wid, nw = (0, 1) if info is None else (info.id, info.num_workers)
        i = self._next
        while True:
            if i % nw == wid:
                yield {"input_ids": self.row(i)}
            i += 1
            if info is None:
                self._next = i

    def state_dict(self) -> dict:
        return {"next_row": self._next}

    def load_state_dict(self, state: dict) -> None:
        self._next = int(state["next_row"])


class RowCollator:
    """Stack rows into ``{"input_ids", "labels"}`` (labels = ids; shifting is the objective's)."""

    def __call__(self, rows):
        ids = torch.as_tensor(np.stack([r["input_ids"] for r in rows]), dtype=torch.long)
        return {"input_ids": ids, "labels": ids.clone()}


class SyntheticBatches:
    """Resumable iterator of ready batches built directly from a Zipf source.

    Cheaper than a DataLoader for benchmarks (no worker processes) while keeping
    the ``state_dict``/``load_state_dict`` contract the prefetcher and
    checkpointer rely on. ``pin=True`` places batches in pinned host memory so
    the host-to-device copy is asynchronous.
    """

    def __init__(self, source: SyntheticZipfRows, micro_batch: int, pin: bool = False):
        self.source = source
        self.micro_batch = micro_batch
        self.pin = pin and torch.cuda.is_available()
        self._batch = 0

    def __iter__(self):
        return self

    def __next__(self):
        b = self._batch
        rows = [self.source.row(b * self.micro_batch + j) for j in range(self.micro_batch)]
        ids = torch.from_numpy(np.stack(rows))
        if self.pin:
            ids = ids.pin_memory()
        self._batch += 1
        return {"input_ids": ids, "labels": ids}

    def state_dict(self) -> dict:
        return {"batch": self._batch}

    def load_state_dict(self, state: dict) -> None:
        self._batch = int(state["batch"])
