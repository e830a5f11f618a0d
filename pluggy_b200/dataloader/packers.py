"""Sequence packers for the dataloader's ``.map`` step.

Parity: reference ``pluggy/dataloader/packers.py:36-255``. The algorithm and its
output must be identical (the reference's packing test compares blocks), so the
steps are the same while the code is this package's own:

* stream packers (``ListPacker``, ``NumpyPacker``, ``TensorPacker``): append
  EOS after every document, concatenate, cut into back-to-back ``seq_len`` rows
  and drop the tail of each map-batch; the three give identical blocks;
* ``ListPackerBestFit``: best-fit-decreasing bin packing (Ding et al. 2024,
  arXiv:2404.10830); long documents are cut into full rows and their remainder
  (plus EOS) is packed with the short documents; open bins are found with a max
  segment tree over free space; unfilled bins are padded with ``pad_id``.

Packers are top-level classes so DataLoader workers can pickle them.
"""

from __future__ import annotations

import numpy as np
import torch

from pluggy_b200.utils import Node


class Packer:
    def __init__(self, tokenizer, seq_len: int, eos_id: int, pad_id: int | None = None,
                 verbose: bool = False):
        self.tokenizer = tokenizer
        self.seq_len = seq_len
        self.eos_id = eos_id
        self.pad_id = eos_id if pad_id is None else pad_id
        self.verbose = verbose

    def __call__(self, examples: dict[str, list]) -> dict[str, list]:
        docs = [enc.ids for enc in self.tokenizer.encode_batch(examples["text"])]
        return {"input_ids": self.pack(docs)}

    def pack(self, docs: list[list[int]]) -> list[list[int]]:
        raise NotImplementedError

    def pack_to_tensor(self, docs: list[list[int]]) -> torch.Tensor:
        rows = self.pack(docs)
        if not rows:
            return torch.empty((0, self.seq_len), dtype=torch.long)
        return torch.tensor(rows, dtype=torch.long)

    def _report(self, n_tokens: int, n_rows: int) -> None:
        if self.verbose:
            print(f"{type(self).__name__}: lost {n_tokens - n_rows * self.seq_len} tokens")


class ListPacker(Packer):
    def pack(self, docs):
        stream: list[int] = []
        for ids in docs:
            stream += ids
            stream.append(self.eos_id)
        n = len(stream) // self.seq_len
        self._report(len(stream), n)
        L = self.seq_len
        return [stream[i * L:(i + 1) * L] for i in range(n)]


class NumpyPacker(Packer):
    def _rows(self, docs) -> np.ndarray:
        if not docs:
            return np.empty((0, self.seq_len), dtype=np.int64)
        lens = np.fromiter((len(d) + 1 for d in docs), dtype=np.int64, count=len(docs))
        stream = np.empty(int(lens.sum()), dtype=np.int64)
        ends = np.cumsum(lens)
        starts = ends - lens
        for d, s, e in zip(docs, starts, ends):
            stream[s:e - 1] = d
            stream[e - 1] = self.eos_id
        n = stream.shape[0] // self.seq_len
        self._report(stream.shape[0], n)
        return stream[: n * self.seq_len].reshape(n, self.seq_len)

    def pack(self, docs):
        return self._rows(docs).tolist()

    def pack_to_tensor(self, docs):
        return torch.from_numpy(self._rows(docs))


class TensorPacker(Packer):
    def _rows(self, docs) -> torch.Tensor:
        if not docs:
            return torch.empty((0, self.seq_len), dtype=torch.long)
        eos = torch.tensor([self.eos_id], dtype=torch.long)
        parts = []
        for d in docs:
            parts.append(torch.as_tensor(d, dtype=torch.long))
            parts.append(eos)
        stream = torch.cat(parts)
        n = stream.shape[0] // self.seq_len
        self._report(stream.shape[0], n)
        return stream[: n * self.seq_len].view(n, self.seq_len)

    def pack(self, docs):
        return self._rows(docs).tolist()

    def pack_to_tensor(self, docs):
        return self._rows(docs)


class ListPackerBestFit(Packer):
    def pack(self, docs):
        L = self.seq_len
        full_rows: list[list[int]] = []
        items: list[list[int]] = []
        for ids in docs:
            k = len(ids) // L
            full_rows.extend(ids[i * L:(i + 1) * L] for i in range(k))
            items.append(ids[k * L:] + [self.eos_id])
        items.sort(key=len, reverse=True)
        tree = Node.build(0, L)
        bins_with_space: dict[int, list[int]] = {}
        bins: list[list[int]] = []
        for item in items:
            size = len(item)
            space = tree.search(size)
            if space is None:
                b = len(bins)
                bins.append([])
                space = L
            else:
                b = bins_with_space[space].pop()
                if not bins_with_space[space]:
                    tree.update(space, available=False)
            bins[b].extend(item)
            left = space - size
            if left > 0:
                bucket = bins_with_space.setdefault(left, [])
                if not bucket:
                    tree.update(left, available=True)
                bucket.append(b)
        for b in bins:
            if len(b) < L:
                b.extend([self.pad_id] * (L - len(b)))
        return full_rows + bins


PACKERS: dict[str, type[Packer]] = {"list": ListPacker, "numpy": NumpyPacker, "tensor": TensorPacker}
BESTFIT_PACKERS: dict[str, type[Packer]] = {"bestfit": ListPackerBestFit}
