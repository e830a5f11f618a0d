"""Host-to-device batch prefetcher with exact-resume state snapshots.

Parity: reference ``pluggy/dataloader/prefetcher.py:22-92``. The copy of batch
N+1 is issued on a side stream while batch N computes; the consumer's stream
waits on it and ``record_stream``s the tensors. The loader's ``state_dict`` is
snapshotted BEFORE each pull, so ``loader_state_dict()`` describes exactly the
batches the caller has consumed (saving the live state would skip the
prefetched batch on resume). On a CPU device the copy is synchronous.

Addition: values that are the same host tensor object (``labels is
input_ids``) are copied once and shared on the device; ``h2d_bytes`` counts
what was actually copied for the last batch. ``background=True`` pulls batches
from the loader on a worker thread (up to ``depth`` ahead, each with the state
snapshot taken right before its pull), so host-side batch generation overlaps the
device work instead of running at the step boundary.
"""

from __future__ import annotations

import queue
import threading

import torch


class CUDAPrefetcher:
    def __init__(self, loader, device: torch.device, background: bool = False, depth: int = 2):
        self.loader = loader
        self.loader_iter = iter(loader)
        self.device = torch.device(device)
        self.stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self.next_batch = None
        self._loader_state = None
        self.h2d_bytes = 0
        self._queue = None
        if background:
            self._queue = queue.Queue(maxsize=max(1, depth))
            threading.Thread(target=self._produce, name="prefetch", daemon=True).start()
        self._preload()

    def _produce(self) -> None:
        # the only user of the loader once started: snapshot, pull, hand over
        while True:
            state = self.loader.state_dict()
            try:
                batch = next(self.loader_iter)
            except StopIteration:
                self._queue.put((state, None))
                return
            except BaseException as e:  # surfaced to the consumer
                self._queue.put((state, e))
                return
            self._queue.put((state, batch))

    def _pull(self):
        if self._queue is None:
            state = self.loader.state_dict()
            try:
                return state, next(self.loader_iter)
            except StopIteration:
                return state, None
        state, batch = self._queue.get()
        if isinstance(batch, BaseException):
            raise batch
        if batch is None:
            self._queue.put((state, None))  # stays exhausted for later pulls
        return state, batch

    def loader_state_dict(self) -> dict:
        return self._loader_state

    def _copy(self, batch: dict) -> dict:
        seen: dict[int, torch.Tensor] = {}
        out = {}
        nbytes = 0
        for k, v in batch.items():
            if id(v) in seen:
                out[k] = seen[id(v)]
                continue
            d = v.to(self.device, non_blocking=self.stream is not None)
            nbytes += v.numel() * v.element_size()
            seen[id(v)] = d
            out[k] = d
        self.h2d_bytes = nbytes
        return out

    def _preload(self) -> None:
        self._loader_state, batch = self._pull()
        if batch is None:
            self.next_batch = None
            return
        if self.stream is None:
            self.next_batch = self._copy(batch)
            return
        with torch.cuda.stream(self.stream):
            self.next_batch = self._copy(batch)

    def __iter__(self):
        return self

    def __next__(self) -> dict:
        if self.next_batch is None:
            raise StopIteration
        batch = self.next_batch
        if self.stream is not None:
            cur = torch.cuda.current_stream(self.device)
            cur.wait_stream(self.stream)
            for v in {id(t): t for t in batch.values()}.values():
                v.record_stream(cur)
        self._preload()
        return batch
