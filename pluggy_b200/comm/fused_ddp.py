"""Fused data-parallel gradient reduction over NVLink peer memory.

``DDP(..., reducer="fused")`` hands its buckets to :class:`BucketReducer`: every
bucket's flat gradient buffer is a slice of one symmetric buffer, and each launch
is a single sm_100a kernel (``csrc/comm.cu``) that averages the bucket across the
axis with direct peer loads and stores and, on the way, accumulates the sum of
squares of the averaged gradients, so the optimizer step needs no separate
grad-norm pass. Launches run on a side stream, overlapping the rest of backward
like the NCCL path.
"""

from __future__ import annotations

import os

import torch

from pluggy_b200.comm.symm import SymmetricBuffer
from pluggy_b200.ops._ext import ext, status_word

_ALIGN = 64  # elements: keeps every bucket 256-byte aligned (float4 paths need 16 bytes)
_FLAG_BYTES = 2 * 8 * 128 * 4
_SLOT_BYTES = 8 * 128 * 4


class _Work:
    def __init__(self, event: torch.cuda.Event):
        self.event = event

    def wait(self) -> None:
        torch.cuda.current_stream().wait_event(self.event)


class BucketReducer:
    def __init__(self, mesh, dim: str, buckets, chunks: int | None = None):
        self.mesh, self.dim = mesh, dim
        self.n, self.rank = mesh.size(dim), mesh.coordinate(dim)
        offs, total = [], 0
        for b in buckets:
            offs.append(total)
            numel = sum(p.numel() for p in b.params)
            total += (numel + _ALIGN - 1) // _ALIGN * _ALIGN
        self.data = SymmetricBuffer(max(total, 1) * 4, mesh, dim)
        self.flags = SymmetricBuffer(_FLAG_BYTES, mesh, dim)
        self.slots = SymmetricBuffer(_SLOT_BYTES, mesh, dim)
        self.offset = {}
        for b, off in zip(buckets, offs, strict=True):
            numel = sum(p.numel() for p in b.params)
            flat = self.data.tensor(off * 4, [numel])
            b.flat = flat
            b.views, o = [], 0
            for p in b.params:
                b.views.append(flat[o:o + p.numel()].view_as(p))
                o += p.numel()
            self.offset[b.index] = (off, numel)
        # 128 CTAs per bucket: measured best from 8 MB up on B200 (the buckets are 25 MB);
        # PLG_COMM_CTAS overrides it for measurements
        self.chunks = chunks or int(os.environ.get("PLG_COMM_CTAS", "128"))
        self.epoch = 0
        self.norm_sq = torch.zeros(1, dtype=torch.float32, device=self.data.device)
        self._first = True
        # high priority: at each kernel boundary the block scheduler places the
        # reduction's CTAs before pending compute CTAs
        self.stream = torch.cuda.Stream(priority=-1)

    def launch(self, b):
        off, numel = self.offset[b.index]
        if len(b.params) == 1 and b.params[0].grad is not b.views[0]:
            # single-param bucket: its grad moves into the symmetric buffer
            b.views[0].copy_(b.params[0].grad)
            b.params[0].grad = b.views[0]
        ready = torch.cuda.Event()
        ready.record()
        self.stream.wait_event(ready)
        self.epoch += 1
        with torch.cuda.stream(self.stream):
            ext().symm_allreduce_avg(self.data.peers, self.flags.peers, self.slots.peers, off, numel,
                                     self.rank, self.epoch, self.chunks, self.norm_sq,
                                     not self._first, status_word(b.flat.device))
        self._first = False
        done = torch.cuda.Event()
        done.record(self.stream)
        return _Work(done)

    def finish(self) -> None:
        """End of a step: the next launch starts a new grad-norm sum."""
        self._first = True

    def reduced_norm_sq(self) -> torch.Tensor:
        """Sum of squares of every averaged gradient of the last step (device scalar)."""
        return self.norm_sq[0]

    def close(self) -> None:
        for buf in (self.data, self.flags, self.slots):
            buf.close()
