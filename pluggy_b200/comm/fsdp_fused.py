"""FSDP parameter all-gather over NVLink peer memory.

Two forms:

* :class:`PeerGather` (fp32): the unit's full fp32 parameters, for models that
  read their parameters directly;
* :class:`SlotGather` (low precision): for the fused-engine models, whose GEMMs
  read bf16 weights. Each rank casts its fp32 shards to bf16 while pushing them
  (half the NVLink bytes) straight into the consumer's buffer, a slot of
  symmetric memory that the GEMMs read in place (no finishing copy, no separate
  cast, no full-size fp32 copy of the unit); 1-D parameters (norm weights) travel
  as fp32. Two slots, alternating by block index, hold the unit being computed
  and the one being prefetched.

A unit's full parameters are one flat buffer (parameter i at ``full_off_i``, its
dim-0 shard of rank r at ``full_off_i + r * shard_len_i``). :meth:`PeerGather.gather`
launches one push kernel (``csrc/comm.cu``: every rank stores each of its parameter
shards into every rank's staging buffer, destinations in rank-rotated order) and one
finishing kernel (flag handshake with bounded waits, then a copy of the staging
buffer into the unit's full storage). Staging is double-buffered by call parity: a
rank can push call e + 2 only after every peer signalled call e + 1, which each does
after copying out call e.
"""

from __future__ import annotations

import torch

from pluggy_b200.comm.symm import SymmetricBuffer
from pluggy_b200.ops._ext import ext, status_word

_KIND = 0
_FLAG_BYTES = 4 * 8 * 4


class PeerGather:
    def __init__(self, mesh, dim: str, max_unit_bytes: int):
        self.mesh, self.dim = mesh, dim
        self.n, self.rank = mesh.size(dim), mesh.coordinate(dim)
        self.half = (int(max_unit_bytes) + 4095) // 4096 * 4096
        self.flags = SymmetricBuffer(_FLAG_BYTES, mesh, dim)
        self.buf = SymmetricBuffer(2 * self.half, mesh, dim)
        self.epoch = 0

    def _table(self, unit) -> torch.Tensor:
        if unit.peer_table is None:
            rows, so, fo = [], 0, 0
            for s in unit.params:
                itemsize = s.param.element_size()
                rows.append([so * itemsize // 16, fo * itemsize // 16, s.shard_numel * itemsize // 16])
                so += s.shard_numel
                fo += s.full_numel
            unit.peer_table = torch.tensor(rows, dtype=torch.int64, device=unit.flat_shard.device)
        return unit.peer_table

    def gather(self, unit) -> None:
        """Fill ``unit.full_flat`` (allocated) from every rank's ``unit.flat_shard``."""
        self.epoch += 1
        e = self.epoch
        bufs = [p + (e % 2) * self.half for p in self.buf.peers]
        st = status_word(unit.flat_shard.device)
        ext().fsdp_push(unit.flat_shard, self._table(unit), self.flags.peers, bufs, self.rank, e,
                        self.half, st)
        out = unit.full_flat.view(torch.int16).view(-1, 8)  # rows of 16 bytes
        n = self.n
        ext().ep_exchange("finish", out, self.flags.peers, bufs, self.rank, e, _KIND, [0] * n, [0] * n,
                          [0] * n, out.shape[0], self.half, st)

    def close(self) -> None:
        self.buf.close()
        self.flags.close()


def _align16(nbytes: int) -> int:
    return (nbytes + 15) // 16 * 16


class SlotLayout:
    """Where each parameter of a unit lives in its slot: matrices first (bf16, in
    block order, so q|k|v and gate|up stay contiguous), then vectors (fp32)."""

    def __init__(self, states, n: int):
        self.entries = []  # (state, kind, byte offset)
        off = 0
        mats = [s for s in states if len(s.full_shape) >= 2]
        vecs = [s for s in states if len(s.full_shape) < 2]
        for s in mats:
            self.entries.append((s, 0, off))
            off = _align16(off + 2 * s.full_numel)
        for s in vecs:
            self.entries.append((s, 1, off))
            off = _align16(off + 4 * s.full_numel)
        self.nbytes = off
        # every rank's shard must be whole 16-byte groups at 16-byte offsets
        self.ok = all((s.shard_numel * (2 if k == 0 else 4)) % 16 == 0 for s, k, _ in self.entries)

    def table(self, shard_order, device) -> tuple[torch.Tensor, int]:
        """The push kernel's rows; ``shard_order``: the states in the order of the
        unit's flat fp32 shard (the source offsets)."""
        rows, g, src = [], 0, 0
        src_off = {}
        for s in shard_order:
            src_off[id(s)] = src
            src += s.shard_numel
        for s, kind, off in self.entries:
            esize = 2 if kind == 0 else 4
            len16 = s.shard_numel * esize // 16
            rows.append([g, src_off[id(s)], off // 16, len16, kind])
            g += len16
        return torch.tensor(rows, dtype=torch.int64, device=device), g


class SlotGather:
    def __init__(self, mesh, dim: str, slot_bytes: int, nslots: int = 2):
        self.mesh, self.dim = mesh, dim
        self.n, self.rank = mesh.size(dim), mesh.coordinate(dim)
        self.slot = (int(slot_bytes) + 4095) // 4096 * 4096
        self.nslots = nslots
        self.flags = SymmetricBuffer(_FLAG_BYTES, mesh, dim)
        self.buf = SymmetricBuffer(nslots * self.slot, mesh, dim)
        self.epoch = 0

    def views(self, layout: SlotLayout, slot: int) -> dict:
        """id(param) -> the parameter's full tensor inside slot ``slot`` (bf16 or fp32)."""
        out = {}
        base = slot * self.slot
        for s, kind, off in layout.entries:
            dt = torch.bfloat16 if kind == 0 else torch.float32
            out[id(s.param)] = self.buf.tensor(base + off, list(s.full_shape), dt)
        return out

    def gather(self, unit, slot: int) -> None:
        """Fill slot ``slot`` of every rank from every rank's ``unit.flat_shard``."""
        self.epoch += 1
        e = self.epoch
        bufs = [p + slot * self.slot for p in self.buf.peers]
        st = status_word(unit.flat_shard.device)
        ext().fsdp_push_lowp(unit.flat_shard, unit.slot_table, unit.slot_groups, self.flags.peers, bufs,
                             self.rank, e, self.slot, st)
        n = self.n
        empty = torch.empty((0, 8), dtype=torch.int16, device=unit.flat_shard.device)
        # handshake only: the pushes already landed in place
        ext().ep_exchange("finish", empty, self.flags.peers, bufs, self.rank, e, _KIND, [0] * n,
                          [0] * n, [0] * n, 0, self.slot, st)

    def close(self) -> None:
        self.buf.close()
        self.flags.close()


_RS_FLAG_BYTES = 2 * 8 * 128 * 4


class PeerReduceScatter:
    """FSDP gradient reduce-scatter over peer memory (``csrc/comm.cu`` ``fsdp_rs_kernel``).

    Each rank copies a unit's full fp32 gradients into a staging slot of symmetric
    memory (two slots alternating by call); one kernel then sums this rank's shard of
    every parameter over all ranks' slots with peer loads, in rank order, scales by
    1/N and writes or accumulates it straight into the rank's flat fp32 grad-shard
    buffer: no NCCL output tensors, no separate accumulate pass."""

    def __init__(self, mesh, dim: str, max_unit_bytes: int, chunks: int = 128):
        self.mesh, self.dim = mesh, dim
        self.n, self.rank = mesh.size(dim), mesh.coordinate(dim)
        self.slot = (int(max_unit_bytes) + 4095) // 4096 * 4096
        self.flags = SymmetricBuffer(_RS_FLAG_BYTES, mesh, dim)
        self.buf = SymmetricBuffer(2 * self.slot, mesh, dim)
        self.chunks = chunks
        self.epoch = 0

    @staticmethod
    def plan(states, device):
        """(table, full offsets) for the states that take gradients, in unit order."""
        rows, so, fo, offs = [], 0, 0, []
        for s in states:
            rows.append([so, fo, s.shard_numel])
            offs.append(fo)
            so += s.shard_numel
            fo += s.full_numel
        return torch.tensor(rows, dtype=torch.int64, device=device), offs

    def reduce(self, unit, grads, accumulate: bool) -> None:
        self.epoch += 1
        e = self.epoch
        base = (e % 2) * self.slot
        views = [self.buf.tensor(base + 4 * off, [s.full_numel])
                 for s, off in zip(unit.rs_states, unit.rs_offsets, strict=True)]
        torch._foreach_copy_(views, [g.reshape(-1) for g in grads])
        ext().fsdp_rs([p + base for p in self.buf.peers], self.flags.peers, unit.rs_table, unit.grad_flat,
                      bool(accumulate), 1.0 / self.n, self.rank, e, self.chunks,
                      status_word(unit.grad_flat.device))

    def close(self) -> None:
        self.buf.close()
        self.flags.close()
