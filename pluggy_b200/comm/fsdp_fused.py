"""FSDP parameter all-gather over NVLink peer memory.

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
