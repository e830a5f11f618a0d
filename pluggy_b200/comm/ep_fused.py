"""Expert-parallel token dispatch and combine over NVLink peer memory.

Replaces the two uneven all-to-alls of :class:`pluggy_b200.parallel.expert_parallel.EPExperts`
with this package's kernels (``csrc/comm.cu``):

* the per-expert pair counts of every rank are pushed into every peer's count table
  (one small peer store per rank) and read back after a bounded flag handshake, so
  every rank knows the whole count matrix and derives all offsets from it;
* dispatch: each rank stores its routed rows (ordered by destination rank, then
  expert) straight into the owning rank's receive buffer at the row offset where
  that source's block begins, then a finishing kernel signals, waits for every
  peer and copies the received rows out (source-major, expert-ordered in each
  source block);
* combine: the expert outputs go back the same way into each source's buffer at
  the source's own row positions.

A dispatch's backward is a combine-direction exchange and vice versa. Buffers are
double-buffered by call parity per direction (the same argument as the tensor-parallel
buffers: a rank reaches call e + 2 of a direction only after every peer signalled
call e + 1, which each does after finishing with call e's buffer) and grow on demand
to the largest block any rank needs (every rank computes that size from the same
count matrix, so the regrowth is a collective step taken by all ranks together).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from pluggy_b200.comm.symm import SymmetricBuffer
from pluggy_b200.ops._ext import ext, status_word

_COUNTS, _TO_OWNERS, _TO_SOURCES = 0, 1, 2
_FLAG_BYTES = 4 * 8 * 4


class EPComm:
    def __init__(self, mesh, dim: str, num_experts: int, hidden: int, capacity_rows: int = 8192):
        self.mesh, self.dim = mesh, dim
        self.n, self.rank = mesh.size(dim), mesh.coordinate(dim)
        self.E, self.H = num_experts, hidden
        self.el = num_experts // self.n
        self.flags = SymmetricBuffer(_FLAG_BYTES, mesh, dim)
        # counts: n rows of E int32 (padded to 16-byte rows), double-buffered
        self.cw = (num_experts * 4 + 15) // 16 * 16 // 2  # row width in 2-byte units
        self.counts = SymmetricBuffer(2 * self.n * self.cw * 2, mesh, dim)
        self.rows = {_TO_OWNERS: 0, _TO_SOURCES: 0}
        self.buf = {_TO_OWNERS: None, _TO_SOURCES: None}
        self.epoch = {_COUNTS: 0, _TO_OWNERS: 0, _TO_SOURCES: 0}
        for k in (_TO_OWNERS, _TO_SOURCES):
            self._grow(k, capacity_rows)

    def _grow(self, kind: int, rows: int) -> None:
        if rows <= self.rows[kind]:
            return
        rows = int(rows * 1.25) + 64
        if self.buf[kind] is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.mesh.get_group(self.dim))
            self.buf[kind].close()
        self.buf[kind] = SymmetricBuffer(2 * rows * self.H * 2, self.mesh, self.dim)
        self.rows[kind] = rows

    def _next(self, kind: int):
        self.epoch[kind] += 1
        return self.epoch[kind]

    def exchange_counts(self, cnt: torch.Tensor) -> np.ndarray:
        """``cnt`` (int32 [E], this rank's pairs per expert) -> the [n, E] matrix on the host."""
        e = self._next(_COUNTS)
        half = self.n * self.cw * 2
        bufs = [p + (e % 2) * half for p in self.counts.peers]
        row = torch.zeros(1, self.cw, dtype=torch.int16, device=cnt.device)
        row.view(torch.int32)[0, :self.E] = cnt.to(torch.int32)
        n = self.n
        st = status_word(cnt.device)
        ext().ep_exchange("push", row, self.flags.peers, bufs, self.rank, e, _COUNTS,
                          [0] * n, [1] * n, [self.rank] * n, 0, half, st)
        out = torch.empty(n, self.cw, dtype=torch.int16, device=cnt.device)
        ext().ep_exchange("finish", out, self.flags.peers, bufs, self.rank, e, _COUNTS,
                          [0] * n, [0] * n, [0] * n, n, half, st)
        return out.view(torch.int32)[:, :self.E].cpu().numpy().astype(np.int64)

    def plan(self, C: np.ndarray) -> dict:
        """Row offsets of both directions from the count matrix ``C[src, expert]``."""
        n, el, me = self.n, self.el, self.rank
        rows = C.reshape(n, n, el).sum(-1)           # rows[s, d]: pairs s sends to d
        start = np.concatenate([np.zeros((n, 1), np.int64), np.cumsum(rows, 1)[:, :-1]], 1)
        recv_off = np.concatenate([[0], np.cumsum(rows[:, me])[:-1]])  # source blocks here
        dst_in_owner = np.concatenate([np.zeros((1, n), np.int64), np.cumsum(rows, 0)[:-1]], 0)
        return {
            "send": rows[me].tolist(), "start": start[me].tolist(),
            "to_owner_off": dst_in_owner[me].tolist(),       # my block inside each owner
            "recv": rows[:, me].tolist(), "recv_off": recv_off.tolist(),
            "back_off": start[:, me].tolist(),                 # my rows inside each source
            "R": int(rows[:, me].sum()), "P": int(rows[me].sum()),
            "R_max": int(rows.sum(0).max()), "P_max": int(rows.sum(1).max()),
            "local_counts": C[:, me * el:(me + 1) * el],     # [src, local expert]
        }

    def _exchange(self, kind, x, src_start, count, dst_off, out_rows):
        need = max(self._plan_max, 1)
        self._grow(kind, need)
        e = self._next(kind)
        half = self.rows[kind] * self.H * 2
        bufs = [p + (e % 2) * half for p in self.buf[kind].peers]
        x2 = x.reshape(-1, self.H).to(torch.bfloat16).contiguous()
        out = torch.empty(out_rows, self.H, dtype=torch.bfloat16, device=x.device)
        st = status_word(x.device)
        if x2.shape[0] == 0:
            x2 = torch.zeros(1, self.H, dtype=torch.bfloat16, device=x.device)
        ext().ep_exchange("push", x2, self.flags.peers, bufs, self.rank, e, kind, src_start, count,
                          dst_off, 0, half, st)
        o = out if out_rows > 0 else torch.empty(1, self.H, dtype=torch.bfloat16, device=x.device)
        ext().ep_exchange("finish", o, self.flags.peers, bufs, self.rank, e, kind, [0] * self.n,
                          [0] * self.n, [0] * self.n, out_rows, half, st)
        return out

    def to_owners(self, x_sorted: torch.Tensor, pl: dict) -> torch.Tensor:
        """[P, H] rows in destination order -> the [R, H] rows this rank's experts receive."""
        self._plan_max = max(pl["R_max"], pl["P_max"])
        return self._exchange(_TO_OWNERS, x_sorted, pl["start"], pl["send"], pl["to_owner_off"], pl["R"])

    def to_sources(self, y: torch.Tensor, pl: dict) -> torch.Tensor:
        """[R, H] rows received by this rank -> back to their sources: [P, H] in this
        rank's own destination order."""
        self._plan_max = max(pl["R_max"], pl["P_max"])
        return self._exchange(_TO_SOURCES, y, pl["recv_off"], pl["recv"], pl["back_off"], pl["P"])

    def close(self) -> None:
        for b in (self.buf[_TO_OWNERS], self.buf[_TO_SOURCES], self.counts, self.flags):
            if b is not None:
                b.close()


class ToOwners(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm, pl):
        ctx.comm, ctx.pl, ctx.dtype = comm, pl, x.dtype
        return comm.to_owners(x, pl).to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        return ctx.comm.to_sources(g.contiguous(), ctx.pl).to(ctx.dtype), None, None


class ToSources(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, comm, pl):
        ctx.comm, ctx.pl, ctx.dtype = comm, pl, y.dtype
        return comm.to_sources(y, pl).to(y.dtype)

    @staticmethod
    def backward(ctx, g):
        return ctx.comm.to_owners(g.contiguous(), ctx.pl).to(ctx.dtype), None, None
