"""DTensor: a local tensor plus its placements over mesh axes (bookkeeping only).

Parity: reference ``pluggy/core/dtensor.py:42-180``. No ``__torch_dispatch__``:
you compute on ``to_local()`` and change layouts explicitly. Redistribution
table (one axis at a time):

==========================  =====================================
from -> to                  collective
==========================  =====================================
Shard(d) -> Replicate        all_gather along d
Replicate -> Shard(d)        local slice, no communication
Partial -> Replicate         all_reduce (on a clone: self stays valid)
Partial -> Shard(d)          reduce_scatter along d
Shard(i) -> Shard(j)         all_to_all (split j, concat i)
==========================  =====================================

Anything -> Partial has no producer and raises. Even shards only; two axes may
not shard the same tensor dim.
"""

from __future__ import annotations

import torch

from pluggy_b200.core.collective import MeshLike, all_gather, all_reduce, all_to_all, reduce_scatter
from pluggy_b200.core.placement import Partial, Placement, Replicate, Shard


def _local_slice(t: torch.Tensor, mesh: MeshLike, axis: str, dim: int) -> torch.Tensor:
    n = mesh.size(axis)
    assert t.shape[dim] % n == 0, (
        f"shape[{dim}]={t.shape[dim]} not divisible by axis {axis!r} of size {n} (even shards only)"
    )
    step = t.shape[dim] // n
    return t.narrow(dim, mesh.coordinate(axis) * step, step)


class DTensor:
    def __init__(self, local: torch.Tensor, mesh: MeshLike, placements: dict[str, Placement]):
        self.local = local
        self.mesh = mesh
        # canonical form: Replicate entries are implicit
        self.placements = {a: p for a, p in placements.items() if not isinstance(p, Replicate)}

    @staticmethod
    def _validate(ndim: int, mesh: MeshLike, placements: dict[str, Placement]) -> None:
        dims = []
        for axis, p in placements.items():
            mesh.size(axis)  # KeyError on unknown axis
            if isinstance(p, Shard):
                assert 0 <= p.dim < ndim, f"Shard({p.dim}) out of range for ndim={ndim}"
                dims.append(p.dim)
        assert len(dims) == len(set(dims)), f"two mesh axes shard the same dim ({dims})"

    @classmethod
    def from_local(cls, local, mesh, placements):
        cls._validate(local.ndim, mesh, placements)
        return cls(local, mesh, placements)

    @classmethod
    def from_full(cls, full, mesh, placements):
        cls._validate(full.ndim, mesh, placements)
        local = full
        for axis, p in placements.items():
            if isinstance(p, Replicate):
                continue
            assert isinstance(p, Shard), f"from_full takes Shard/Replicate only, got {axis}: {p}"
            local = _local_slice(local, mesh, axis, p.dim)
        return cls(local.contiguous().clone(), mesh, placements)

    def to_local(self) -> torch.Tensor:
        return self.local

    @property
    def global_shape(self) -> tuple[int, ...]:
        shape = list(self.local.shape)
        for axis, p in self.placements.items():
            if isinstance(p, Shard):
                shape[p.dim] *= self.mesh.size(axis)
        return tuple(shape)

    def placement(self, axis: str) -> Placement:
        return self.placements.get(axis, Replicate())

    def redistribute(self, axis: str, to: Placement) -> "DTensor":
        src = self.placement(axis)
        if src == to:
            return self
        if isinstance(src, Shard) and isinstance(to, Replicate):
            new = all_gather(self.local, self.mesh, axis, gather_dim=src.dim)
        elif isinstance(src, Replicate) and isinstance(to, Shard):
            new = _local_slice(self.local, self.mesh, axis, to.dim).contiguous().clone()
        elif isinstance(src, Partial) and isinstance(to, Replicate):
            new = all_reduce(self.local.clone(), self.mesh, axis, src.op)
        elif isinstance(src, Partial) and isinstance(to, Shard):
            new = reduce_scatter(self.local, self.mesh, axis, src.op, scatter_dim=to.dim)
        elif isinstance(src, Shard) and isinstance(to, Shard):
            new = all_to_all(self.local, self.mesh, axis, split_dim=to.dim, concat_dim=src.dim)
        else:
            raise AssertionError(f"unsupported redistribute {src} -> {to} on axis {axis!r}")
        pl = dict(self.placements)
        pl[axis] = to
        return DTensor(new, self.mesh, pl)

    def full_tensor(self) -> torch.Tensor:
        out = self
        for axis, p in list(out.placements.items()):
            if isinstance(p, Partial):
                out = out.redistribute(axis, Replicate())
        for axis, p in list(out.placements.items()):
            if isinstance(p, Shard):
                out = out.redistribute(axis, Replicate())
        return out.local

    def __repr__(self) -> str:
        pl = ", ".join(f"{a}: {p}" for a, p in self.placements.items()) or "Replicate()"
        return f"DTensor(local_shape={tuple(self.local.shape)}, global_shape={self.global_shape}, {pl})"
