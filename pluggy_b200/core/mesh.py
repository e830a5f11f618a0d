"""Named device mesh over the flat torch.distributed rank space.

Parity: reference ``pluggy/core/mesh.py:8-114`` (``Mesh``: row-major named axes,
last axis fastest; one process group per axis slice; ``flatten`` virtual axes;
``size/get_group/coordinate``).

Layout: a spec ``{"dp": 2, "tp": 4}`` maps global rank ``r`` to coordinates with
the LAST axis varying fastest, i.e. ``coord[ax] = (r // stride[ax]) % size[ax]``
where ``stride`` is the product of the sizes of every axis after ``ax``.

``dist.new_group`` is itself a collective: every rank must create every group
in the same order, including groups it is not a member of. The constructor and
``flatten`` therefore walk all slices on every rank.
"""

from __future__ import annotations

import itertools

import torch.distributed as dist


def _row_major_strides(sizes: dict[str, int]) -> dict[str, int]:
    strides: dict[str, int] = {}
    acc = 1
    for axis in reversed(list(sizes)):
        strides[axis] = acc
        acc *= sizes[axis]
    return strides


def axis_slices(sizes: dict[str, int], axis: str) -> list[list[int]]:
    """Every rank list that forms one group along ``axis`` (deterministic order).

    Pure function of the spec so it is unit-testable without a process group.
    """
    strides = _row_major_strides(sizes)
    others = [a for a in sizes if a != axis]
    slices = []
    for coords in itertools.product(*(range(sizes[a]) for a in others)):
        base = sum(c * strides[a] for a, c in zip(others, coords))
        slices.append([base + i * strides[axis] for i in range(sizes[axis])])
    slices.sort(key=lambda m: m[0])
    return slices


class Mesh:
    """Named axes over ``dist.get_world_size()`` ranks.

    ``Mesh({"dp": 8})`` is the DDP/FSDP2 mesh; ``Mesh({"dp": 2, "tp": 4})``
    places the 4 TP peers of one data shard on consecutive ranks (NVSwitch makes
    every pair equidistant on a B200 box, so consecutive placement only matters
    for readability).
    """

    def __init__(self, spec: dict[str, int]):
        assert dist.is_initialized(), "init_process_group() must run before Mesh()"
        self.world_size = dist.get_world_size()
        total = 1
        for v in spec.values():
            total *= int(v)
        assert total == self.world_size, (
            f"mesh {spec} spans {total} ranks but the world has {self.world_size}"
        )
        self.sizes: dict[str, int] = {k: int(v) for k, v in spec.items()}
        self.strides = _row_major_strides(self.sizes)
        self._real_axes = list(self.sizes)
        self._flat_coords: dict[str, int] = {}
        self._flat_members: dict[str, list[int]] = {}
        self.groups: dict[str, dist.ProcessGroup] = {}
        self._members: dict[str, list[int]] = {}
        rank = dist.get_rank()
        for axis in self._real_axes:
            for members in axis_slices(self.sizes, axis):
                group = dist.new_group(members)
                if rank in members:
                    self.groups[axis] = group
                    self._members[axis] = members

    # ------------------------------------------------------------------ queries
    def size(self, dim: str) -> int:
        return self.sizes[dim]

    def get_group(self, dim: str) -> dist.ProcessGroup:
        return self.groups[dim]

    def members(self, dim: str) -> list[int]:
        """Global ranks of this rank's group along ``dim``, in coordinate order."""
        return list(self._members[dim])

    def coordinate(self, dim: str) -> int:
        if dim in self._flat_coords:
            return self._flat_coords[dim]
        return (dist.get_rank() // self.strides[dim]) % self.sizes[dim]

    # ------------------------------------------------------------------ flatten
    def flatten(self, axes: tuple[str, ...], name: str) -> None:
        """Register virtual axis ``name`` = the real ``axes`` taken as one axis.

        ``axes`` must be distinct real axes listed in spec order, so that the
        coordinate on the flat axis (the index in the group's rank order) equals
        the row-major mixed-radix coordinate. Collective: call it on every rank
        with the same arguments (reference ``pluggy/core/mesh.py:55-103``).
        """
        axes = tuple(axes)
        assert axes and len(set(axes)) == len(axes), f"bad axes {axes}"
        assert all(a in self.strides for a in axes), f"unknown axis in {axes}"
        order = [a for a in self._real_axes if a in axes]
        assert list(axes) == order, f"{axes} must follow spec order {order}"
        assert name not in self.sizes, f"axis {name!r} already exists"
        rest = [a for a in self._real_axes if a not in axes]
        rank = dist.get_rank()
        buckets: dict[tuple[int, ...], list[int]] = {}
        for r in range(self.world_size):
            key = tuple((r // self.strides[a]) % self.sizes[a] for a in rest)
            buckets.setdefault(key, []).append(r)
        for key in sorted(buckets):
            members = buckets[key]
            group = dist.new_group(members)
            if rank in members:
                self.groups[name] = group
                self._members[name] = members
                self._flat_coords[name] = members.index(rank)
        flat = 1
        for a in axes:
            flat *= self.sizes[a]
        self.sizes[name] = flat

    def __repr__(self) -> str:
        return f"Mesh({self.sizes})"


class FlatMesh:
    """A one-axis stand-in over an explicit process group (tests, tooling)."""

    def __init__(self, name: str = "dp", group: dist.ProcessGroup | None = None):
        self.name = name
        self.group = group if group is not None else dist.group.WORLD
        self.sizes = {name: dist.get_world_size(self.group)}

    def size(self, dim: str) -> int:
        return self.sizes[dim]

    def get_group(self, dim: str):
        return self.group

    def coordinate(self, dim: str) -> int:
        return dist.get_rank(self.group)

    def members(self, dim: str) -> list[int]:
        return [dist.get_global_rank(self.group, i) for i in range(self.size(dim))]
