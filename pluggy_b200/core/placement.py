"""Placement value types: how a logical tensor maps onto one mesh axis.

Parity: reference ``pluggy/core/placement.py:25-42``. Frozen dataclasses so they
hash, compare and serialise into checkpoint metadata.
"""

from __future__ import annotations

from dataclasses import dataclass

from pluggy_b200.core.collective import ReduceOpName


@dataclass(frozen=True)
class Placement:
    pass


@dataclass(frozen=True)
class Shard(Placement):
    """The logical tensor is split evenly along ``dim``; a rank holds slice ``coord``."""

    dim: int


@dataclass(frozen=True)
class Replicate(Placement):
    """Every rank holds the whole logical tensor."""


@dataclass(frozen=True)
class Partial(Placement):
    """Every rank holds a term; the logical tensor is their ``op`` reduction."""

    op: ReduceOpName = "sum"


def to_meta(p: Placement) -> dict:
    """JSON-able description (sharded checkpoint metadata)."""
    if isinstance(p, Shard):
        return {"type": "shard", "dim": p.dim}
    if isinstance(p, Partial):
        return {"type": "partial", "op": p.op}
    return {"type": "replicate"}


def from_meta(d: dict) -> Placement:
    t = d["type"]
    if t == "shard":
        return Shard(int(d["dim"]))
    if t == "partial":
        return Partial(d["op"])
    return Replicate()
