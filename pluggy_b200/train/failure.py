"""Host-side notice of a rank's failure to the other ranks.

A rank that fails between collectives (a data error, a failed checkpoint write, a
status word that reports a timed-out device wait) would otherwise leave the other
ranks blocked in their next collective until the process group's timeout (10 minutes
by default, ``pluggy/train/train.py:69-71`` of the reference). Here the failing rank
writes one key into the process group's key-value store (the TCP store every rank
already shares) and every rank checks that key, without blocking, before each step:
the survivors stop before they launch that step's collectives, with an error that
names the failed rank. A rank that dies without writing (killed, ``os._exit``) is
still caught by the process group: its peers' next collective fails on the closed
connection or at the timeout.
"""

from __future__ import annotations

import torch.distributed as dist

_KEY = "plg/failed_rank"


class PeerFailure(RuntimeError):
    """Another rank announced that it failed."""


class FailureNotice:
    def __init__(self, rank: int, enabled: bool = True):
        self.rank = rank
        self.store = None
        if enabled and dist.is_initialized() and dist.get_world_size() > 1:
            try:
                self.store = dist.distributed_c10d._get_default_store()
            except (AttributeError, RuntimeError):
                self.store = None

    def check(self) -> None:
        """Raise :class:`PeerFailure` if any rank has announced a failure."""
        if self.store is not None and self.store.check([_KEY]):
            raise PeerFailure(f"stopping: {self.store.get(_KEY).decode(errors='replace')}")

    def announce(self, exc: BaseException) -> None:
        """Tell the other ranks that this rank is failing with ``exc`` (a failure that
        is itself a peer's notice is not re-announced)."""
        if self.store is None or isinstance(exc, PeerFailure):
            return
        msg = f"rank {self.rank} failed: {type(exc).__name__}: {exc}"[:500]
        try:
            self.store.set(_KEY, msg)
        except Exception:  # noqa: BLE001 - the store itself may be gone; nothing to add
            pass
