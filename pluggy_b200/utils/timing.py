"""Device-side timing: CUDA events on the launching stream, max over ranks.

Every benchmark number this package reports comes from here: ``W`` untimed
warm-up iterations, a barrier plus ``torch.cuda.synchronize()`` on both sides of
the timed window, the elapsed time between two events recorded on the current
stream, and (multi-rank) the MAX over ranks via an all-reduce.
"""

from __future__ import annotations

import time

import torch
import torch.distributed as dist


def _barrier():
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def max_over_ranks(value: float, device=None) -> float:
    if not (dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1):
        return value
    t = torch.tensor([value], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def device_time(fn, steps: int, warmup: int, between=None) -> float:
    """Milliseconds per ``fn()`` call, timed on the device, max over ranks.

    ``between`` (optional) runs before every timed call but outside the timed
    events, e.g. an L2 flush.
    """
    for _ in range(warmup):
        if between is not None:
            between()
        fn()
    if not torch.cuda.is_available():
        _barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            if between is not None:
                between()
            fn()
        _barrier()
        return max_over_ranks((time.perf_counter() - t0) * 1e3 / steps)
    torch.cuda.synchronize()
    _barrier()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(steps):
        if between is not None:
            between()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        end.synchronize()
        total += start.elapsed_time(end)
    torch.cuda.synchronize()
    _barrier()
    return max_over_ranks(total / steps, device=torch.device("cuda", torch.cuda.current_device()))


class L2Flush:
    """Writes a buffer larger than the 126 MB L2 so the next kernel starts cold."""

    def __init__(self, nbytes: int = 256 << 20, device=None):
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device or "cuda")

    def __call__(self):
        self.buf.fill_(1)
