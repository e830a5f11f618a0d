"""Run a function on N gloo ranks (spawned processes) and surface every rank's failure."""

from __future__ import annotations

import os
import socket
import traceback
from datetime import timedelta

import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn, args, q, timeout_s, backend="gloo"):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(rank)
            kw["device_id"] = torch.device("cuda", rank)
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=timedelta(seconds=timeout_s), **kw)
        fn(rank, world, *args)
        q.put((rank, None))
    except BaseException:  # noqa: BLE001 - reported to the parent
        q.put((rank, traceback.format_exc()))
    finally:
        try:
            if dist.is_initialized():
                dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def run_ranks(fn, world: int, *args, timeout_s: float = 60.0, join_s: float = 180.0,
              backend: str = "gloo"):
    """``backend="nccl"``: rank r drives GPU r (needs ``world`` GPUs)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn, args, q, timeout_s, backend))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for p in procs:
        p.join(join_s)
    for p in procs:
        if p.is_alive():
            p.kill()
    while not q.empty():
        r, err = q.get()
        results[r] = err
    errs = {r: e for r, e in results.items() if e}
    missing = [r for r in range(world) if r not in results]
    if errs or missing:
        msg = "\n".join(f"--- rank {r} ---\n{e}" for r, e in sorted(errs.items()))
        raise AssertionError(f"ranks failed: {sorted(errs)} missing: {missing}\n{msg}")
