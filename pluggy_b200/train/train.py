"""Training entry point: ``python -m pluggy_b200.train.train --config X [--steps N]``.

Parity: reference ``pluggy/train/train.py:31-87``: env defaults for a
single-process launch, ``set_device(local_rank)`` before
``init_process_group`` (10 min timeout so a wedged collective fails), the
Trainer, and ``destroy_process_group`` in a ``finally``. ``--steps`` is the
benchmark mode (fixed step count, no checkpoints, no wandb). The backend is
NCCL on GPUs and gloo on CPU-only hosts.
"""

from __future__ import annotations

import argparse
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--config", required=True, help="path to the train config json")
    p.add_argument("--steps", type=int, default=None,
                   help="benchmark mode: run exactly N steps (no checkpointing)")
    return p.parse_args(argv)


def init_distributed(timeout_min: float = 10.0) -> tuple[int, int, int]:
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("LOCAL_RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    rank = int(os.environ["RANK"])
    local_rank = int(os.environ["LOCAL_RANK"])
    world = int(os.environ["WORLD_SIZE"])
    if torch.cuda.is_available():
        torch.cuda.set_device(local_rank)
        backend = "nccl"
    else:
        backend = "gloo"
    if not dist.is_initialized():
        kw = {"device_id": torch.device("cuda", local_rank)} if backend == "nccl" else {}
        dist.init_process_group(backend=backend, timeout=timedelta(minutes=timeout_min), **kw)
    return rank, local_rank, world


def main(argv=None) -> None:
    args = parse_args(argv)
    rank, local_rank, world = init_distributed()
    from pluggy_b200.train.trainer import Trainer

    try:
        trainer = Trainer(args.config, rank=rank, local_rank=local_rank, world_size=world,
                          benchmark=args.steps is not None)
        if args.steps is not None:
            trainer.train_n_step_test(args.steps)
        else:
            trainer.train()
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
