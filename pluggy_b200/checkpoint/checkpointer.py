"""Resume-everything checkpointer, one directory per completed step.

Parity: reference ``pluggy/checkpoint/checkpointer.py:18-123``. Layout:

``<root>/<completed_step>/{model.pt, optimizer.pt, scheduler.pt, trainer.pt,
rng_rank{r}.pt, dataloader_dp{c}.pt, .complete}``

``.complete`` is written last (after a barrier in the trainer); ``latest()`` and
``valid_step()`` only see completed directories, so a torn save is invisible.
Loads use ``map_location="cpu"`` and ``weights_only=True`` except for the
dataloader state (arbitrary picklable iterator state).

Sharded additions (FSDP2 / TP / EP): ``save_sharded_model`` writes
``model_shard_rank{r}.pt`` per rank plus ``placements.json`` describing how
each tensor is laid out; ``consolidate`` reassembles a plain ``model.pt`` that
a replicated run (or the reference) loads unchanged.
"""

from __future__ import annotations

import json
import os

import torch
import torch.nn as nn


class Checkpointer:
    def __init__(self, checkpoint_save_path: str):
        self.checkpoint_save_path = checkpoint_save_path
        os.makedirs(checkpoint_save_path, exist_ok=True)

    # --------------------------------------------------------------- discovery
    def _steps(self) -> list[int]:
        return [int(d) for d in os.listdir(self.checkpoint_save_path)
                if d.isdigit() and self.is_complete(int(d))]

    def latest(self) -> int | None:
        return max(self._steps(), default=None)

    def valid_step(self, step: int) -> int | None:
        return step if step in self._steps() else None

    def _step_dir(self, step: int, create: bool = False) -> str:
        d = os.path.join(self.checkpoint_save_path, str(step))
        if create:
            os.makedirs(d, exist_ok=True)
        return d

    def _path(self, step: int, name: str, create: bool = False) -> str:
        return os.path.join(self._step_dir(step, create), name)

    def _save(self, obj, step: int, name: str) -> None:
        torch.save(obj.state_dict(), self._path(step, name, create=True))

    def _load(self, step: int, name: str, weights_only: bool = True):
        return torch.load(self._path(step, name), map_location="cpu", weights_only=weights_only)

    # -------------------------------------------------------------- components
    def save_model(self, model: nn.Module, step: int) -> None:
        self._save(model, step, "model.pt")

    def load_model(self, model: nn.Module, step: int) -> None:
        model.load_state_dict(self._load(step, "model.pt"))

    def save_optimizer(self, optimizer, step: int) -> None:
        self._save(optimizer, step, "optimizer.pt")

    def load_optimizer(self, optimizer, step: int) -> None:
        optimizer.load_state_dict(self._load(step, "optimizer.pt"))

    def save_scheduler(self, scheduler, step: int) -> None:
        self._save(scheduler, step, "scheduler.pt")

    def load_scheduler(self, scheduler, step: int) -> None:
        scheduler.load_state_dict(self._load(step, "scheduler.pt"))

    def save_trainer(self, state: dict, step: int) -> None:
        torch.save(state, self._path(step, "trainer.pt", create=True))

    def load_trainer(self, step: int) -> dict:
        return self._load(step, "trainer.pt")

    def save_dataloader(self, dataloader, step: int, dp_rank: int = 0) -> None:
        self.save_dataloader_state(dataloader.state_dict(), step, dp_rank)

    def save_dataloader_state(self, state: dict, step: int, dp_rank: int = 0) -> None:
        torch.save(state, self._path(step, f"dataloader_dp{dp_rank}.pt", create=True))

    def load_dataloader(self, dataloader, step: int, dp_rank: int = 0) -> None:
        dataloader.load_state_dict(self._load(step, f"dataloader_dp{dp_rank}.pt", weights_only=False))

    def save_rng(self, state: dict, step: int, rank: int = 0) -> None:
        torch.save(state, self._path(step, f"rng_rank{rank}.pt", create=True))

    def load_rng(self, step: int, rank: int = 0) -> dict | None:
        p = self._path(step, f"rng_rank{rank}.pt")
        if not os.path.exists(p):
            return None
        return torch.load(p, map_location="cpu", weights_only=True)

    # ------------------------------------------------------------- completion
    def _complete_path(self, step: int) -> str:
        return self._path(step, ".complete")

    def mark_complete(self, step: int) -> None:
        open(self._complete_path(step), "w").close()

    def is_complete(self, step: int) -> bool:
        return os.path.exists(self._complete_path(step))

    # ---------------------------------------------------------------- sharded
    def save_sharded_model(self, local_state: dict[str, torch.Tensor], placements: dict[str, dict],
                           step: int, rank: int, world_size: int) -> None:
        """Write this rank's shard and (rank 0) the placement metadata.

        ``placements[name] = {"axis_size": n, "coord": c, "dim": d}`` for a tensor
        sharded evenly along ``d`` over ``n`` ranks (``dim = None`` = replicated).
        """
        torch.save({k: v.detach().cpu() for k, v in local_state.items()},
                   self._path(step, f"model_shard_rank{rank}.pt", create=True))
        meta_path = self._path(step, f"placements_rank{rank}.json", create=True)
        with open(meta_path, "w") as f:
            json.dump({"world_size": world_size, "placements": placements}, f)

    def consolidate(self, step: int, world_size: int) -> dict[str, torch.Tensor]:
        """Reassemble the full state dict from every rank's shard file; writes model.pt."""
        shards, metas = [], []
        for r in range(world_size):
            shards.append(self._load(step, f"model_shard_rank{r}.pt"))
            with open(self._path(step, f"placements_rank{r}.json")) as f:
                metas.append(json.load(f)["placements"])
        full: dict[str, torch.Tensor] = {}
        for name in shards[0]:
            dim = metas[0][name].get("dim")
            if dim is None:
                full[name] = shards[0][name]
                continue
            pieces = sorted(((metas[r][name]["coord"], metas[r][name].get("group", 0), shards[r][name])
                             for r in range(world_size)), key=lambda t: (t[1], t[0]))
            group0 = [p for p in pieces if p[1] == pieces[0][1]]
            full[name] = torch.cat([p[2] for p in group0], dim=dim)
        torch.save(full, self._path(step, "model.pt", create=True))
        return full
