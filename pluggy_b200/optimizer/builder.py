"""Optimizer / scheduler registries and builders.

Parity: reference ``pluggy/optimizer/builder.py:20-55``: two param groups
(weight decay on tensors with >= 2 dims, none on 1-D), the rest of the config
passed straight to the constructor. ``adamw`` maps to :class:`FusedAdamW` (a
``torch.optim.AdamW`` whose CUDA step is this package's kernel).
"""

from __future__ import annotations

import torch.nn as nn
import torch.optim as optim

from pluggy_b200.optimizer.fused_adamw import FusedAdamW
from pluggy_b200.optimizer.scheduler import CosineAnnealingScheduler, WarmupStableDecaySchedulder

OPTIMIZER_REGISTRY = {
    "adamw": FusedAdamW,
    "sgd": optim.SGD,
}

SCHEDULER_REGISTRY = {
    "wsd": WarmupStableDecaySchedulder,
    "cosine": CosineAnnealingScheduler,
}


def param_groups(model: nn.Module, weight_decay: float) -> list[dict]:
    params = [p for p in model.parameters() if p.requires_grad]
    return [
        {"params": [p for p in params if p.dim() >= 2], "weight_decay": weight_decay},
        {"params": [p for p in params if p.dim() < 2], "weight_decay": 0.0},
    ]


def build_optimizer(model: nn.Module, optim_name: str, optim_config: dict) -> optim.Optimizer:
    assert optim_name in OPTIMIZER_REGISTRY, f"unknown optimizer {optim_name!r}"
    cfg = dict(optim_config)
    wd = cfg.pop("weight_decay", 0.0)
    if "betas" in cfg:
        cfg["betas"] = tuple(cfg["betas"])
    return OPTIMIZER_REGISTRY[optim_name](param_groups(model, wd), **cfg)


def build_scheduler(optimizer: optim.Optimizer, scheduler_config: dict):
    cfg = dict(scheduler_config)
    kind = cfg.pop("type")
    assert kind in SCHEDULER_REGISTRY, f"unknown scheduler {kind!r}"
    return SCHEDULER_REGISTRY[kind](optimizer=optimizer, **cfg)
