"""LR schedules: warmup-stable-decay and warmup-cosine.

Parity: reference ``pluggy/optimizer/scheduler.py:12-65``. Both warm up with
``(step + 1) / W`` where ``W = max(1, round(total_steps * warmup_ratio))``, so
step ``W-1`` reaches scale 1.0.

* WSD: flat after warmup; linear decay to 0 starting at
  ``total_steps * (1 - decay_ratio)``, clamped at 0.
* Cosine: half-cosine from 1 to ``min_lr_ratio`` over the steps after warmup,
  held at the floor past ``total_steps``.

The class name ``WarmupStableDecaySchedulder`` keeps the reference's spelling so
that pickled scheduler state and configs stay interchangeable; the correctly
spelled alias is the same class.
"""

from __future__ import annotations

import math

from torch.optim.lr_scheduler import LRScheduler


def _warmup_steps(total_steps: int, warmup_ratio: float) -> int:
    return max(1, round(total_steps * warmup_ratio))


def wsd_scale(step: int, total_steps: int, warmup_ratio: float, decay_ratio: float) -> float:
    w = _warmup_steps(total_steps, warmup_ratio)
    decay_start = total_steps * (1 - decay_ratio)
    if step < w:
        return (step + 1) / w
    if step >= decay_start:
        return max(0.0, 1 - (step - decay_start) / (decay_ratio * total_steps))
    return 1.0


def cosine_scale(step: int, total_steps: int, warmup_ratio: float, min_lr_ratio: float) -> float:
    w = _warmup_steps(total_steps, warmup_ratio)
    if step < w:
        return (step + 1) / w
    progress = min(1.0, (step - w) / max(1, total_steps - w))
    return min_lr_ratio + (1 - min_lr_ratio) * 0.5 * (1 + math.cos(math.pi * progress))


class WarmupStableDecaySchedulder(LRScheduler):
    def __init__(self, optimizer, total_steps, warmup_ratio, decay_ratio, last_epoch=-1):
        self.total_steps = total_steps
        self.warmup_ratio = warmup_ratio
        self.decay_ratio = decay_ratio
        super().__init__(optimizer, last_epoch)

    def get_lr(self):
        s = wsd_scale(self.last_epoch, self.total_steps, self.warmup_ratio, self.decay_ratio)
        return [base * s for base in self.base_lrs]


WarmupStableDecayScheduler = WarmupStableDecaySchedulder


class CosineAnnealingScheduler(LRScheduler):
    def __init__(self, optimizer, total_steps, warmup_ratio, min_lr_ratio=0.0, last_epoch=-1):
        self.total_steps = total_steps
        self.warmup_ratio = warmup_ratio
        self.min_lr_ratio = min_lr_ratio
        super().__init__(optimizer, last_epoch)

    def get_lr(self):
        s = cosine_scale(self.last_epoch, self.total_steps, self.warmup_ratio, self.min_lr_ratio)
        return [base * s for base in self.base_lrs]
