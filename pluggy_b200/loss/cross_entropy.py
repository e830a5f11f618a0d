"""Plain next-token cross entropy over full logits.

Parity: reference ``pluggy/loss/cross_entropy.py:7-35``: position t predicts
token t+1; logits are flattened and the shifted labels use ``ignore_index``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def cross_entropy_loss(labels: torch.Tensor, logits: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    shift_logits = logits[:, :-1, :].contiguous()
    shift_labels = labels[:, 1:].contiguous()
    return F.cross_entropy(shift_logits.view(-1, shift_logits.size(-1)).float(),
                           shift_labels.view(-1), ignore_index=ignore_index)
