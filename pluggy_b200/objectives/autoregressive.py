"""Autoregressive (next-token) objective.

Parity: reference ``pluggy/objectives/autoregressive.py:16-57``:

* ``fused_linear_ce=True``: ``model(ids, return_final_hidden=True)``, labels
  shifted so position t predicts t+1 (last position = ignore_index), then the
  chunked fused linear-CE against ``model.lm_head.weight``;
* otherwise full logits + ``cross_entropy_loss``;
* ``model.aux_loss()`` (MoE load-balance / z-loss) is added when present.

On CUDA the fused path passes the model's cached bf16 LM-head weight so the
head GEMMs never re-cast the fp32 master weight.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from pluggy_b200.loss.cross_entropy import cross_entropy_loss
from pluggy_b200.loss.fused_linear_ce import fused_linear_cross_entropy


def shift_labels(labels: torch.Tensor, ignore_index: int) -> torch.Tensor:
    out = torch.full_like(labels, ignore_index)
    out[:, :-1] = labels[:, 1:]
    return out


class ARObjective:
    def __init__(self, ignore_index: int = -100, fused_linear_ce: bool = True, ce_chunk_size: int = 4096):
        self.ignore_index = ignore_index
        self.fused_linear_ce = fused_linear_ce
        self.ce_chunk_size = ce_chunk_size

    def compute_loss(self, model: nn.Module, batch: dict[str, torch.Tensor]) -> torch.Tensor:
        core = getattr(model, "module", model)
        tp = getattr(core, "tp", None)
        cp = getattr(core, "cp", None)
        if cp is not None and cp.mesh.size(cp.dim) > 1:
            # context parallel: labels shifted on the full sequence, then each rank
            # keeps its zigzag tokens; the loss is this rank's share of the global mean
            from pluggy_b200.core.collective import all_reduce

            assert self.fused_linear_ce, "context parallelism needs fused_linear_ce=True"
            labels = shift_labels(batch["labels"], self.ignore_index)
            ids, labels, pos = cp.shard_batch(batch["input_ids"], labels)
            hidden = model(ids, return_final_hidden=True, position_ids=pos)
            n_local = (labels != self.ignore_index).sum().float()
            n_all = all_reduce(n_local.clone(), cp.mesh, cp.dim, "sum")
            loss = fused_linear_cross_entropy(hidden, core.lm_head.weight, labels, self.ignore_index,
                                              self.ce_chunk_size) * (n_local / n_all.clamp(min=1))
        elif tp is not None and tp.mesh.size(tp.dim) > 1:
            # vocabulary-parallel head: full-sequence hidden against the local vocab rows
            from pluggy_b200.parallel.tensor_parallel import (tp_hidden_for_head,
                                                              vocab_parallel_cross_entropy)

            assert self.fused_linear_ce, "tensor parallelism needs fused_linear_ce=True"
            hidden = tp_hidden_for_head(core, model(batch["input_ids"], return_final_hidden=True))
            labels = shift_labels(batch["labels"], self.ignore_index)
            lowp_fn = getattr(core, "lm_head_lowp", None)
            lowp = lowp_fn() if (callable(lowp_fn) and hidden.is_cuda) else None
            loss = vocab_parallel_cross_entropy(hidden.reshape(-1, hidden.shape[-1]),
                                                core.lm_head.weight, labels.reshape(-1), tp.vstart,
                                                tp.mesh, tp.dim, self.ignore_index,
                                                self.ce_chunk_size, w_lowp=lowp)
        elif self.fused_linear_ce:
            hidden = model(batch["input_ids"], return_final_hidden=True)
            labels = shift_labels(batch["labels"], self.ignore_index)
            lowp_fn = getattr(core, "lm_head_lowp", None)
            lowp = lowp_fn() if (callable(lowp_fn) and hidden.is_cuda) else None
            loss = fused_linear_cross_entropy(hidden, core.lm_head.weight, labels, self.ignore_index,
                                              self.ce_chunk_size, weight_lowp=lowp)
        else:
            logits = model(batch["input_ids"])
            loss = cross_entropy_loss(batch["labels"], logits, self.ignore_index)
        aux_fn = getattr(core, "aux_loss", None)
        if callable(aux_fn):
            aux = aux_fn()
            if aux is not None:
                loss = loss + aux
        return loss
