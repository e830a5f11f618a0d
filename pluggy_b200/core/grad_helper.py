"""Global grad-norm clipping across mesh axes.

Parity: reference ``pluggy/core/grad_helper.py:8-34``: L2 norm over all grads,
squared norms summed over ``shard_dims`` when grads are sharded, clip
coefficient ``clamp(max_norm / (total + 1e-6), max=1)``, returns the pre-clip
norm, ``max_norm=None`` only measures.

On CUDA the per-tensor norms and the scaling run in this package's sm_100a
multi-tensor kernels (``pluggy_b200.ops.optim``) with no host synchronisation:
the coefficient stays on the device. ``fold_into_optimizer=True`` skips the
scaling pass and returns the coefficient so the fused AdamW kernel applies it
while it reads the grads anyway.
"""

from __future__ import annotations

import torch

from pluggy_b200.core.collective import all_reduce


def _grads(params) -> list[torch.Tensor]:
    grads = [p.grad for p in params if p.grad is not None]
    assert grads, "clip_grad_norm got no grads; backward didn't run, or all params are frozen"
    return grads


def grad_norm_sq(grads: list[torch.Tensor]) -> torch.Tensor:
    """Sum of squares of every element of ``grads`` as an fp32 0-d tensor."""
    if grads[0].is_cuda:
        from pluggy_b200.ops import optim as _optim

        return _optim.multi_tensor_sumsq(grads)
    norms = torch._foreach_norm(grads, 2.0)
    return torch.linalg.vector_norm(torch.stack(norms).float(), 2.0) ** 2


def _norm_sq(grads: list[torch.Tensor]) -> torch.Tensor:
    if grads[0].is_cuda:
        return grad_norm_sq(grads)
    norms = torch._foreach_norm(grads, 2.0)
    return torch.linalg.vector_norm(torch.stack(norms), 2.0) ** 2


def clip_grad_norm(params, mesh, max_norm, shard_dims=(), *, fold_into_optimizer: bool = False,
                   partial_over=None, precomputed_sq: torch.Tensor | None = None):
    """``partial_over``: a list of ``(dims, param_ids)`` (or one such pair). Those
    params are further sharded over ``dims`` (tensor or expert parallelism), so
    their squared norms are summed over ``dims`` too; params in no group are
    replicated and counted once. The groups must be disjoint.

    ``precomputed_sq``: the global sum of squares, already computed (the fused
    data-parallel reducer produces it while it averages the grads)."""
    params = list(params)
    grads = _grads(params)
    if precomputed_sq is not None:
        sq = precomputed_sq.reshape(())
        shard_dims = ()
    elif partial_over is None:
        sq = _norm_sq(grads)
    else:
        groups = [partial_over] if isinstance(partial_over, tuple) else list(partial_over)
        claimed: set[int] = set()
        sq = torch.zeros((), device=grads[0].device)
        for dims, ids in groups:
            part = [p.grad for p in params if p.grad is not None and id(p) in ids]
            claimed |= set(ids)
            gsq = _norm_sq(part) if part else torch.zeros((), device=grads[0].device)
            for dim in dims:
                all_reduce(gsq, mesh, dim, "sum")
            sq = sq + gsq
        rep = [p.grad for p in params if p.grad is not None and id(p) not in claimed]
        if rep:
            sq = sq + _norm_sq(rep)
    for dim in shard_dims:
        all_reduce(sq, mesh, dim, "sum")
    total = sq.sqrt()
    if max_norm is None:
        return (total, None) if fold_into_optimizer else total
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    if fold_into_optimizer:
        return total, coef
    if grads[0].is_cuda:
        from pluggy_b200.ops import optim as _optim

        _optim.multi_tensor_scale_(grads, coef)
    else:
        torch._foreach_mul_(grads, coef)
    return total
