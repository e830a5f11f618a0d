"""Multi-tensor optimizer kernels: AdamW step, grad sum-of-squares, grad scaling.

Each op is ONE launch over every tensor of the list: a small int64 table of
(pointers, numel, first chunk) is built on the host, copied with a pinned
non-blocking H2D copy, and the kernel grid-strides over 64K-element chunks,
locating each chunk's tensor by binary search in the table. Tables are kept by
content (the same pointers give the same table), so a steady-state step uploads
nothing, and a step captured into a CUDA graph keeps the table it was captured
with alive.
"""

from __future__ import annotations

from collections import OrderedDict

import torch

from pluggy_b200.ops._ext import ext

CHUNK = 65536


_TABLES: OrderedDict = OrderedDict()
_TABLES_MAX = 64


def _table(rows: list[list[int]], numels: list[int], device) -> tuple[torch.Tensor, int]:
    data, start = [], 0
    for r, n in zip(rows, numels, strict=True):
        data.append(r + [n, start])
        start += (n + CHUNK - 1) // CHUNK
    key = (str(device), tuple(tuple(r) for r in data))
    hit = _TABLES.get(key)
    if hit is not None:
        _TABLES.move_to_end(key)
        return hit[1], start
    host = torch.tensor(data, dtype=torch.int64).pin_memory()
    dev = host.to(device, non_blocking=True)
    # the pinned source stays referenced: a copy captured into a CUDA graph reads it
    # again on every replay
    _TABLES[key] = (host, dev)
    capturing = dev.is_cuda and torch.cuda.is_current_stream_capturing()
    if len(_TABLES) > _TABLES_MAX and not capturing:
        _TABLES.popitem(last=False)
    return dev, start


def _ptr(t: torch.Tensor | None) -> int:
    return 0 if t is None else t.data_ptr()


def multi_tensor_sumsq(tensors: list[torch.Tensor]) -> torch.Tensor:
    """Sum of squares of all elements of fp32 ``tensors`` (0-d fp32 tensor, deterministic)."""
    ts = [t for t in tensors if t.numel() > 0]
    dev = ts[0].device
    for t in ts:
        assert t.dtype == torch.float32 and t.is_contiguous(), "sumsq takes contiguous fp32 tensors"
    table, chunks = _table([[_ptr(t), 0, 0, 0, 0] for t in ts], [t.numel() for t in ts], dev)
    out = torch.empty(1 + chunks, dtype=torch.float32, device=dev)
    ext().multi_sumsq(table, len(ts), chunks, out)
    return out[0]


def multi_tensor_scale_(tensors: list[torch.Tensor], coef: torch.Tensor) -> None:
    ts = [t for t in tensors if t.numel() > 0]
    table, chunks = _table([[_ptr(t), 0, 0, 0, 0] for t in ts], [t.numel() for t in ts],
                           ts[0].device)
    ext().multi_scale(table, len(ts), chunks, coef.reshape(1).float())


def adamw_step(params, grads, exp_avgs, exp_avg_sqs, shadows, *, lr, beta1, beta2, eps,
               weight_decay, bias_correction1, bias_correction2, grad_scale=None,
               hyper=None) -> None:
    """``hyper``: optional fp32 device tensor (lr, bias_correction1, bias_correction2)
    read by the kernel in place of the scalar arguments."""
    rows, numels = [], []
    for p, g, m, v, s in zip(params, grads, exp_avgs, exp_avg_sqs, shadows, strict=True):
        if p.numel() == 0:
            continue
        assert p.dtype == torch.float32 and g.dtype == torch.float32, "AdamW kernel takes fp32"
        assert p.is_contiguous() and g.is_contiguous() and m.is_contiguous() and v.is_contiguous()
        rows.append([_ptr(p), _ptr(g), _ptr(m), _ptr(v), _ptr(s)])
        numels.append(p.numel())
    if not rows:
        return
    table, chunks = _table(rows, numels, params[0].device)
    gs = None if grad_scale is None else grad_scale.reshape(1).float()
    ext().adamw_multi(table, len(rows), chunks, float(lr), float(beta1), float(beta2), float(eps),
                      float(weight_decay), float(bias_correction1), float(bias_correction2), gs,
                      hyper)
