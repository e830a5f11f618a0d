"""Grouped (per-expert) SwiGLU FFN over expert-sorted rows.

``grouped_swiglu_ffn(x, experts, counts, gate_up_proj, down_proj)``: row ``i`` of
``x`` belongs to expert ``experts[i]`` (rows sorted by expert, ``counts[e]`` rows
for expert ``e``); for each expert ``y_e = (silu(x_e Wg_e^T) * x_e Wu_e^T) Wd_e^T``
with the reference's packed weights ``gate_up_proj (E, 2I, H)`` and ``down_proj
(E, H, I)``. Replaces the reference's two ``F.grouped_mm`` launches per
direction (``pluggy/kernels/moe.py:68-124``).

CUDA: the rows are laid out in a padded per-expert layout (each expert's rows
start on a 128-row tile boundary, the padding rows are zero), computed on the
device from the counts, so nothing is read back to the host. Each projection is
ONE launch of the tcgen05 GEMM in its grouped modes over all experts:

* forward / input-gradient (mode 1): every 128-row tile belongs to one expert,
  whose weight block the tile's B loads select (tiles past the last expert are
  skipped);
* weight-gradient (mode 2): expert ``e`` sums over its own row range only and
  writes its own ``[E]`` slice of the fp32 gradient; an expert without rows
  writes zeros.

The GLU between the projections is the sm_100a kernel; the zero padding rows
stay zero through it, so they add nothing to the weight gradients. bf16 expert
weights come from the caller (the model's weight cache, which the optimizer
keeps current) or are cast once per call.
"""

from __future__ import annotations

import torch

from pluggy_b200.ops.elementwise import SILU, glu_bwd, glu_fwd

TILE = 128  # rows per GEMM m tile: each expert's rows start on a tile boundary


def expert_layout(counts: torch.Tensor, P: int):
    """Padded row layout of ``P`` expert-sorted rows (device tensors only).

    Returns ``(poff, shift, tile_group, R)``: ``poff`` int32 [E + 1] padded row
    offsets (multiples of 128); ``shift`` int64 [E] = padded minus packed offset of
    each expert (row ``i`` of expert ``e`` goes to ``i + shift[e]``); ``tile_group``
    int32 [R / 128], the expert of each tile or -1 past the last; ``R`` the
    worst-case padded row count (a host int: every expert adds < 128 rows)."""
    E = counts.numel()
    counts = counts.to(torch.int64)
    pad = (counts + TILE - 1) // TILE * TILE
    poff = torch.zeros(E + 1, dtype=torch.int64, device=counts.device)
    poff[1:] = torch.cumsum(pad, 0)
    off = torch.cumsum(counts, 0) - counts
    shift = poff[:-1] - off
    tiles = (P + E * (TILE - 1) + TILE - 1) // TILE
    starts = torch.arange(tiles, device=counts.device, dtype=torch.int64) * TILE
    g = torch.searchsorted(poff[1:].contiguous(), starts, right=True)
    tile_group = torch.where(g >= E, torch.full_like(g, -1), g).to(torch.int32)
    return poff.to(torch.int32), shift, tile_group, tiles * TILE


def _gg(a, b, b_mn_major, c, mode, table, groups, b_rows):
    from pluggy_b200.ops._ext import ext, status_word

    ext().gemm_grouped(a, b, b_mn_major, c, mode, table, groups, b_rows, 1.0, 0.0,
                       status_word(a.device))
    return c


class _GroupedSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, experts, counts, gate_up_proj, down_proj, gu_lowp, dn_lowp):
        E, I2, H = gate_up_proj.shape
        I = I2 // 2
        P = x.shape[0]
        dev = x.device
        poff, shift, tile_g, R = expert_layout(counts, P)
        dst = torch.arange(P, device=dev, dtype=torch.int64) + shift[experts]
        x_pad = torch.zeros((R, H), dtype=torch.bfloat16, device=dev)
        x_pad.index_copy_(0, dst, x.to(torch.bfloat16))
        gu_w = (gu_lowp if gu_lowp is not None else gate_up_proj.detach().to(torch.bfloat16))
        dn_w = (dn_lowp if dn_lowp is not None else down_proj.detach().to(torch.bfloat16))
        gu_w2, dn_w2 = gu_w.reshape(E * I2, H), dn_w.reshape(E * H, I)
        gu = _gg(x_pad, gu_w2, False, torch.empty((R, I2), dtype=torch.bfloat16, device=dev), 1,
                 tile_g, E, I2)
        act = glu_fwd(gu, SILU)
        y_pad = _gg(act, dn_w2, False, torch.empty((R, H), dtype=torch.bfloat16, device=dev), 1,
                    tile_g, E, H)
        ctx.save_for_backward(x_pad, gu, act, gu_w2, dn_w2, dst, poff, tile_g)
        ctx.dims = (E, I, H, R)
        ctx.x_dtype = x.dtype
        return y_pad.index_select(0, dst).to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        x_pad, gu, act, gu_w2, dn_w2, dst, poff, tile_g = ctx.saved_tensors
        E, I, H, R = ctx.dims
        dev = dy.device
        dy_pad = torch.zeros((R, H), dtype=torch.bfloat16, device=dev)
        dy_pad.index_copy_(0, dst, dy.to(torch.bfloat16))
        dact = _gg(dy_pad, dn_w2, True, torch.empty((R, I), dtype=torch.bfloat16, device=dev), 1,
                   tile_g, E, H)
        ddn = _gg(dy_pad, act, True, torch.empty((E * H, I), dtype=torch.float32, device=dev), 2,
                  poff, E, 0)
        dgu = glu_bwd(gu, dact, SILU)
        dx_pad = _gg(dgu, gu_w2, True, torch.empty((R, H), dtype=torch.bfloat16, device=dev), 1,
                     tile_g, E, 2 * I)
        dgu_w = _gg(dgu, x_pad, True, torch.empty((E * 2 * I, H), dtype=torch.float32, device=dev),
                    2, poff, E, 0)
        dx = dx_pad.index_select(0, dst).to(ctx.x_dtype)
        return dx, None, None, dgu_w.view(E, 2 * I, H), ddn.view(E, H, I), None, None


def grouped_swiglu_ffn(x, experts, counts, gate_up_proj, down_proj, gu_lowp=None, dn_lowp=None):
    """``experts`` [P] expert of each (expert-sorted) row, ``counts`` [E] rows per expert."""
    if x.is_cuda:
        return _GroupedSwiGLU.apply(x, experts, counts, gate_up_proj, down_proj, gu_lowp, dn_lowp)
    out = []
    off = 0
    for e, n in enumerate(counts.tolist()):
        if n == 0:
            continue
        xe = x[off:off + n]
        g, u = torch.nn.functional.linear(xe, gate_up_proj[e].to(x.dtype)).chunk(2, dim=-1)
        out.append(torch.nn.functional.linear(torch.nn.functional.silu(g) * u,
                                              down_proj[e].to(x.dtype)))
        off += n
    return torch.cat(out, 0) if out else x.new_zeros((0, down_proj.shape[1]))
