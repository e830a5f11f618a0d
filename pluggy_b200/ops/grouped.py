"""Grouped (per-expert) SwiGLU FFN over expert-sorted rows.

``grouped_swiglu_ffn(x, counts, gate_up_proj, down_proj)``: rows of ``x`` are
sorted by expert and ``counts[e]`` rows belong to expert ``e``; for each expert
``y_e = (silu(x_e Wg_e^T) * x_e Wu_e^T) Wd_e^T`` with the reference's packed
weights ``gate_up_proj (E, 2I, H)`` and ``down_proj (E, H, I)``.

CUDA: every per-expert product is a tcgen05 GEMM from ``pluggy_b200.ops.gemm``
on views of one bf16 copy of the expert weights; the GLU runs in the sm_100a
kernel. Empty experts launch nothing. The per-expert row counts are read on the
host once per call (one small device-to-host copy).
"""

from __future__ import annotations

import torch

from pluggy_b200.ops.elementwise import SILU, glu_bwd, glu_fwd
from pluggy_b200.ops.gemm import linear_dgrad, linear_fwd, linear_wgrad


class _GroupedSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, counts, gate_up_proj, down_proj):
        E, I2, H = gate_up_proj.shape
        I = I2 // 2
        xs = x.to(torch.bfloat16).contiguous()
        gu_w = gate_up_proj.detach().to(torch.bfloat16)
        dn_w = down_proj.detach().to(torch.bfloat16)
        cnt = counts.tolist()
        P = xs.shape[0]
        gu = torch.empty((P, I2), dtype=torch.bfloat16, device=x.device)
        act = torch.empty((P, I), dtype=torch.bfloat16, device=x.device)
        y = torch.empty((P, H), dtype=torch.bfloat16, device=x.device)
        off = 0
        for e, n in enumerate(cnt):
            if n == 0:
                continue
            linear_fwd(xs[off:off + n], gu_w[e], out=gu[off:off + n])
            act[off:off + n] = glu_fwd(gu[off:off + n], SILU)
            linear_fwd(act[off:off + n], dn_w[e], out=y[off:off + n])
            off += n
        ctx.save_for_backward(xs, gu, act, gu_w, dn_w)
        ctx.cnt = cnt
        ctx.x_dtype = x.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        xs, gu, act, gu_w, dn_w = ctx.saved_tensors
        dy = dy.to(torch.bfloat16).contiguous()
        E = gu_w.shape[0]
        dx = torch.empty_like(xs)
        dgu_w = torch.zeros(gu_w.shape, dtype=torch.float32, device=xs.device)
        ddn_w = torch.zeros(dn_w.shape, dtype=torch.float32, device=xs.device)
        off = 0
        for e, n in enumerate(ctx.cnt):
            if n == 0:
                continue
            sl = slice(off, off + n)
            da = linear_dgrad(dy[sl], dn_w[e])
            linear_wgrad(dy[sl], act[sl], out=ddn_w[e])
            dgu = glu_bwd(gu[sl], da, SILU)
            linear_dgrad(dgu, gu_w[e], out=dx[sl])
            linear_wgrad(dgu, xs[sl], out=dgu_w[e])
            off += n
        return dx.to(ctx.x_dtype), None, dgu_w, ddn_w


def grouped_swiglu_ffn(x, counts, gate_up_proj, down_proj):
    if x.is_cuda:
        return _GroupedSwiGLU.apply(x, counts, gate_up_proj, down_proj)
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
