"""RMSNorm and fused QK-norm + RoPE.

Public ``rms_norm(x, weight=None, eps=1e-6)`` matches the reference's free
function (``pluggy/kernels/rms_norm.py:13-29``: fp32 math, optional weight,
output in the input dtype) and is differentiable. On CUDA forward and backward
are this package's sm_100a kernels; on CPU it is the same math in eager torch.

The model fast path calls the raw launchers (``rmsnorm_fwd``/``rmsnorm_bwd``,
``qk_norm_rope_fwd``/``qk_norm_rope_bwd``) inside its own autograd Functions.
"""

from __future__ import annotations

import weakref

import torch

from pluggy_b200.ops._ext import ext, status_word

DW_BLOCKS = 592  # 4 CTAs per SM on 148 SMs: dw partial sums reduced by the caller


def _colsum(part: torch.Tensor) -> torch.Tensor:
    """Deterministic column sum of the per-block dw partials [DW_BLOCKS, D]."""
    out = torch.empty(part.shape[1], dtype=torch.float32, device=part.device)
    ext().colsum(part, out)
    return out


def rms_norm_reference(x, weight=None, eps=1e-6):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    if weight is not None:
        y = y * weight.float()
    return y.to(x.dtype)


def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor | None, eps: float, out_dtype=torch.bfloat16):
    """Returns (y, rstd) with y [rows, D] in ``out_dtype`` and rstd fp32 [rows]."""
    D = x.shape[-1]
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    rstd = torch.empty(x.numel() // D, dtype=torch.float32, device=x.device)
    ext().rmsnorm_fwd(x, w, y, rstd, float(eps))
    return y, rstd


def rmsnorm_bwd(dy, x, w, rstd, *, dres=None, want_f32=True, want_bf16=False, want_dw=True):
    """Returns (dx_f32 | None, dx_bf16 | None, dw | None)."""
    D = x.shape[-1]
    dxf = torch.empty(x.shape, dtype=torch.float32, device=x.device) if want_f32 else None
    dxb = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device) if want_bf16 else None
    part = (torch.empty((DW_BLOCKS, D), dtype=torch.float32, device=x.device)
            if (want_dw and w is not None) else None)
    ext().rmsnorm_bwd(dy, x, w, rstd, dres, dxf, dxb, part)
    dw = _colsum(part) if part is not None else None
    return dxf, dxb, dw


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        xc = x.contiguous()
        y, rstd = rmsnorm_fwd(xc, weight, eps, out_dtype=x.dtype)
        ctx.save_for_backward(xc, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        want_bf16 = x.dtype == torch.bfloat16
        dxf, dxb, dw = rmsnorm_bwd(dy.contiguous(), x, w, rstd, want_f32=not want_bf16,
                                   want_bf16=want_bf16, want_dw=w is not None and ctx.needs_input_grad[1])
        dx = dxb if want_bf16 else dxf.to(x.dtype)
        return dx, dw, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    if x.is_cuda and x.shape[-1] % 128 == 0 and x.dtype in (torch.float32, torch.bfloat16):
        return _RMSNorm.apply(x, weight, eps)
    return rms_norm_reference(x, weight, eps)


_ROPE_TABLES: dict = {}


def rope_table(inv_freq: torch.Tensor, S: int, rot_dim: int) -> torch.Tensor:
    """fp32 [S, 2, rot_dim/2] table of cos and sin of ``pos * inv_freq`` (the same
    fp32 products the reference's rotary embedding takes cos/sin of), built once per
    (frequencies, length) on the device so the kernels skip per-token sincos."""
    # keyed on the frequency tensor object itself (a weak reference guards against a
    # new tensor reusing a freed one's id or storage)
    key = (id(inv_freq), inv_freq._version, int(S), int(rot_dim))
    hit = _ROPE_TABLES.get(key)
    if hit is not None and hit[0]() is inv_freq:
        return hit[1]
    pos = torch.arange(S, dtype=torch.float32, device=inv_freq.device)
    ang = torch.outer(pos, inv_freq[: rot_dim // 2].float())
    t = torch.stack((ang.cos(), ang.sin()), dim=1).contiguous()
    if len(_ROPE_TABLES) > 16:
        _ROPE_TABLES.clear()
    _ROPE_TABLES[key] = (weakref.ref(inv_freq), t)
    return t


def qk_norm_rope_fwd(qkv, *, S, Hq, Hk, d, wq, wk, inv_freq, positions=None, eps=1e-6,
                     rot_dim=None, k_offset=None):
    """Normalise+rotate q and k of a fused projection ``qkv [T, (Hq+2Hk)*d]``.

    ``positions`` (int32 [T], optional) must stay below ``S`` (the cos/sin table length).

    Returns (q [T,Hq,d], k [T,Hk,d], rstd [T, Hq+Hk]); v stays in ``qkv``.
    """
    T = qkv.shape[0]
    q = torch.empty((T, Hq, d), dtype=torch.bfloat16, device=qkv.device)
    k = torch.empty((T, Hk, d), dtype=torch.bfloat16, device=qkv.device)
    rstd = torch.empty((T, Hq + Hk), dtype=torch.float32, device=qkv.device)
    rd = int(d if rot_dim is None else rot_dim)
    table = rope_table(inv_freq, S, rd) if rd > 0 else None
    ext().qk_norm_rope_fwd(qkv, q, k, rstd, wq, wk, inv_freq, positions, int(S), int(Hq), int(Hk),
                           int(d), rd, float(eps), int(Hq if k_offset is None else k_offset), table,
                           status_word(qkv.device))
    return q, k, rstd


def qk_norm_rope_bwd(qkv, rstd, dq, dk, dqkv, *, S, Hq, Hk, d, wq, wk, inv_freq, positions=None,
                     eps=1e-6, rot_dim=None, k_offset=None):
    """Writes dq/dk (pre-norm) into the q and k columns of ``dqkv``; returns (dwq, dwk)."""
    pq = torch.empty((DW_BLOCKS, d), dtype=torch.float32, device=qkv.device) if wq is not None else None
    pk = torch.empty((DW_BLOCKS, d), dtype=torch.float32, device=qkv.device) if wk is not None else None
    rd = int(d if rot_dim is None else rot_dim)
    table = rope_table(inv_freq, S, rd) if rd > 0 else None
    ext().qk_norm_rope_bwd(qkv, rstd, wq, wk, inv_freq, positions, int(S), int(Hq), int(Hk), int(d),
                           rd, float(eps), int(Hq if k_offset is None else k_offset), dq, dk, dqkv,
                           pq, pk, DW_BLOCKS, table, status_word(qkv.device))
    return (_colsum(pq) if pq is not None else None), (_colsum(pk) if pk is not None else None)
