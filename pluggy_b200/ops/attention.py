"""Flash attention (causal / sliding-window, GQA) on the sm_100a tensor cores.

``flash_attention(q, k, v, causal=True, window=0, scale=None)`` takes
``[B, S, H, d]`` tensors (heads packed, any token stride: k and v may be column
views of a fused QKV projection) and returns ``o [B, S, Hq, d]``. It replaces the
reference's ``F.scaled_dot_product_attention(is_causal=True, enable_gqa=True)``
(``pluggy/models/qwen3/qwen3.py:166-181``) and its dense S x S sliding-window
masks (``pluggy/models/olmo3/olmo3.py:109-143``).

CPU tensors use the same math through SDPA (the test oracle).
"""

from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from pluggy_b200.ops._ext import ext, status_word


def attention_reference(q, k, v, causal=True, window=0, scale=None):
    """fp32 math on [B, S, H, d] inputs; returns [B, S, Hq, d] in q's dtype."""
    B, S, Hq, d = q.shape
    Hk = k.shape[2]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    if Hk != Hq:
        kf = kf.repeat_interleave(Hq // Hk, dim=1)
        vf = vf.repeat_interleave(Hq // Hk, dim=1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    i = torch.arange(S, device=q.device)
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device)
    if causal:
        mask &= i[None, :] <= i[:, None]
    if window and window > 0:
        mask &= (i[:, None] - i[None, :]) < window
    s = s.masked_fill(~mask, float("-inf"))
    o = torch.softmax(s, dim=-1) @ vf
    return o.transpose(1, 2).to(q.dtype)


def attn_fwd(q, k, v, *, causal=True, window=0, scale=None):
    B, S, Hq, d = q.shape
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    o = torch.empty((B, S, Hq, d), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty((B, Hq, S), dtype=torch.float32, device=q.device)
    ext().attn_fwd(q, k, v, o, lse, float(scale), bool(causal), int(window or 0),
                   status_word(q.device))
    return o, lse


def _attn_bwd_d64_padded(q, k, v, o, lse, do, causal, window, scale, dq, dk, dv):
    """head_dim 64 through the head_dim-128 backward kernel (``PLG_ATTN_D64_PAD=1``): q,
    k, v, o and dO are zero-padded to 128 channels (the padded channels add 0 to every
    score and to rowsum(dO * O), so lse and the softmax are unchanged) and the
    gradients' first 64 channels are the result. Kept as a cross-check of the native
    head_dim-64 instance of the pipelined kernel, which is the default."""
    pad = [F.pad(t, (0, 64)) for t in (q, k, v, o, do)]
    dq_p, dk_p, dv_p = attn_bwd(*pad[:4], lse, pad[4], causal=causal, window=window, scale=scale)
    outs = []
    for g, out in ((dq_p, dq), (dk_p, dk), (dv_p, dv)):
        if out is None:
            outs.append(g[..., :64].contiguous())
        else:
            out.copy_(g[..., :64])
            outs.append(out)
    return tuple(outs)


def attn_bwd(q, k, v, o, lse, do, *, causal=True, window=0, scale=None, dq=None, dk=None, dv=None,
             trace=None):
    """Backward of flash attention: one pipelined kernel for head_dim 64 and 128 (the
    earlier single-group head_dim-64 kernel stays selectable with
    ``PLG_ATTN_BWD64=group``). ``trace`` (int64 [12, 256] on the device) receives
    SM-clock stamps of the first CTA's pipeline events per step, for timeline analysis
    of the kernel."""
    B, S, Hq, d = q.shape
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    if d == 64 and trace is None and os.environ.get("PLG_ATTN_D64_PAD", "0") == "1":
        return _attn_bwd_d64_padded(q, k, v, o, lse, do, causal, window, scale, dq, dk, dv)
    dq = torch.empty_like(q, memory_format=torch.contiguous_format) if dq is None else dq
    dk = torch.empty(k.shape, dtype=k.dtype, device=k.device) if dk is None else dk
    dv = torch.empty(v.shape, dtype=v.dtype, device=v.device) if dv is None else dv
    do = do.contiguous()
    dq_acc = torch.empty((B, S, Hq, d), dtype=torch.float32, device=q.device)
    # [B * Hq][2][S rounded up to 64]: -lse*log2(e) and -scale*rowsum(dO*O)
    delta = torch.empty(B * Hq * 2 * ((S + 63) // 64 * 64), dtype=torch.float32, device=q.device)
    ext().attn_bwd(q, k, v, o, lse, do, dq, dk, dv, dq_acc, delta, float(scale), bool(causal),
                   int(window or 0), status_word(q.device), trace)
    return dq, dk, dv


class _FlashAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, window, scale):
        o, lse = attn_fwd(q, k, v, causal=causal, window=window, scale=scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.cfg = (causal, window, scale)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        causal, window, scale = ctx.cfg
        dq, dk, dv = attn_bwd(q, k, v, o, lse, do.contiguous(), causal=causal, window=window,
                              scale=scale)
        return dq, dk, dv, None, None, None


def supported(q: torch.Tensor) -> bool:
    return q.is_cuda and q.shape[-1] in (64, 128)


def flash_attention(q, k, v, causal: bool = True, window: int = 0, scale: float | None = None):
    if q.is_cuda:
        if not supported(q):
            raise NotImplementedError(
                f"sm_100a flash attention supports head_dim 64/128, got {q.shape[-1]}")
        return _FlashAttention.apply(q, k, v, causal, window, scale)
    return attention_reference(q, k, v, causal, window, scale)


def sdpa_bhsd(q, k, v, causal=True, window=0, scale=None):
    """Convenience for [B, H, S, d] callers (the reference layout)."""
    o = flash_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), causal, window, scale)
    return o.transpose(1, 2)


def sdpa_masked(q, k, v, attn_mask, scale=None):
    """Arbitrary boolean-mask attention ([B,H,S,d]); used only by the padded eval path."""
    Hq, Hk = q.shape[1], k.shape[1]
    return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, scale=scale,
                                          enable_gqa=Hq != Hk)
