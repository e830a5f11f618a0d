"""Fused transformer sublayers on the sm_100a kernels (the CUDA training path).

Each sublayer is ONE autograd Function whose forward and backward are a fixed
sequence of this package's kernels, so a block runs no PyTorch math on the hot
path and saves exactly what its backward needs:

``AttnSublayer`` (pre-norm attention, residual fused into the o-proj epilogue)
  h   = RMSNorm(x)                         rmsnorm kernel, bf16 out
  qkv = h Wqkv^T                           tcgen05 GEMM, q|k|v in one product
  q,k = RoPE(QKNorm(qkv))                  fused qk-norm+rope kernel
  o   = FlashAttn(q, k, v)                 tcgen05 attention (v read in place)
  x'  = x + o Wo^T                         tcgen05 GEMM, fp32 residual epilogue
``MlpSublayer`` (pre-norm GLU MLP)
  h   = RMSNorm(x'); gu = h Wgu^T (gate|up in one GEMM); a = act(g) * u
  x'' = x' + a Wd^T                        fp32 residual epilogue

Backward mirrors it with dgrad/wgrad GEMMs (weight grads straight out of the
fp32 accumulator), the attention backward kernel and the norm backward kernels
(which fuse the residual-gradient add and emit the bf16 copy the next GEMM
reads). The residual stream stays fp32 like the reference's autocast path
(fp32 embedding output + bf16 sublayer outputs).

Parity: reference ``pluggy/models/qwen3/qwen3.py:73-248`` (GQA with per-head
q/k norm, SwiGLU, pre-norm block), ``pluggy/models/llama3/llama3.py`` (no qk
norm), ``pluggy/models/qwen3_moe/qwen3_moe.py`` (same attention).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from pluggy_b200.ops import attention as _attn
from pluggy_b200.ops import norm as _norm
from pluggy_b200.ops._ext import ext
from pluggy_b200.ops.elementwise import glu_bwd, glu_fwd
from pluggy_b200.ops.gemm import linear_dgrad, linear_fwd, linear_wgrad


@dataclass
class AttnCfg:
    B: int
    S: int
    Hq: int
    Hk: int
    d: int
    eps: float
    qk_eps: float
    causal: bool = True
    window: int = 0
    scale: float | None = None
    qk_norm: bool = True


def _to_bf16(x: torch.Tensor) -> torch.Tensor:
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    ext().cast_f32_bf16(x.contiguous(), y)
    return y


def _grad_bf16(dy: torch.Tensor) -> torch.Tensor:
    """bf16 copy of the residual-stream gradient. The norm backward of the sublayer
    above writes it next to the fp32 gradient and hangs it on that tensor; autograd
    hands the same tensor object down when nothing was summed into it, otherwise
    (or for the first sublayer) it is cast here."""
    lp = getattr(dy, "_plg_bf16", None)
    if lp is not None and lp.shape == dy.shape:
        return lp
    return _to_bf16(dy)


def _norm_bwd_with_bf16(dh, x, n_w, r, dy):
    dx, dxb, dnw = _norm.rmsnorm_bwd(dh, x, n_w, r, dres=dy, want_f32=True, want_bf16=True)
    dx._plg_bf16 = dxb
    return dx, dnw


class AttnSublayer(torch.autograd.Function):
    """x [T,H] fp32 -> x + Attn(RMSNorm(x)) [T,H] fp32."""

    @staticmethod
    def forward(ctx, x, n_w, wq, wk, wv, wo, qn_w, kn_w, lowp, cfg: AttnCfg, inv_freq):
        w_qkv, w_o = lowp
        T = x.shape[0]
        Hq, Hk, d = cfg.Hq, cfg.Hk, cfg.d
        h, r = _norm.rmsnorm_fwd(x, n_w, cfg.eps)
        qkv = linear_fwd(h, w_qkv)
        q, k, rqk = _norm.qk_norm_rope_fwd(qkv, S=cfg.S, Hq=Hq, Hk=Hk, d=d,
                                           wq=qn_w if cfg.qk_norm else None,
                                           wk=kn_w if cfg.qk_norm else None,
                                           inv_freq=inv_freq, eps=cfg.qk_eps)
        v = qkv[:, (Hq + Hk) * d:].view(cfg.B, cfg.S, Hk, d)
        o, lse = _attn.attn_fwd(q.view(cfg.B, cfg.S, Hq, d), k.view(cfg.B, cfg.S, Hk, d), v,
                                causal=cfg.causal, window=cfg.window, scale=cfg.scale)
        o2 = o.view(T, Hq * d)
        y = linear_fwd(o2, w_o, out_dtype=torch.float32, residual=x)
        ctx.save_for_backward(x, n_w, r, h, qkv, q, k, rqk, o, lse, qn_w, kn_w, inv_freq)
        ctx.lowp = lowp
        ctx.cfg = cfg
        return y

    @staticmethod
    def backward(ctx, dy):
        x, n_w, r, h, qkv, q, k, rqk, o, lse, qn_w, kn_w, inv_freq = ctx.saved_tensors
        w_qkv, w_o = ctx.lowp
        cfg = ctx.cfg
        Hq, Hk, d, B, S = cfg.Hq, cfg.Hk, cfg.d, cfg.B, cfg.S
        T = x.shape[0]
        dy = dy.contiguous()
        dy_b = _grad_bf16(dy)
        o2 = o.view(T, Hq * d)
        do = linear_dgrad(dy_b, w_o)
        dWo = linear_wgrad(dy_b, o2)
        W = qkv.shape[1]
        dqkv = torch.empty((T, W), dtype=torch.bfloat16, device=x.device)
        v = qkv[:, (Hq + Hk) * d:].view(B, S, Hk, d)
        dv = dqkv[:, (Hq + Hk) * d:].view(B, S, Hk, d)
        dq, dk, _ = _attn.attn_bwd(q.view(B, S, Hq, d), k.view(B, S, Hk, d), v, o, lse,
                                   do.view(B, S, Hq, d), causal=cfg.causal, window=cfg.window,
                                   scale=cfg.scale, dv=dv)
        dqn, dkn = _norm.qk_norm_rope_bwd(qkv, rqk, dq, dk, dqkv, S=S, Hq=Hq, Hk=Hk, d=d,
                                          wq=qn_w if cfg.qk_norm else None,
                                          wk=kn_w if cfg.qk_norm else None,
                                          inv_freq=inv_freq, eps=cfg.qk_eps)
        dh = linear_dgrad(dqkv, w_qkv)
        dWqkv = linear_wgrad(dqkv, h)
        dx, dnw = _norm_bwd_with_bf16(dh, x, n_w, r, dy)
        nq, nk = Hq * d, Hk * d
        return (dx, dnw, dWqkv[:nq], dWqkv[nq:nq + nk], dWqkv[nq + nk:], dWo, dqn, dkn,
                None, None, None)


class MlpSublayer(torch.autograd.Function):
    """x [T,H] fp32 -> x + Wd act(Wg h) * (Wu h), h = RMSNorm(x)."""

    @staticmethod
    def forward(ctx, x, n_w, wg, wu, wd, lowp, eps: float, kind: int):
        w_gu, w_d = lowp
        h, r = _norm.rmsnorm_fwd(x, n_w, eps)
        gu = linear_fwd(h, w_gu)
        a = glu_fwd(gu, kind)
        y = linear_fwd(a, w_d, out_dtype=torch.float32, residual=x)
        ctx.save_for_backward(x, n_w, r, h, gu, a)
        ctx.lowp = lowp
        ctx.kind = kind
        return y

    @staticmethod
    def backward(ctx, dy):
        x, n_w, r, h, gu, a = ctx.saved_tensors
        w_gu, w_d = ctx.lowp
        dy = dy.contiguous()
        dy_b = _grad_bf16(dy)
        da = linear_dgrad(dy_b, w_d)
        dWd = linear_wgrad(dy_b, a)
        dgu = glu_bwd(gu, da, ctx.kind)
        dh = linear_dgrad(dgu, w_gu)
        dWgu = linear_wgrad(dgu, h)
        dx, dnw = _norm_bwd_with_bf16(dh, x, n_w, r, dy)
        Fh = gu.shape[1] // 2
        return dx, dnw, dWgu[:Fh], dWgu[Fh:], dWd, None, None, None


class Embedding(torch.autograd.Function):
    """ids [T] -> w[ids] * scale as fp32 [T, D]; backward sums each id's rows in token
    order (ids sorted once; deterministic, no atomics)."""

    @staticmethod
    def forward(ctx, ids, w, scale: float):
        ids = ids.reshape(-1).contiguous()
        out = torch.empty((ids.numel(), w.shape[1]), dtype=torch.float32, device=w.device)
        ext().embedding_fwd(ids, w.detach().contiguous(), out, float(scale))
        ctx.save_for_backward(ids)
        ctx.shape = w.shape
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        dw = torch.zeros(ctx.shape, dtype=torch.float32, device=dy.device)
        ids_sorted, pos = torch.sort(ids, stable=True)
        ext().embedding_bwd_sorted(ids_sorted, pos, dy.contiguous().float(), dw, float(ctx.scale))
        return None, dw, None


class FinalNorm(torch.autograd.Function):
    """RMSNorm of the fp32 residual to a bf16 hidden (input of the LM head)."""

    @staticmethod
    def forward(ctx, x, w, eps: float):
        h, r = _norm.rmsnorm_fwd(x, w, eps)
        ctx.save_for_backward(x, w, r)
        return h

    @staticmethod
    def backward(ctx, dh):
        x, w, r = ctx.saved_tensors
        dx, _, dw = _norm.rmsnorm_bwd(dh.contiguous(), x, w, r, want_f32=True)
        return dx, dw, None
