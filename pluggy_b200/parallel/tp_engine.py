"""Tensor- and sequence-parallel transformer sublayers on the sm_100a kernels.

The single-GPU engine (:mod:`pluggy_b200.models._engine`) runs a block as two
autograd Functions over this package's kernels. These are their tensor-parallel
forms (Megatron-style TP with sequence parallelism, the layout the reference's
roadmap describes in ``notes/ROADMAP.md:327-378``): the residual stream ``x`` is
sequence-sharded ([B * S / tp, D] fp32 per rank), the projections hold this
rank's heads / FFN columns, and every collective is one of the peer-memory
kernels of :mod:`pluggy_b200.comm.tp_fused`:

``TPAttnSublayer``
  h   = AG(RMSNorm(x))                 norm fused with the sequence all-gather
  qkv = h Wqkv_r^T                     tcgen05 GEMM, this rank's q|k|v heads
  q,k = RoPE(QKNorm(qkv)); o = FlashAttn(q, k, v)
  x'  = x + RS(o Wo_r^T)               GEMM whose epilogue reduce-scatters over NVLink
``TPMlpSublayer``
  h = AG(RMSNorm(x')); gu = h Wgu_r^T; a = act(g) * u; x'' = x' + RS(a Wd_r^T)

Backward: the incoming gradient is all-gathered once per sublayer (peer push),
the input-gradient GEMM of the first projection is the fused GEMM ->
reduce-scatter again, and the norm backward runs on this rank's rows. Weight
gradients stay local (sharded parameters); the norm and per-head q/k-norm weight
gradients are partial and are summed over the axis by
``TensorParallel.sync_replicated_grads``.
"""

from __future__ import annotations

import torch

from pluggy_b200.models._engine import AttnCfg, _grad_bf16, _norm_bwd_with_bf16
from pluggy_b200.ops import attention as _attn
from pluggy_b200.ops import norm as _norm
from pluggy_b200.ops.elementwise import glu_bwd, glu_fwd
from pluggy_b200.ops.gemm import linear_dgrad, linear_fwd, linear_wgrad


class TPAttnSublayer(torch.autograd.Function):
    """x [B*S/tp, D] fp32 -> x + RS(Attn_r(AG(RMSNorm(x)))) [B*S/tp, D] fp32."""

    @staticmethod
    def forward(ctx, x, n_w, wq, wk, wv, wo, qn_w, kn_w, lowp, cfg: AttnCfg, inv_freq, comm):
        w_qkv, w_o = lowp
        B, S, Hq, Hk, d = cfg.B, cfg.S, cfg.Hq, cfg.Hk, cfg.d
        n = comm.n
        D = x.shape[1]
        h, r = comm.norm_all_gather_seq(x.view(B, S // n, D), n_w, cfg.eps)
        h2 = h.view(B * S, D)
        qkv = linear_fwd(h2, w_qkv)
        q, k, rqk = _norm.qk_norm_rope_fwd(qkv, S=S, Hq=Hq, Hk=Hk, d=d,
                                           wq=qn_w if cfg.qk_norm else None,
                                           wk=kn_w if cfg.qk_norm else None,
                                           inv_freq=inv_freq, eps=cfg.qk_eps)
        v = qkv[:, (Hq + Hk) * d:].view(B, S, Hk, d)
        o, lse = _attn.attn_fwd(q.view(B, S, Hq, d), k.view(B, S, Hk, d), v,
                                causal=cfg.causal, window=cfg.window, scale=cfg.scale)
        y = comm.gemm_reduce_scatter(o.view(B, S, Hq * d), w_o)
        out = x + y.view(-1, D).float()
        ctx.save_for_backward(x, n_w, r, h2, qkv, q, k, rqk, o, lse, qn_w, kn_w, inv_freq)
        ctx.lowp, ctx.cfg, ctx.comm = lowp, cfg, comm
        return out

    @staticmethod
    def backward(ctx, dy):
        x, n_w, r, h2, qkv, q, k, rqk, o, lse, qn_w, kn_w, inv_freq = ctx.saved_tensors
        w_qkv, w_o = ctx.lowp
        cfg, comm = ctx.cfg, ctx.comm
        B, S, Hq, Hk, d = cfg.B, cfg.S, cfg.Hq, cfg.Hk, cfg.d
        n, D = comm.n, x.shape[1]
        T = B * S
        dy = dy.contiguous()
        dy_full = comm.all_gather_seq(_grad_bf16(dy).view(B, S // n, D)).view(T, D)
        o2 = o.view(T, Hq * d)
        do = linear_dgrad(dy_full, w_o)
        dWo = linear_wgrad(dy_full, o2)
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
        # input gradient of the q|k|v projection, reduce-scattered by the GEMM epilogue
        dh = comm.gemm_reduce_scatter(dqkv.view(B, S, W), w_qkv, w_mn_major=True).view(-1, D)
        dWqkv = linear_wgrad(dqkv, h2)
        dx, dnw = _norm_bwd_with_bf16(dh, x, n_w, r, dy)
        nq, nk = Hq * d, Hk * d
        return (dx, dnw, dWqkv[:nq], dWqkv[nq:nq + nk], dWqkv[nq + nk:], dWo, dqn, dkn,
                None, None, None, None)


class TPMlpSublayer(torch.autograd.Function):
    """x [B*S/tp, D] fp32 -> x + RS(Wd_r act(Wg_r h) * (Wu_r h)), h = AG(RMSNorm(x))."""

    @staticmethod
    def forward(ctx, x, n_w, wg, wu, wd, lowp, eps: float, kind: int, B: int, S: int, comm):
        w_gu, w_d = lowp
        n, D = comm.n, x.shape[1]
        h, r = comm.norm_all_gather_seq(x.view(B, S // n, D), n_w, eps)
        h2 = h.view(B * S, D)
        gu = linear_fwd(h2, w_gu)
        a = glu_fwd(gu, kind)
        y = comm.gemm_reduce_scatter(a.view(B, S, -1), w_d)
        out = x + y.view(-1, D).float()
        ctx.save_for_backward(x, n_w, r, h2, gu, a)
        ctx.lowp, ctx.kind, ctx.comm, ctx.BS = lowp, kind, comm, (B, S)
        return out

    @staticmethod
    def backward(ctx, dy):
        x, n_w, r, h2, gu, a = ctx.saved_tensors
        w_gu, w_d = ctx.lowp
        comm = ctx.comm
        B, S = ctx.BS
        n, D = comm.n, x.shape[1]
        dy = dy.contiguous()
        dy_full = comm.all_gather_seq(_grad_bf16(dy).view(B, S // n, D)).view(B * S, D)
        da = linear_dgrad(dy_full, w_d)
        dWd = linear_wgrad(dy_full, a)
        dgu = glu_bwd(gu, da, ctx.kind)
        dh = comm.gemm_reduce_scatter(dgu.view(B, S, -1), w_gu, w_mn_major=True).view(-1, D)
        dWgu = linear_wgrad(dgu, h2)
        dx, dnw = _norm_bwd_with_bf16(dh, x, n_w, r, dy)
        Fh = gu.shape[1] // 2
        return dx, dnw, dWgu[:Fh], dWgu[Fh:], dWd, None, None, None, None, None, None
