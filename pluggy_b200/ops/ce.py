"""Chunked fused linear + cross-entropy.

Parity: reference ``pluggy/loss/fused_linear_ce.py:31-136``. Per chunk of
``chunk_size`` rows: logits = h W^T, loss = lse - target logit (ignore_index
rows contribute 0), grad_logits = softmax - onehot; grad_h and grad_W are
computed in the FORWARD pass and stashed; backward scales them in place by
``grad_out / n_valid`` and hands them out (so a second backward raises).

CUDA path (all sm_100a kernels, no (chunk, V) fp32 tensor ever exists):
  1. logits chunk (bf16) = tcgen05 GEMM h_c W^T
  2. one CTA per row: online max/sum-exp, target gather, loss sum, and the
     gradient (softmax - onehot) written IN PLACE over the logits (bf16)
  3. grad_h_c = G_c W     (tcgen05 GEMM, B N-major)
  4. grad_W  += G_c^T h_c (tcgen05 GEMM, A and B M/N-major, fp32 accumulate
     fused into the epilogue)
"""

from __future__ import annotations

import torch

from pluggy_b200.ops._ext import ext
from pluggy_b200.ops.gemm import gemm


def _chunk_reference(h, w, labels, ignore_index):
    logits = (h @ w.t()).float()
    valid = labels != ignore_index
    safe = torch.where(valid, labels, 0).unsqueeze(1)
    lse = torch.logsumexp(logits, dim=-1)
    tgt = logits.gather(1, safe).squeeze(1)
    loss_sum = ((lse - tgt) * valid).sum()
    probs = torch.exp(logits - lse.unsqueeze(1)) * valid.unsqueeze(1)
    probs.scatter_add_(1, safe, -valid.float().unsqueeze(1))
    g = probs.to(h.dtype)
    return loss_sum, g @ w, g.t() @ h


class _FusedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, labels, ignore_index, chunk_size, w_lowp, softcap):
        N, D = hidden.shape
        dev = hidden.device
        n_valid = (labels != ignore_index).sum().clamp_min(1)
        need_w = weight.requires_grad
        if hidden.is_cuda:
            h = hidden.to(torch.bfloat16).contiguous()
            w = w_lowp if w_lowp is not None else weight.to(torch.bfloat16)
            V = w.shape[0]
            # per-row losses, summed once in a fixed order (deterministic)
            row_loss = torch.empty(N, dtype=torch.float32, device=dev)
            grad_h = torch.empty((N, D), dtype=torch.bfloat16, device=dev)
            # the first chunk's wgrad GEMM writes grad_w (beta = 0), later ones accumulate
            grad_w = torch.empty((V, D), dtype=torch.float32, device=dev) if need_w else None
            logits = torch.empty((min(chunk_size, N), V), dtype=torch.bfloat16, device=dev)
            lab = labels.contiguous()
            for s in range(0, N, chunk_size):
                e = min(s + chunk_size, N)
                lg = logits[: e - s]
                gemm(h[s:e], w, out=lg)
                ext().ce_rows(lg, lab[s:e], int(ignore_index), 1.0, float(softcap or 0.0), None,
                              None, None, row_loss[s:e])
                gemm(lg, w, b_mn_major=True, out=grad_h[s:e])
                if need_w:
                    gemm(lg, h[s:e], a_mn_major=True, b_mn_major=True, out=grad_w,
                         addend=grad_w if s > 0 else None, beta=1.0)
            if N == 0 and grad_w is not None:
                grad_w.zero_()
            loss_sum = row_loss.sum()
            grad_h = grad_h.to(hidden.dtype)
        else:
            assert not softcap, "softcap on the fused-CE path is a CUDA-only option"
            w = weight.to(hidden.dtype)
            loss_sum = torch.zeros((), dtype=torch.float32, device=dev)
            grad_h = torch.empty_like(hidden)
            grad_w = torch.zeros_like(weight, dtype=torch.float32) if need_w else None
            for s in range(0, N, chunk_size):
                e = min(s + chunk_size, N)
                ls, gh, gw = _chunk_reference(hidden[s:e], w, labels[s:e], ignore_index)
                loss_sum += ls
                grad_h[s:e] = gh
                if grad_w is not None:
                    grad_w += gw
        ctx.n_valid = n_valid
        ctx.grad_hidden = grad_h
        ctx.grad_weight = grad_w
        ctx.w_dtype = weight.dtype
        return loss_sum / n_valid

    @staticmethod
    def backward(ctx, grad_out):
        if ctx.n_valid is None:
            raise RuntimeError(
                "fused_linear_cross_entropy: backward called twice; the stashed grads are "
                "consumed in place on the first call, so retain_graph does not work through this op")
        gh, gw = ctx.grad_hidden, ctx.grad_weight
        scale = grad_out / ctx.n_valid
        ctx.grad_hidden = ctx.grad_weight = ctx.n_valid = None
        gh.mul_(scale.to(gh.dtype))
        if gw is not None:
            gw.mul_(scale)
            if gw.dtype != ctx.w_dtype:
                gw = gw.to(ctx.w_dtype)
        return gh, gw, None, None, None, None, None


def fused_linear_cross_entropy(hidden, weight, labels, ignore_index: int = -100,
                               chunk_size: int = 1024, *, weight_lowp=None, softcap=None):
    """Mean CE of ``hidden @ weight^T`` against ``labels`` without full logits."""
    if hidden.dim() == 3:
        hidden = hidden.reshape(-1, hidden.shape[-1])
        labels = labels.reshape(-1)
    return _FusedLinearCE.apply(hidden, weight, labels, ignore_index, chunk_size, weight_lowp,
                                softcap)
