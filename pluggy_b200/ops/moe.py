"""Dropless top-k MoE expert FFN.

Parity: reference ``pluggy/kernels/moe.py:38-168`` (``moe_expert_ffn``: sort the
(token, expert) pairs by expert, per-expert SwiGLU FFN with packed weights
``gate_up_proj (E, 2I, H)`` / ``down_proj (E, H, I)``, scale by the routing
weight, scatter-add back). The loop and grouped forms give identical results.

CUDA path: pairs are sorted once by expert; each of the FFN's projections is
ONE launch of this package's grouped tcgen05 GEMM over all experts
(:func:`pluggy_b200.ops.grouped.grouped_swiglu_ffn`: a device-computed padded
per-expert row layout, no host synchronisation) and the GLU is the sm_100a
kernel; the combine is a scatter-add of the route-weighted rows.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from pluggy_b200.ops.elementwise import swiglu_mul


def expert_histogram(idx: torch.Tensor, n: int) -> torch.Tensor:
    """int64 [n]: how many entries of ``idx`` (values in [0, n)) equal each value.
    A scatter-add, so it stays on the device: ``torch.bincount`` on CUDA reads the
    input's minimum and maximum back to the host to size its output."""
    flat = idx.reshape(-1).to(torch.int64)
    out = torch.zeros(n, dtype=torch.int64, device=idx.device)
    return out.scatter_add_(0, flat, torch.ones_like(flat))


def _expert_ffn_loop(hidden, top_indices, top_weights, gate_up_proj, down_proj):
    T, H = hidden.shape
    E = gate_up_proj.shape[0]
    out = torch.zeros(T, H, device=hidden.device, dtype=hidden.dtype)
    mask = F.one_hot(top_indices, num_classes=E).permute(2, 1, 0)  # (E, K, T)
    hit = mask.sum(dim=(-1, -2)).nonzero(as_tuple=False).flatten()
    gu = gate_up_proj.to(hidden.dtype)
    dn = down_proj.to(hidden.dtype)
    for e in hit.tolist():
        k_pos, tok = torch.where(mask[e])
        if tok.numel() == 0:
            continue
        g, u = F.linear(hidden[tok], gu[e]).chunk(2, dim=-1)
        y = F.linear(swiglu_mul(g, u), dn[e]) * top_weights[tok, k_pos, None]
        out.index_add_(0, tok, y.to(out.dtype))
    return out


def _expert_ffn_sorted(hidden, top_indices, top_weights, gate_up_proj, down_proj, gu_lowp=None,
                       dn_lowp=None):
    from pluggy_b200.ops.grouped import grouped_swiglu_ffn

    T, H = hidden.shape
    E = gate_up_proj.shape[0]
    K = top_indices.shape[1]
    tok = torch.arange(T, device=hidden.device).unsqueeze(1).expand(T, K).reshape(-1)
    exp = top_indices.reshape(-1)
    w = top_weights.reshape(-1)
    order = torch.argsort(exp, stable=True)
    s_tok, s_w, s_exp = tok[order], w[order], exp[order]
    counts = expert_histogram(exp, E)
    x = hidden[s_tok]
    y = grouped_swiglu_ffn(x, s_exp, counts, gate_up_proj, down_proj, gu_lowp, dn_lowp)
    y = y * s_w.unsqueeze(1).to(y.dtype)
    out = torch.zeros(T, H, device=hidden.device, dtype=y.dtype)
    out.index_add_(0, s_tok, y)
    return out.to(hidden.dtype)


def moe_expert_ffn(hidden, top_indices, top_weights, gate_up_proj, down_proj, *,
                   use_grouped_mm: bool | None = None, gu_lowp=None, dn_lowp=None):
    """Dropless top-k expert FFN; ``use_grouped_mm`` None = auto (CUDA -> sorted grouped path)."""
    assert hidden.dim() == 2 and top_indices.shape == top_weights.shape
    assert top_indices.shape[0] == hidden.shape[0]
    assert gate_up_proj.dim() == 3 and down_proj.dim() == 3
    if use_grouped_mm is None:
        use_grouped_mm = hidden.is_cuda
    if use_grouped_mm:
        return _expert_ffn_sorted(hidden, top_indices, top_weights, gate_up_proj, down_proj,
                                  gu_lowp, dn_lowp)
    return _expert_ffn_loop(hidden, top_indices, top_weights, gate_up_proj, down_proj)
