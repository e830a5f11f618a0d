"""Qwen3-MoE: Qwen3 attention + dropless top-k sparse MLP.

Parity: reference ``pluggy/models/qwen3_moe/qwen3_moe.py:140-444``:

* router: fp32 softmax over ``F.linear(h, W_router)``, top-k, optional
  renormalisation; the router weight is a bare Parameter initialised to zeros
  and ``init_weights`` leaves it there (it only draws ``nn.Linear`` /
  ``nn.Embedding`` weights and the packed experts), as in the reference;
* packed experts ``gate_up_proj (E, 2I, H)`` / ``down_proj (E, H, I)``;
* dense blocks from ``decoder_sparse_step`` / ``mlp_only_layers``;
* Switch load-balance loss and ST-MoE z-loss over the step's router logits,
  ``aux_loss()`` returns their weighted sum (None when no sparse layer ran);
* ``last_tokens_per_expert`` per-expert token counts for logging.

CUDA path: the attention sublayer is the fused ``_engine.AttnSublayer``; the
sparse MLP composes this package's kernels (RMSNorm, router GEMM, one grouped
tcgen05 GEMM launch per expert projection over all experts + the GLU kernel). Under expert parallelism the ``experts`` module is
replaced by ``pluggy_b200.parallel.expert_parallel.EPExperts``.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from pluggy_b200.models import _engine
from pluggy_b200.models.common import (GQAttention, RotaryEmbedding, SwiGLU, default_ffn_dim,
                                       norm_eps, position_ids_for)
from pluggy_b200.models.qwen3 import Qwen3TransformerBlock
from pluggy_b200.ops.linear import WeightCache, linear
from pluggy_b200.ops.moe import expert_histogram, moe_expert_ffn


class _RouterTopK(torch.autograd.Function):
    """Softmax (fp32) + top-k + optional renormalisation in one sm_100a kernel launch;
    the backward is the chain rule through the renormalisation and the softmax."""

    @staticmethod
    def forward(ctx, logits, k: int, renorm: bool):
        from pluggy_b200.ops._ext import ext

        lg = logits.contiguous()
        T, E = lg.shape
        probs = torch.empty((T, E), dtype=torch.float32, device=lg.device)
        w = torch.empty((T, k), dtype=torch.float32, device=lg.device)
        idx = torch.empty((T, k), dtype=torch.int64, device=lg.device)
        ext().router_topk(lg, k, renorm, probs, w, idx)
        ctx.save_for_backward(probs, w, idx)
        ctx.renorm, ctx.dtype = renorm, logits.dtype
        ctx.mark_non_differentiable(idx)
        return w, idx

    @staticmethod
    def backward(ctx, dw, _didx):
        probs, w, idx = ctx.saved_tensors
        dw = dw.float()
        if ctx.renorm:
            # w = p_sel / S, S = sum of the selected p: dL/dp_sel = (dw - <dw, w>) / S
            s = probs.gather(1, idx).sum(-1, keepdim=True)
            dsel = (dw - (dw * w).sum(-1, keepdim=True)) / s
        else:
            dsel = dw
        dp = torch.zeros_like(probs).scatter_add_(1, idx, dsel)
        dlogits = probs * (dp - (dp * probs).sum(-1, keepdim=True))
        return dlogits.to(ctx.dtype), None, None


class Qwen3MoeTopKRouter(nn.Module):
    def __init__(self, emb_dim: int, num_experts: int, top_k: int, norm_topk_prob: bool = True):
        super().__init__()
        assert 1 <= top_k <= num_experts
        self.top_k, self.num_experts, self.norm_topk_prob = top_k, num_experts, norm_topk_prob
        self.weight = nn.Parameter(torch.zeros(num_experts, emb_dim))

    def forward(self, h):
        logits = linear(h, self.weight) if h.is_cuda else F.linear(h, self.weight)
        E = logits.shape[-1]
        if logits.is_cuda and E % 32 == 0 and E <= 512 and self.top_k <= min(32, E):
            w, idx = _RouterTopK.apply(logits, self.top_k, self.norm_topk_prob)
            return logits, w.to(h.dtype), idx
        probs = F.softmax(logits, dim=-1, dtype=torch.float32)
        w, idx = torch.topk(probs, self.top_k, dim=-1)
        if self.norm_topk_prob:
            w = w / w.sum(dim=-1, keepdim=True)
        return logits, w.to(h.dtype), idx


class Qwen3MoeExperts(nn.Module):
    def __init__(self, emb_dim: int, moe_ffn_dim: int, num_experts: int):
        super().__init__()
        self.num_experts, self.emb_dim, self.moe_ffn_dim = num_experts, emb_dim, moe_ffn_dim
        self.gate_up_proj = nn.Parameter(torch.empty(num_experts, 2 * moe_ffn_dim, emb_dim))
        self.down_proj = nn.Parameter(torch.empty(num_experts, emb_dim, moe_ffn_dim))

    def forward(self, h, top_indices, top_weights):
        gu_lp = dn_lp = None
        cache = getattr(self, "weight_cache", None)
        if cache is not None and h.is_cuda:
            gu_lp, dn_lp = cache.get(self.gate_up_proj), cache.get(self.down_proj)
        return moe_expert_ffn(h, top_indices, top_weights, self.gate_up_proj, self.down_proj,
                              gu_lowp=gu_lp, dn_lowp=dn_lp)


class Qwen3MoeSparseMLP(nn.Module):
    def __init__(self, emb_dim, moe_ffn_dim, num_experts, top_k, norm_topk_prob=True):
        super().__init__()
        self.router = Qwen3MoeTopKRouter(emb_dim, num_experts, top_k, norm_topk_prob)
        self.experts = Qwen3MoeExperts(emb_dim, moe_ffn_dim, num_experts)
        self.last_router_logits: torch.Tensor | None = None
        self.last_top_idx: torch.Tensor | None = None

    def forward(self, x):
        shp = x.shape
        flat = x.reshape(-1, shp[-1])
        logits, w, idx = self.router(flat)
        self.last_router_logits = logits
        self.last_top_idx = idx.detach()
        return self.experts(flat, idx, w).reshape(shp)


class Qwen3MoeTransformerBlock(Qwen3TransformerBlock):
    def __init__(self, num_heads, emb_dim, num_kv_heads, head_dim, *, use_moe: bool,
                 ffn_dim=None, moe_ffn_dim=None, num_experts=128, top_k=8, norm_topk_prob=True):
        nn.Module.__init__(self)
        self.gqa = GQAttention(num_heads, emb_dim, num_kv_heads, head_dim, qk_norm=True)
        self.norm1 = nn.RMSNorm(emb_dim)
        self.norm2 = nn.RMSNorm(emb_dim)
        self.use_moe = use_moe
        if use_moe:
            assert moe_ffn_dim is not None, "moe_ffn_dim required for sparse layers"
            self.ffn = Qwen3MoeSparseMLP(emb_dim, moe_ffn_dim, num_experts, top_k, norm_topk_prob)
        else:
            self.ffn = SwiGLU(emb_dim, ffn_dim if ffn_dim is not None else default_ffn_dim(emb_dim))

    def fused_forward(self, x, cache: WeightCache, cfg, inv_freq, idx: int):
        if not self.use_moe:
            return super().fused_forward(x, cache, cfg, inv_freq, idx)
        g = self.gqa
        w_qkv = cache.get_cat([g.q_proj.weight, g.k_proj.weight, g.v_proj.weight], f"b{idx}.qkv")
        w_o = cache.get(g.o_proj.weight)
        x = _engine.AttnSublayer.apply(x, self.norm1.weight, g.q_proj.weight, g.k_proj.weight,
                                       g.v_proj.weight, g.o_proj.weight, g.q_norm.weight,
                                       g.k_norm.weight, (w_qkv, w_o), cfg, inv_freq)
        h = _engine.FinalNorm.apply(x, self.norm2.weight, norm_eps(self.norm2))
        return x + self.ffn(h).float()


def load_balancing_loss(router_logits, num_experts: int, top_k: int):
    if not router_logits:
        return torch.tensor(0.0)
    logits = torch.cat([g.float() for g in router_logits], dim=0)
    probs = F.softmax(logits, dim=-1)
    _, top = torch.topk(probs, top_k, dim=-1)
    # the reference's one_hot(top, E).mean(0) summed over the k slots: the fraction of
    # (token, slot) pairs routed to each expert, counted without the [T, k, E] one-hot
    frac = expert_histogram(top, num_experts).float() / top.shape[0]
    return (frac * probs.mean(dim=0)).sum() * num_experts


def router_z_loss(router_logits):
    if not router_logits:
        return torch.tensor(0.0)
    logits = torch.cat([g.float() for g in router_logits], dim=0)
    return torch.square(torch.logsumexp(logits, dim=-1)).mean()


class Qwen3Moe(nn.Module):
    def __init__(self, num_layers: int, num_heads: int, num_kv_heads: int, emb_dim: int,
                 head_dim: int, vocab_size: int, moe_ffn_dim: int, num_experts: int = 128,
                 top_k: int = 8, ffn_dim: int | None = None, norm_topk_prob: bool = True,
                 decoder_sparse_step: int = 1, mlp_only_layers: list[int] | None = None,
                 router_aux_loss_coef: float = 0.001, router_z_loss_coef: float = 0.001,
                 rope_base: float = 1_000_000.0, tie_embeddings: bool = False,
                 router_init_std: float = 0.0):
        super().__init__()
        mlp_only = set(mlp_only_layers or [])
        # 0 keeps the routers at zeros through init_weights (the reference's init: every
        # token's top-k then ties on the same experts until training spreads them);
        # > 0 draws them N(0, router_init_std), a router that already spreads tokens
        self.router_init_std = router_init_std
        self.num_experts, self.top_k = num_experts, top_k
        self.router_aux_loss_coef, self.router_z_loss_coef = router_aux_loss_coef, router_z_loss_coef
        self.head_dim, self.emb_dim = head_dim, emb_dim
        self.token_emb = nn.Embedding(vocab_size, emb_dim)
        self.rope = RotaryEmbedding(head_dim, base=rope_base)
        self.blocks = nn.ModuleList(
            Qwen3MoeTransformerBlock(
                num_heads, emb_dim, num_kv_heads, head_dim,
                use_moe=(i not in mlp_only and num_experts > 0 and (i + 1) % decoder_sparse_step == 0),
                ffn_dim=ffn_dim, moe_ffn_dim=moe_ffn_dim, num_experts=num_experts, top_k=top_k,
                norm_topk_prob=norm_topk_prob)
            for i in range(num_layers))
        self.norm = nn.RMSNorm(emb_dim)
        self.lm_head = nn.Linear(emb_dim, vocab_size, bias=False)
        if tie_embeddings:
            self.lm_head.weight = self.token_emb.weight
        self._router_logits: list[torch.Tensor] = []
        self.last_tokens_per_expert: torch.Tensor | None = None
        self.weight_cache = WeightCache()
        # the expert banks' bf16 copies come from the same cache (kept current by the
        # optimizer instead of a cast of the whole bank on every forward)
        for b in self.blocks:
            if b.use_moe:
                b.ffn.experts.weight_cache = self.weight_cache

    def init_weights(self, std: float = 0.02) -> None:
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, 0.0, std)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, 0.0, std)
            elif isinstance(m, nn.RMSNorm) and m.weight is not None:
                nn.init.ones_(m.weight)
        for b in self.blocks:
            if isinstance(b.ffn, Qwen3MoeSparseMLP):
                nn.init.normal_(b.ffn.experts.gate_up_proj, 0.0, std)
                nn.init.normal_(b.ffn.experts.down_proj, 0.0, std)
                if self.router_init_std > 0:
                    nn.init.normal_(b.ffn.router.weight, 0.0, self.router_init_std)
        s = (2 * len(self.blocks)) ** -0.5
        for b in self.blocks:
            b.gqa.o_proj.weight.data.mul_(s)
            if isinstance(b.ffn, Qwen3MoeSparseMLP):
                b.ffn.experts.down_proj.data.mul_(s)
            else:
                b.ffn.down_proj.weight.data.mul_(s)

    def _collect(self):
        return [b.ffn.last_router_logits for b in self.blocks
                if isinstance(b.ffn, Qwen3MoeSparseMLP) and b.ffn.last_router_logits is not None]

    def _update_expert_counts(self, logits) -> None:
        """Tokens routed to each expert this forward, summed over the sparse layers
        (from the routers' own top-k choices)."""
        if not logits:
            self.last_tokens_per_expert = None
            return
        counts = torch.zeros(self.num_experts, device=logits[0].device)
        with torch.no_grad():
            for b in self.blocks:
                idx = getattr(b.ffn, "last_top_idx", None) if isinstance(b.ffn, Qwen3MoeSparseMLP) \
                    else None
                if idx is not None:
                    counts += expert_histogram(idx, self.num_experts).float()
        self.last_tokens_per_expert = counts

    def aux_loss(self):
        logits = self._router_logits
        if not logits:
            return None
        loss = torch.zeros((), device=logits[0].device)
        if self.router_aux_loss_coef != 0.0:
            loss = loss + self.router_aux_loss_coef * load_balancing_loss(logits, self.num_experts,
                                                                          self.top_k)
        if self.router_z_loss_coef != 0.0:
            loss = loss + self.router_z_loss_coef * router_z_loss(logits)
        return loss

    def forward(self, x, attention_mask=None, return_hidden_states: bool = False,
                return_final_hidden: bool = False, position_ids=None):
        for b in self.blocks:
            if isinstance(b.ffn, Qwen3MoeSparseMLP):
                b.ffn.last_router_logits = None
                b.ffn.last_top_idx = None
        self._router_logits = []
        B, S = x.shape
        fused = (x.is_cuda and attention_mask is None and not return_hidden_states
                 and position_ids is None and getattr(self, "tp", None) is None
                 and getattr(self, "cp", None) is None
                 and self.head_dim in (64, 128) and self.emb_dim % 128 == 0)
        if fused:
            h = _engine.Embedding.apply(x, self.token_emb.weight, 1.0)
            fs = getattr(self, "_plg_fsdp", None)
            for i, blk in enumerate(self.blocks):
                cfg = _engine.AttnCfg(B=B, S=S, Hq=blk.gqa.num_heads, Hk=blk.gqa.num_kv_heads,
                                      d=blk.gqa.head_dim, eps=norm_eps(blk.norm1),
                                      qk_eps=norm_eps(blk.gqa.q_norm, torch.bfloat16))
                if fs is not None:
                    fs.fused_block_enter(i)
                h = blk.fused_forward(h, self.weight_cache, cfg, self.rope.inv_freq, i)
                if fs is not None:
                    fs.fused_block_exit(i, h)
            self._router_logits = self._collect()
            self._update_expert_counts(self._router_logits)
            hidden = _engine.FinalNorm.apply(h, self.norm.weight, norm_eps(self.norm)).view(B, S, -1)
            if return_final_hidden:
                return hidden
            return linear(hidden, self.lm_head.weight, self.weight_cache.get(self.lm_head.weight))
        pos, cacheable, am = position_ids_for(x, attention_mask)
        if position_ids is not None:
            pos, cacheable = position_ids, False
        h = self.token_emb(x)
        cos, sin = self.rope(pos, cacheable=cacheable)
        hs = [h] if return_hidden_states else []
        for blk in self.blocks:
            h = blk(h, cos, sin, am)
            if return_hidden_states:
                hs.append(h)
        self._router_logits = self._collect()
        self._update_expert_counts(self._router_logits)
        if return_final_hidden:
            return self.norm(h)
        logits = self.lm_head(self.norm(h))
        return (logits, hs) if return_hidden_states else logits

    def lm_head_lowp(self):
        w = self.lm_head.weight
        return self.weight_cache.get(w) if w.is_cuda else None
