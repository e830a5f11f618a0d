"""Qwen3 dense decoder.

Parity: reference ``pluggy/models/qwen3/qwen3.py:18-338``: token embedding,
RoPE (base 1e6), GQA with per-head q_norm/k_norm, SwiGLU (ffn default 8/3*d
rounded to 256), pre-norm blocks, tied ``lm_head``, ``init_weights`` with the
1/sqrt(2L) residual scaling, and ``forward(x, attention_mask=None,
return_hidden_states=False, return_final_hidden=False)`` returning logits,
``(logits, hidden_states)`` or the post-norm final hidden.

Execution: on CUDA, an unmasked forward (the packed training path) runs every
block as two fused sm_100a sublayers (``_engine.AttnSublayer`` +
``_engine.MlpSublayer``) over an fp32 residual stream, with the embedding and
final norm in their own kernels and bf16 weights taken from a
:class:`~pluggy_b200.ops.linear.WeightCache` (one cast per optimizer step, not
per forward). The eager path (CPU, padded masks, ``return_hidden_states``) is
the reference math.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from pluggy_b200.models import _engine
from pluggy_b200.models.common import (GQAttention, RotaryEmbedding, SwiGLU, default_ffn_dim,
                                       init_decoder_weights, norm_eps, position_ids_for)
from pluggy_b200.ops.elementwise import SILU
from pluggy_b200.ops.linear import WeightCache, linear


class Qwen3TransformerBlock(nn.Module):
    attn_name = "gqa"   # attribute name of the attention module (Llama3 calls it "attn")
    qk_norm = True

    def __init__(self, num_heads, emb_dim, num_kv_heads=8, head_dim=None, ffn_dim=None):
        super().__init__()
        setattr(self, self.attn_name,
                GQAttention(num_heads, emb_dim, num_kv_heads, head_dim, qk_norm=self.qk_norm))
        self.norm1 = nn.RMSNorm(emb_dim)
        self.norm2 = nn.RMSNorm(emb_dim)
        self.ffn = SwiGLU(emb_dim, ffn_dim if ffn_dim is not None else default_ffn_dim(emb_dim))

    @property
    def attention(self) -> GQAttention:
        return getattr(self, self.attn_name)

    def forward(self, x, cos, sin, attention_mask=None):
        x = x + self.attention(self.norm1(x), cos, sin, attention_mask)
        return x + self.ffn(self.norm2(x))

    # ---------------------------------------------------------------- fused path
    def fused_forward(self, x, cache: WeightCache, cfg: _engine.AttnCfg, inv_freq, idx: int):
        g = self.attention
        w_qkv = cache.get_cat([g.q_proj.weight, g.k_proj.weight, g.v_proj.weight], f"b{idx}.qkv")
        w_o = cache.get(g.o_proj.weight)
        qn = g.q_norm.weight if g.qk_norm else None
        kn = g.k_norm.weight if g.qk_norm else None
        x = _engine.AttnSublayer.apply(x, self.norm1.weight, g.q_proj.weight, g.k_proj.weight,
                                       g.v_proj.weight, g.o_proj.weight, qn, kn, (w_qkv, w_o), cfg,
                                       inv_freq)
        f = self.ffn
        w_gu = cache.get_cat([f.gate_proj.weight, f.up_proj.weight], f"b{idx}.gu")
        w_d = cache.get(f.down_proj.weight)
        return _engine.MlpSublayer.apply(x, self.norm2.weight, f.gate_proj.weight, f.up_proj.weight,
                                         f.down_proj.weight, (w_gu, w_d), norm_eps(self.norm2), SILU)


    def fused_forward_tp(self, x, cache: WeightCache, cfg: _engine.AttnCfg, inv_freq, idx: int, comm):
        """Tensor/sequence-parallel form of :meth:`fused_forward`: ``x`` is this rank's
        sequence shard [B*S/tp, D] fp32; the weights are this rank's head/column shards."""
        from pluggy_b200.parallel.tp_engine import TPAttnSublayer, TPMlpSublayer

        g = self.attention
        w_qkv = cache.get_cat([g.q_proj.weight, g.k_proj.weight, g.v_proj.weight], f"b{idx}.qkv")
        w_o = cache.get(g.o_proj.weight)
        qn = g.q_norm.weight if g.qk_norm else None
        kn = g.k_norm.weight if g.qk_norm else None
        x = TPAttnSublayer.apply(x, self.norm1.weight, g.q_proj.weight, g.k_proj.weight,
                                 g.v_proj.weight, g.o_proj.weight, qn, kn, (w_qkv, w_o), cfg, inv_freq,
                                 comm)
        f = self.ffn
        w_gu = cache.get_cat([f.gate_proj.weight, f.up_proj.weight], f"b{idx}.gu")
        w_d = cache.get(f.down_proj.weight)
        return TPMlpSublayer.apply(x, self.norm2.weight, f.gate_proj.weight, f.up_proj.weight,
                                   f.down_proj.weight, (w_gu, w_d), norm_eps(self.norm2), SILU,
                                   cfg.B, cfg.S, comm)


class Qwen3(nn.Module):
    # the forward calls ``_plg_param_gate.enter`` (ZeRO-1 DDP: wait for each block's
    # parameter all-gather just before the block)
    param_gate_aware = True
    # the CUDA path reads every matrix weight as bf16 through ``weight_cache`` (FSDP2
    # can then gather them in low precision straight into the GEMMs' buffers)
    fused_engine = True
    rope_base = 1_000_000
    tie_default = True
    block_cls = Qwen3TransformerBlock

    def __init__(self, num_layers: int, num_heads: int, num_kv_heads: int, emb_dim: int,
                 head_dim: int | None, vocab_size: int, ffn_dim: int | None = None,
                 tie_embeddings: bool | None = None, rope_base: float | None = None):
        super().__init__()
        head_dim = head_dim if head_dim is not None else emb_dim // num_heads
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.emb_dim, self.vocab_size = emb_dim, vocab_size
        self.token_emb = nn.Embedding(vocab_size, emb_dim)
        self.rope = RotaryEmbedding(head_dim, base=rope_base if rope_base is not None else self.rope_base)
        self.blocks = nn.ModuleList(self._make_block(num_heads, emb_dim, num_kv_heads, head_dim, ffn_dim)
                                    for _ in range(num_layers))
        self.norm = nn.RMSNorm(emb_dim)
        self.lm_head = nn.Linear(emb_dim, vocab_size, bias=False)
        tie = self.tie_default if tie_embeddings is None else tie_embeddings
        if tie:
            self.lm_head.weight = self.token_emb.weight
        self.weight_cache = WeightCache()

    def _make_block(self, num_heads, emb_dim, num_kv_heads, head_dim, ffn_dim):
        return self.block_cls(num_heads, emb_dim, num_kv_heads, head_dim, ffn_dim)

    def init_weights(self, std: float = 0.02) -> None:
        init_decoder_weights(self, self.blocks, std)

    # ------------------------------------------------------------------ paths
    def _use_fused(self, x, attention_mask, return_hidden_states) -> bool:
        return (x.is_cuda and attention_mask is None and not return_hidden_states
                and getattr(self, "tp", None) is None and getattr(self, "cp", None) is None
                and self.token_emb.weight.dtype == torch.float32
                and self.head_dim in (64, 128) and self.emb_dim % 128 == 0)

    def _use_fused_tp(self, x, attention_mask, return_hidden_states) -> bool:
        """Tensor parallelism with sequence parallelism on the peer-memory collectives,
        with the pre-norms fused into the gathers: the blocks run as TP sublayers."""
        tp = getattr(self, "tp", None)
        if not (x.is_cuda and attention_mask is None and not return_hidden_states and tp is not None
                and tp.comm is not None and tp.sp and getattr(self, "cp", None) is None
                and self.head_dim in (64, 128) and self.emb_dim % 128 == 0
                and x.shape[1] % tp.comm.n == 0):
            return False
        from pluggy_b200.comm.tp_fused import TPNormGather

        return all(isinstance(b.norm1, TPNormGather) and isinstance(b.norm2, TPNormGather)
                   and hasattr(b, "fused_forward_tp") for b in self.blocks)

    def fused_hidden_tp(self, x: torch.Tensor) -> torch.Tensor:
        """Packed causal forward under TP + SP on the sm_100a kernels; returns this
        rank's sequence shard of the final hidden, bf16 [B, S/tp, D]."""
        B, S = x.shape
        comm = self.tp.comm
        h = self.token_emb(x)  # vocabulary-parallel lookup, reduce-scattered along the sequence
        D = h.shape[-1]
        h = h.reshape(-1, D).float().contiguous()
        inv = self.rope.inv_freq
        for i, blk in enumerate(self.blocks):
            h = blk.fused_forward_tp(h, self.weight_cache, self._attn_cfg(B, S, blk), inv, i, comm)
        out = _engine.FinalNorm.apply(h, self.norm.weight, norm_eps(self.norm))
        return out.view(B, S // comm.n, D)

    def _attn_cfg(self, B, S, block) -> _engine.AttnCfg:
        g = block.attention
        return _engine.AttnCfg(B=B, S=S, Hq=g.num_heads, Hk=g.num_kv_heads, d=g.head_dim,
                               eps=norm_eps(block.norm1),
                               qk_eps=norm_eps(g.q_norm, torch.bfloat16) if g.qk_norm else 1e-6,
                               qk_norm=g.qk_norm)

    def fused_hidden(self, x: torch.Tensor) -> torch.Tensor:
        """Packed causal forward on the sm_100a kernels; returns bf16 [B, S, D]."""
        B, S = x.shape
        gate = getattr(self, "_plg_param_gate", None)
        if gate is not None:
            gate.enter("emb")
        h = _engine.Embedding.apply(x, self.token_emb.weight, 1.0)
        inv = self.rope.inv_freq
        fs = getattr(self, "_plg_fsdp", None)
        for i, blk in enumerate(self.blocks):
            if gate is not None:
                gate.enter(i)
            if fs is not None:
                fs.fused_block_enter(i)
            h = blk.fused_forward(h, self.weight_cache, self._attn_cfg(B, S, blk), inv, i)
            if fs is not None:
                fs.fused_block_exit(i, h)
        if gate is not None:
            gate.enter("all")
        out = _engine.FinalNorm.apply(h, self.norm.weight, norm_eps(self.norm))
        return out.view(B, S, -1)

    def forward(self, x, attention_mask=None, return_hidden_states: bool = False,
                return_final_hidden: bool = False, position_ids=None):
        """``position_ids`` (optional [B, S]) overrides the packed arange positions
        (context parallelism feeds each rank's zigzag positions)."""
        if (position_ids is None and return_final_hidden
                and self._use_fused_tp(x, attention_mask, return_hidden_states)):
            return self.fused_hidden_tp(x)
        if position_ids is None and self._use_fused(x, attention_mask, return_hidden_states):
            hidden = self.fused_hidden(x)
            if return_final_hidden:
                return hidden
            return linear(hidden, self.lm_head.weight, self.weight_cache.get(self.lm_head.weight))
        gate = getattr(self, "_plg_param_gate", None)
        if gate is not None:
            gate.enter("all")
        fs = getattr(self, "_plg_fsdp", None)
        if fs is not None and getattr(fs, "_slots", None) is not None and x.is_cuda:
            raise RuntimeError("FSDP2 low-precision gathers serve the fused packed path only; build "
                               "FSDP2(..., lowp_gather=False) for masked or hidden-state forwards")
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
        if return_final_hidden:
            return self.norm(h)
        logits = self.lm_head(self.norm(h))
        return (logits, hs) if return_hidden_states else logits

    def lm_head_lowp(self):
        """bf16 copy of the LM head weight for the fused linear-CE (CUDA only)."""
        w = self.lm_head.weight
        return self.weight_cache.get(w) if w.is_cuda else None
