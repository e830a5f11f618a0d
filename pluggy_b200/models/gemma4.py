"""Gemma-4 dense text decoder.

Parity: reference ``pluggy/models/gemma4/gemma4.py:38-531``:

* sandwich norms ``x = x + post(sublayer(pre(x)))`` for attention and FFN;
* hybrid attention (``default_layer_types``: 5 sliding : 1 full, last layer
  forced full); sliding layers use ``head_dim`` and RoPE theta 1e4, full layers
  ``global_head_dim`` with proportional partial RoPE (factor 0.25, theta 1e6;
  the unrotated channels get inv_freq 0, i.e. identity);
* per-head q/k RMSNorm, scale-free v RMSNorm, attention scale 1.0;
* GeGLU (gelu-tanh), embedding scaled by sqrt(d), tied head by default;
* KV sharing across the last ``num_kv_shared_layers`` (donor = last earlier
  layer of the same type), ``attention_k_eq_v`` on full layers, double-wide
  MLP on shared layers, per-layer embeddings (PLE);
* final logit softcap on the logits path (skipped by the fused linear-CE path,
  which consumes ``return_final_hidden``).

On CUDA the projections run on the tcgen05 GEMM, norms and GeGLU on this
package's kernels, and attention on the sm_100a flash kernel with the window
applied in-kernel when the layer's head_dim is 64 or 128. Wider global heads
(256/512) use PyTorch SDPA with a causal/band mask: the flash kernel's TMEM
budget covers head_dim <= 128.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from pluggy_b200.models.common import apply_norm, attend, position_ids_for
from pluggy_b200.ops.attention import flash_attention
from pluggy_b200.ops.elementwise import apply_rotary, geglu_mul, logit_softcap
from pluggy_b200.ops.linear import WeightCache, linear


def default_layer_types(num_layers: int, pattern: int = 6) -> list[str]:
    t = ["sliding_attention" if (i + 1) % pattern else "full_attention" for i in range(num_layers)]
    if t:
        t[-1] = "full_attention"
    return t


def rms_norm_no_scale(x: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps).to(x.dtype)


class Gemma4RotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, base: float = 10_000.0, partial_rotary_factor: float = 1.0,
                 proportional: bool = False):
        super().__init__()
        assert head_dim % 2 == 0, "RoPE requires even head_dim"
        self.head_dim = head_dim
        if proportional and partial_rotary_factor < 1.0:
            n_rot = int(partial_rotary_factor * head_dim // 2)
            inv = 1.0 / (base ** (torch.arange(0, 2 * n_rot, 2).float() / head_dim))
            nope = head_dim // 2 - n_rot
            if nope > 0:
                inv = torch.cat([inv, torch.zeros(nope)])
        else:
            inv = 1.0 / (base ** (torch.arange(0, head_dim, 2).float() / head_dim))
        self.register_buffer("inv_freq", inv, persistent=False)
        self._cache: dict = {}

    def _cos_sin(self, pos):
        f = pos.float()[:, :, None] * self.inv_freq[None, None, :]
        e = torch.cat([f, f], dim=-1)
        return e.cos()[:, None], e.sin()[:, None]

    def forward(self, pos, cacheable: bool = False):
        if not cacheable:
            return self._cos_sin(pos)
        key = (pos.shape[1], pos.device)
        if key not in self._cache:
            self._cache[key] = self._cos_sin(pos[:1])  # batch-1 table broadcasts to any B
        return self._cache[key]


class GeGLU(nn.Module):
    def __init__(self, hidden_dim: int, ffn_dim: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_dim, ffn_dim, bias=False)
        self.up_proj = nn.Linear(hidden_dim, ffn_dim, bias=False)
        self.down_proj = nn.Linear(ffn_dim, hidden_dim, bias=False)

    def forward(self, x, cache: WeightCache | None = None):
        if cache is not None:
            g = linear(x, self.gate_proj.weight, cache.get(self.gate_proj.weight))
            u = linear(x, self.up_proj.weight, cache.get(self.up_proj.weight))
            return linear(geglu_mul(g, u), self.down_proj.weight, cache.get(self.down_proj.weight))
        return self.down_proj(geglu_mul(self.gate_proj(x), self.up_proj(x)))


def _lin(mod: nn.Linear, x, cache):
    return linear(x, mod.weight, cache.get(mod.weight)) if cache is not None else mod(x)


class Gemma4Attention(nn.Module):
    def __init__(self, emb_dim, num_heads, num_kv_heads, head_dim, layer_type, sliding_window,
                 is_kv_shared_layer, store_full_length_kv, attention_k_eq_v, rms_norm_eps=1e-6):
        super().__init__()
        assert num_heads % num_kv_heads == 0 and num_heads >= num_kv_heads
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.layer_type = layer_type
        self.sliding_window = sliding_window if layer_type == "sliding_attention" else None
        self.is_kv_shared_layer = is_kv_shared_layer
        self.store_full_length_kv = store_full_length_kv
        self.use_k_eq_v = bool(attention_k_eq_v) and layer_type == "full_attention"
        self.rms_norm_eps = rms_norm_eps
        self.scale = 1.0
        q_out, kv_out = num_heads * head_dim, num_kv_heads * head_dim
        self.q_proj = nn.Linear(emb_dim, q_out, bias=False)
        self.q_norm = nn.RMSNorm(head_dim, eps=rms_norm_eps)
        self.o_proj = nn.Linear(q_out, emb_dim, bias=False)
        if not is_kv_shared_layer:
            self.k_proj = nn.Linear(emb_dim, kv_out, bias=False)
            self.k_norm = nn.RMSNorm(head_dim, eps=rms_norm_eps)
            self.v_proj = None if self.use_k_eq_v else nn.Linear(emb_dim, kv_out, bias=False)
        else:
            self.k_proj = self.k_norm = self.v_proj = None

    def _split(self, x, n):
        B, S, _ = x.shape
        return x.reshape(B, S, n, self.head_dim).transpose(1, 2)

    def forward(self, x, cos, sin, attention_mask, shared_kv, cache=None):
        Q = apply_rotary(apply_norm(self.q_norm, self._split(_lin(self.q_proj, x, cache), self.num_heads)),
                         cos, sin)
        if self.is_kv_shared_layer:
            K, V = shared_kv[self.layer_type]
            K, V = K.to(Q.device, Q.dtype), V.to(Q.device, Q.dtype)
        else:
            K = self._split(_lin(self.k_proj, x, cache), self.num_kv_heads)
            V = K if (self.use_k_eq_v or self.v_proj is None) else \
                self._split(_lin(self.v_proj, x, cache), self.num_kv_heads)
            K = apply_rotary(apply_norm(self.k_norm, K), cos, sin)
            V = rms_norm_no_scale(V, self.rms_norm_eps)
            if self.store_full_length_kv:
                shared_kv[self.layer_type] = (K, V)
        S = Q.shape[-2]
        window = self.sliding_window if (self.sliding_window is not None and self.sliding_window < S) else 0
        if cache is not None and attention_mask is None and self.head_dim in (64, 128):
            o = flash_attention(Q.transpose(1, 2).contiguous(), K.transpose(1, 2).contiguous(),
                                V.transpose(1, 2).contiguous(), True, window, self.scale).transpose(1, 2)
        else:
            o = attend(Q, K, V, attention_mask, window, scale=self.scale)
        B = o.shape[0]
        return _lin(self.o_proj, o.transpose(1, 2).reshape(B, S, -1), cache)


class Gemma4TransformerBlock(nn.Module):
    def __init__(self, emb_dim, num_heads, num_kv_heads, head_dim, ffn_dim, layer_type, sliding_window,
                 is_kv_shared_layer, store_full_length_kv, attention_k_eq_v, ple_dim=0,
                 rms_norm_eps=1e-6):
        super().__init__()
        self.attn = Gemma4Attention(emb_dim, num_heads, num_kv_heads, head_dim, layer_type,
                                    sliding_window, is_kv_shared_layer, store_full_length_kv,
                                    attention_k_eq_v, rms_norm_eps)
        self.ffn = GeGLU(emb_dim, ffn_dim)
        self.input_norm = nn.RMSNorm(emb_dim, eps=rms_norm_eps)
        self.post_attn_norm = nn.RMSNorm(emb_dim, eps=rms_norm_eps)
        self.pre_ffn_norm = nn.RMSNorm(emb_dim, eps=rms_norm_eps)
        self.post_ffn_norm = nn.RMSNorm(emb_dim, eps=rms_norm_eps)
        self.ple_dim = ple_dim
        if ple_dim > 0:
            self.ple_gate = nn.Linear(emb_dim, ple_dim, bias=False)
            self.ple_proj = nn.Linear(ple_dim, emb_dim, bias=False)
            self.ple_norm = nn.RMSNorm(emb_dim, eps=rms_norm_eps)

    def forward(self, x, cos, sin, attention_mask, shared_kv, ple_input=None, cache=None):
        a = self.attn(apply_norm(self.input_norm, x), cos, sin, attention_mask, shared_kv, cache)
        x = x + apply_norm(self.post_attn_norm, a)
        x = x + apply_norm(self.post_ffn_norm, self.ffn(apply_norm(self.pre_ffn_norm, x), cache))
        if self.ple_dim > 0 and ple_input is not None:
            gated = F.gelu(_lin(self.ple_gate, x, cache), approximate="tanh") * ple_input
            x = x + apply_norm(self.ple_norm, _lin(self.ple_proj, gated, cache))
        return x


class Gemma4(nn.Module):
    def __init__(self, num_layers: int, num_heads: int, num_kv_heads: int, emb_dim: int,
                 vocab_size: int, ffn_dim: int, head_dim: int = 256, global_head_dim: int = 512,
                 num_global_kv_heads: int | None = None, sliding_window: int | None = 512,
                 layer_types: list[str] | None = None, layer_pattern: int = 6,
                 rope_theta_sliding: float = 10_000.0, rope_theta_full: float = 1_000_000.0,
                 partial_rotary_factor: float = 0.25, final_logit_softcapping: float | None = 30.0,
                 num_kv_shared_layers: int = 0, attention_k_eq_v: bool = False,
                 use_double_wide_mlp: bool = False, hidden_size_per_layer_input: int = 0,
                 vocab_size_per_layer_input: int | None = None, rms_norm_eps: float = 1e-6,
                 tie_embeddings: bool = True):
        super().__init__()
        layer_types = list(layer_types) if layer_types is not None else \
            default_layer_types(num_layers, layer_pattern)
        assert len(layer_types) == num_layers, "layer_types length must equal num_layers"
        for t in layer_types:
            assert t in ("full_attention", "sliding_attention"), f"bad layer type {t!r}"
        if layer_types:
            layer_types[-1] = "full_attention"
        num_global_kv_heads = num_kv_heads if num_global_kv_heads is None else num_global_kv_heads
        vocab_size_per_layer_input = vocab_size if vocab_size_per_layer_input is None else \
            vocab_size_per_layer_input
        self.layer_types, self.sliding_window = layer_types, sliding_window
        self.final_logit_softcapping = final_logit_softcapping
        self.ple_dim = int(hidden_size_per_layer_input)
        self.num_kv_shared_layers = num_kv_shared_layers
        self.emb_dim = emb_dim
        self.token_emb = nn.Embedding(vocab_size, emb_dim)
        self.embed_scale = emb_dim ** 0.5
        self.rope_sliding = Gemma4RotaryEmbedding(head_dim, base=rope_theta_sliding)
        self.rope_full = Gemma4RotaryEmbedding(global_head_dim, base=rope_theta_full,
                                               partial_rotary_factor=partial_rotary_factor,
                                               proportional=True)
        first_shared = num_layers - num_kv_shared_layers
        prev = layer_types[:first_shared] if num_kv_shared_layers > 0 else list(layer_types)
        donor = {lt: i for i, lt in enumerate(prev)}
        blocks = []
        for i, lt in enumerate(layer_types):
            full = lt == "full_attention"
            shared = num_kv_shared_layers > 0 and i >= first_shared and lt in donor
            blocks.append(Gemma4TransformerBlock(
                emb_dim, num_heads, num_global_kv_heads if full else num_kv_heads,
                global_head_dim if full else head_dim,
                ffn_dim * (2 if (use_double_wide_mlp and shared) else 1), lt, sliding_window, shared,
                (not shared) and donor.get(lt) == i, attention_k_eq_v, self.ple_dim, rms_norm_eps))
        self.blocks = nn.ModuleList(blocks)
        self.norm = nn.RMSNorm(emb_dim, eps=rms_norm_eps)
        self.lm_head = nn.Linear(emb_dim, vocab_size, bias=False)
        if tie_embeddings:
            self.lm_head.weight = self.token_emb.weight
        if self.ple_dim > 0:
            self.embed_tokens_per_layer = nn.Embedding(vocab_size_per_layer_input,
                                                       num_layers * self.ple_dim)
            self.ple_embed_scale = self.ple_dim ** 0.5
            self.per_layer_model_projection = nn.Linear(emb_dim, num_layers * self.ple_dim, bias=False)
            self.per_layer_model_projection_scale = emb_dim ** -0.5
            self.per_layer_projection_norm = nn.RMSNorm(self.ple_dim, eps=rms_norm_eps)
            self.per_layer_input_scale = 2.0 ** -0.5
        self.weight_cache = WeightCache()

    def _ple_inputs(self, ids, emb):
        B, S = ids.shape
        L = len(self.blocks)
        tok = (self.embed_tokens_per_layer(ids) * self.ple_embed_scale).reshape(B, S, L, self.ple_dim)
        ctx = self.per_layer_model_projection(emb) * self.per_layer_model_projection_scale
        ctx = self.per_layer_projection_norm(ctx.reshape(B, S, L, self.ple_dim))
        return (ctx + tok) * self.per_layer_input_scale

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
        s = (2 * len(self.blocks)) ** -0.5
        for b in self.blocks:
            b.attn.o_proj.weight.data.mul_(s)
            b.ffn.down_proj.weight.data.mul_(s)
            if b.ple_dim > 0:
                b.ple_proj.weight.data.mul_(s)

    def forward(self, x, attention_mask=None, return_hidden_states: bool = False,
                return_final_hidden: bool = False):
        pos, cacheable, am = position_ids_for(x, attention_mask)
        h = self.token_emb(x) * self.embed_scale
        ple = self._ple_inputs(x, h) if self.ple_dim > 0 else None
        ropes = {"sliding_attention": self.rope_sliding(pos, cacheable=cacheable),
                 "full_attention": self.rope_full(pos, cacheable=cacheable)}
        cache = self.weight_cache if (x.is_cuda and am is None) else None
        shared: dict = {}
        hs = [h] if return_hidden_states else []
        for i, blk in enumerate(self.blocks):
            cos, sin = ropes[self.layer_types[i]]
            h = blk(h, cos, sin, am, shared, ple[:, :, i, :] if ple is not None else None, cache)
            if return_hidden_states:
                hs.append(h)
        if return_final_hidden:
            return apply_norm(self.norm, h)
        logits = logit_softcap(self.lm_head(apply_norm(self.norm, h)), self.final_logit_softcapping)
        return (logits, hs) if return_hidden_states else logits
