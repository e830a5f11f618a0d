"""OLMo-3 decoder: post-norm blocks, full-width q/k norm, hybrid sliding attention.

Parity: reference ``pluggy/models/olmo3/olmo3.py:25-330``:

* post-norm residual ``x = x + Norm(sublayer(x))`` (``post_attention_norm``,
  ``post_ffn_norm``), no pre-norm on the residual stream;
* q/k RMSNorm over the FULL projected width (``q_norm: RMSNorm(Hq*d)``) before
  the head split;
* layer pattern 3 sliding + 1 full (``default_layer_types``), window 4096;
* untied head, RoPE base 5e5.

B200 difference: the sliding window is applied inside the flash-attention
kernel (a band test per tile) instead of a dense S x S boolean mask, so the
windowed layers keep the O(S) memory and the tile skipping of the causal path.
On CUDA every product runs on the tcgen05 GEMM and the norms/attention on this
package's kernels (composed differentiable ops).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from pluggy_b200.models.common import RotaryEmbedding, SwiGLU, apply_norm, attend, position_ids_for
from pluggy_b200.ops.attention import flash_attention
from pluggy_b200.ops.elementwise import apply_rotary
from pluggy_b200.ops.linear import WeightCache, linear
from pluggy_b200.ops.norm import rms_norm


def default_layer_types(num_layers: int) -> list[str]:
    return ["full_attention" if (i + 1) % 4 == 0 else "sliding_attention" for i in range(num_layers)]


def _eps(m: nn.RMSNorm) -> float:
    return torch.finfo(torch.float32).eps if m.eps is None else m.eps


class Olmo3Attention(nn.Module):
    def __init__(self, num_heads, emb_dim, num_kv_heads, head_dim, sliding_window=None):
        super().__init__()
        assert num_heads % num_kv_heads == 0 and num_heads >= num_kv_heads
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.emb_dim, self.sliding_window = emb_dim, sliding_window
        q_out, kv_out = num_heads * head_dim, num_kv_heads * head_dim
        self.q_proj = nn.Linear(emb_dim, q_out, bias=False)
        self.k_proj = nn.Linear(emb_dim, kv_out, bias=False)
        self.v_proj = nn.Linear(emb_dim, kv_out, bias=False)
        self.o_proj = nn.Linear(q_out, emb_dim, bias=False)
        self.q_norm = nn.RMSNorm(q_out)
        self.k_norm = nn.RMSNorm(kv_out)

    def _window(self, S: int) -> int:
        return self.sliding_window if (self.sliding_window is not None and self.sliding_window < S) else 0

    def forward(self, x, cos, sin, attention_mask=None, cache: WeightCache | None = None):
        B, S, _ = x.shape
        if x.is_cuda and attention_mask is None and cache is not None:
            q = rms_norm(linear(x, self.q_proj.weight, cache.get(self.q_proj.weight)),
                         self.q_norm.weight, _eps(self.q_norm))
            k = rms_norm(linear(x, self.k_proj.weight, cache.get(self.k_proj.weight)),
                         self.k_norm.weight, _eps(self.k_norm))
            v = linear(x, self.v_proj.weight, cache.get(self.v_proj.weight))
            q = apply_rotary(q.view(B, S, self.num_heads, self.head_dim).transpose(1, 2), cos, sin)
            k = apply_rotary(k.view(B, S, self.num_kv_heads, self.head_dim).transpose(1, 2), cos, sin)
            o = flash_attention(q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous(),
                                v.view(B, S, self.num_kv_heads, self.head_dim), True, self._window(S))
            return linear(o.reshape(B, S, -1), self.o_proj.weight, cache.get(self.o_proj.weight))
        Q = self.q_norm(self.q_proj(x)).reshape(B, S, self.num_heads, self.head_dim).transpose(1, 2)
        K = self.k_norm(self.k_proj(x)).reshape(B, S, self.num_kv_heads, self.head_dim).transpose(1, 2)
        V = self.v_proj(x).reshape(B, S, self.num_kv_heads, self.head_dim).transpose(1, 2)
        Q, K = apply_rotary(Q, cos, sin), apply_rotary(K, cos, sin)
        o = attend(Q, K, V, attention_mask, self._window(S))
        return self.o_proj(o.transpose(1, 2).reshape(B, S, -1))


class Olmo3TransformerBlock(nn.Module):
    def __init__(self, num_heads, emb_dim, num_kv_heads, head_dim, ffn_dim, sliding_window=None):
        super().__init__()
        self.attn = Olmo3Attention(num_heads, emb_dim, num_kv_heads, head_dim, sliding_window)
        self.ffn = SwiGLU(emb_dim, ffn_dim)
        self.post_attention_norm = nn.RMSNorm(emb_dim)
        self.post_ffn_norm = nn.RMSNorm(emb_dim)

    def forward(self, x, cos, sin, attention_mask=None, cache: WeightCache | None = None):
        if x.is_cuda and attention_mask is None and cache is not None:
            a = self.attn(x, cos, sin, None, cache)
            x = x + rms_norm(a, self.post_attention_norm.weight, _eps(self.post_attention_norm)).float()
            f = self.ffn
            from pluggy_b200.ops.elementwise import swiglu_mul

            g = linear(x, f.gate_proj.weight, cache.get(f.gate_proj.weight))
            u = linear(x, f.up_proj.weight, cache.get(f.up_proj.weight))
            y = linear(swiglu_mul(g, u), f.down_proj.weight, cache.get(f.down_proj.weight))
            return x + rms_norm(y, self.post_ffn_norm.weight, _eps(self.post_ffn_norm)).float()
        x = x + self.post_attention_norm(self.attn(x, cos, sin, attention_mask))
        return x + self.post_ffn_norm(self.ffn(x))


class Olmo3(nn.Module):
    def __init__(self, num_layers: int, num_heads: int, num_kv_heads: int, emb_dim: int,
                 vocab_size: int, ffn_dim: int, head_dim: int | None = None,
                 rope_base: float = 500_000.0, sliding_window: int | None = 4096,
                 layer_types: list[str] | None = None):
        super().__init__()
        head_dim = head_dim if head_dim is not None else emb_dim // num_heads
        layer_types = layer_types if layer_types is not None else default_layer_types(num_layers)
        assert len(layer_types) == num_layers, "layer_types length must equal num_layers"
        for t in layer_types:
            assert t in ("full_attention", "sliding_attention"), f"unknown layer type {t!r}"
        self.layer_types, self.sliding_window = list(layer_types), sliding_window
        self.token_emb = nn.Embedding(vocab_size, emb_dim)
        self.rope = RotaryEmbedding(head_dim, base=rope_base)
        self.blocks = nn.ModuleList(
            Olmo3TransformerBlock(num_heads, emb_dim, num_kv_heads, head_dim, ffn_dim,
                                  sliding_window if t == "sliding_attention" else None)
            for t in self.layer_types)
        self.norm = nn.RMSNorm(emb_dim)
        self.lm_head = nn.Linear(emb_dim, vocab_size, bias=False)
        self.weight_cache = WeightCache()

    def init_weights(self, std: float = 0.02) -> None:
        from pluggy_b200.models.common import init_decoder_weights

        init_decoder_weights(self, self.blocks, std, out_projs=("attn.o_proj", "ffn.down_proj"))

    def forward(self, x, attention_mask=None, return_hidden_states: bool = False,
                return_final_hidden: bool = False):
        pos, cacheable, am = position_ids_for(x, attention_mask)
        h = self.token_emb(x)
        cos, sin = self.rope(pos, cacheable=cacheable)
        cache = self.weight_cache if (x.is_cuda and am is None) else None
        hs = [h] if return_hidden_states else []
        for blk in self.blocks:
            h = blk(h, cos, sin, am, cache)
            if return_hidden_states:
                hs.append(h)
        if return_final_hidden:
            return apply_norm(self.norm, h)
        logits = self.lm_head(apply_norm(self.norm, h))
        return (logits, hs) if return_hidden_states else logits
