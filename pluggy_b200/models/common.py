"""Building blocks shared by the decoder families.

Module and parameter names follow the reference models so ``state_dict`` keys
are identical and checkpoints move between the two frameworks
(``pluggy/models/qwen3/qwen3.py:18-296``):

* ``RotaryEmbedding``: ``inv_freq = 1 / base^(2i/d)`` (non-persistent buffer),
  cos/sin of shape (B, 1, S, d) cached per (seq_len, device) on the packed path;
* ``GQAttention``: ``q_proj/k_proj/v_proj/o_proj`` + optional per-head
  ``q_norm/k_norm`` (``nn.RMSNorm(head_dim)``);
* ``SwiGLU``: ``gate_proj/up_proj/down_proj``;
* ``DecoderBlock``: pre-norm ``x + attn(norm1(x))``, ``x + ffn(norm2(x))``.

The eager forward here is the CPU / oracle path. The CUDA training path lives
in ``pluggy_b200.models._engine`` and reads the same parameters.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from pluggy_b200.ops.attention import attention_reference, flash_attention, sdpa_masked
from pluggy_b200.ops.elementwise import apply_rotary, swiglu_mul

FP32_EPS = torch.finfo(torch.float32).eps


def default_ffn_dim(emb_dim: int) -> int:
    """8/3 * d rounded up to a multiple of 256 (reference qwen3.py:234)."""
    return 256 * ((int(8 * emb_dim / 3) + 255) // 256)


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, base: float = 1_000_000, rot_dim: int | None = None):
        super().__init__()
        assert head_dim % 2 == 0, "RoPE requires even head_dim"
        rd = head_dim if rot_dim is None else rot_dim
        inv = 1.0 / (base ** (torch.arange(0, rd, 2).float() / rd))
        self.register_buffer("inv_freq", inv, False)
        self.head_dim = head_dim
        self._cache: dict = {}

    def _cos_sin(self, position_ids):
        f = position_ids.float()[:, :, None] * self.inv_freq[None, None, :]
        emb = torch.cat([f, f], dim=-1)
        return emb.cos()[:, None], emb.sin()[:, None]

    def forward(self, position_ids, cacheable: bool = False):
        if not cacheable:
            return self._cos_sin(position_ids)
        key = (position_ids.shape[1], position_ids.device)
        hit = self._cache.get(key)
        if hit is None:
            # packed path: every row is arange(S), so one batch-1 table broadcasts to any B
            hit = self._cos_sin(position_ids[:1])
            self._cache[key] = hit
        return hit


class GQAttention(nn.Module):
    def __init__(self, num_heads: int, emb_dim: int, num_kv_heads: int = 8, head_dim: int | None = None,
                 qk_norm: bool = True, norm_eps: float | None = None):
        super().__init__()
        assert num_heads % num_kv_heads == 0 and num_heads >= num_kv_heads, \
            "num_heads must be a positive multiple of num_kv_heads"
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.emb_dim = emb_dim
        self.head_dim = head_dim if head_dim is not None else emb_dim // num_heads
        q_out, kv_out = num_heads * self.head_dim, num_kv_heads * self.head_dim
        self.q_proj = nn.Linear(emb_dim, q_out, bias=False)
        self.k_proj = nn.Linear(emb_dim, kv_out, bias=False)
        self.v_proj = nn.Linear(emb_dim, kv_out, bias=False)
        self.o_proj = nn.Linear(q_out, emb_dim, bias=False)
        self.qk_norm = qk_norm
        if qk_norm:
            self.q_norm = nn.RMSNorm(self.head_dim, eps=norm_eps)
            self.k_norm = nn.RMSNorm(self.head_dim, eps=norm_eps)

    def split(self, x, n):
        return x.reshape(*x.shape[:2], n, self.head_dim).transpose(1, 2)

    def forward(self, x, cos, sin, attention_mask=None, window: int = 0):
        Q = self.split(self.q_proj(x), self.num_heads)
        K = self.split(self.k_proj(x), self.num_kv_heads)
        V = self.split(self.v_proj(x), self.num_kv_heads)
        if self.qk_norm:
            Q, K = self.q_norm(Q), self.k_norm(K)
        Q, K = apply_rotary(Q, cos, sin), apply_rotary(K, cos, sin)
        cp = getattr(self, "cp", None)
        if cp is not None and cp.mesh.size(cp.dim) > 1:
            # context parallel: this rank's zigzag tokens, keys/values around the ring
            from pluggy_b200.parallel.context_parallel import ring_attention

            assert attention_mask is None and not window, "context parallelism is causal-only"
            o = ring_attention(Q.transpose(1, 2), K.transpose(1, 2), V.transpose(1, 2), cp.mesh,
                               cp.dim).transpose(1, 2)
        else:
            o = attend(Q, K, V, attention_mask, window)
        B, _, S, _ = o.shape
        return self.o_proj(o.transpose(1, 2).reshape(B, S, -1))


def attend(Q, K, V, attention_mask=None, window: int = 0, scale=None):
    """[B,H,S,d] attention: causal (+window) fast form, or padded boolean mask."""
    if attention_mask is None:
        q, k, v = Q.transpose(1, 2), K.transpose(1, 2), V.transpose(1, 2)
        if q.is_cuda and q.shape[-1] in (64, 128):
            o = flash_attention(q.to(torch.bfloat16).contiguous(), k.to(torch.bfloat16).contiguous(),
                                v.to(torch.bfloat16).contiguous(), True, window, scale).to(Q.dtype)
        elif q.is_cuda:
            # head_dim outside the sm_100a kernels' {64, 128} (Gemma-4's 256/512 global
            # heads): PyTorch SDPA in bf16, as the reference does for every head
            # (pluggy/models/gemma4/gemma4.py:187-217); never the fp32 S x S math
            return sdpa_causal_bf16(Q, K, V, window, scale).to(Q.dtype)
        else:
            o = attention_reference(q, k, v, causal=True, window=window, scale=scale)
        return o.transpose(1, 2)
    S = Q.shape[-2]
    i = torch.arange(S, device=Q.device)
    m = i[None, :] <= i[:, None]
    if window:
        m = m & ((i[:, None] - i[None, :]) < window)
    m = m[None, None] & attention_mask[:, None, None, :].bool()
    return sdpa_masked(Q, K, V, m, scale=scale)


def sdpa_causal_bf16(Q, K, V, window: int = 0, scale=None):
    """[B,H,S,d] causal (+ sliding window) attention through PyTorch SDPA in bf16."""
    Hq, Hk = Q.shape[1], K.shape[1]
    q, k, v = (t.to(torch.bfloat16) for t in (Q, K, V))
    if not window:
        return F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale,
                                              enable_gqa=Hq != Hk)
    S = Q.shape[-2]
    i = torch.arange(S, device=Q.device)
    m = (i[None, :] <= i[:, None]) & ((i[:, None] - i[None, :]) < window)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=m, scale=scale, enable_gqa=Hq != Hk)


class SwiGLU(nn.Module):
    def __init__(self, hidden_dim: int, ffn_dim: int):
        super().__init__()
        self.gate_proj = nn.Linear(hidden_dim, ffn_dim, bias=False)
        self.up_proj = nn.Linear(hidden_dim, ffn_dim, bias=False)
        self.down_proj = nn.Linear(ffn_dim, hidden_dim, bias=False)

    def forward(self, x):
        return self.down_proj(swiglu_mul(self.gate_proj(x), self.up_proj(x)))


def position_ids_for(x: torch.Tensor, attention_mask):
    B, S = x.shape
    if attention_mask is None:
        return torch.arange(S, device=x.device).unsqueeze(0).expand(B, -1), True, None
    am = attention_mask.bool()
    pos = (am.long().cumsum(dim=1) - 1).masked_fill(~am, 0)
    return pos, False, am


def init_decoder_weights(model: nn.Module, blocks, std: float = 0.02, out_projs=("gqa.o_proj",
                                                                             "ffn.down_proj")):
    """N(0, std) for Linear/Embedding, ones for RMSNorm, then the residual
    writers scaled by 1/sqrt(2L) (reference qwen3.py:273-296)."""
    for m in model.modules():
        if isinstance(m, nn.Linear):
            nn.init.normal_(m.weight, 0.0, std)
            if m.bias is not None:
                nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, 0.0, std)
        elif isinstance(m, nn.RMSNorm) and m.weight is not None:
            nn.init.ones_(m.weight)
    s = (2 * len(blocks)) ** -0.5
    for b in blocks:
        for path in out_projs:
            mod = b
            ok = True
            for part in path.split("."):
                if not hasattr(mod, part):
                    ok = False
                    break
                mod = getattr(mod, part)
            if ok:
                mod.weight.data.mul_(s)


def norm_eps(module: nn.RMSNorm, dtype: torch.dtype = torch.float32) -> float:
    """The eps ``nn.RMSNorm(eps=None)`` resolves to for an input of ``dtype``."""
    return torch.finfo(dtype).eps if module.eps is None else float(module.eps)


def apply_norm(module: nn.RMSNorm, x: torch.Tensor) -> torch.Tensor:
    """``module(x)``; CUDA inputs whose width the RMSNorm kernel takes run it (fp32
    statistics, the module's weight and resolved eps, output in x's dtype)."""
    from pluggy_b200.ops.norm import rms_norm

    if x.is_cuda and x.shape[-1] % 128 == 0 and x.dtype in (torch.float32, torch.bfloat16):
        return rms_norm(x, module.weight, norm_eps(module, x.dtype))
    return module(x)


def scaled_init_std(d: int) -> float:
    return 1.0 / math.sqrt(d)


__all__ = ["RotaryEmbedding", "GQAttention", "SwiGLU", "attend", "default_ffn_dim",
           "init_decoder_weights", "position_ids_for", "norm_eps", "F"]
