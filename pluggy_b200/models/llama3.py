"""Llama-3 decoder: Qwen3's block without q/k norm, RoPE base 5e5.

Parity: reference ``pluggy/models/llama3/llama3.py:17-243`` (attention module
named ``attn``; ``head_dim`` defaults to ``emb_dim // num_heads``; untied LM
head). Addition: ``tie_embeddings`` (default False, the reference behaviour)
ties ``lm_head`` to ``token_emb`` as the Llama-3.2-1B benchmark config asks.
Runs on the same fused sm_100a sublayers as Qwen3 on CUDA.
"""

from __future__ import annotations

from pluggy_b200.models.qwen3 import Qwen3, Qwen3TransformerBlock


class Llama3TransformerBlock(Qwen3TransformerBlock):
    attn_name = "attn"
    qk_norm = False


class Llama3(Qwen3):
    rope_base = 500_000.0
    tie_default = False
    block_cls = Llama3TransformerBlock

    def __init__(self, num_layers: int, num_heads: int, num_kv_heads: int, emb_dim: int,
                 vocab_size: int, head_dim: int | None = None, ffn_dim: int | None = None,
                 rope_base: float = 500_000.0, tie_embeddings: bool = False):
        super().__init__(num_layers=num_layers, num_heads=num_heads, num_kv_heads=num_kv_heads,
                         emb_dim=emb_dim, head_dim=head_dim, vocab_size=vocab_size, ffn_dim=ffn_dim,
                         tie_embeddings=tie_embeddings, rope_base=rope_base)

    def init_weights(self, std: float = 0.02) -> None:
        from pluggy_b200.models.common import init_decoder_weights

        init_decoder_weights(self, self.blocks, std, out_projs=("attn.o_proj", "ffn.down_proj"))
