"""The model contract holds for every registered decoder family (CPU), and the checker
catches a model that breaks it."""

import pytest
import torch

CFGS = {
    "qwen3_dense": dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=64, head_dim=16,
                        vocab_size=128, ffn_dim=128),
    "llama3_2": dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=64, head_dim=16,
                     vocab_size=128, ffn_dim=128),
    "qwen3_moe": dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=64, head_dim=16,
                      vocab_size=128, moe_ffn_dim=32, num_experts=4, top_k=2, ffn_dim=128),
    "olmo3": dict(num_layers=4, num_heads=4, num_kv_heads=2, emb_dim=64, head_dim=16,
                  vocab_size=128, ffn_dim=128, sliding_window=8),
    "gemma4": dict(num_layers=3, num_heads=4, num_kv_heads=2, emb_dim=64, head_dim=16,
                   global_head_dim=32, vocab_size=128, ffn_dim=128, sliding_window=8,
                   layer_pattern=3, num_kv_shared_layers=1, hidden_size_per_layer_input=8),
}


@pytest.mark.parametrize("name", sorted(CFGS))
def test_registered_models_pass(name):
    from pluggy_b200.models.contract import build, check

    assert check(build(name, CFGS[name])) == []


def test_checker_catches_non_causal_model():
    from pluggy_b200.models.contract import build, check

    m = build("qwen3_dense", CFGS["qwen3_dense"])
    orig = m.forward

    def leaky(x, *a, **k):
        # every position sees the mean of the whole sequence's embeddings
        out = orig(x, *a, **k)
        if isinstance(out, torch.Tensor) and out.dim() == 3 and not k.get("return_final_hidden"):
            out = out + m.token_emb(x).mean(dim=1, keepdim=True).sum(-1, keepdim=True)
        return out

    m.forward = leaky
    fails = check(m)
    assert any("not causal" in f for f in fails), fails


def test_cli(capsys):
    import json

    from pluggy_b200.models.contract import main

    assert main(["--model", "qwen3_dense", "--config", json.dumps(CFGS["qwen3_dense"])]) == 0
    assert "contract: OK" in capsys.readouterr().out
