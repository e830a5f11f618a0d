"""HF checkpoint import: safetensors round trip, name map, sharded index, loud failures."""

import json
import os

import pytest
import torch

TINY = dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=32, head_dim=8, vocab_size=64,
            ffn_dim=64)


def _export(model, attn="gqa"):
    from pluggy_b200.models.hf_import import local_to_hf

    out = {}
    for n, p in model.named_parameters():
        hf = local_to_hf(n, attn)
        assert hf is not None, n
        out[hf] = p.detach().to(torch.bfloat16)
    return out


def test_safetensors_round_trip(tmp_path):
    from safetensors.torch import load_file

    from pluggy_b200.models.hf_import import read_safetensors, write_safetensors

    ts = {"a": torch.randn(3, 5), "b": torch.arange(7, dtype=torch.int64),
          "c": torch.randn(2, 2).bfloat16(), "empty": torch.zeros(0)}
    p = str(tmp_path / "x.safetensors")
    write_safetensors(ts, p, metadata={"format": "pt"})
    back = read_safetensors(p)
    theirs = load_file(p)  # the published reader agrees with ours
    for k, v in ts.items():
        assert torch.equal(back[k], v) and torch.equal(theirs[k], v)


@pytest.mark.parametrize("cls,attn", [("qwen3", "gqa"), ("llama3", "attn")])
def test_load_hf_weights_sharded(tmp_path, cls, attn):
    from pluggy_b200.models.hf_import import load_hf_weights, write_safetensors
    from pluggy_b200.models.llama3 import Llama3
    from pluggy_b200.models.qwen3 import Qwen3

    C = Qwen3 if cls == "qwen3" else Llama3
    torch.manual_seed(0)
    src = C(**TINY, tie_embeddings=True)
    src.init_weights()
    hf = _export(src, attn)
    hf.pop("lm_head.weight", None)  # tied: HF checkpoints omit it
    names = sorted(hf)
    half = len(names) // 2
    shards = {"model-00001-of-00002.safetensors": names[:half],
              "model-00002-of-00002.safetensors": names[half:]}
    wm = {}
    for fn, keys in shards.items():
        write_safetensors({k: hf[k] for k in keys}, str(tmp_path / fn))
        wm.update({k: fn for k in keys})
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"weight_map": wm}, f)
    dst = C(**TINY, tie_embeddings=True)
    n = load_hf_weights(dst, str(tmp_path))
    assert n == len(hf)
    for (a, p), (_, q) in zip(src.named_parameters(), dst.named_parameters()):
        assert q.dtype == torch.float32
        assert torch.equal(q, p.detach().bfloat16().float()), a


def test_load_hf_weights_fails_loudly(tmp_path):
    from pluggy_b200.models.hf_import import load_hf_weights, write_safetensors
    from pluggy_b200.models.qwen3 import Qwen3

    torch.manual_seed(0)
    m = Qwen3(**TINY, tie_embeddings=True)
    hf = _export(m)
    hf.pop("lm_head.weight", None)
    before = {k: v.clone() for k, v in m.state_dict().items()}

    def attempt(tensors, err):
        d = tmp_path / f"case{len(os.listdir(tmp_path))}"
        d.mkdir()
        write_safetensors(tensors, str(d / "model.safetensors"))
        with pytest.raises(err):
            load_hf_weights(m, str(d))
        for k, v in m.state_dict().items():  # nothing was modified
            assert torch.equal(v, before[k])

    extra = dict(hf)
    extra["model.layers.0.mlp.router.weight"] = torch.zeros(2, 2)
    attempt(extra, KeyError)
    missing = dict(hf)
    missing.pop("model.layers.1.mlp.down_proj.weight")
    attempt(missing, KeyError)
    wrong = dict(hf)
    wrong["model.norm.weight"] = torch.zeros(31)
    attempt(wrong, ValueError)
