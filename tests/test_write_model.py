"""Model-writer agent with a scripted LLM: write -> scaffold -> contract -> repair -> register."""

import json
import subprocess
import sys

from pluggy_b200.synth import write_model as wm
from pluggy_b200.synth.llm import ScriptedClient

GOOD = '''
import torch
from pluggy_b200.models.qwen3 import Qwen3


class TinyQ(Qwen3):
    """Qwen3 under another name."""


if __name__ == "__main__":
    m = TinyQ(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=64, head_dim=16, vocab_size=128,
              ffn_dim=128)
    m.init_weights()
    print(tuple(m(torch.randint(0, 128, (1, 8))).shape), sum(p.numel() for p in m.parameters()))
'''

CFG = {"num_layers": 4, "num_heads": 16, "num_kv_heads": 8, "emb_dim": 1024, "head_dim": 128,
       "vocab_size": 151936, "ffn_dim": 3072}


def _answer(code):
    return json.dumps({"registry_key": "tiny_q", "class_name": "TinyQ", "model_code": code,
                       "helpers": [], "config_json": json.dumps(CFG), "summary": "A renamed Qwen3."})


def test_write_repair_register(tmp_path, monkeypatch):
    pkg = tmp_path / "plg_gen_test"
    monkeypatch.setenv("PLG_GENERATED_DIR", str(pkg))
    monkeypatch.setenv("PLG_GENERATED_PACKAGE", "plg_gen_test")
    monkeypatch.setenv("PYTHONPATH", str(tmp_path))
    monkeypatch.setenv("PLG_MODEL_REGISTRY_FILES", str(pkg / "registry.json"))
    prompts = []

    def fn(prompt, system, max_tokens):
        prompts.append(prompt)
        if len(prompts) == 1:
            return _answer(GOOD.replace('    m.init_weights()', '    raise RuntimeError("boom")'))
        return _answer(GOOD)

    rc = wm.main(["--name", "tiny_q", "--description", "Qwen3 again, renamed, for a test run.",
                  "--no-kernels", "--repairs", "1"], client=ScriptedClient(fn))
    assert rc == 0
    assert len(prompts) == 2 and "boom" in prompts[1]  # the failure was handed back
    assert "The model contract" in prompts[0] and "qwen3.py" in prompts[0]
    reg = json.loads((pkg / "registry.json").read_text())
    assert reg == {"tiny_q": "plg_gen_test.tiny_q:TinyQ"}
    assert (pkg / "tiny_q.py").read_text().startswith("# " + wm.MARK)
    # a fresh interpreter builds it through the registry
    code = ("from pluggy_b200.models.builder import build_model; "
            "m = build_model('tiny_q', dict(num_layers=1, num_heads=2, num_kv_heads=1, emb_dim=32, "
            "head_dim=16, vocab_size=64, ffn_dim=64)); print(type(m).__name__)")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300,
                         env={**__import__("os").environ, "PYTHONPATH": f"{tmp_path}:{wm.ROOT}"})
    assert out.stdout.strip() == "TinyQ", out.stderr


def test_unvalidated_model_is_not_registered(tmp_path, monkeypatch):
    pkg = tmp_path / "plg_gen_test2"
    monkeypatch.setenv("PLG_GENERATED_DIR", str(pkg))
    monkeypatch.setenv("PLG_GENERATED_PACKAGE", "plg_gen_test2")
    monkeypatch.setenv("PYTHONPATH", str(tmp_path))
    bad = GOOD.replace('    m.init_weights()', '    raise RuntimeError("boom")')
    rc = wm.main(["--name", "bad_q", "--description", "a model that never constructs properly",
                  "--repairs", "1"], client=ScriptedClient(lambda *a: _answer(bad)))
    assert rc == 1
    assert (pkg / "bad_q.py").exists() and not (pkg / "registry.json").exists()


def test_shrink_and_references():
    s = wm.shrink({**CFG, "num_layers": 28, "num_experts": 128, "top_k": 8, "tie_embeddings": True})
    assert s["num_layers"] == 8 and s["emb_dim"] == 128 and s["num_experts"] == 4 and s["top_k"] == 2
    assert s["tie_embeddings"] is True
    assert wm.pick_references("a sparse mixture of experts") == ["models/qwen3.py", "models/qwen3_moe.py"]
    assert wm.pick_references("plain dense") == ["models/qwen3.py"]
