"""Model-writer agent: an LLM writes a new architecture into the tree, validated.

Parity: reference ``pluggy/synth/write_model.py:1-477``.

    python -m pluggy_b200.synth.write_model --name rwkv_like --description "..."
    python -m pluggy_b200.synth.write_model --name x --description "..." --no-kernels

Steps:

1. prompt the model (grok by default; any ``claude-*`` name goes to Anthropic) with
   the model contract, an index of the tree, the registry, the nearest existing
   implementation(s) chosen by keywords in the description, and, unless
   ``--no-kernels``, the fused-op surface it may import (``pluggy_b200.ops``);
2. write ``pluggy_b200/models/generated/<name>.py`` (with a provenance banner) and
   any helper modules it asked for as ``<name>_<helper>.py`` beside it;
3. run the file's own ``__main__`` scaffold (constructs, initialises, one forward);
4. run the contract check (``pluggy_b200.models.contract``) on the same
   architecture shrunk to CPU size, keeping its depth;
5. on a failure, hand the output back for a bounded number of repair rounds;
6. only then add ``key -> module:Class`` to ``models/generated/registry.json``,
   and check in a fresh interpreter that the registry resolves it; on any
   failure the registry file is restored, so an unvalidated model is never
   registered (its file stays on disk for inspection).

The registry is a JSON file rather than an edit to ``builder.py``: the trainer
imports the builder for every run, and a registry entry is only imported when a
run asks for that key, so a bad generated file cannot break other runs.

The last line on success is ``RESULT {json}``, which the web front end reads.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
from pathlib import Path

from pluggy_b200.synth.llm import build_client

PKG = Path(__file__).resolve().parents[1]
ROOT = PKG.parent
MARK = "written by pluggy_b200.synth.write_model"
BANNER = (f"# {MARK}: it passed its own scaffold and the model contract check,\n"
          "# but no person has reviewed it. Treat its patterns as unproven.\n")

# keyword triggers -> the closest existing implementation to show the model
REFERENCES = [
    (("moe", "mixture of experts", "expert", "router", "sparse"), "models/qwen3_moe.py"),
    (("sliding", "hybrid", "local attention", "softcap", "geglu", "per-layer"), "models/gemma4.py"),
]
BASE_REFERENCE = "models/qwen3.py"

SCHEMA = {
    "type": "object",
    "required": ["registry_key", "class_name", "model_code", "helpers", "config_json", "summary"],
    "properties": {
        "registry_key": {"type": "string"},
        "class_name": {"type": "string"},
        "model_code": {"type": "string"},
        "helpers": {"type": "array", "items": {
            "type": "object", "required": ["filename", "code", "why"],
            "properties": {"filename": {"type": "string"}, "code": {"type": "string"},
                           "why": {"type": "string"}}}},
        "config_json": {"type": "string"},
        "summary": {"type": "string"},
    },
}

SYSTEM = ("You write PyTorch language-model architectures for pluggy_b200, a training "
          "framework for NVIDIA B200 GPUs. The trainer, the fused-CE objective and the "
          "parallelism layer reach into models by attribute name, so the contract you are "
          "given is binding: a deviation shows up as a wrong loss curve, not an error. "
          "Return complete files, never diffs or ellipses.")

CONTRACT = """\
A model is an nn.Module whose __init__ keyword arguments are the config schema (the
trainer calls Class(**config), so every argument is a plain JSON value). It has:
- token_emb (nn.Embedding), blocks (nn.ModuleList), norm (the final norm), lm_head
  (nn.Linear, bias-free; weight tied to token_emb when tie_embeddings is set);
- forward(input_ids, attention_mask=None, return_hidden_states=False,
  return_final_hidden=False): logits [B, S, V]; with return_hidden_states,
  (logits, [embedding output] + one hidden state per block); with
  return_final_hidden, the post-norm hidden [B, S, D] and lm_head is NOT applied
  (the fused linear-CE objective applies it chunk by chunk);
- causal attention: the packed-training path (no mask) and a padded path
  (attention_mask [B, S] of 0/1) that stays finite;
- init_weights(std=0.02): normal(0, std) weights, and std / sqrt(2 * num_layers)
  on every projection that writes into the residual stream (attention output and
  FFN down projections);
- a fresh model's cross entropy is close to ln(vocab_size).
The check that enforces this is pluggy_b200.models.contract.check (source below)."""


def log(msg: str) -> None:
    print(msg, flush=True)


def gen_dir() -> Path:
    return Path(os.environ.get("PLG_GENERATED_DIR", PKG / "models" / "generated"))


def gen_package() -> str:
    return os.environ.get("PLG_GENERATED_PACKAGE", "pluggy_b200.models.generated")


def registry_file() -> Path:
    return gen_dir() / "registry.json"


def pick_references(description: str) -> list[str]:
    want = description.lower()
    return [BASE_REFERENCE] + [p for keys, p in REFERENCES if any(k in want for k in keys)]


def tree_index() -> str:
    lines = ["Model families in the tree (follow the nearest one rather than reinventing it):"]
    generated = []
    for path in sorted((PKG / "models").glob("*.py")) + sorted(gen_dir().glob("*.py")):
        if path.stem.startswith("_") or path.stem in ("builder", "contract", "hf_import"):
            continue
        text = path.read_text()
        entry = f"- {path.relative_to(path.parents[1])} ({len(text.splitlines())} lines)"
        (generated if MARK in text else lines).append(entry)
    if generated:
        lines.append("Also present but written by this tool and never reviewed; take no patterns "
                     "from these:")
        lines += generated
    return "\n".join(lines)


def build_prompt(name: str, description: str, references: list[str], kernels: bool) -> str:
    parts = ["# The model contract\n\n" + CONTRACT,
             "# pluggy_b200/models/contract.py\n\n```python\n" + (PKG / "models" / "contract.py").read_text() + "```",
             "# " + tree_index()]
    for ref in references:
        parts.append(f"# Reference implementation: pluggy_b200/{ref}\n\n```python\n"
                     f"{(PKG / ref).read_text()}```")
    if kernels:
        parts.append("# Fused ops you may import\n\n```python\n" + (PKG / "ops" / "__init__.py").read_text()
                     + "```\nEach runs a hand-written sm_100a kernel on CUDA tensors and the same math in "
                     "eager PyTorch on CPU, so a model that uses them still runs on CPU. Prefer them "
                     "over re-implementing attention, norms, GLUs or cross entropy.")
    parts.append(
        f"# The task\n\nWrite `{gen_package()}.{name}` (one file) implementing:\n\n{description.strip()}\n\n"
        "Rules: torch, the standard library and pluggy_b200 imports only. "
        + ("Helper modules may be returned in `helpers` (file names end in .py; each is saved "
           f"as `{name}_<filename>` beside the model and imported from `{gen_package()}`). "
           if kernels else "Return an empty `helpers` list and use plain torch ops. ")
        + "End the file with an `if __name__ == \"__main__\":` scaffold that builds a small "
        "instance, calls init_weights(), runs one forward on random ids and prints the "
        "parameter count; it is the first check that runs. `config_json` is the model.config "
        "block (the exact __init__ kwargs) at roughly 1B parameters; `registry_key` matches "
        "[a-z0-9_]+; `summary` says in two or three sentences what the architecture is.")
    return "\n\n---\n\n".join(parts)


def write_files(name: str, result: dict, kernels: bool) -> list[Path]:
    d = gen_dir()
    d.mkdir(parents=True, exist_ok=True)
    init = d / "__init__.py"
    if not init.exists():
        init.write_text('"""Generated model families."""\n')
    path = d / f"{name}.py"
    path.write_text(BANNER + result["model_code"])
    out = [path]
    for h in (result.get("helpers") or []) if kernels else []:
        fn = Path(str(h.get("filename", ""))).name
        if not fn.endswith(".py") or fn == "__init__.py" or not re.fullmatch(r"[A-Za-z0-9_]+\.py", fn):
            log(f"  skipped a helper with an unusable file name {h.get('filename')!r}")
            continue
        hp = d / f"{name}_{fn}"
        hp.write_text(BANNER + h["code"])
        out.append(hp)
        log(f"  helper {hp.name}: {h.get('why', '')}")
    return out


def _run(args: list[str], timeout: int = 900) -> tuple[bool, str]:
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(p for p in (str(ROOT), env.get("PYTHONPATH", "")) if p)
    p = subprocess.run([sys.executable, *args], cwd=ROOT, capture_output=True, text=True,
                       timeout=timeout, env=env)
    return p.returncode == 0, (p.stdout + p.stderr)[-4000:]


def scaffold(name: str) -> tuple[bool, str]:
    return _run(["-m", f"{gen_package()}.{name}"])


def shrink(config: dict) -> dict:
    """The same architecture at CPU-test size; depth is kept (residual scaling reads it)."""
    small = dict(config)
    caps = {"emb_dim": 128, "head_dim": 32, "global_head_dim": 32, "num_heads": 4, "num_kv_heads": 2,
            "vocab_size": 2000, "ffn_dim": 256, "moe_ffn_dim": 64, "num_experts": 4, "top_k": 2}
    for k, cap in caps.items():
        if isinstance(small.get(k), int) and not isinstance(small[k], bool):
            small[k] = min(small[k], cap)
    if isinstance(small.get("num_layers"), int):
        small["num_layers"] = min(small["num_layers"], 8)
    if small.get("num_kv_heads", 1) > small.get("num_heads", 1):
        small["num_kv_heads"] = small["num_heads"]
    return small


def contract(name: str, cls: str, config: dict) -> tuple[bool, str]:
    return _run(["-m", "pluggy_b200.models.contract", "--module", f"{gen_package()}.{name}",
                 "--class", cls, "--config", json.dumps(shrink(config))])


def register(key: str, name: str, cls: str) -> None:
    reg = registry_file()
    cur = json.loads(reg.read_text()) if reg.exists() else {}
    cur[key] = f"{gen_package()}.{name}:{cls}"
    tmp = reg.with_name(reg.name + ".tmp")
    tmp.write_text(json.dumps(cur, indent=2, sort_keys=True) + "\n")
    os.replace(tmp, reg)


def _config(result: dict) -> dict:
    try:
        c = json.loads(result.get("config_json") or "{}")
        return c if isinstance(c, dict) else {}
    except json.JSONDecodeError:
        return {}


def generate(name: str, description: str, model: str, kernels: bool, repairs: int,
             max_tokens: int, client=None) -> dict:
    client = client if client is not None else build_client(
        {"model": model, "generation": {"temperature": 0.2}})
    refs = pick_references(description)
    log("references: " + ", ".join(refs))
    prompt = build_prompt(name, description, refs, kernels)
    log(f"prompting {model} ({len(prompt) // 4} tokens of context)")
    result = client.generate_json(prompt, SCHEMA, system=SYSTEM, max_tokens=max_tokens)
    if result is None:
        raise RuntimeError("the model returned nothing usable (often: the answer hit "
                           f"max_tokens={max_tokens}; raise --max-tokens)")
    if not re.fullmatch(r"[a-z0-9_]+", result["registry_key"]) or \
            not re.fullmatch(r"[A-Za-z_][A-Za-z0-9_]*", result["class_name"]):
        raise RuntimeError(f"unusable registry_key/class_name: {result['registry_key']!r}, "
                           f"{result['class_name']!r}")
    reg = registry_file()
    before = reg.read_text() if reg.exists() else None
    try:
        for attempt in range(repairs + 1):
            write_files(name, result, kernels)
            log(f"validating: python -m {gen_package()}.{name}")
            stage = "its own __main__ scaffold"
            ok, out = scaffold(name)
            if ok:
                log(out.strip()[-500:])
                log("checking the model contract")
                stage = "the model contract check"
                ok, out = contract(name, result["class_name"], _config(result))
                if ok:
                    log(out.strip()[-800:])
                    break
            log(f"  failed:\n{out.strip()[-1500:]}")
            if attempt == repairs:
                raise RuntimeError(f"the model still fails {stage} after {repairs} repair round(s); "
                                   f"it is left unregistered in {gen_dir() / (name + '.py')}")
            log(f"repair round {attempt + 1}/{repairs}")
            result = client.generate_json(
                f"The file you wrote fails {stage}. Return the complete corrected answer (same "
                f"schema, whole files).\n\n# Output\n\n```\n{out}\n```\n\n# The file\n\n```python\n"
                f"{result['model_code']}```", SCHEMA, system=SYSTEM, max_tokens=max_tokens) or result
        key = result["registry_key"]
        register(key, name, result["class_name"])
        ok, out = _run(["-c", "from pluggy_b200.models.builder import resolve; "
                              f"assert resolve({key!r}) is not None"], timeout=300)
        if not ok:
            raise RuntimeError("the registry does not resolve the new key:\n" + out[-1500:])
    except Exception:
        if before is None:
            reg.unlink(missing_ok=True)
        else:
            reg.write_text(before)
        raise
    return {"registry_key": key, "class_name": result["class_name"],
            "model_file": str(gen_dir() / f"{name}.py"),
            "helpers": [h["filename"] for h in result.get("helpers") or []] if kernels else [],
            "config": _config(result), "summary": result["summary"]}


def main(argv=None, client=None) -> int:
    p = argparse.ArgumentParser(description="have an LLM write a validated model family")
    p.add_argument("--name", required=True, help="module name, [A-Za-z0-9_]+")
    p.add_argument("--description", required=True)
    p.add_argument("--model", default="grok-4")
    p.add_argument("--no-kernels", dest="kernels", action="store_false")
    p.add_argument("--repairs", type=int, default=2)
    p.add_argument("--max-tokens", type=int, default=32768)
    p.add_argument("--overwrite", action="store_true")
    a = p.parse_args(argv)
    if not re.fullmatch(r"[A-Za-z0-9_]+", a.name):
        print("--name must match [A-Za-z0-9_]+ (it becomes a module name)")
        return 2
    if (gen_dir() / f"{a.name}.py").exists() and not a.overwrite:
        print(f"{gen_dir() / (a.name + '.py')} exists; pass --overwrite or pick another name")
        return 2
    try:
        res = generate(a.name, a.description, a.model, a.kernels, a.repairs, a.max_tokens, client)
    except Exception as e:  # noqa: BLE001 - reported on the log the front end shows
        log(f"FAILED: {e}")
        return 1
    log(f"registered {res['registry_key']} -> {res['class_name']}")
    log(res["summary"])
    log("RESULT " + json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
