"""Model contract checker: what the trainer, objective and checkpointer rely on.

Parity: reference ``pluggy/models/contract.py:58-229``. On CPU, for a model built
from the registry (or given directly), it checks:

* attributes: ``token_emb``, ``blocks``, ``norm``, ``lm_head``, ``init_weights``;
* the three forward modes and their shapes: logits ``[B, S, V]``,
  ``(logits, hidden_states)`` with one state per block plus the embedding, and the
  post-norm final hidden ``[B, S, D]``;
* the padded (attention-mask) path runs and stays finite;
* causality: changing a later token leaves earlier logits unchanged;
* reachability: token 0 moves the last position's logits;
* residual scaling: the residual writers (o/down projections) start at
  ``std / sqrt(2 L)``;
* a fresh model's cross-entropy is ln(V) within 1.5;
* the fused linear-CE objective reaches every parameter with a gradient;
* one block's forward + backward finishes within a time budget (the reference
  checks that a block compiles in 30 s; this framework does not compile blocks,
  so the same budget bounds an eager step instead).

``check`` returns the list of failures; ``python -m pluggy_b200.models.contract
--model NAME --config JSON`` prints them and exits non-zero on any.
"""

from __future__ import annotations

import argparse
import json
import math
import sys
import time

import torch
import torch.nn as nn


class ContractError(AssertionError):
    pass


def build(name: str, config: dict) -> nn.Module:
    from pluggy_b200.models.builder import build_model

    return build_model(name, config)


def _residual_writers(model):
    for blk in model.blocks:
        for path in ("gqa.o_proj", "attn.o_proj", "attention.o_proj", "ffn.down_proj"):
            mod = blk
            for part in path.split("."):
                mod = getattr(mod, part, None)
                if mod is None:
                    break
            if isinstance(mod, nn.Linear):
                yield path, mod.weight


def check(model: nn.Module, *, batch: int = 2, seq: int = 16, seed: int = 0,
          std: float = 0.02, block_budget_s: float = 30.0) -> list[str]:
    """Run every check on CPU; returns human-readable failures (empty = pass)."""
    from pluggy_b200.objectives.autoregressive import ARObjective

    fails: list[str] = []
    torch.manual_seed(seed)
    for attr in ("token_emb", "blocks", "norm", "lm_head"):
        if not hasattr(model, attr):
            fails.append(f"missing attribute {attr}")
    if not callable(getattr(model, "init_weights", None)):
        fails.append("missing init_weights()")
    if fails:
        return fails
    model = model.cpu().float()
    model.init_weights(std) if "std" in model.init_weights.__code__.co_varnames else model.init_weights()
    V = model.lm_head.weight.shape[0]
    D = model.token_emb.weight.shape[1]
    L = len(model.blocks)
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, V, (batch, seq), generator=g)

    with torch.no_grad():
        logits = model(ids)
        if tuple(logits.shape) != (batch, seq, V):
            fails.append(f"logits shape {tuple(logits.shape)} != {(batch, seq, V)}")
        out = model(ids, return_hidden_states=True)
        if not (isinstance(out, tuple) and len(out) == 2 and len(out[1]) == L + 1):
            fails.append("return_hidden_states must give (logits, [embedding] + one state per block)")
        hid = model(ids, return_final_hidden=True)
        if tuple(hid.shape) != (batch, seq, D):
            fails.append(f"final hidden shape {tuple(hid.shape)} != {(batch, seq, D)}")
        mask = torch.ones(batch, seq, dtype=torch.long)
        mask[0, : seq // 4] = 0  # left padding on the first row
        padded = model(ids, attention_mask=mask)
        if not torch.isfinite(padded[mask.bool()]).all():
            fails.append("padded path produced non-finite logits")
        t = seq // 2
        ids2 = ids.clone()
        ids2[:, t] = (ids2[:, t] + 1) % V
        l2 = model(ids2)
        if not torch.allclose(l2[:, :t], logits[:, :t], atol=1e-5, rtol=1e-5):
            fails.append(f"not causal: changing token {t} moved earlier logits")
        ids3 = ids.clone()
        ids3[:, 0] = (ids3[:, 0] + 1) % V
        l3 = model(ids3)
        if torch.allclose(l3[:, -1], logits[:, -1], atol=1e-7, rtol=0):
            fails.append("token 0 does not reach the last position")
        ce = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, V), ids[:, 1:].reshape(-1))
        if abs(ce.item() - math.log(V)) > 1.5:
            fails.append(f"fresh CE {ce.item():.3f} not within 1.5 of ln(V)={math.log(V):.3f}")

    want = std / math.sqrt(2 * L)
    for path, w in _residual_writers(model):
        s = w.detach().std().item()
        if not (0.5 * want < s < 1.5 * want):
            fails.append(f"residual writer {path} std {s:.4g}, expected ~{want:.4g}")
            break

    model.zero_grad(set_to_none=True)
    loss = ARObjective(ce_chunk_size=max(1, batch * seq // 2)).compute_loss(
        model, {"input_ids": ids, "labels": ids})
    loss.backward()
    for n, p in model.named_parameters():
        if p.requires_grad and (p.grad is None or not torch.isfinite(p.grad).all()):
            fails.append(f"no finite grad for {n} through the fused CE")
    model.zero_grad(set_to_none=True)

    blk = model.blocks[0]
    x = torch.randn(batch, seq, D, requires_grad=True)
    cos_sin = model.rope(torch.arange(seq).unsqueeze(0).expand(batch, -1), cacheable=False) \
        if hasattr(model, "rope") else (None, None)
    t0 = time.perf_counter()
    try:
        y = blk(x, *cos_sin)
        y.float().sum().backward()
    except TypeError:
        pass  # blocks with a different signature are covered by the full-model checks
    if time.perf_counter() - t0 > block_budget_s:
        fails.append(f"one block forward+backward took more than {block_budget_s} s")
    return fails


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="check a model against the contract")
    p.add_argument("--model", help="registry key")
    p.add_argument("--module", help="module of an unregistered model (with --class)")
    p.add_argument("--class", dest="cls", help="class name inside --module")
    p.add_argument("--config", required=True, help="JSON model config (or @file.json)")
    a = p.parse_args(argv)
    cfg = a.config
    if cfg.startswith("@"):
        with open(cfg[1:]) as f:
            cfg = f.read()
    cfg = json.loads(cfg)
    if a.module:
        import importlib

        if not a.cls:
            p.error("--module needs --class")
        model = getattr(importlib.import_module(a.module), a.cls)(**cfg)
    elif a.model:
        model = build(a.model, cfg)
    else:
        p.error("give --model, or --module and --class")
    fails = check(model)
    for f in fails:
        print(f"FAIL {f}")
    print("contract: OK" if not fails else f"contract: {len(fails)} failure(s)")
    return 1 if fails else 0


if __name__ == "__main__":
    sys.exit(main())
