"""Model registry: config name -> class; the config dict is the constructor kwargs.

Parity: reference ``pluggy/models/builder.py:11-24`` (same registry names).
The reference also imports two modules that are absent from its tree
(``grokathon_model``, ``hybrid_test``); this registry only lists families that
exist. Families written by the model-writer agent are listed in JSON registry
files (``{"key": "package.module:ClassName"}``): ``models/generated/registry.json``
and any files named in ``PLG_MODEL_REGISTRY_FILES`` (``os.pathsep``-separated).
They are imported on first use, so a broken generated file can only fail the run
that asks for it.
"""

from __future__ import annotations

import importlib
import json
import os

import torch.nn as nn

from pluggy_b200.models.gemma4 import Gemma4
from pluggy_b200.models.llama3 import Llama3
from pluggy_b200.models.olmo3 import Olmo3
from pluggy_b200.models.qwen3 import Qwen3
from pluggy_b200.models.qwen3_moe import Qwen3Moe

MODEL_REGISTRY: dict[str, type[nn.Module]] = {
    "qwen3_dense": Qwen3,
    "qwen3_moe": Qwen3Moe,
    "llama3_2": Llama3,
    "olmo3": Olmo3,
    "gemma4": Gemma4,
}


def register_model(name: str, dotted: str) -> None:
    """Register ``package.module:ClassName`` under ``name``."""
    mod, cls = dotted.split(":")
    MODEL_REGISTRY[name] = getattr(importlib.import_module(mod), cls)


GENERATED_REGISTRY = os.path.join(os.path.dirname(os.path.abspath(__file__)), "generated",
                                  "registry.json")


def generated_entries() -> dict[str, str]:
    """Registry key -> ``module:Class`` of the generated families (later files win)."""
    out: dict[str, str] = {}
    extra = [p for p in os.environ.get("PLG_MODEL_REGISTRY_FILES", "").split(os.pathsep) if p]
    for path in [GENERATED_REGISTRY, *extra]:
        try:
            with open(path) as f:
                out.update(json.load(f))
        except FileNotFoundError:
            continue
    return out


def resolve(model_name: str) -> type[nn.Module]:
    if model_name not in MODEL_REGISTRY:
        dotted = generated_entries().get(model_name)
        if dotted is None:
            raise KeyError(f"model name {model_name!r} not in registry: "
                           f"{sorted(MODEL_REGISTRY) + sorted(generated_entries())}")
        register_model(model_name, dotted)
    return MODEL_REGISTRY[model_name]


def build_model(model_name: str, model_config: dict) -> nn.Module:
    return resolve(model_name)(**model_config)
