"""Model registry: config name -> class; the config dict is the constructor kwargs.

Parity: reference ``pluggy/models/builder.py:11-24`` (same registry names).
The reference also imports two modules that are absent from its tree
(``grokathon_model``, ``hybrid_test``); this registry only lists families that
exist. ``register_model`` lets the model-writer agent add generated families.
"""

from __future__ import annotations

import importlib

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


def build_model(model_name: str, model_config: dict) -> nn.Module:
    assert model_name in MODEL_REGISTRY, f"model name {model_name!r} not in registry"
    return MODEL_REGISTRY[model_name](**model_config)
