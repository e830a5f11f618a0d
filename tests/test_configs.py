"""Every shipped config validates (train configs against the registries and constructor
signatures, the synthetic-data config against the front end's checks)."""

import glob
import json
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CONFIGS = sorted(glob.glob(os.path.join(ROOT, "configs", "*.json")))


@pytest.mark.parametrize("path", CONFIGS, ids=[os.path.basename(p) for p in CONFIGS])
def test_config_validates(path):
    with open(path) as f:
        cfg = json.load(f)
    if "seed_domains" in cfg or "grounding" in cfg:
        from pluggy_b200.synth.server import validate_synth

        assert validate_synth(cfg) is None
    else:
        from pluggy_b200.train.validate import validate_config

        validate_config(cfg)


def test_configs_present():
    assert len(CONFIGS) >= 6


def test_cuda_graph_key_is_checked():
    from pluggy_b200.train.validate import ConfigError, validate_config

    with open(os.path.join(ROOT, "configs", "qwen3_0.6b_ddp_synthetic.json")) as f:
        cfg = json.load(f)
    cfg["mesh"] = {"dp": 1}
    cfg["cuda_graph"] = True
    validate_config(cfg)
    for bad in ({"cuda_graph": "yes"}, {"cuda_graph": True, "mesh": {"dp": 2}},
                {"cuda_graph": True, "parallelism": "fsdp2"}):
        c = dict(cfg, **bad)
        with pytest.raises(ConfigError, match="cuda_graph"):
            validate_config(c)
