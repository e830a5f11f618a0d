"""Objective registry (reference ``pluggy/objectives/builder.py:9-16``)."""

from pluggy_b200.objectives.autoregressive import ARObjective

OBJECTIVE_REGISTRY = {"AR": ARObjective}


def build_objective(objective_name: str, objective_config: dict):
    assert objective_name in OBJECTIVE_REGISTRY, f"objective {objective_name!r} not in registry"
    return OBJECTIVE_REGISTRY[objective_name](**objective_config)
