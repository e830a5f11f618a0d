"""Startup validation of a training config (structure + constructor signatures).

The reference validates configs only inside its web server
(``pluggy/synth/server.py:281-384``: constructor signatures are the schema) and
its roadmap asks for a startup ``validate()``; this module is that pass, shared
by the trainer and the web server.
"""

from __future__ import annotations

import inspect

REQUIRED_TOP = ("model", "mesh", "optimizer", "objective", "data", "run_name")


class ConfigError(ValueError):
    pass


def kwarg_error(cls, cfg: dict, what: str) -> str | None:
    sig = inspect.signature(cls.__init__)
    params = {k: p for k, p in sig.parameters.items() if k != "self"}
    if any(p.kind == p.VAR_KEYWORD for p in params.values()):
        return None
    unknown = sorted(set(cfg) - set(params))
    if unknown:
        return f"{what}: unknown argument(s) {unknown}"
    missing = sorted(k for k, p in params.items()
                     if p.default is p.empty and p.kind not in (p.VAR_POSITIONAL, p.VAR_KEYWORD)
                     and k not in cfg and k != "optimizer")
    if missing:
        return f"{what}: missing required argument(s) {missing}"
    return None


def validate_config(cfg: dict) -> None:
    errs = [f"missing top-level key {k!r}" for k in REQUIRED_TOP if k not in cfg]
    if errs:
        raise ConfigError("; ".join(errs))
    from pluggy_b200.models.builder import resolve
    from pluggy_b200.objectives.builder import OBJECTIVE_REGISTRY
    from pluggy_b200.optimizer.builder import OPTIMIZER_REGISTRY, SCHEDULER_REGISTRY

    for k in ("model", "mesh", "optimizer", "objective", "data"):
        if not isinstance(cfg[k], dict):
            raise ConfigError(f"config block {k!r} must be an object")
    m = cfg["model"]
    try:
        e = kwarg_error(resolve(m.get("name")), m.get("config", {}), "model.config")
        if e:
            errs.append(e)
    except (KeyError, ImportError, AttributeError) as exc:
        errs.append(f"model.name: {exc}")
    mesh = cfg["mesh"]
    if not isinstance(mesh, dict) or "dp" not in mesh or any(int(v) < 1 for v in mesh.values()):
        errs.append("mesh must map axis names (including 'dp') to positive sizes")
    if cfg.get("parallelism", "ddp") not in ("ddp", "fsdp2"):
        errs.append(f"parallelism must be 'ddp' or 'fsdp2', got {cfg.get('parallelism')!r}")
    if "cuda_graph" in cfg and not isinstance(cfg["cuda_graph"], bool):
        errs.append("cuda_graph must be true or false")
    if cfg.get("cuda_graph") and (cfg.get("parallelism", "ddp") != "ddp"
                                  or any(int(v) != 1 for v in mesh.values() if isinstance(mesh, dict))
                                  or any(k in cfg for k in ("tp", "cp", "ep"))):
        errs.append("cuda_graph runs one GPU with plain data parallelism (mesh of size 1, no tp/cp/ep)")
    o = cfg["optimizer"]
    if o.get("name") not in OPTIMIZER_REGISTRY:
        errs.append(f"optimizer.name {o.get('name')!r} not in {sorted(OPTIMIZER_REGISTRY)}")
    sch = o.get("scheduler", {})
    if not isinstance(sch.get("total_steps"), int) or sch["total_steps"] < 1:
        errs.append("optimizer.scheduler.total_steps must be a positive integer")
    if sch.get("type") not in SCHEDULER_REGISTRY:
        errs.append(f"optimizer.scheduler.type {sch.get('type')!r} not in {sorted(SCHEDULER_REGISTRY)}")
    else:
        e = kwarg_error(SCHEDULER_REGISTRY[sch["type"]], {k: v for k, v in sch.items() if k != "type"},
                        "optimizer.scheduler")
        if e:
            errs.append(e)
    ob = cfg["objective"]
    if ob.get("name") not in OBJECTIVE_REGISTRY:
        errs.append(f"objective.name {ob.get('name')!r} not in {sorted(OBJECTIVE_REGISTRY)}")
    else:
        e = kwarg_error(OBJECTIVE_REGISTRY[ob["name"]], ob.get("config", {}), "objective.config")
        if e:
            errs.append(e)
    d = cfg["data"]
    for k in ("global_batch_size", "micro_batch_size", "seq_len"):
        if not isinstance(d.get(k), int) or d[k] < 1:
            errs.append(f"data.{k} must be a positive integer")
    if not errs or all(not e.startswith("data.") for e in errs):
        dp = mesh.get("dp", 1) if isinstance(mesh, dict) else 1
        if isinstance(d.get("global_batch_size"), int) and isinstance(d.get("micro_batch_size"), int) \
                and d["global_batch_size"] % (d["micro_batch_size"] * dp):
            errs.append(f"data.global_batch_size {d['global_batch_size']} must be divisible by "
                        f"micro_batch_size {d['micro_batch_size']} x dp {dp}")
    if not d.get("synthetic") and not any(k in d for k in ("sources", "name", "data_files")):
        errs.append("data needs 'name' (hub dataset), 'data_files', 'sources' or 'synthetic'")
    if not d.get("synthetic"):
        for k in ("tokenizer", "eos_token", "pad_token", "num_workers", "seed"):
            if k not in d:
                errs.append(f"data.{k} is required for a dataset-backed run")
    if errs:
        raise ConfigError("; ".join(errs))
