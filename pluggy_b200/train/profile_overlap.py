"""Communication/compute overlap profiler.

Parity: reference ``pluggy/train/profile_overlap.py:63-206``: after warm-up steps,
a ``torch.profiler`` chrome trace of a few training steps is captured; the GPU
kernels are split into communication (NCCL kernels, and this framework's fused
collective kernels) and compute; each set is merged into a union of intervals,
and the report gives hidden communication (intersection with compute), exposed
communication (communication minus hidden), per-kernel exposure and per-stream
busy time.

``python -m pluggy_b200.train.profile_overlap --config X [--warmup 3] [--steps 2]
[--out trace.json]`` profiles a run (one process per GPU, like the trainer);
``analyze(trace_path)`` works on any saved chrome trace.
"""

from __future__ import annotations

import argparse
import json
import os
from collections import defaultdict

# kernel-name fragments that mark communication: NCCL's kernels and the fused
# collective kernels of this package (pluggy_b200.comm)
COMM_MARKERS = ("nccl", "plg::comm::", "comm::allreduce_avg", "sumsq_total", "tp_rs_", "tp_ag_",
                "tp_norm_ag", "ep_push", "ep_finish", "fsdp_push", "zero1_rs", "zero1_adamw_ag")


def union(intervals: list[tuple[float, float]]) -> list[tuple[float, float]]:
    out: list[list[float]] = []
    for s, e in sorted(intervals):
        if out and s <= out[-1][1]:
            out[-1][1] = max(out[-1][1], e)
        else:
            out.append([s, e])
    return [(s, e) for s, e in out]


def total(intervals) -> float:
    return sum(e - s for s, e in intervals)


def intersect_len(a: list[tuple[float, float]], b: list[tuple[float, float]]) -> float:
    """Length of the intersection of two unions of disjoint sorted intervals."""
    i = j = 0
    acc = 0.0
    while i < len(a) and j < len(b):
        s = max(a[i][0], b[j][0])
        e = min(a[i][1], b[j][1])
        if e > s:
            acc += e - s
        if a[i][1] < b[j][1]:
            i += 1
        else:
            j += 1
    return acc


def is_comm(name: str) -> bool:
    n = name.lower()
    return any(m in n for m in COMM_MARKERS)


def analyze(trace_path: str) -> dict:
    with open(trace_path) as f:
        tr = json.load(f)
    events = tr["traceEvents"] if isinstance(tr, dict) else tr
    kernels = [e for e in events if e.get("ph") == "X" and e.get("cat") in ("kernel", "gpu_memcpy")
               and "dur" in e]
    comm, comp = [], []
    per_stream = defaultdict(float)
    per_kernel = defaultdict(lambda: [0.0, 0])
    for e in kernels:
        iv = (float(e["ts"]), float(e["ts"]) + float(e["dur"]))
        (comm if is_comm(e["name"]) else comp).append((iv, e["name"]))
        per_stream[str(e.get("tid"))] += float(e["dur"])
    cu = union([iv for iv, _ in comm])
    pu = union([iv for iv, _ in comp])
    hidden = intersect_len(cu, pu)
    exposed = total(cu) - hidden
    for iv, name in comm:
        ex = (iv[1] - iv[0]) - intersect_len([iv], pu)
        per_kernel[name[:80]][0] += ex
        per_kernel[name[:80]][1] += 1
    allu = union([iv for iv, _ in comm + comp])
    span = (allu[-1][1] - allu[0][0]) if allu else 0.0
    return {
        # span: first kernel start to last kernel end; busy: time any kernel runs. The
        # difference is device idle time (host-bound launches, synchronisations).
        "span_us": span, "busy_us": total(allu), "idle_us": span - total(allu),
        "comm_us": total(cu), "compute_us": total(pu), "hidden_us": hidden, "exposed_us": exposed,
        "hidden_frac": hidden / total(cu) if cu else 1.0,
        "per_kernel_exposed_us": {k: v[0] for k, v in sorted(per_kernel.items(), key=lambda kv: -kv[1][0])},
        "per_stream_busy_us": dict(per_stream),
    }


SYNC_MARKERS = ("cudaStreamSynchronize", "cudaDeviceSynchronize", "cudaEventSynchronize",
                "aten::_local_scalar_dense", "aten::item")


def idle_gaps(trace_path: str, top: int = 8) -> dict:
    """Where the device idles: the ``top`` longest gaps between consecutive kernels
    (with the kernels on both sides) and the host calls that wait for the device."""
    with open(trace_path) as f:
        tr = json.load(f)
    events = tr["traceEvents"] if isinstance(tr, dict) else tr
    ks = sorted((float(e["ts"]), float(e["ts"]) + float(e["dur"]), e["name"]) for e in events
                if e.get("ph") == "X" and e.get("cat") in ("kernel", "gpu_memcpy", "gpu_memset")
                and "dur" in e)
    gaps = []
    end, last = None, None
    for t0, t1, name in ks:
        if end is not None and t0 > end:
            gaps.append((t0 - end, short_name(last), short_name(name)))
        if end is None or t1 > end:
            end, last = t1, name
    gaps.sort(reverse=True)
    syncs = defaultdict(lambda: [0, 0.0])
    for e in events:
        if e.get("ph") == "X" and any(m == e.get("name") for m in SYNC_MARKERS):
            syncs[e["name"]][0] += 1
            syncs[e["name"]][1] += float(e.get("dur", 0.0))
    return {"gaps_us": [(round(g, 1), a, b) for g, a, b in gaps[:top]],
            "host_waits": {k: {"calls": v[0], "us": round(v[1], 1)} for k, v in syncs.items()}}


def short_name(name: str) -> str:
    """Kernel function name without namespaces, template arguments or parameters."""
    n = name.replace("(anonymous namespace)::", "").split("(")[0]
    depth, out = 0, []
    for ch in n:  # drop <...> (nested)
        if ch == "<":
            depth += 1
        elif ch == ">":
            depth = max(0, depth - 1)
        elif depth == 0:
            out.append(ch)
    n = "".join(out).strip()
    n = n.split(" ")[-1]
    return n.split("::")[-1] or name[:60]


def kernel_table(trace_path: str, steps: int = 1) -> list[dict]:
    """Per-kernel device time per step from a chrome trace: name, ms/step,
    launches/step and share of the summed kernel time, largest first."""
    with open(trace_path) as f:
        tr = json.load(f)
    events = tr["traceEvents"] if isinstance(tr, dict) else tr
    acc = defaultdict(lambda: [0.0, 0])
    for e in events:
        if e.get("ph") == "X" and e.get("cat") in ("kernel", "gpu_memcpy", "gpu_memset") and "dur" in e:
            k = short_name(e["name"])
            acc[k][0] += float(e["dur"])
            acc[k][1] += 1
    tot = sum(v[0] for v in acc.values()) or 1.0
    rows = [{"kernel": k, "ms_per_step": v[0] / 1e3 / steps, "launches_per_step": v[1] / steps,
             "share": v[0] / tot} for k, v in acc.items()]
    return sorted(rows, key=lambda r: -r["ms_per_step"])


def capture(config, warmup: int, steps: int, out: str, rank: int, local_rank: int,
            world: int, raw: bool = False) -> str:
    """Profile ``steps`` training steps after ``warmup`` (``config``: dict or JSON path).
    ``raw`` runs the step without the per-step timing synchronisations, as the
    throughput benchmark does."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from pluggy_b200.train.trainer import Trainer

    tr = Trainer(config, rank=rank, local_rank=local_rank, world_size=world, benchmark=True)
    step = tr._train_step if raw else tr.train_step
    for _ in range(warmup):
        step()
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    with profile(activities=acts) as prof:
        for _ in range(steps):
            step()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    path = out if world == 1 else f"{os.path.splitext(out)[0]}_rank{rank}.json"
    prof.export_chrome_trace(path)
    if torch.cuda.is_available():
        ms = torch.cuda.memory_stats()
        # allocator retries (cudaFree + retry under memory pressure) synchronise the device
        print(json.dumps({"rank": rank, "max_mem_gib": torch.cuda.max_memory_allocated() / 2**30,
                          "alloc_retries": ms.get("num_alloc_retries", 0)}))
    return path


def main(argv=None) -> None:
    import torch.distributed as dist

    from pluggy_b200.train.train import init_distributed

    p = argparse.ArgumentParser()
    p.add_argument("--config", required=True)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--out", default="overlap_trace.json")
    p.add_argument("--raw", action="store_true",
                   help="profile the step without its timing synchronisations (as bench.py runs it)")
    p.add_argument("--kernels", type=int, default=0,
                   help="also print the N largest kernels (device ms per step)")
    a = p.parse_args(argv)
    rank, local_rank, world = init_distributed()
    try:
        path = capture(a.config, a.warmup, a.steps, a.out, rank, local_rank, world, raw=a.raw)
        rep = analyze(path)
        if rank == 0:
            print(json.dumps({k: v for k, v in rep.items() if k != "per_kernel_exposed_us"}, indent=1))
            for k, v in list(rep["per_kernel_exposed_us"].items())[:10]:
                print(f"  exposed {v:10.1f} us  {k}")
            print(json.dumps(idle_gaps(path), indent=1))
            if a.kernels:
                rows = kernel_table(path, a.steps)
                print(f"{'kernel':48s} {'ms/step':>9s} {'launches':>9s} {'share':>7s}")
                for r in rows[:a.kernels]:
                    print(f"{r['kernel'][:48]:48s} {r['ms_per_step']:9.3f} "
                          f"{r['launches_per_step']:9.0f} {100 * r['share']:6.1f}%")
                print(f"{'total':48s} {sum(r['ms_per_step'] for r in rows):9.3f} "
                      f"{sum(r['launches_per_step'] for r in rows):9.0f}")
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
