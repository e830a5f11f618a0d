"""Overlap analysis on a synthetic chrome trace, and a CPU capture end to end."""

import json


def test_interval_algebra():
    from pluggy_b200.train.profile_overlap import intersect_len, total, union

    u = union([(5, 7), (0, 2), (1, 3), (6, 9)])
    assert u == [(0, 3), (5, 9)] and total(u) == 7
    assert intersect_len(u, union([(2, 6)])) == 2


def test_analyze_synthetic_trace(tmp_path):
    from pluggy_b200.train.profile_overlap import analyze

    ev = [
        {"ph": "X", "cat": "kernel", "name": "gemm_kernel", "ts": 0, "dur": 100, "tid": 7},
        {"ph": "X", "cat": "kernel", "name": "ncclDevKernel_AllReduce", "ts": 50, "dur": 100, "tid": 9},
        {"ph": "X", "cat": "kernel", "name": "attn_bwd3_kernel", "ts": 120, "dur": 10, "tid": 7},
        {"ph": "X", "cat": "cpu_op", "name": "aten::mm", "ts": 0, "dur": 500},
    ]
    p = tmp_path / "t.json"
    p.write_text(json.dumps({"traceEvents": ev}))
    r = analyze(str(p))
    assert r["comm_us"] == 100 and r["compute_us"] == 110
    assert r["hidden_us"] == 60 and r["exposed_us"] == 40
    assert abs(r["hidden_frac"] - 0.6) < 1e-9
    assert r["per_kernel_exposed_us"]["ncclDevKernel_AllReduce"] == 40
    assert r["per_stream_busy_us"] == {"7": 110.0, "9": 100.0}


def test_capture_cpu(tmp_path):
    import torch.distributed as dist

    from tests._dist import free_port
    from pluggy_b200.train.profile_overlap import analyze, capture

    cfg = {
        "run_name": "prof", "seed": 0, "mesh": {"dp": 1}, "parallelism": "ddp",
        "model": {"name": "qwen3_dense", "config": dict(num_layers=1, num_heads=2, num_kv_heads=1,
                                                         emb_dim=32, head_dim=16, vocab_size=64,
                                                         ffn_dim=64)},
        "objective": {"name": "AR", "config": {"ce_chunk_size": 16}},
        "optimizer": {"name": "adamw", "config": {"lr": 1e-3},
                      "scheduler": {"type": "cosine", "warmup_ratio": 0.1, "total_steps": 4},
                      "max_norm": 1.0},
        "data": {"synthetic": {"kind": "uniform"}, "seq_len": 16, "micro_batch_size": 2,
                 "global_batch_size": 2, "seed": 0},
        "checkpointing": {"save_steps": 10**9, "resume": None},
    }
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1)
    try:
        path = capture(cfg, 1, 1, str(tmp_path / "trace.json"), 0, 0, 1)
    finally:
        dist.destroy_process_group()
    r = analyze(path)
    assert r["exposed_us"] == 0 and r["comm_us"] == 0
