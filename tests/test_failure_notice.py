"""Host-side fault injection on gloo ranks (no GPU): a rank that fails between steps
stops the others before their next step with an error naming it; a rank that dies
without a word makes its peers' next collective fail instead of hanging."""

import json
import os
import time

import pytest

from tests._dist import run_ranks

CFG = {
    "run_name": "failure_notice", "seed": 0, "parallelism": "ddp", "mesh": {"dp": 2},
    "ddp": {"bucket_mb": 25},
    "model": {"name": "qwen3_dense", "config": {
        "num_layers": 2, "emb_dim": 128, "num_heads": 4, "num_kv_heads": 2, "head_dim": 32,
        "ffn_dim": 256, "vocab_size": 1024}},
    "optimizer": {"name": "adamw", "config": {"lr": 3e-4, "weight_decay": 0.1, "betas": [0.9, 0.95]},
                  "max_norm": 1.0, "scheduler": {"type": "cosine", "total_steps": 10, "warmup_ratio": 0.2}},
    "objective": {"name": "AR", "config": {"ignore_index": -100, "fused_linear_ce": True,
                                           "ce_chunk_size": 256}},
    "data": {"synthetic": {"kind": "uniform"}, "seq_len": 64, "micro_batch_size": 2,
             "global_batch_size": 4, "seed": 0},
}


def _trainer(rank, world, root):
    from pluggy_b200.train.trainer import Trainer

    return Trainer(json.loads(json.dumps(CFG)), rank=rank, local_rank=rank, world_size=world,
                   checkpoint_root=root)


def _fail_between_steps(rank, world, root, out):
    tr = _trainer(rank, world, root)
    steps, checks = {"n": 0}, {"n": 0}
    real_step, real_check = tr.train_step, tr.failure_notice.check

    def step():
        steps["n"] += 1
        if rank == 1 and steps["n"] == 2:
            raise RuntimeError("injected data error")
        return real_step()

    def check():
        checks["n"] += 1
        if rank == 0 and checks["n"] == 2:
            time.sleep(3)  # rank 1 has failed and announced by now
        real_check()

    tr.train_step, tr.failure_notice.check = step, check
    t0 = time.time()
    try:
        tr.train_n_step_test(4)
        msg = "no error"
    except Exception as e:  # noqa: BLE001 - the outcome is what the test checks
        msg = f"{type(e).__name__}: {e}"
    with open(f"{out}.{rank}", "w") as f:
        json.dump({"msg": msg, "steps": steps["n"], "secs": time.time() - t0}, f)


def test_a_failing_rank_stops_the_others_before_their_next_step(tmp_path):
    out = str(tmp_path / "res")
    run_ranks(_fail_between_steps, 2, str(tmp_path / "ck"), out, timeout_s=60, join_s=300)
    r0, r1 = (json.load(open(f"{out}.{r}")) for r in (0, 1))
    assert r1["msg"] == "RuntimeError: injected data error", r1
    assert r0["msg"].startswith("PeerFailure: stopping: rank 1 failed: RuntimeError: injected data error"), r0
    assert r0["steps"] == 1 and r0["secs"] < 30  # no collective of step 2 was entered


def _die_between_steps(rank, world, root, out):
    tr = _trainer(rank, world, root)
    steps = {"n": 0}
    real_step = tr.train_step

    def step():
        steps["n"] += 1
        if rank == 1 and steps["n"] == 2:
            os._exit(3)  # gone without a word: no notice, no process-group teardown
        return real_step()

    tr.train_step = step
    t0 = time.time()
    try:
        tr.train_n_step_test(4)
        msg = "no error"
    except Exception as e:  # noqa: BLE001
        msg = f"{type(e).__name__}: {e}"
    with open(f"{out}.{rank}", "w") as f:
        json.dump({"msg": msg, "steps": steps["n"], "secs": time.time() - t0}, f)


def test_a_vanished_rank_fails_the_next_collective(tmp_path):
    out = str(tmp_path / "res")
    with pytest.raises(AssertionError, match=r"missing: \[1\]"):
        run_ranks(_die_between_steps, 2, str(tmp_path / "ck"), out, timeout_s=20, join_s=300)
    r0 = json.load(open(f"{out}.0"))
    assert r0["msg"] != "no error" and r0["steps"] == 2, r0
    assert r0["secs"] < 120, r0
    assert not os.path.exists(f"{out}.1")
