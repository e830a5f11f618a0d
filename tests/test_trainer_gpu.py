"""The trainer reads the kernels' status word: a bounded wait that gave up
during a step stops training (and a checkpoint) with an error on that rank."""

import json

import pytest

from tests._dist import run_ranks

pytestmark = pytest.mark.gpu

CFG = {
    "run_name": "status_check", "seed": 0, "parallelism": "ddp", "mesh": {"dp": 1},
    "model": {"name": "qwen3_dense", "config": {
        "num_layers": 2, "emb_dim": 256, "num_heads": 4, "num_kv_heads": 2, "head_dim": 128,
        "ffn_dim": 512, "vocab_size": 1024}},
    "optimizer": {"name": "adamw", "config": {"lr": 1e-3, "weight_decay": 0.1, "betas": [0.9, 0.95]},
                  "max_norm": 1.0, "scheduler": {"type": "cosine", "total_steps": 10, "warmup_ratio": 0.1}},
    "objective": {"name": "AR", "config": {"ignore_index": -100, "fused_linear_ce": True,
                                           "ce_chunk_size": 256}},
    "data": {"synthetic": {"kind": "uniform"}, "seq_len": 256, "micro_batch_size": 2,
             "global_batch_size": 2, "seed": 0},
}


def _run(rank, world, root, out):
    from pluggy_b200.ops import _ext
    from pluggy_b200.train.trainer import Trainer

    tr = Trainer(json.loads(json.dumps(CFG)), rank=rank, local_rank=rank, world_size=world,
                 checkpoint_root=root)
    tr.train_n_step_test(1)  # healthy step: no error
    res = {}
    # a kernel that timed out waiting for a peer leaves status 5 behind
    _ext.status_word(tr.device).fill_(5)
    try:
        tr.train_n_step_test(1)
        res["step"] = "no error"
    except RuntimeError as e:
        res["step"] = str(e)
    _ext.status_word(tr.device).fill_(5)
    try:
        tr.checkpoint(2)
        res["checkpoint"] = "no error"
    except RuntimeError as e:
        res["checkpoint"] = str(e)
    tr.train_n_step_test(1)  # the word was reset by the check: training can go on
    with open(out, "w") as f:
        json.dump(res, f)


def test_trainer_raises_on_kernel_status(tmp_path):
    out = str(tmp_path / "res.json")
    run_ranks(_run, 1, str(tmp_path / "ck"), out, timeout_s=120, join_s=600, backend="nccl")
    r = json.load(open(out))
    assert "status 5" in r["step"], r
    assert "status 5" in r["checkpoint"], r


def _graph_vs_eager(rank, world, root, out):
    import torch

    from pluggy_b200.train.trainer import Trainer

    res = {}
    for mode in (False, True):
        cfg = json.loads(json.dumps(CFG))
        cfg["run_name"] = f"graph_{mode}"
        cfg["cuda_graph"] = mode
        tr = Trainer(cfg, rank=rank, local_rank=rank, world_size=world, checkpoint_root=root)
        losses = []
        for _ in range(5):
            m = tr._train_step()
            losses.append(float(m["loss"].item()))
        torch.cuda.synchronize()
        res[str(mode)] = {"losses": losses,
                          "params": [p.detach().double().sum().item() for p in tr.model.parameters()],
                          "steps": [float(s["step"]) for s in tr.optimizer.state.values()][:3],
                          "captured": tr._graph is not None}
        del tr
    with open(out, "w") as f:
        json.dump(res, f)


def test_cuda_graph_step_matches_eager(tmp_path):
    """The whole step replayed from a CUDA graph (after one eager step) gives the losses
    and parameters of eager steps: the graph reads the learning rate and bias corrections
    the host uploads each step. Not bitwise: the attention dQ accumulation adds fp32
    partials in arrival order."""
    out = str(tmp_path / "res.json")
    run_ranks(_graph_vs_eager, 1, str(tmp_path / "ck"), out, timeout_s=120, join_s=600,
              backend="nccl")
    r = json.load(open(out))
    assert r["True"]["captured"] and not r["False"]["captured"]
    assert r["True"]["steps"] == r["False"]["steps"] == [5.0, 5.0, 5.0]
    for a, b in zip(r["True"]["losses"], r["False"]["losses"], strict=True):
        assert abs(a - b) <= 1e-4 * abs(b), r
    for a, b in zip(r["True"]["params"], r["False"]["params"], strict=True):
        assert abs(a - b) <= 1e-3 * max(1.0, abs(b)), (a, b)
