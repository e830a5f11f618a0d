"""Tensor (+ sequence) parallelism on gloo ranks against the unsharded model that every
rank recomputes locally: same loss, and each rank's gradient shard equals the
matching slice of the full model's gradient."""

import copy

import pytest
import torch

from tests._dist import run_ranks

TINY = dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=32, head_dim=8, vocab_size=64,
            ffn_dim=64)


def _model(cls="qwen3", tie=True):
    from pluggy_b200.models.llama3 import Llama3
    from pluggy_b200.models.qwen3 import Qwen3

    torch.manual_seed(0)
    m = (Qwen3 if cls == "qwen3" else Llama3)(**TINY, tie_embeddings=tie)
    m.init_weights()
    return m


def _batch(S=16, B=2):
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 64, (B, S), generator=g)
    return {"input_ids": ids, "labels": ids}


def _tp_case(rank, world, sp, cls, tie):
    from pluggy_b200.core.grad_helper import clip_grad_norm
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.objectives.autoregressive import ARObjective
    from pluggy_b200.parallel.tensor_parallel import (ColumnParallelLinear, RowParallelLinear,
                                                      VocabParallelEmbedding, parallelize_tp)

    mesh = Mesh({"tp": world})
    ref = _model(cls, tie)
    m = copy.deepcopy(ref)
    tp = parallelize_tp(m, mesh, "tp", sequence_parallel=sp)
    obj = ARObjective(ce_chunk_size=8)
    b = _batch()
    loss_ref = obj.compute_loss(ref, b)
    loss_ref.backward()
    loss = obj.compute_loss(m, b)
    loss.backward()
    tp.sync_replicated_grads()
    bad = []
    if not torch.allclose(loss, loss_ref, atol=1e-5, rtol=1e-5):
        bad.append(("loss", loss.item(), loss_ref.item()))
    full = dict(ref.named_parameters())
    r, n = mesh.coordinate("tp"), world
    for name, p in m.named_parameters():
        q = full[name]
        mod = m.get_submodule(name.rpartition(".")[0])
        if isinstance(mod, (ColumnParallelLinear, VocabParallelEmbedding)) or name == "lm_head.weight":
            k = q.shape[0] // n
            want = q.grad[r * k:(r + 1) * k]
        elif isinstance(mod, RowParallelLinear):
            k = q.shape[1] // n
            want = q.grad[:, r * k:(r + 1) * k]
        else:
            want = q.grad
        if p.grad is None or not torch.allclose(p.grad, want, atol=1e-5, rtol=1e-4):
            bad.append((name, None if p.grad is None else (p.grad - want).abs().max().item()))
    # the clip norm of the sharded model equals the full model's
    g_ref = clip_grad_norm(ref.parameters(), mesh, None)
    g = clip_grad_norm(m.parameters(), mesh, None, partial_over=(("tp",), tp.sharded_param_ids()))
    if not torch.allclose(g, g_ref, rtol=1e-5):
        bad.append(("grad_norm", g.item(), g_ref.item()))
    # gathering the shards gives back the full state dict
    sd = tp.full_state_dict()
    for k, v in ref.state_dict().items():
        if not torch.equal(sd[k], v):
            bad.append(("state_dict", k))
    assert not bad, bad


@pytest.mark.parametrize("sp", [True, False])
def test_tp2_qwen3_matches_unsharded(sp):
    run_ranks(_tp_case, 2, sp, "qwen3", True)


def test_tp2_llama3_untied_sp():
    run_ranks(_tp_case, 2, True, "llama3", False)


def _tp_dp_trainer(rank, world):
    """tp=2 x dp=2 through the Trainer: two optimizer steps run and every rank agrees
    on the loss (the dp average) while tp ranks hold different shards."""
    import torch.distributed as dist

    from pluggy_b200.train.trainer import Trainer

    cfg = {
        "run_name": "tp_dp", "seed": 0, "mesh": {"dp": 2, "tp": 2}, "parallelism": "ddp",
        "model": {"name": "qwen3_dense", "config": dict(TINY, tie_embeddings=True)},
        "objective": {"name": "AR", "config": {"ce_chunk_size": 8}},
        "optimizer": {"name": "adamw", "config": {"lr": 1e-3, "weight_decay": 0.1},
                      "scheduler": {"type": "cosine", "warmup_ratio": 0.1, "total_steps": 4},
                      "max_norm": 1.0},
        "data": {"synthetic": {"kind": "uniform"}, "seq_len": 16, "micro_batch_size": 2,
                 "global_batch_size": 4, "seed": 0},
        "checkpointing": {"save_steps": 10**9, "resume": None},
    }
    tr = Trainer(cfg, rank=rank, local_rank=rank, world_size=world, benchmark=True)
    losses = []
    for _ in range(2):
        metrics = tr._train_step()
        losses.append(float(metrics["loss"]))
    t = torch.tensor(losses)
    all_t = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(all_t, t)
    for o in all_t:
        assert torch.allclose(o, t), (o, t)
    assert all(torch.isfinite(t))


def test_tp2_dp2_trainer_steps():
    run_ranks(_tp_dp_trainer, 4)
