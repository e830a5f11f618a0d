"""Context parallelism (zigzag ring attention) on gloo ranks against the full model
recomputed locally: ring attention equals full causal attention, and the CP model's
loss and (axis-summed) grads equal the unsharded model's."""

import copy

import pytest
import torch

from tests._dist import run_ranks

TINY = dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=32, head_dim=8, vocab_size=64,
            ffn_dim=64)


def _ring_case(rank, world):
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.ops.attention import attention_reference
    from pluggy_b200.parallel.context_parallel import ring_attention, zigzag_shard

    mesh = Mesh({"cp": world})
    g = torch.Generator().manual_seed(0)
    B, S, Hq, Hk, d = 2, 8 * world, 4, 2, 8
    q = torch.randn(B, S, Hq, d, generator=g, dtype=torch.float32)
    k = torch.randn(B, S, Hk, d, generator=g, dtype=torch.float32)
    v = torch.randn(B, S, Hk, d, generator=g, dtype=torch.float32)
    do = torch.randn(B, S, Hq, d, generator=g, dtype=torch.float32)
    qf, kf, vf = (t.clone().requires_grad_(True) for t in (q, k, v))
    o_full = attention_reference(qf, kf, vf, causal=True)
    o_full.backward(do)
    ql, kl, vl = (zigzag_shard(t, mesh, "cp").requires_grad_(True) for t in (q, k, v))
    o = ring_attention(ql, kl, vl, mesh, "cp")
    o.backward(zigzag_shard(do, mesh, "cp"))
    bad = []
    for name, got, want in (("o", o, o_full), ("dq", ql.grad, qf.grad), ("dk", kl.grad, kf.grad),
                            ("dv", vl.grad, vf.grad)):
        w = zigzag_shard(want.detach(), mesh, "cp")
        if not torch.allclose(got.detach(), w, atol=1e-5, rtol=1e-5):
            bad.append((name, (got.detach() - w).abs().max().item()))
    assert not bad, bad


@pytest.mark.parametrize("world", [2, 3])
def test_ring_attention_matches_full(world):
    run_ranks(_ring_case, world)


def _cp_model_case(rank, world):
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.models.qwen3 import Qwen3
    from pluggy_b200.objectives.autoregressive import ARObjective
    from pluggy_b200.parallel.context_parallel import parallelize_cp

    mesh = Mesh({"cp": world})
    torch.manual_seed(0)
    ref = Qwen3(**TINY)
    ref.init_weights()
    m = copy.deepcopy(ref)
    cp = parallelize_cp(m, mesh, "cp")
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 64, (2, 8 * world), generator=g)
    b = {"input_ids": ids, "labels": ids}
    obj = ARObjective(ce_chunk_size=8)
    loss_ref = obj.compute_loss(ref, b)
    loss_ref.backward()
    loss = obj.compute_loss(m, b)
    loss.backward()
    cp.sync_grads()
    total = loss.detach().clone()
    import torch.distributed as dist

    dist.all_reduce(total)
    bad = []
    if not torch.allclose(total, loss_ref.detach(), atol=1e-5, rtol=1e-5):
        bad.append(("loss", total.item(), loss_ref.item()))
    full = dict(ref.named_parameters())
    for name, p in m.named_parameters():
        if p.grad is None or not torch.allclose(p.grad, full[name].grad, atol=1e-5, rtol=1e-4):
            bad.append((name, None if p.grad is None else (p.grad - full[name].grad).abs().max().item()))
    assert not bad, bad


def test_cp2_model_matches_full():
    run_ranks(_cp_model_case, 2)
