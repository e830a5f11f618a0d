"""DDP and FSDP2 parity on gloo ranks against a single-process reference that every rank
recomputes locally (no extra collectives needed for the comparison)."""

import copy

import torch

from tests._dist import run_ranks

TINY = dict(num_layers=2, num_heads=2, num_kv_heads=1, emb_dim=32, head_dim=16, vocab_size=64, ffn_dim=64)


def _model(seed=0):
    from pluggy_b200.models.qwen3 import Qwen3

    torch.manual_seed(seed)
    m = Qwen3(**TINY)
    m.init_weights()
    return m


def _batch(n, seed=1, S=16):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, 64, (n, S), generator=g)
    return {"input_ids": ids, "labels": ids}


def _loss(m, b):
    from pluggy_b200.objectives.autoregressive import ARObjective

    return ARObjective(ce_chunk_size=8).compute_loss(m, b)


def grad_mismatches(a, b, tol):
    """Collect (not raise) so no rank bails out while others are inside collectives."""
    out = []
    for (n, p), (_, q) in zip(a.named_parameters(), b.named_parameters()):
        if p.grad is None or q.grad is None:
            out.append((n, "missing"))
        elif not torch.allclose(p.grad, q.grad, atol=tol, rtol=tol):
            out.append((n, (p.grad - q.grad).abs().max().item()))
    return out


def _ddp(rank, world, bucket_mb):
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.parallel.ddp import DDP

    mesh = Mesh({"dp": world})
    ref = _model(seed=100)  # rank 0's init: what the broadcast replicates
    m = _model(seed=100 + rank)  # different init: the broadcast must make replicas identical
    ddp = DDP(m, mesh, "dp", bucket_mb=bucket_mb)
    for (n, p), (_, q) in zip(m.named_parameters(), ref.named_parameters()):
        assert torch.equal(p, q), f"replica differs after broadcast: {n}"
    full = _batch(world * 2)
    bad = []
    for cycle in range(2):
        m.zero_grad(set_to_none=True)
        ref.zero_grad(set_to_none=True)
        mine = {k: v[rank * 2:(rank + 1) * 2] for k, v in full.items()}
        _loss(m, mine).backward()
        ddp.sync()
        _loss(ref, full).backward()
        bad += grad_mismatches(m, ref, 1e-5)
    # accumulation: 2 microbatches, no_sync on the first
    m.zero_grad(set_to_none=True)
    ref.zero_grad(set_to_none=True)
    ddp.requires_sync = False
    (_loss(m, {k: v[rank * 2:rank * 2 + 1] for k, v in full.items()}) / 2).backward()
    assert not ddp._works, "no_sync must not launch any reduction"
    ddp.requires_sync = True
    (_loss(m, {k: v[rank * 2 + 1:rank * 2 + 2] for k, v in full.items()}) / 2).backward()
    ddp.sync()
    # reference of the accumulated grads: mean over every rank's two microbatches
    for r in range(world):
        for j in range(2):
            (_loss(ref, {k: v[r * 2 + j:r * 2 + j + 1] for k, v in full.items()}) / (2 * world)).backward()
    bad += grad_mismatches(m, ref, 1e-5)
    assert not bad, bad


def test_ddp_parity_single_bucket():
    run_ranks(_ddp, 4, 25)


def test_ddp_parity_many_buckets():
    run_ranks(_ddp, 2, 0.008)


def test_ddp_parity_all_in_place():
    run_ranks(_ddp, 2, 0)


def _fsdp(rank, world):
    from pluggy_b200.core.grad_helper import clip_grad_norm
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.parallel.fsdp2 import FSDP2

    mesh = Mesh({"dp": world})
    ref = _model(seed=7)
    m = _model(seed=7 + rank)
    fs = FSDP2(m, mesh, "dp")
    # shard shapes and the tie survive sharding
    for (n, p), (_, q) in zip(m.named_parameters(), ref.named_parameters()):
        assert p.shape[0] * world == q.shape[0], n
        assert torch.equal(p.data, q.data.chunk(world)[rank]), n
    assert m.lm_head.weight is m.token_emb.weight
    full = _batch(world * 2, seed=3)
    bad = []
    for accum in (1, 2):
        m.zero_grad(set_to_none=True)
        ref.zero_grad(set_to_none=True)
        for j in range(accum):
            lo = rank * 2 + j * (2 // accum) if accum == 2 else rank * 2
            sl = slice(rank * 2 + j, rank * 2 + j + 1) if accum == 2 else slice(rank * 2, rank * 2 + 2)
            (_loss(m, {k: v[sl] for k, v in full.items()}) / accum).backward()
            del lo
        fs.sync()
        for r in range(world):
            for j in range(accum):
                sl = slice(r * 2 + j, r * 2 + j + 1) if accum == 2 else slice(r * 2, r * 2 + 2)
                (_loss(ref, {k: v[sl] for k, v in full.items()}) / (accum * world)).backward()
        for (n, p), (_, q) in zip(m.named_parameters(), ref.named_parameters()):
            if not torch.allclose(p.grad, q.grad.chunk(world)[rank], atol=1e-5, rtol=1e-5):
                bad.append((accum, n, (p.grad - q.grad.chunk(world)[rank]).abs().max().item()))
        # storage: block units freed after backward (root may stay gathered)
        for u in fs.units[:-1]:
            for s in u.params:
                if s.full.untyped_storage().nbytes() != 0:
                    bad.append(("storage", u.name))
    # sharded clip == global clip of the full grads
    norm = clip_grad_norm(list(m.parameters()), mesh, None, shard_dims=("dp",))
    ref_norm = torch.linalg.vector_norm(torch.stack([q.grad.norm() for q in ref.parameters()]))
    if abs(norm.item() - ref_norm.item()) > 1e-4 * ref_norm.item():
        bad.append(("clip", norm.item(), ref_norm.item()))
    # SGD steps: shard optimizer == full optimizer on the shards
    opt = torch.optim.SGD(m.parameters(), lr=0.1)
    ropt = torch.optim.SGD(ref.parameters(), lr=0.1)
    for step in range(3):
        opt.zero_grad(set_to_none=True)
        ropt.zero_grad(set_to_none=True)
        _loss(m, {k: v[rank * 2:rank * 2 + 2] for k, v in full.items()}).backward()
        fs.sync()
        opt.step()
        for r in range(world):
            (_loss(ref, {k: v[r * 2:r * 2 + 2] for k, v in full.items()}) / world).backward()
        ropt.step()
    for (n, p), (_, q) in zip(m.named_parameters(), ref.named_parameters()):
        if not torch.allclose(p.data, q.data.chunk(world)[rank], atol=1e-5, rtol=1e-4):
            bad.append(("sgd", n))
    assert not bad, bad


def test_fsdp2_parity_gloo2():
    run_ranks(_fsdp, 2)


def test_fsdp2_and_ddp_noop_single_rank():
    run_ranks(_single, 1)


def _single(rank, world):
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.parallel.ddp import DDP
    from pluggy_b200.parallel.fsdp2 import FSDP2

    mesh = Mesh({"dp": 1})
    m = _model()
    before = copy.deepcopy(m.state_dict())
    FSDP2(m, mesh)
    DDP(m, mesh).sync()
    for k, v in m.state_dict().items():
        assert torch.equal(v, before[k])


def _clip(rank, world):
    from pluggy_b200.core.grad_helper import clip_grad_norm
    from pluggy_b200.core.mesh import Mesh

    mesh = Mesh({"dp": world})
    m = _model()
    _loss(m, _batch(2)).backward()
    ref = copy.deepcopy(m)
    for p, q in zip(m.parameters(), ref.parameters()):
        q.grad = p.grad.clone()
    tot = clip_grad_norm(m.parameters(), mesh, 0.1)
    rt = torch.nn.utils.clip_grad_norm_(ref.parameters(), 0.1)
    assert abs(tot.item() - rt.item()) < 1e-5 * rt.item()
    for p, q in zip(m.parameters(), ref.parameters()):
        assert torch.allclose(p.grad, q.grad, atol=1e-7, rtol=1e-5)
    # below threshold: bitwise no-op
    g0 = [p.grad.clone() for p in m.parameters()]
    clip_grad_norm(m.parameters(), mesh, 1e9)
    assert all(torch.equal(p.grad, g) for p, g in zip(m.parameters(), g0))
    # None only measures
    n1 = clip_grad_norm(m.parameters(), mesh, None)
    assert all(torch.equal(p.grad, g) for p, g in zip(m.parameters(), g0)) and n1.item() > 0
    # sharded norm of a known split vector: ranks hold [3, 4] chunks of a norm-5*sqrt(w) vector
    p = torch.nn.Parameter(torch.zeros(2))
    p.grad = torch.tensor([3.0, 4.0])
    n2 = clip_grad_norm([p], mesh, None, shard_dims=("dp",))
    assert abs(n2.item() - 5.0 * world ** 0.5) < 1e-5
    # replicated grads must not be reduced
    n3 = clip_grad_norm([p], mesh, None)
    assert abs(n3.item() - 5.0) < 1e-6
    try:
        clip_grad_norm([torch.nn.Parameter(torch.zeros(1))], mesh, 1.0)
        raise RuntimeError("no grads must assert")
    except AssertionError:
        pass


def test_grad_clip_gloo2():
    run_ranks(_clip, 2)
