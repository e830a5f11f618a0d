"""Collectives and mesh on 4 gloo ranks (closed-form per-rank values, like the reference's
tests/collective.py): every op, src-as-coordinate, subgroup isolation, flatten."""

import torch

from tests._dist import run_ranks


def pattern(rank, shape=(4, 3)):
    return torch.arange(torch.Size(shape).numel(), dtype=torch.float32).view(shape) * (rank + 1)


def _ops(rank, world):
    from pluggy_b200.core import collective as C
    from pluggy_b200.core.mesh import FlatMesh, Mesh

    m = FlatMesh("dp")
    n = world
    tot = sum(range(1, n + 1))
    x = pattern(rank)
    assert torch.equal(C.all_reduce(x.clone(), m, "dp", "sum"), pattern(0) * tot)
    assert torch.allclose(C.all_reduce(x.clone(), m, "dp", "avg"), pattern(0) * tot / n)
    assert torch.equal(C.all_reduce(x.clone(), m, "dp", "max"), pattern(n - 1))
    assert torch.equal(C.all_reduce(x.clone(), m, "dp", "min"), pattern(0))
    b = C.broadcast(x.clone(), m, "dp", src=1)
    assert torch.equal(b, pattern(1))
    g = C.all_gather(x, m, "dp", gather_dim=0)
    assert torch.equal(g, torch.cat([pattern(r) for r in range(n)], 0))
    g1 = C.all_gather(x, m, "dp", gather_dim=-1)
    assert torch.equal(g1, torch.cat([pattern(r) for r in range(n)], -1))
    nc = pattern(rank, (3, 4)).t()  # non-contiguous input
    assert torch.equal(C.all_gather(nc, m, "dp", 0), torch.cat([pattern(r, (3, 4)).t() for r in range(n)], 0))
    big = torch.arange(4 * n * 2, dtype=torch.float32).view(4 * n, 2) * (rank + 1)
    rs = C.reduce_scatter(big, m, "dp", "sum")
    full = torch.arange(4 * n * 2, dtype=torch.float32).view(4 * n, 2) * tot
    assert torch.equal(rs, full.chunk(n)[rank])
    rsa = C.reduce_scatter(big, m, "dp", "avg")
    assert torch.allclose(rsa, full.chunk(n)[rank] / n)
    try:
        C.reduce_scatter(torch.zeros(n + 1, 2), m, "dp")
        raise AssertionError("non-divisible reduce_scatter must assert")
    except AssertionError as e:
        assert "divisible" in str(e)
    # FSDP identity: AG(RS(x)) == AR(x)
    assert torch.equal(C.all_gather(C.reduce_scatter(big, m, "dp"), m, "dp"), C.all_reduce(big.clone(), m, "dp"))
    a2a = C.all_to_all(big, m, "dp", 0, 0)
    back = C.all_to_all(a2a, m, "dp", 0, 0)
    assert torch.equal(back, big)  # involution
    # uneven all_to_all: rank r sends (j + 1) rows to coordinate j
    send = torch.cat([torch.full((j + 1, 2), float(rank * 10 + j)) for j in range(n)])
    recv = C.all_to_all(send, m, "dp", input_splits=[j + 1 for j in range(n)],
                        output_splits=[rank + 1] * n)
    exp = torch.cat([torch.full((rank + 1, 2), float(s * 10 + rank)) for s in range(n)])
    assert torch.equal(recv, exp)
    # ring
    y = x.clone()
    for _ in range(n):
        y = C.ring_send_recv(y, m, "dp")
    assert torch.equal(y, x)
    assert torch.equal(C.ring_send_recv(x, m, "dp"), pattern((rank - 1) % n))
    r2, w = C.ring_send_recv(x, m, "dp", async_op=True)
    w.wait()
    assert torch.equal(r2, pattern((rank - 1) % n))
    # async == sync
    t, work = C.all_reduce(x.clone(), m, "dp", "avg", async_op=True)
    work.wait()
    assert torch.allclose(t, pattern(0) * tot / n)
    C.barrier()

    # 2x2 mesh: dp groups {0,2},{1,3}; tp groups {0,1},{2,3}; powers of two make wrong groups visible
    mesh = Mesh({"dp": 2, "tp": 2})
    assert mesh.coordinate("tp") == rank % 2 and mesh.coordinate("dp") == rank // 2
    v = torch.tensor([float(2 ** rank)])
    s_dp = C.all_reduce(v.clone(), mesh, "dp")
    s_tp = C.all_reduce(v.clone(), mesh, "tp")
    assert s_dp.item() == sum(2 ** r for r in range(4) if r % 2 == rank % 2)
    assert s_tp.item() == sum(2 ** r for r in range(4) if r // 2 == rank // 2)
    b2 = C.broadcast(v.clone(), mesh, "dp", src=1)
    assert b2.item() == 2 ** (2 + rank % 2)
    mesh.flatten(("dp", "tp"), "dptp")
    assert mesh.size("dptp") == 4 and mesh.coordinate("dptp") == rank
    gg = C.all_gather(v, mesh, "dptp")
    assert gg.tolist() == [float(2 ** r) for r in range(4)]


def test_collectives_and_mesh_gloo4():
    run_ranks(_ops, 4)


def test_axis_slices_layout():
    from pluggy_b200.core.mesh import axis_slices

    sizes = {"pp": 2, "dp": 2, "tp": 2}
    assert axis_slices(sizes, "tp") == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert axis_slices(sizes, "dp") == [[0, 2], [1, 3], [4, 6], [5, 7]]
    assert axis_slices(sizes, "pp") == [[0, 4], [1, 5], [2, 6], [3, 7]]


def _dtensor(rank, world):
    from pluggy_b200.core.dtensor import DTensor
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.core.placement import Partial, Replicate, Shard

    mesh = Mesh({"dp": 2, "tp": 2})
    full = torch.arange(8 * 4, dtype=torch.float32).view(8, 4)
    d = DTensor.from_full(full, mesh, {"dp": Shard(0)})
    assert d.local.shape == (4, 4) and d.global_shape == (8, 4)
    assert torch.equal(d.full_tensor(), full)
    r = d.redistribute("dp", Replicate())
    assert torch.equal(r.local, full)
    s = r.redistribute("tp", Shard(1))
    assert torch.equal(s.full_tensor(), full)
    ss = d.redistribute("dp", Shard(1))  # Shard(0) -> Shard(1) via all_to_all
    assert ss.local.shape == (8, 2) and torch.equal(ss.full_tensor(), full)
    p = DTensor.from_local(full * (rank + 1), mesh, {"dp": Partial("sum")})
    before = p.local.clone()
    pr = p.redistribute("dp", Replicate())
    assert torch.equal(p.local, before)  # clone, not mutate
    dp_ranks = [r for r in range(4) if r % 2 == rank % 2]
    assert torch.equal(pr.local, full * sum(r + 1 for r in dp_ranks))
    ps = p.redistribute("dp", Shard(0))
    assert torch.equal(ps.local, (full * sum(r + 1 for r in dp_ranks)).chunk(2)[mesh.coordinate("dp")])
    multi = DTensor.from_local((full * (rank + 1)).chunk(2, 1)[mesh.coordinate("tp")], mesh,
                               {"tp": Shard(1), "dp": Partial("sum")})
    exp = torch.cat([full.chunk(2, 1)[c] * sum(r + 1 for r in range(4) if r % 2 == c) for c in (0, 1)], 1)
    assert torch.equal(multi.full_tensor(), exp)
    try:
        DTensor.from_full(full, mesh, {"dp": Shard(0), "tp": Shard(0)})
        raise AssertionError("two axes on one dim must assert")
    except AssertionError as e:
        assert "same dim" in str(e)
    try:
        d.redistribute("dp", Partial())
        raise AssertionError("-> Partial must assert")
    except AssertionError as e:
        assert "unsupported" in str(e)


def test_dtensor_gloo4():
    run_ranks(_dtensor, 4)
