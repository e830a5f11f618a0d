"""Fused NVLink collectives on 2+ GPUs (one process per GPU, NCCL as the oracle).
Skipped with fewer than 2 GPUs."""

import pytest
import torch

from tests._dist import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _need(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _allreduce_case(rank, world):
    import torch.distributed as dist

    from pluggy_b200.comm.symm import SymmetricBuffer
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.ops import _ext

    mesh = Mesh({"dp": world})
    total = 1 << 20
    data = SymmetricBuffer(total * 4, mesh, "dp")
    flags = SymmetricBuffer(2 * 8 * 128 * 4, mesh, "dp")
    slots = SymmetricBuffer(8 * 128 * 4, mesh, "dp")
    buf = data.tensor(0, [total])
    g = torch.Generator(device="cuda").manual_seed(rank)
    buf.copy_(torch.randn(total, device="cuda", generator=g))
    ref = buf.clone()
    dist.all_reduce(ref, op=dist.ReduceOp.AVG)
    norm = torch.zeros(1, device="cuda")
    bad = []
    epoch = 0
    for off, n, chunks in ((0, 1000, 4), (1024, 123457, 64), (131072, total - 131072, 128), (4, 3, 8)):
        before = buf[off:off + n].clone()
        epoch += 1
        _ext.ext().symm_allreduce_avg(data.peers, flags.peers, slots.peers, off, n, rank, epoch, chunks,
                                      norm, False, _ext.status_word(buf.device))
        torch.cuda.synchronize()
        _ext.check_status(buf.device)
        if off == 4:  # a re-reduction of already averaged data leaves it unchanged
            want = before
        else:
            want = ref[off:off + n]
        if not torch.allclose(buf[off:off + n], want, rtol=1e-5, atol=1e-6):
            bad.append(("data", off, (buf[off:off + n] - want).abs().max().item()))
        ss = float(want.double().pow(2).sum())
        if abs(float(norm) - ss) > 1e-4 * ss:
            bad.append(("norm", off, float(norm), ss))
    for b in (data, flags, slots):
        b.close()
    assert not bad, bad


def test_fused_allreduce_matches_nccl():
    _need(2)
    run_ranks(_allreduce_case, 2, backend="nccl")


def _ddp_case(rank, world):
    import copy

    from pluggy_b200.core.grad_helper import clip_grad_norm
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.models.qwen3 import Qwen3
    from pluggy_b200.objectives.autoregressive import ARObjective
    from pluggy_b200.parallel.ddp import DDP

    mesh = Mesh({"dp": world})
    torch.manual_seed(0)
    base = Qwen3(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=256, head_dim=64,
                 vocab_size=1024, ffn_dim=512).cuda()
    base.init_weights()
    models = {r: copy.deepcopy(base) for r in ("nccl", "fused")}
    ddps = {r: DDP(models[r], mesh, "dp", bucket_mb=1, reducer=r) for r in models}
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    ids = torch.randint(0, 1024, (2, 256), device="cuda", generator=g)
    b = {"input_ids": ids, "labels": ids}
    norms = {}
    for r, m in models.items():
        for _ in range(2):
            m.zero_grad(set_to_none=True)
            ARObjective(ce_chunk_size=256).compute_loss(m, b).backward()
            ddps[r].sync()
        pre = ddps[r].reduced_norm_sq()
        norms[r] = clip_grad_norm(m.parameters(), mesh, None, precomputed_sq=pre)
    bad = []
    for (n, p), (_, q) in zip(models["nccl"].named_parameters(), models["fused"].named_parameters()):
        if not torch.allclose(p.grad, q.grad, rtol=1e-4, atol=1e-6):
            bad.append((n, (p.grad - q.grad).abs().max().item()))
    if not torch.allclose(norms["nccl"], norms["fused"], rtol=1e-4):
        bad.append(("norm", norms["nccl"].item(), norms["fused"].item()))
    ddps["fused"]._fused.close()
    assert not bad, bad


def test_fused_ddp_matches_nccl_ddp():
    _need(2)
    run_ranks(_ddp_case, 2, backend="nccl")
