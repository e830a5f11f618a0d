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


def _zero1_case(rank, world):
    import copy

    import torch.distributed as dist

    from pluggy_b200.core.grad_helper import clip_grad_norm
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.models.qwen3 import Qwen3
    from pluggy_b200.objectives.autoregressive import ARObjective
    from pluggy_b200.ops import _ext
    from pluggy_b200.optimizer.builder import build_optimizer
    from pluggy_b200.parallel.ddp import DDP

    mesh = Mesh({"dp": world})
    torch.manual_seed(0)
    base = Qwen3(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=256, head_dim=128,
                 vocab_size=1024, ffn_dim=512).cuda()
    base.init_weights()
    init = {n: p.detach().clone() for n, p in base.named_parameters()}
    cfg = {"lr": 1e-3, "weight_decay": 0.1, "betas": [0.9, 0.95]}
    models, ddps, opts = {}, {}, {}
    for r in ("nccl", "zero1"):
        models[r] = copy.deepcopy(base)
        ddps[r] = DDP(models[r], mesh, "dp", bucket_mb=1, reducer=r)
        opts[r] = ddps[r].zero1_optimizer(build_optimizer(models[r], "adamw", dict(cfg)))
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    bad = []
    for step in range(3):
        ids = torch.randint(0, 1024, (2, 256), device="cuda", generator=g)
        b = {"input_ids": ids, "labels": ids}
        norms = {}
        for r, m in models.items():
            ARObjective(ce_chunk_size=256).compute_loss(m, b).backward()
            ddps[r].sync()
            gn, coef = clip_grad_norm(m.parameters(), mesh, 1.0, fold_into_optimizer=True,
                                      precomputed_sq=ddps[r].reduced_norm_sq())
            norms[r] = float(gn)
            opts[r].set_grad_scale(coef)
            opts[r].step()
            opts[r].zero_grad()
        opts["zero1"].wait_params()
        torch.cuda.synchronize()
        if abs(norms["nccl"] - norms["zero1"]) > 1e-4 * norms["nccl"]:
            bad.append(("norm", step, norms))
        for (n, p), (_, q) in zip(models["nccl"].named_parameters(), models["zero1"].named_parameters()):
            upd = (p.detach() - init[n]).norm().item()
            diff = (p.detach() - q.detach()).norm().item()
            if diff > 1e-2 * max(upd, 1e-12):
                bad.append((step, n, diff, upd))
    # the replicas are bitwise identical on every rank
    flat = torch.cat([p.detach().reshape(-1) for p in models["zero1"].parameters()])
    allf = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(allf, flat)
    if not all(torch.equal(allf[0], x) for x in allf[1:]):
        bad.append("replicas differ")
    _ext.check_status()
    ddps["zero1"].zero1.close()
    assert not bad, bad


def test_zero1_ddp_matches_nccl_ddp():
    _need(2)
    run_ranks(_zero1_case, 2, backend="nccl")


def _tp_collectives_case(rank, world):
    import torch.distributed as dist

    from pluggy_b200.comm.tp_fused import TPComm
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.ops import _ext

    mesh = Mesh({"tp": world})
    comm = TPComm(mesh, "tp", capacity_bytes=1 << 20)  # small: forces a regrow below
    bad = []
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    for it, (B, S, W) in enumerate([(2, 256, 512), (1, 1024, 256), (2, 256, 512), (3, 64, 1024),
                                    (2, 2048, 1024)]):
        part = torch.randn(B, S, W, device="cuda", generator=g).bfloat16()
        got = comm.reduce_scatter_seq(part)
        full = part.float()
        dist.all_reduce(full)
        want = full.view(B, world, S // world, W)[:, rank]
        err = (got.float() - want).abs().max().item()
        if err > 0.05 * want.abs().max().item():
            bad.append(("rs", it, err))
        shard = torch.randn(B, S // world, W, device="cuda", generator=g).bfloat16()
        gathered = comm.all_gather_seq(shard)
        parts = [torch.empty_like(shard) for _ in range(world)]
        dist.all_gather(parts, shard.contiguous())
        ref = torch.cat(parts, dim=1)
        if not torch.equal(gathered, ref):
            bad.append(("ag", it))
        # fused GEMM -> reduce-scatter against GEMM + NCCL reduce-scatter
        K, N = 256, W
        x = torch.randn(B, S, K, device="cuda", generator=g).bfloat16()
        w = torch.randn(N, K, device="cuda", generator=g).bfloat16() * 0.05
        y = comm.gemm_reduce_scatter(x, w)
        yf = (x.float().reshape(-1, K) @ w.float().t()).view(B, S, N)
        dist.all_reduce(yf)
        want = yf.view(B, world, S // world, N)[:, rank]
        rel = ((y.float() - want).norm() / want.norm()).item()
        if rel > 1e-2:
            bad.append(("gemm_rs", it, rel))
    torch.cuda.synchronize()
    _ext.check_status()
    comm.close()
    assert not bad, bad


def test_tp_peer_collectives_match_nccl():
    _need(2)
    run_ranks(_tp_collectives_case, 2, backend="nccl")


def _vocab_ce_case(rank, world):
    import torch.distributed as dist

    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.ops.ce import fused_linear_cross_entropy
    from pluggy_b200.parallel.tensor_parallel import vocab_parallel_cross_entropy

    mesh = Mesh({"tp": world})
    torch.manual_seed(0)  # same full problem on every rank
    N, D, V = 1500, 256, 6000
    h = (torch.randn(N, D, device="cuda") * 0.5).bfloat16()
    w = torch.randn(V, D, device="cuda") * 0.05
    lab = torch.randint(0, V, (N,), device="cuda")
    lab[::5] = -100
    Vl = V // world
    hl = h.clone().requires_grad_(True)
    wl = w[rank * Vl:(rank + 1) * Vl].clone().requires_grad_(True)
    loss = vocab_parallel_cross_entropy(hl, wl, lab, rank * Vl, mesh, "tp", -100, 512)
    loss.backward()
    gh = hl.grad.float().clone()
    dist.all_reduce(gh)  # the TP entry collective sums the ranks' grad_hidden shares
    hr = h.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    ref = fused_linear_cross_entropy(hr, wr, lab, -100, 512)
    ref.backward()
    bad = []
    if abs(loss.item() - ref.item()) > 1e-3 * ref.item():
        bad.append(("loss", loss.item(), ref.item()))
    rh = ((gh - hr.grad.float()).norm() / hr.grad.float().norm()).item()
    rw = ((wl.grad - wr.grad[rank * Vl:(rank + 1) * Vl]).norm() / wr.grad.norm()).item()
    if rh > 2e-2 or rw > 2e-2:
        bad.append(("grads", rh, rw))
    assert not bad, bad


def test_vocab_parallel_ce_matches_single_gpu():
    _need(2)
    run_ranks(_vocab_ce_case, 2, backend="nccl")


def _tp_model_case(rank, world):
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.models.qwen3 import Qwen3
    from pluggy_b200.objectives.autoregressive import ARObjective
    from pluggy_b200.ops import _ext
    from pluggy_b200.parallel.tensor_parallel import parallelize_tp

    mesh = Mesh({"tp": world})
    cfg = dict(num_layers=2, num_heads=8, num_kv_heads=4, emb_dim=512, head_dim=64, vocab_size=4096,
               ffn_dim=1024, tie_embeddings=True)
    losses, grads = {}, {}
    ids = torch.randint(0, 4096, (2, 512), generator=torch.Generator().manual_seed(0)).cuda()
    for fused in (False, True):
        torch.manual_seed(0)
        m = Qwen3(**cfg).cuda()
        m.init_weights()
        # the TP engine runs the per-head q/k norms in bf16 (eps = bf16 eps, as the
        # reference under autocast): give the eager NCCL path the same eps
        for mod in m.modules():
            if isinstance(mod, torch.nn.RMSNorm) and mod.normalized_shape[0] == cfg["head_dim"]:
                mod.eps = torch.finfo(torch.bfloat16).eps
        tp = parallelize_tp(m, mesh, "tp", sequence_parallel=True, fused=fused)
        loss = ARObjective(ce_chunk_size=512).compute_loss(m, {"input_ids": ids, "labels": ids})
        loss.backward()
        tp.sync_replicated_grads()
        losses[fused] = float(loss)
        grads[fused] = {n: p.grad.float().clone() for n, p in m.named_parameters() if p.grad is not None}
        tp.close()
    torch.cuda.synchronize()
    _ext.check_status()
    assert abs(losses[True] - losses[False]) < 2e-2 * abs(losses[False]), losses
    bad = []
    for n, gref in grads[False].items():
        gf = grads[True][n]
        rel = ((gf - gref).norm() / (gref.norm() + 1e-12)).item()
        if rel > 5e-2:
            bad.append((n, rel))
    assert not bad, bad


def test_tp2_fused_model_matches_nccl_path():
    _need(2)
    run_ranks(_tp_model_case, 2, backend="nccl")


def _ep_model_case(rank, world):
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.models.qwen3_moe import Qwen3Moe
    from pluggy_b200.objectives.autoregressive import ARObjective
    from pluggy_b200.ops import _ext
    from pluggy_b200.parallel.expert_parallel import parallelize_ep

    mesh = Mesh({"dp": world})
    cfg = dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=256, head_dim=64, vocab_size=2048,
               moe_ffn_dim=128, num_experts=8, top_k=2, ffn_dim=512, decoder_sparse_step=1)
    g = torch.Generator().manual_seed(10 + rank)  # every rank routes its own tokens
    batches = [torch.randint(0, 2048, (2, 256), generator=g).cuda() for _ in range(3)]
    res = {}
    for fused in (False, True):
        torch.manual_seed(0)
        m = Qwen3Moe(**cfg).cuda()
        m.init_weights()
        for blk in m.blocks:
            if blk.use_moe:
                torch.nn.init.normal_(blk.ffn.router.weight, 0.0, 0.5)
        ep = parallelize_ep(m, mesh, "dp", fused=fused)
        assert (ep.comm is not None) == fused
        losses = []
        for ids in batches:
            m.zero_grad(set_to_none=True)
            loss = ARObjective(ce_chunk_size=256).compute_loss(m, {"input_ids": ids, "labels": ids})
            loss.backward()
            losses.append(float(loss))
        res[fused] = (losses, {n: p.grad.float().clone() for n, p in m.named_parameters()
                               if p.grad is not None})
        ep.close()
    torch.cuda.synchronize()
    _ext.check_status()
    l0, g0 = res[False]
    l1, g1 = res[True]
    assert all(abs(a - b) < 2e-2 * abs(a) for a, b in zip(l0, l1)), (l0, l1)
    bad = [(n, ((g1[n] - g).norm() / (g.norm() + 1e-12)).item()) for n, g in g0.items()
           if ((g1[n] - g).norm() / (g.norm() + 1e-12)).item() > 5e-2]
    assert not bad, bad


def test_ep2_peer_exchange_matches_nccl_path():
    _need(2)
    run_ranks(_ep_model_case, 2, backend="nccl")


def _fsdp_peer_case(rank, world):
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.models.qwen3 import Qwen3
    from pluggy_b200.objectives.autoregressive import ARObjective
    from pluggy_b200.ops import _ext
    from pluggy_b200.parallel.fsdp2 import FSDP2

    mesh = Mesh({"dp": world})
    cfg = dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=256, head_dim=64, vocab_size=2048,
               ffn_dim=512, tie_embeddings=True)
    g = torch.Generator().manual_seed(20 + rank)
    batches = [torch.randint(0, 2048, (2, 128), generator=g).cuda() for _ in range(3)]
    # the unsharded model's first loss on this rank's batch is the FSDP2 target
    torch.manual_seed(0)
    plain = Qwen3(**cfg).cuda()
    plain.init_weights()
    with torch.no_grad():
        want0 = float(ARObjective(ce_chunk_size=256).compute_loss(
            plain, {"input_ids": batches[0], "labels": batches[0]}))
    del plain
    res = {}
    for mode in ("nccl", "peer", "peer_fp32", "peer_rs"):
        torch.manual_seed(0)
        m = Qwen3(**cfg).cuda()
        m.init_weights()
        fs = FSDP2(m, mesh, "dp", gather="nccl" if mode == "nccl" else "peer",
                   lowp_gather=mode in ("peer", "peer_rs"),
                   reduce="peer" if mode == "peer_rs" else "nccl")
        assert (fs._peer is not None) == (mode != "nccl")
        # "peer": block units gathered as bf16 straight into the GEMMs' slots
        assert (fs._slots is not None) == (mode in ("peer", "peer_rs"))
        # "peer_rs": gradients reduce-scattered by the peer-memory kernel
        assert (fs._peer_rs is not None) == (mode == "peer_rs")
        losses = []
        for ids in batches:
            loss = ARObjective(ce_chunk_size=256).compute_loss(m, {"input_ids": ids, "labels": ids})
            loss.backward()
            fs.sync()
            losses.append(float(loss))
            grads = {n: p.grad.float().clone() for n, p in m.named_parameters() if p.grad is not None}
            m.zero_grad(set_to_none=True)
        res[mode] = (losses, grads)
        fs.close()
    torch.cuda.synchronize()
    _ext.check_status()
    assert abs(res["nccl"][0][0] - want0) < 1e-3 * abs(want0), (res["nccl"][0][0], want0)
    # the gathers are exact copies; the remaining differences come from float atomics
    # elsewhere in the step (loss sum, dQ accumulation)
    for mode in ("peer", "peer_fp32", "peer_rs"):
        for a, b in zip(res["nccl"][0], res[mode][0]):
            assert abs(a - b) < 1e-5 * abs(a), (mode, res["nccl"][0], res[mode][0])
        for n, gref in res["nccl"][1].items():
            g = res[mode][1][n]
            assert ((g - gref).norm() / (gref.norm() + 1e-12)).item() < 1e-3, (mode, n)


def test_fsdp2_peer_gather_matches_nccl():
    _need(2)
    run_ranks(_fsdp_peer_case, 2, backend="nccl")
