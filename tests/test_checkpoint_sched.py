"""Checkpointer round trip and completion markers; prefetcher exact resume; LR schedules."""

import math
import os

import pytest
import torch
import torch.nn as nn

from pluggy_b200.checkpoint.checkpointer import Checkpointer
from pluggy_b200.dataloader.prefetcher import CUDAPrefetcher
from pluggy_b200.dataloader.synthetic import SyntheticBatches, SyntheticZipfRows
from pluggy_b200.optimizer.builder import build_scheduler
from pluggy_b200.optimizer.scheduler import (CosineAnnealingScheduler, WarmupStableDecaySchedulder,
                                             cosine_scale, wsd_scale)


def _mlp():
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(8, 16), nn.GELU(), nn.Linear(16, 4))


def _train(model, opt, sched, batches, n):
    for _ in range(n):
        b = next(batches)
        x = b["input_ids"][:, :8].float() / 500
        loss = model(x).pow(2).mean()
        loss.backward()
        opt.step()
        opt.zero_grad()
        sched.step()


def test_round_trip_resumes_exactly(tmp_path):
    ck = Checkpointer(str(tmp_path / "run"))
    m = _mlp()
    opt = torch.optim.AdamW(m.parameters(), lr=1e-2)
    sch = CosineAnnealingScheduler(opt, total_steps=20, warmup_ratio=0.1)
    data = CUDAPrefetcher(SyntheticBatches(SyntheticZipfRows(500, 16, seed=1), 4), torch.device("cpu"))
    _train(m, opt, sch, data, 5)
    ck.save_model(m, 5)
    ck.save_optimizer(opt, 5)
    ck.save_scheduler(sch, 5)
    ck.save_trainer({"step": 5}, 5)
    ck.save_rng({"cpu_rng": torch.get_rng_state()}, 5, rank=0)
    ck.save_dataloader_state(data.loader_state_dict(), 5, dp_rank=0)
    assert ck.latest() is None  # not complete yet: invisible
    ck.mark_complete(5)
    assert ck.latest() == 5 and ck.valid_step(5) == 5 and ck.valid_step(4) is None
    _train(m, opt, sch, data, 5)
    want = [p.detach().clone() for p in m.parameters()]

    m2 = _mlp()
    with torch.no_grad():
        for p in m2.parameters():
            p.add_(1.0)  # different from the saved state
    opt2 = torch.optim.AdamW(m2.parameters(), lr=1e-2)
    sch2 = CosineAnnealingScheduler(opt2, total_steps=20, warmup_ratio=0.1)
    loader2 = SyntheticBatches(SyntheticZipfRows(500, 16, seed=1), 4)
    ck.load_model(m2, 5)
    ck.load_optimizer(opt2, 5)
    ck.load_scheduler(sch2, 5)
    ck.load_dataloader(loader2, 5, dp_rank=0)
    torch.set_rng_state(ck.load_rng(5, rank=0)["cpu_rng"])
    assert ck.load_trainer(5)["step"] == 5 and ck.load_rng(5, rank=3) is None
    _train(m2, opt2, sch2, CUDAPrefetcher(loader2, torch.device("cpu")), 5)
    for a, b in zip(want, m2.parameters()):
        assert torch.equal(a, b)


def test_prefetcher_state_is_the_consumed_state():
    """The prefetcher pulls one batch ahead; its saved state must not skip that batch."""
    loader = SyntheticBatches(SyntheticZipfRows(500, 16, seed=2), 2)
    pf = CUDAPrefetcher(loader, torch.device("cpu"))
    for _ in range(3):
        next(pf)
    st = pf.loader_state_dict()
    assert loader.state_dict() != st  # the live state is one ahead (negative control)
    want = next(pf)["input_ids"]
    l2 = SyntheticBatches(SyntheticZipfRows(500, 16, seed=2), 2)
    l2.load_state_dict(st)
    assert torch.equal(next(CUDAPrefetcher(l2, torch.device("cpu")))["input_ids"], want)


def test_torn_directories_are_ignored(tmp_path):
    ck = Checkpointer(str(tmp_path))
    for s in (2, 4, 6):
        ck.save_trainer({"step": s}, s)
    ck.mark_complete(2)
    ck.mark_complete(4)
    os.makedirs(tmp_path / "notastep")
    assert ck.latest() == 4  # 6 is torn (no marker)
    assert ck.valid_step(6) is None


def test_sharded_consolidate(tmp_path):
    ck = Checkpointer(str(tmp_path))
    full = {"w": torch.arange(24.).view(6, 4), "b": torch.ones(3)}
    for r in range(3):
        ck.save_sharded_model({"w": full["w"][2 * r: 2 * r + 2], "b": full["b"]},
                              {"w": {"dim": 0, "coord": r, "axis_size": 3}, "b": {"dim": None}}, 7, r, 3)
    out = ck.consolidate(7, 3)
    assert torch.equal(out["w"], full["w"]) and torch.equal(out["b"], full["b"])
    assert torch.equal(torch.load(tmp_path / "7" / "model.pt")["w"], full["w"])


def test_wsd_and_cosine_shapes():
    T = 100
    w = [wsd_scale(s, T, 0.1, 0.2) for s in range(T)]
    assert w[0] == pytest.approx(0.1) and w[9] == pytest.approx(1.0)
    assert all(v == 1.0 for v in w[10:80])
    assert w[80] == pytest.approx(1.0) and w[90] == pytest.approx(0.5) and w[99] == pytest.approx(0.05)
    c = [cosine_scale(s, T, 0.1, 0.1) for s in range(T + 20)]
    assert c[9] == pytest.approx(1.0)
    mid = 10 + (T - 10) // 2
    assert c[mid] == pytest.approx(0.1 + 0.9 * 0.5 * (1 + math.cos(math.pi * (mid - 10) / 90)))
    assert all(v == pytest.approx(0.1) for v in c[T:])  # held at the floor


@pytest.mark.parametrize("kind", ["wsd", "cosine"])
def test_scheduler_resume(kind):
    cfg = {"type": kind, "total_steps": 50, "warmup_ratio": 0.1}
    cfg.update({"decay_ratio": 0.3} if kind == "wsd" else {"min_lr_ratio": 0.05})

    def make():
        opt = torch.optim.SGD([nn.Parameter(torch.zeros(1))], lr=2.0)
        return opt, build_scheduler(opt, cfg)

    opt, s = make()
    lrs = []
    for _ in range(50):
        lrs.append(s.get_last_lr()[0])
        opt.step()
        s.step()
    opt2, s2 = make()
    for _ in range(20):
        opt2.step()
        s2.step()
    state = s2.state_dict()
    opt3, s3 = make()
    s3.load_state_dict(state)
    rest = []
    for _ in range(30):
        rest.append(s3.get_last_lr()[0])
        opt3.step()
        s3.step()
    assert rest == pytest.approx(lrs[20:])
    cls = WarmupStableDecaySchedulder if kind == "wsd" else CosineAnnealingScheduler
    assert isinstance(s, cls)


def test_fused_adamw_device_hyper_bookkeeping():
    """CUDA-graph steps keep the host bookkeeping out of the graph: ``advance`` counts
    the step and writes this step's (lr, 1 - b1^t, 1 - b2^t) per group, and the state
    dict keeps the same step counts as eager steps."""
    from pluggy_b200.optimizer.fused_adamw import FusedAdamW

    ps = [nn.Parameter(torch.randn(4, 3)), nn.Parameter(torch.randn(3))]
    opt = FusedAdamW([{"params": ps[:1], "weight_decay": 0.1}, {"params": ps[1:], "weight_decay": 0.0}],
                     lr=1e-3, betas=(0.9, 0.95))
    for p in ps:
        p.grad = torch.randn_like(p)
    opt.step()  # eager first step creates the state
    opt.use_device_hyper("cpu")
    for g in opt.param_groups:
        g["lr"] = 5e-4
    opt.advance()
    opt.advance()
    assert [float(opt.state[p]["step"]) for p in ps] == [3.0, 3.0]
    for hyper in opt._hyper:
        assert torch.allclose(hyper, torch.tensor([5e-4, 1 - 0.9 ** 3, 1 - 0.95 ** 3]))
    sd = opt.state_dict()
    assert all(float(s["step"]) == 3.0 for s in sd["state"].values())


def test_background_prefetcher_matches_inline():
    """Pulling batches on a worker thread gives the same batches and the same
    consumed-state snapshots as pulling them inline, and stops at the end."""
    def run(background):
        loader = SyntheticBatches(SyntheticZipfRows(500, 16, seed=3), 2)
        pf = CUDAPrefetcher(loader, torch.device("cpu"), background=background, depth=3)
        out = []
        for _ in range(6):
            b = next(pf)["input_ids"].clone()
            out.append((b, dict(pf.loader_state_dict())))
        return out

    a, b = run(False), run(True)
    for (x, sx), (y, sy) in zip(a, b, strict=True):
        assert torch.equal(x, y) and sx == sy

    class Short:
        def __init__(self):
            self.i = 0

        def __iter__(self):
            return self

        def __next__(self):
            if self.i == 2:
                raise StopIteration
            self.i += 1
            return {"x": torch.full((2,), self.i)}

        def state_dict(self):
            return {"i": self.i}

    pf = CUDAPrefetcher(Short(), torch.device("cpu"), background=True)
    assert [int(next(pf)["x"][0]) for _ in range(2)] == [1, 2]
    with pytest.raises(StopIteration):
        next(pf)
    with pytest.raises(StopIteration):
        next(pf)
