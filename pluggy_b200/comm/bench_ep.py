"""Expert-parallel token exchange microbenchmark: peer-memory kernels vs NCCL.

``torchrun --nproc-per-node N -m pluggy_b200.comm.bench_ep [--tokens 8192 --top-k 8
--hidden 2048 --experts 128]`` routes ``tokens x top_k`` pairs per rank to random
experts (uniform: every rank sends about 1/N of its rows to each rank), then times
dispatch + combine (rows out to the expert owners and back) with CUDA events over
back-to-back calls, max over ranks:

* peer: :class:`pluggy_b200.comm.ep_fused.EPComm` (peer stores into the owners'
  buffers, flag handshakes); the count-matrix exchange is timed separately;
* nccl: ``all_to_all_single`` with uneven splits both ways (splits known on the host).

Roofline: the bytes each GPU must send both ways, 2 x (N-1)/N x rows x hidden x 2,
at the measured 770 GB/s per-direction peer bandwidth. Defaults: the Qwen3-MoE EP
config (micro-batch 2 x 4096 tokens, top-8 of 128 experts, hidden 2048).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _time(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def main(argv=None) -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=8192)
    p.add_argument("--top-k", type=int, default=8)
    p.add_argument("--hidden", type=int, default=2048)
    p.add_argument("--experts", type=int, default=128)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    a = p.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from pluggy_b200.comm.ep_fused import EPComm
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.ops import _ext

    mesh = Mesh({"ep": world})
    grp = mesh.get_group("ep")
    H, E, n = a.hidden, a.experts, world
    P = a.tokens * a.top_k
    g = torch.Generator(device="cuda").manual_seed(rank)
    exp = torch.sort(torch.randint(0, E, (P,), device="cuda", generator=g)).values
    x = torch.randn(P, H, device="cuda", generator=g).bfloat16()
    comm = EPComm(mesh, "ep", E, H, capacity_rows=2 * P)
    cnt = torch.bincount(exp, minlength=E)
    C = comm.exchange_counts(cnt)
    pl = comm.plan(C)

    def peer():
        y = comm.to_owners(x, pl)
        comm.to_sources(y, pl)

    send, recv = pl["send"], pl["recv"]
    ybuf = torch.empty(pl["R"], H, device="cuda", dtype=torch.bfloat16)
    back = torch.empty(P, H, device="cuda", dtype=torch.bfloat16)

    def nccl():
        dist.all_to_all_single(ybuf, x, recv, send, group=grp)
        dist.all_to_all_single(back, ybuf, send, recv, group=grp)

    t_peer = _time(peer, a.iters, a.warmup)
    t_nccl = _time(nccl, a.iters, a.warmup)
    t_cnt = _time(lambda: comm.exchange_counts(cnt), a.iters, a.warmup)
    nv = 2.0 * (n - 1) / n * P * H * 2
    roof = nv / (NVLINK_GBS * 1e9) * 1e3
    if rank == 0:
        print(json.dumps({"op": "moe_dispatch_combine", "n_gpus": n,
                          "shape": {"pairs": P, "hidden": H, "experts": E},
                          "ms_peer": round(t_peer, 4), "ms_nccl": round(t_nccl, 4),
                          "speedup": round(t_nccl / t_peer, 3), "roofline_ms": round(roof, 4),
                          "frac_of_roofline": round(roof / t_peer, 3),
                          "ms_count_exchange_with_host_copy": round(t_cnt, 4)}), flush=True)
    torch.cuda.synchronize()
    _ext.check_status()
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
