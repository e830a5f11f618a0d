"""Tensor-parallel collective microbenchmark: peer-memory kernels vs NCCL.

``torchrun --nproc-per-node N -m pluggy_b200.comm.bench_tp [--B 2 --S 8192 --H 2048]``
times, on every rank with CUDA events (after warm-up, back-to-back calls whose
operands exceed L2) and reports the max over ranks:

* ``gemm_rs``: row-parallel linear ``[B*S, H/n] @ [H, H/n]^T`` reduce-scattered
  along the sequence — the fused GEMM (reduce-scatter epilogue over NVLink) vs
  the same tcgen05 GEMM followed by NCCL ``reduce_scatter_tensor``;
* ``ag``: sequence all-gather of ``[B, S/n, H]`` bf16 — peer pull vs NCCL;
* ``rs``: sequence reduce-scatter of ``[B, S, H]`` bf16 partials — peer push vs NCCL.

Roofline for each: the slower of FLOPs at the measured bf16 GEMM peak and the
bytes that must leave each GPU over NVLink at 770 GB/s per direction (measured
peer-copy bandwidth on this hardware). Defaults: the Llama-3.2-1B TP config
(hidden 2048, micro-batch 2 x 8192 tokens).
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _time(fn, iters, warmup, flush):
    """Mean device ms per call over ``iters`` back-to-back calls (the calls pace
    each other through their handshakes, so per-call skew between ranks does not
    enter), max over ranks. Inputs and outputs exceed L2 for the default shapes."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    flush.fill_(1)
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
    p.add_argument("--B", type=int, default=2)
    p.add_argument("--S", type=int, default=8192)
    p.add_argument("--H", type=int, default=2048)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    a = p.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from pluggy_b200.comm.tp_fused import TPComm
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.ops import _ext
    from pluggy_b200.ops.gemm import gemm
    from pluggy_b200.ops.microbench import peaks

    _, bf16_peak, label = peaks()
    mesh = Mesh({"tp": world})
    comm = TPComm(mesh, "tp", capacity_bytes=a.B * a.S * a.H * 2)
    grp = mesh.get_group("tp")
    B, S, H, n = a.B, a.S, a.H, world
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(rank)
    x = torch.randn(B, S, H // n, device="cuda", generator=g).bfloat16()
    w = (torch.randn(H, H // n, device="cuda", generator=g) * 0.02).bfloat16()
    part = torch.randn(B, S, H, device="cuda", generator=g).bfloat16()
    shard = torch.randn(B, S // n, H, device="cuda", generator=g).bfloat16()
    y = torch.empty(B * S, H, device="cuda", dtype=torch.bfloat16)
    out_rs = torch.empty(B * S // n, H, device="cuda", dtype=torch.bfloat16)
    out_ag = torch.empty(n * B * (S // n), H, device="cuda", dtype=torch.bfloat16)

    def nccl_gemm_rs():
        gemm(x.view(B * S, H // n), w, out=y)
        # NCCL scatters along rows: [n, B*S/n] blocks of a sequence-major copy
        t = y.view(B, n, S // n, H).transpose(0, 1).contiguous()
        dist.reduce_scatter_tensor(out_rs, t.view(n * B * (S // n), H), group=grp)

    def nccl_ag():
        dist.all_gather_into_tensor(out_ag, shard.reshape(-1, H), group=grp)

    def nccl_rs():
        t = part.view(B, n, S // n, H).transpose(0, 1).contiguous()
        dist.reduce_scatter_tensor(out_rs, t.view(-1, H), group=grp)

    cases = {
        "gemm_rs": (lambda: comm.gemm_reduce_scatter(x, w), nccl_gemm_rs,
                    2.0 * B * S * H * (H // n), B * S * H * 2 * (n - 1) / n),
        "ag": (lambda: comm.all_gather_seq(shard), nccl_ag, 0.0, B * S * H * 2 * (n - 1) / n),
        "rs": (lambda: comm.reduce_scatter_seq(part), nccl_rs, 0.0, B * S * H * 2 * (n - 1) / n),
    }
    for name, (ours, ref, flops, nv_bytes) in cases.items():
        t_ours = _time(ours, a.iters, a.warmup, flush)
        t_ref = _time(ref, a.iters, a.warmup, flush)
        roof = max(flops / bf16_peak * 1e3, nv_bytes / (NVLINK_GBS * 1e9) * 1e3)
        if rank == 0:
            print(json.dumps({"op": name, "n_gpus": n, "shape": {"B": B, "S": S, "H": H},
                              "ms_peer": round(t_ours, 4), "ms_nccl": round(t_ref, 4),
                              "speedup": round(t_ref / t_ours, 3), "roofline_ms": round(roof, 4),
                              f"frac_of_roofline_{label}": round(roof / t_ours, 3)}), flush=True)
    torch.cuda.synchronize()
    _ext.check_status()
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
