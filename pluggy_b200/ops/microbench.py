"""Per-op microbenchmarks of the sm_100a kernels, against the measured roofline.

``python -m pluggy_b200.ops.microbench --op attn_bwd [--iters 20] [--warmup 5]``
times one op with CUDA events on its stream, after warm-up, with the L2 flushed
(a 256 MiB buffer written) before every timed launch, and prints one JSON line
per op: milliseconds, the algorithmic FLOP/s or bytes/s, and the fraction of the
peak measured on this hardware (``MEASURED_PEAKS.json`` at the repository root if
present: a STREAM-style copy and a cuBLAS bf16 GEMM; otherwise 6.65 TB/s and
1.59 PFLOP/s). ``--op all`` runs every case; ``--small`` shrinks each case to a
size meant for profiler captures (still larger than L2). Shapes default to the
Qwen3-0.6B training step at micro-batch 8 x 4096 tokens.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

PEAKS_FILE = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                          "MEASURED_PEAKS.json")


def peaks() -> tuple[float, float, str]:
    """(bytes/s, bf16 FLOP/s, label) of the roofline denominators."""
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return p["hbm_gbs"] * 1e9, p["bf16_tflops"] * 1e12, "measured"
    except (OSError, KeyError, ValueError):
        return 6.65e12, 1.59e15, "fallback"


class _Flush:
    def __init__(self, dev):
        self.buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def __call__(self):
        self.buf.fill_(1)


def time_op(fn, iters: int, warmup: int, flush: bool = True) -> float:
    """Mean device milliseconds of ``fn`` over ``iters`` launches (L2 flushed before each)."""
    fl = _Flush(torch.cuda.current_device()) if flush else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    for i in range(iters):
        if fl is not None:
            fl()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / iters


def _bf16(*shape, dev="cuda"):
    return torch.randn(*shape, device=dev).to(torch.bfloat16)


def case_gemm(a, small):
    from pluggy_b200.ops.gemm import gemm

    M, N, K = (16384, 4096, 1024) if small else (a.m, a.n, a.k)
    if a.layout == "nt":  # forward: x[M,K] @ w[N,K]^T
        x, w = _bf16(M, K), _bf16(N, K)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        fn = lambda: gemm(x, w, out=out)  # noqa: E731
    elif a.layout == "nn":  # dgrad: dy[M,K] @ w[K,N]
        x, w = _bf16(M, K), _bf16(K, N)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        fn = lambda: gemm(x, w, b_mn_major=True, out=out)  # noqa: E731
    else:  # "tn" wgrad: dy[K,M]^T @ x[K,N], fp32 out
        x, w = _bf16(K, M), _bf16(K, N)
        out = torch.empty(M, N, device="cuda", dtype=torch.float32)
        fn = lambda: gemm(x, w, a_mn_major=True, b_mn_major=True, out=out)  # noqa: E731
    return fn, {"flops": 2.0 * M * N * K, "shape": {"M": M, "N": N, "K": K, "layout": a.layout}}


def _attn_inputs(a, small):
    B = 2 if small else a.batch
    S, Hq, Hk, d = a.seq, a.heads, a.kv_heads, a.head_dim
    q, k, v = _bf16(B, S, Hq, d), _bf16(B, S, Hk, d), _bf16(B, S, Hk, d)
    flops = 4.0 * B * Hq * S * S * d / 2  # causal
    return q, k, v, flops, {"B": B, "S": S, "Hq": Hq, "Hk": Hk, "d": d, "causal": True}


def case_attn_fwd(a, small):
    from pluggy_b200.ops.attention import attn_fwd

    q, k, v, flops, shape = _attn_inputs(a, small)
    return (lambda: attn_fwd(q, k, v)), {"flops": flops, "shape": shape}


def case_attn_bwd(a, small):
    from pluggy_b200.ops.attention import attn_bwd, attn_fwd

    q, k, v, flops, shape = _attn_inputs(a, small)
    o, lse = attn_fwd(q, k, v)
    do = torch.randn_like(o)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    fn = lambda: attn_bwd(q, k, v, o, lse, do, dq=dq, dk=dk, dv=dv)  # noqa: E731
    return fn, {"flops": 2.5 * flops, "shape": shape}


def _tokens(a, small):
    return (2 if small else a.batch) * a.seq


def case_qk_rope_fwd(a, small):
    from pluggy_b200.ops.norm import qk_norm_rope_fwd

    T, Hq, Hk, d = _tokens(a, small), a.heads, a.kv_heads, a.head_dim
    qkv = _bf16(T, (Hq + 2 * Hk) * d)
    wq, wk = torch.ones(d, device="cuda"), torch.ones(d, device="cuda")
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device="cuda").float() / d))
    pos = (torch.arange(T, device="cuda", dtype=torch.int32) % a.seq)
    fn = lambda: qk_norm_rope_fwd(qkv, S=a.seq, Hq=Hq, Hk=Hk, d=d, wq=wq, wk=wk,  # noqa: E731
                                  inv_freq=inv, positions=pos)
    byt = T * (Hq + Hk) * d * 2 * 2 + T * (Hq + Hk) * 4
    return fn, {"bytes": byt, "shape": {"T": T, "Hq": Hq, "Hk": Hk, "d": d}}


def case_qk_rope_bwd(a, small):
    from pluggy_b200.ops.norm import qk_norm_rope_bwd, qk_norm_rope_fwd

    T, Hq, Hk, d = _tokens(a, small), a.heads, a.kv_heads, a.head_dim
    qkv = _bf16(T, (Hq + 2 * Hk) * d)
    wq, wk = torch.ones(d, device="cuda"), torch.ones(d, device="cuda")
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device="cuda").float() / d))
    pos = (torch.arange(T, device="cuda", dtype=torch.int32) % a.seq)
    _, _, rstd = qk_norm_rope_fwd(qkv, S=a.seq, Hq=Hq, Hk=Hk, d=d, wq=wq, wk=wk, inv_freq=inv,
                                  positions=pos)
    dq, dk = _bf16(T, Hq, d), _bf16(T, Hk, d)
    dqkv = torch.empty_like(qkv)
    fn = lambda: qk_norm_rope_bwd(qkv, rstd, dq, dk, dqkv, S=a.seq, Hq=Hq, Hk=Hk, d=d,  # noqa: E731
                                  wq=wq, wk=wk, inv_freq=inv, positions=pos)
    byt = T * (Hq + Hk) * d * 2 * 3 + T * (Hq + Hk) * 4
    return fn, {"bytes": byt, "shape": {"T": T, "Hq": Hq, "Hk": Hk, "d": d}}


def case_rmsnorm_fwd(a, small):
    from pluggy_b200.ops.norm import rmsnorm_fwd

    T, D = _tokens(a, small), a.dim
    x, w = _bf16(T, D), torch.ones(D, device="cuda")
    return (lambda: rmsnorm_fwd(x, w, 1e-6)), {"bytes": T * D * 4 + T * 4,
                                               "shape": {"T": T, "D": D}}


def case_rmsnorm_bwd(a, small):
    from pluggy_b200.ops.norm import rmsnorm_bwd, rmsnorm_fwd

    T, D = _tokens(a, small), a.dim
    x, w = _bf16(T, D), torch.ones(D, device="cuda")
    _, rstd = rmsnorm_fwd(x, w, 1e-6)[:2]
    dy = _bf16(T, D)
    fn = lambda: rmsnorm_bwd(dy, x, w, rstd, want_f32=False, want_bf16=True)  # noqa: E731
    return fn, {"bytes": T * D * 6 + T * 4, "shape": {"T": T, "D": D}}


def case_glu_fwd(a, small):
    from pluggy_b200.ops.elementwise import glu_fwd

    T, F = _tokens(a, small), a.ffn
    gu = _bf16(T, 2 * F)
    return (lambda: glu_fwd(gu)), {"bytes": T * F * 6, "shape": {"T": T, "F": F}}


def case_glu_bwd(a, small):
    from pluggy_b200.ops.elementwise import glu_bwd

    T, F = _tokens(a, small), a.ffn
    gu, dout = _bf16(T, 2 * F), _bf16(T, F)
    out = torch.empty_like(gu)
    return (lambda: glu_bwd(gu, dout, out=out)), {"bytes": T * F * 10, "shape": {"T": T, "F": F}}


def case_ce_rows(a, small):
    """The fused CE's per-row pass over one logits chunk (bf16, in place)."""
    from pluggy_b200.ops._ext import ext

    N, V = (1024 if small else 4096), a.vocab
    logits = _bf16(N, V)
    labels = torch.randint(0, V, (N,), device="cuda")
    loss = torch.zeros(1, device="cuda")
    fn = lambda: ext().ce_rows(logits, labels, -100, 1.0, 0.0, None, loss, None)  # noqa: E731
    return fn, {"bytes": N * V * 4, "shape": {"rows": N, "V": V}}


def case_adamw(a, small):
    from pluggy_b200.ops.optim import adamw_step

    n = (64 if small else 256) << 20
    p, g, m, v = (torch.randn(n, device="cuda") for _ in range(4))
    sh = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    fn = lambda: adamw_step([p], [g], [m], [v], [sh], lr=1e-4, beta1=0.9, beta2=0.95,  # noqa: E731
                            eps=1e-8, weight_decay=0.1, bias_correction1=0.9,
                            bias_correction2=0.95)
    return fn, {"bytes": n * (4 * 4 + 3 * 4 + 2), "shape": {"params": n}}


def case_sumsq(a, small):
    from pluggy_b200.ops.optim import multi_tensor_sumsq

    ts = [torch.randn(n, device="cuda") for n in ([8 << 20] * (4 if small else 32))]
    return (lambda: multi_tensor_sumsq(ts)), {"bytes": sum(t.numel() for t in ts) * 4,
                                              "shape": {"tensors": len(ts)}}


def case_embedding(a, small):
    from pluggy_b200.ops._ext import ext

    T, D, V = _tokens(a, small), a.dim, a.vocab
    w = torch.randn(V, D, device="cuda")
    ids = torch.randint(0, V, (T,), device="cuda")
    out = torch.empty(T, D, device="cuda")
    fn = lambda: ext().embedding_fwd(ids, w, out, 1.0)  # noqa: E731
    return fn, {"bytes": T * D * 8, "shape": {"T": T, "D": D, "V": V}}


def case_embedding_bwd(a, small):
    """Deterministic (sorted) embedding backward with Zipf(1.1)-distributed ids."""
    from pluggy_b200.ops._ext import ext

    T, D, V = _tokens(a, small), a.dim, a.vocab
    r = torch.arange(1, V + 1, device="cuda", dtype=torch.float64)
    p = r.pow(-1.1)
    ids = torch.multinomial((p / p.sum()).float(), T, replacement=True)
    dout = torch.randn(T, D, device="cuda")
    dw = torch.zeros(V, D, device="cuda")

    def fn():
        s, pos = torch.sort(ids, stable=True)
        ext().embedding_bwd_sorted(s, pos, dout, dw, 1.0)
    # algorithmic bytes: dout read once, the touched rows of dw read and written
    touched = int(torch.unique(ids).numel())
    return fn, {"bytes": T * D * 4 + touched * D * 8, "shape": {"T": T, "D": D, "unique_ids": touched}}


def case_grouped_gemm(a, small):
    """One MoE expert projection over all experts (grouped tcgen05 GEMM, mode 1):
    T tokens x top-k rows routed uniformly over E experts, [E, N, K] weights."""
    from pluggy_b200.ops._ext import ext
    from pluggy_b200.ops.grouped import expert_layout

    E, topk, K, N = a.experts, a.topk, a.dim, a.n
    P = (2048 if small else 8192) * topk
    ex = torch.randint(0, E, (P,), device="cuda").sort().values
    counts = torch.bincount(ex, minlength=E)
    poff, shift, tg, R = expert_layout(counts, P)
    x = torch.zeros(R, K, device="cuda", dtype=torch.bfloat16)
    x[torch.arange(P, device="cuda") + shift[ex]] = _bf16(P, K)
    w = _bf16(E * N, K)
    out = torch.empty(R, N, device="cuda", dtype=torch.bfloat16)
    if a.layout == "tn":  # weight gradient (mode 2): dW_e = dy_e^T x_e
        dy = _bf16(R, N)
        dw = torch.empty(E * N, K, device="cuda", dtype=torch.float32)
        fn = lambda: ext().gemm_grouped(dy, x, True, dw, 2, poff, E, 0, 1.0, 0.0)  # noqa: E731
    else:
        fn = lambda: ext().gemm_grouped(x, w, False, out, 1, tg, E, N, 1.0, 0.0)  # noqa: E731
    return fn, {"flops": 2 * P * N * K, "shape": {"rows": P, "padded_rows": int(poff[-1]),
                                                   "E": E, "N": N, "K": K, "layout": a.layout}}


def case_zero1(a, small):
    """ZeRO-1 reduce-scatter and AdamW+all-gather kernels on one rank (no peers: the
    local memory side of the kernels; NVLink rates come from the multi-GPU runs)."""
    from pluggy_b200.comm.symm import SymmetricBuffer
    from pluggy_b200.core.mesh import Mesh
    from pluggy_b200.ops._ext import ext, status_word

    import torch.distributed as dist

    if not dist.is_initialized():
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29533", rank=0, world_size=1)
    mesh = Mesh({"dp": 1})
    n = (64 if small else 256) << 20
    g = SymmetricBuffer(n * 4, mesh, "dp")
    pa = SymmetricBuffer(n * 4, mesh, "dp")
    fl = SymmetricBuffer(3 * 8 * 128 * 4, mesh, "dp")
    sl = SymmetricBuffer(8 * 128 * 4, mesh, "dp")
    g.tensor(0, [n]).normal_()
    pa.tensor(0, [n]).normal_()
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    rows = torch.tensor([[0, n, 0]], dtype=torch.int64, device="cuda")
    norm = torch.zeros(1, device="cuda")
    ep = [0, 0]
    st = status_word()

    def rs():
        ep[0] += 1
        ext().zero1_rs(g.peers, pa.peers, fl.peers, sl.peers, 0, n, 0, ep[0], 128, norm, False, st)

    def ag():
        ep[1] += 1
        ext().zero1_adamw_ag(g.peers, pa.peers, fl.peers, sl.peers, 0, n, 0, ep[1], 128, [1e-4], [0.1],
                             0.9, 0.95, 1e-8, 0.9, 0.95, None, rows, m, v, st)
    fn = ag if a.layout == "tn" else rs
    nbytes = n * (4 + 4) if fn is rs else n * (4 * 4 + 3 * 4)
    return fn, {"bytes": nbytes, "shape": {"elements": n, "kernel": "adamw_ag" if fn is ag else "rs"}}


def case_rope(a, small):
    """RoPE on a transposed [B, S, H, d] projection view (the OLMo-3 / Gemma-4 path)."""
    from pluggy_b200.ops.elementwise import apply_rotary

    T, H, d = _tokens(a, small), a.heads, a.head_dim
    B = max(1, T // a.seq)
    S = T // B
    x = _bf16(B, S, H, d).transpose(1, 2)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device="cuda").float() / d))
    f = torch.arange(S, device="cuda").float()[:, None] * inv
    emb = torch.cat([f, f], -1)
    cos, sin = emb.cos()[None, None], emb.sin()[None, None]
    fn = lambda: apply_rotary(x, cos, sin)  # noqa: E731
    return fn, {"bytes": B * S * H * d * 2 * 2 + S * d * 8, "shape": {"B": B, "S": S, "H": H, "d": d}}


def case_router(a, small):
    """MoE router: softmax + top-k + renormalisation + histogram over [T, E] logits."""
    from pluggy_b200.ops._ext import ext

    T, E, k = _tokens(a, small), a.experts, a.topk
    logits = _bf16(T, E)
    probs = torch.empty(T, E, device="cuda")
    w = torch.empty(T, k, device="cuda")
    idx = torch.empty(T, k, dtype=torch.int64, device="cuda")
    counts = torch.zeros(E, dtype=torch.int32, device="cuda")
    fn = lambda: ext().router_topk(logits, k, True, probs, w, idx, counts)  # noqa: E731
    return fn, {"bytes": T * E * (2 + 4) + T * k * 12, "shape": {"T": T, "E": E, "k": k}}


CASES = {
    "gemm": case_gemm, "attn_fwd": case_attn_fwd, "attn_bwd": case_attn_bwd,
    "qk_rope_fwd": case_qk_rope_fwd, "qk_rope_bwd": case_qk_rope_bwd,
    "rmsnorm_fwd": case_rmsnorm_fwd, "rmsnorm_bwd": case_rmsnorm_bwd,
    "glu_fwd": case_glu_fwd, "glu_bwd": case_glu_bwd,
    "ce_rows": case_ce_rows, "adamw": case_adamw, "sumsq": case_sumsq, "embedding": case_embedding,
    "embedding_bwd": case_embedding_bwd, "grouped_gemm": case_grouped_gemm, "zero1": case_zero1,
    "rope": case_rope, "router": case_router,
}


def run_case(name: str, a) -> dict:
    from pluggy_b200.ops._ext import check_status

    fn, info = CASES[name](a, a.small)
    ms = time_op(fn, a.iters, a.warmup, flush=not a.no_flush)
    check_status()
    bw, fl, label = peaks()
    rec = {"op": name, "ms": round(ms, 4), **info}
    if "flops" in info:
        rec["tflops"] = round(info["flops"] / ms / 1e9, 1)
        rec[f"frac_of_{label}_bf16"] = round(info["flops"] / ms * 1e3 / fl, 3)
    else:
        rec["gbs"] = round(info["bytes"] / ms / 1e6, 1)
        rec[f"frac_of_{label}_hbm"] = round(info["bytes"] / ms * 1e3 / bw, 3)
    return rec


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="time one sm_100a op against the roofline")
    p.add_argument("--op", default="all", choices=["all", *CASES])
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--small", action="store_true", help="profiler-sized case (> L2, a few GB at most)")
    p.add_argument("--no-flush", action="store_true")
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--seq", type=int, default=4096)
    p.add_argument("--heads", type=int, default=16)
    p.add_argument("--kv-heads", type=int, default=8)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--dim", type=int, default=1024)
    p.add_argument("--ffn", type=int, default=3072)
    p.add_argument("--vocab", type=int, default=151936)
    p.add_argument("--m", type=int, default=32768)
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--k", type=int, default=1024)
    p.add_argument("--layout", default="nt", choices=["nt", "nn", "tn"])
    p.add_argument("--experts", type=int, default=128)
    p.add_argument("--topk", type=int, default=8)
    a = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("microbench needs a CUDA device")
    torch.manual_seed(0)
    for name in (CASES if a.op == "all" else [a.op]):
        print(json.dumps(run_case(name, a)), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
