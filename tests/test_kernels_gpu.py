"""Numerics of every sm_100a kernel against a plain fp32 PyTorch reference of the same op."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(autouse=True)
def _status():
    from pluggy_b200.ops import _ext

    _ext.ext()
    yield
    torch.cuda.synchronize()
    _ext.check_status()


# ---------------------------------------------------------------------- GEMM
# every stride must stay 16-byte aligned (multiples of 8 bf16): M, N, K % 8 == 0 where they are
# a leading dimension; edges that are not multiples of the 128x256x64 tile are exercised
GEMM_SHAPES = [(128, 256, 64), (256, 512, 128), (296, 200, 136), (1000, 384, 520), (4096, 4096, 1024),
               (136, 1032, 72), (8192, 1024, 3072), (200, 1000, 8)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("layout", ["fwd", "dgrad", "wgrad"])
def test_gemm_layouts(M, N, K, layout):
    from pluggy_b200.ops.gemm import gemm

    torch.manual_seed(M + N + K)
    A = torch.randn(M, K, device=DEV).bfloat16()
    B = torch.randn(N, K, device=DEV).bfloat16()
    ref = A.float() @ B.float().t()
    if layout == "fwd":
        out = gemm(A, B)
    elif layout == "dgrad":  # B given as [K, N]
        out = gemm(A, B.t().contiguous(), b_mn_major=True)
    else:  # A given as [K, M] and B as [K, N], fp32 out
        out = gemm(A.t().contiguous(), B.t().contiguous(), a_mn_major=True, b_mn_major=True,
                   out_dtype=torch.float32)
    assert rel(out, ref) < 1e-2, (layout, M, N, K, rel(out, ref))


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_tile_widths_and_fp32_out(bn):
    from pluggy_b200.ops.gemm import gemm

    A = torch.randn(777, 320, device=DEV).bfloat16()
    B = torch.randn(640, 320, device=DEV).bfloat16()
    out = gemm(A, B, out_dtype=torch.float32, bn=bn)
    assert rel(out, A.float() @ B.float().t()) < 5e-3


def test_gemm_residual_epilogue():
    from pluggy_b200.ops.gemm import linear_fwd

    x = torch.randn(1024, 512, device=DEV).bfloat16()
    w = torch.randn(384, 512, device=DEV).bfloat16() * 0.05
    r = torch.randn(1024, 384, device=DEV)
    out = linear_fwd(x, w, out_dtype=torch.float32, residual=r)
    assert rel(out, r + x.float() @ w.float().t()) < 5e-3


def test_gemm_split_k_and_accumulate():
    from pluggy_b200.ops.gemm import gemm, linear_wgrad

    dy = torch.randn(16384, 256, device=DEV).bfloat16()
    x = torch.randn(16384, 128, device=DEV).bfloat16()
    ref = dy.float().t() @ x.float()
    out = linear_wgrad(dy, x)  # small output, long K: split-K with fp32 atomics
    assert rel(out, ref) < 5e-3
    acc = torch.ones(256, 128, device=DEV)
    linear_wgrad(dy, x, out=acc, accumulate=True)
    assert rel(acc, ref + 1) < 5e-3
    for s in (1, 3, 7):
        o = gemm(dy, x, a_mn_major=True, b_mn_major=True, out_dtype=torch.float32, splits=s)
        assert rel(o, ref) < 5e-3, s


def test_gemm_rejects_misaligned_and_mismatched():
    from pluggy_b200.ops.gemm import gemm

    a = torch.randn(64, 100, device=DEV).bfloat16()  # K = 100: rows not 16-byte aligned
    with pytest.raises(Exception):
        gemm(a, a)
    x = torch.randn(64, 128, device=DEV).bfloat16()
    with pytest.raises(ValueError):
        gemm(x, torch.randn(64, 256, device=DEV).bfloat16())


# ---------------------------------------------------------------- norms, rope
@pytest.mark.parametrize("D", [128, 1024, 2560])
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
def test_rmsnorm_fwd_bwd(D, xdt):
    from pluggy_b200.ops.norm import rms_norm, rms_norm_reference

    x = torch.randn(333, D, device=DEV, dtype=xdt, requires_grad=True)
    w = (1 + 0.1 * torch.randn(D, device=DEV)).requires_grad_(True)
    y = rms_norm(x, w, 1e-6)
    g = torch.randn_like(y)
    (y * g).sum().backward()
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    yr = rms_norm_reference(xr, wr, 1e-6)
    (yr * g.float()).sum().backward()
    tol = 1e-2 if xdt == torch.bfloat16 else 1e-5
    assert rel(y, yr) < tol
    assert rel(x.grad, xr.grad) < max(tol, 1e-4)
    assert rel(w.grad, wr.grad) < 1e-3


def _ref_qk_rope(qkv, S, Hq, Hk, d, wq, wk, inv, eps, rot_dim=None):
    T = qkv.shape[0]
    rd = d if rot_dim is None else rot_dim
    q = qkv[:, :Hq * d].view(T, Hq, d)
    k = qkv[:, Hq * d:(Hq + Hk) * d].view(T, Hk, d)

    def nrm(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    q, k = nrm(q, wq), nrm(k, wk)
    pos = (torch.arange(T, device=qkv.device) % S).float()
    f = pos[:, None] * inv[None, : rd // 2]
    cos = torch.cat([f, f], -1).cos()[:, None]
    sin = torch.cat([f, f], -1).sin()[:, None]

    def rot(x):
        # rotate-half over the first rd channels (HF partial rotary), the rest pass through
        xr, xp = x[..., :rd], x[..., rd:]
        h = rd // 2
        xr = xr * cos + torch.cat([-xr[..., h:], xr[..., :h]], -1) * sin
        return torch.cat([xr, xp], -1)

    return rot(q), rot(k)


@pytest.mark.parametrize("d,rot_frac,Hq,Hk", [(64, 1, 4, 2), (128, 1, 4, 2), (128, 1, 16, 8),
                                               (128, 0.5, 4, 2), (256, 1, 3, 1), (128, 0, 2, 1)])
def test_qk_norm_rope_fwd_bwd(d, rot_frac, Hq, Hk):
    from pluggy_b200.ops.norm import qk_norm_rope_bwd, qk_norm_rope_fwd

    B, S = 2, 192
    T = B * S
    rd = int(d * rot_frac)
    W = (Hq + 2 * Hk) * d
    qkv = torch.randn(T, W, device=DEV).bfloat16()
    wq = 1 + 0.1 * torch.randn(d, device=DEV)
    wk = 1 + 0.1 * torch.randn(d, device=DEV)
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device=DEV).float() / d))
    q, k, rstd = qk_norm_rope_fwd(qkv, S=S, Hq=Hq, Hk=Hk, d=d, wq=wq, wk=wk, inv_freq=inv, eps=1e-6,
                                  rot_dim=rd)
    x = qkv.float().requires_grad_(True)
    wqr, wkr = wq.clone().requires_grad_(True), wk.clone().requires_grad_(True)
    qr, kr = _ref_qk_rope(x, S, Hq, Hk, d, wqr, wkr, inv, 1e-6, rot_dim=rd)
    assert rel(q, qr) < 1e-2 and rel(k, kr) < 1e-2
    gq, gk = torch.randn_like(qr), torch.randn_like(kr)
    ((qr * gq).sum() + (kr * gk).sum()).backward()
    dqkv = torch.zeros(T, W, device=DEV, dtype=torch.bfloat16)
    dwq, dwk = qk_norm_rope_bwd(qkv, rstd, gq.bfloat16(), gk.bfloat16(), dqkv, S=S, Hq=Hq, Hk=Hk,
                                d=d, wq=wq, wk=wk, inv_freq=inv, eps=1e-6, rot_dim=rd)
    assert rel(dqkv[:, :(Hq + Hk) * d], x.grad[:, :(Hq + Hk) * d]) < 2e-2
    assert rel(dwq, wqr.grad) < 2e-2 and rel(dwk, wkr.grad) < 2e-2


@pytest.mark.parametrize("norm", [True, False])
def test_qk_rope_positions_odd_tokens(norm):
    """Explicit positions, a token count that does not fill the last tile, and the
    no-norm (Llama) path of the TMA-fed kernels."""
    from pluggy_b200.ops.norm import qk_norm_rope_bwd, qk_norm_rope_fwd

    d, Hq, Hk, S, T = 128, 16, 8, 300, 257
    W = (Hq + 2 * Hk) * d
    qkv = torch.randn(T, W, device=DEV).bfloat16()
    wq = (1 + 0.1 * torch.randn(d, device=DEV)) if norm else None
    wk = (1 + 0.1 * torch.randn(d, device=DEV)) if norm else None
    inv = 1.0 / (1e6 ** (torch.arange(0, d, 2, device=DEV).float() / d))
    pos = torch.randint(0, S, (T,), device=DEV, dtype=torch.int32)
    q, k, rstd = qk_norm_rope_fwd(qkv, S=S, Hq=Hq, Hk=Hk, d=d, wq=wq, wk=wk, inv_freq=inv, eps=1e-6,
                                  positions=pos)
    x = qkv.float().requires_grad_(True)
    H = Hq + Hk
    xs = x[:, :H * d].view(T, H, d)
    if norm:
        w = torch.cat([wq.expand(Hq, d), wk.expand(Hk, d)], 0)
        xn = xs * torch.rsqrt(xs.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    else:
        xn = xs
    ang = pos.float()[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None, :]
    h = d // 2
    ref = xn * cos + torch.cat([-xn[..., h:], xn[..., :h]], -1) * sin
    assert rel(q, ref[:, :Hq]) < 1e-2 and rel(k, ref[:, Hq:]) < 1e-2
    g = torch.randn_like(ref)
    (ref * g).sum().backward()
    dqkv = torch.zeros(T, W, device=DEV, dtype=torch.bfloat16)
    qk_norm_rope_bwd(qkv, rstd, g[:, :Hq].bfloat16().contiguous(), g[:, Hq:].bfloat16().contiguous(),
                     dqkv, S=S, Hq=Hq, Hk=Hk, d=d, wq=wq, wk=wk, inv_freq=inv, eps=1e-6, positions=pos)
    assert rel(dqkv[:, :H * d], x.grad[:, :H * d]) < 2e-2


# ----------------------------------------------------------------- pointwise
@pytest.mark.parametrize("kind", [0, 1])
def test_glu_fwd_bwd(kind):
    from pluggy_b200.ops.elementwise import glu_bwd, glu_fwd

    gu = torch.randn(513, 2 * 384, device=DEV).bfloat16()
    g, u = gu.float()[:, :384].requires_grad_(True), gu.float()[:, 384:].requires_grad_(True)
    act = torch.nn.functional.silu(g) if kind == 0 else torch.nn.functional.gelu(g, approximate="tanh")
    ref = act * u
    out = glu_fwd(gu, kind)
    assert rel(out, ref) < 1e-2
    do = torch.randn_like(ref)
    (ref * do).sum().backward()
    dgu = glu_bwd(gu, do.bfloat16(), kind)
    assert rel(dgu[:, :384], g.grad) < 2e-2 and rel(dgu[:, 384:], u.grad) < 2e-2


def test_embedding_fwd_bwd():
    from pluggy_b200.models._engine import Embedding

    w = torch.randn(1000, 256, device=DEV, requires_grad=True)
    ids = torch.randint(0, 1000, (4, 64), device=DEV)
    out = Embedding.apply(ids, w, 1.5)
    assert torch.allclose(out, w.detach()[ids.view(-1)] * 1.5)
    g = torch.randn_like(out)
    out.backward(g)
    ref = torch.zeros_like(w).index_add_(0, ids.view(-1), g * 1.5)
    assert rel(w.grad, ref) < 1e-6


def test_embedding_bwd_deterministic_with_a_hot_id():
    """Zipf-like ids (one id on a third of the positions, runs longer than a CTA):
    the sorted backward matches index_add in fp64 and is bitwise identical on a rerun."""
    from pluggy_b200.models._engine import Embedding

    torch.manual_seed(3)
    V, D, T = 5000, 1024, 4096
    ids = torch.randint(0, V, (T,), device=DEV)
    ids[::3] = 7
    w = torch.randn(V, D, device=DEV, requires_grad=True)
    g = torch.randn(T, D, device=DEV)
    grads = []
    for _ in range(2):
        w.grad = None
        Embedding.apply(ids, w, 1.0).backward(g)
        grads.append(w.grad.clone())
    assert torch.equal(grads[0], grads[1])
    ref = torch.zeros(V, D, dtype=torch.float64, device=DEV).index_add_(0, ids, g.double())
    assert rel(grads[0], ref) < 1e-6


def test_kernels_rerun_bitwise():
    """Kernels whose summation order is fixed (no atomics on floats) give bitwise
    identical results on a second run: a race would show up as a difference."""
    from pluggy_b200.ops import optim
    from pluggy_b200.ops.attention import attn_fwd
    from pluggy_b200.ops.ce import fused_linear_cross_entropy
    from pluggy_b200.ops.gemm import linear_dgrad, linear_fwd
    from pluggy_b200.ops.norm import rmsnorm_bwd, rmsnorm_fwd

    torch.manual_seed(4)
    x = torch.randn(3000, 1024, device=DEV).bfloat16()
    w = (torch.randn(1536, 1024, device=DEV) * 0.05).bfloat16()
    dy = torch.randn(3000, 1536, device=DEV).bfloat16()
    q = torch.randn(2, 512, 4, 128, device=DEV).bfloat16()
    k = torch.randn(2, 512, 2, 128, device=DEV).bfloat16()
    v = torch.randn(2, 512, 2, 128, device=DEV).bfloat16()
    xf = torch.randn(3000, 1024, device=DEV)
    nw = torch.rand(1024, device=DEV) + 0.5
    dn = torch.randn(3000, 1024, device=DEV)
    h = (torch.randn(700, 256, device=DEV) * 0.5).bfloat16()
    wv = (torch.randn(3000, 256, device=DEV) * 0.05)
    lab = torch.randint(0, 3000, (700,), device=DEV)
    ts = [torch.randn(n, device=DEV) for n in (100, 70000, 65536 * 3)]

    def run():
        out = [linear_fwd(x, w), linear_dgrad(dy, w), attn_fwd(q, k, v)[0]]
        yb, r = rmsnorm_fwd(xf, nw, 1e-6)
        out += [yb, r]
        out += list(rmsnorm_bwd(dn, xf, nw, r))
        out.append(fused_linear_cross_entropy(h, wv, lab, -100, 256))
        out.append(optim.multi_tensor_sumsq(ts))
        return out

    a, b = run(), run()
    for i, (u, t) in enumerate(zip(a, b)):
        if isinstance(u, torch.Tensor):
            assert torch.equal(u, t), i


# ------------------------------------------------------------- fused lin-CE
@pytest.mark.parametrize("N,chunk", [(1000, 256), (2048, 2048), (333, 4096)])
def test_fused_linear_ce(N, chunk):
    from pluggy_b200.ops.ce import fused_linear_cross_entropy

    D, V = 256, 5000
    h = (torch.randn(N, D, device=DEV) * 0.5).bfloat16().requires_grad_(True)
    w = (torch.randn(V, D, device=DEV) * 0.05).requires_grad_(True)
    lab = torch.randint(0, V, (N,), device=DEV)
    lab[::7] = -100
    loss = fused_linear_cross_entropy(h, w, lab, -100, chunk)
    loss.backward()
    hr = h.detach().float().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    logits = hr.bfloat16().float() @ wr.bfloat16().float().t()
    lr = torch.nn.functional.cross_entropy(logits, lab, ignore_index=-100)
    lr.backward()
    assert abs(loss.item() - lr.item()) < 2e-2 * max(1.0, abs(lr.item()))
    assert rel(h.grad, hr.grad) < 3e-2
    assert rel(w.grad, wr.grad) < 3e-2


# ----------------------------------------------------------------- optimizer
def test_fused_adamw_matches_torch():
    from pluggy_b200.optimizer.fused_adamw import FusedAdamW

    torch.manual_seed(0)
    shapes = [(300, 17), (1024,), (7,), (65536 + 5,)]
    ps = [torch.randn(s, device=DEV, requires_grad=True) for s in shapes]
    qs = [p.detach().clone().requires_grad_(True) for p in ps]
    a = FusedAdamW([{"params": ps[:2], "weight_decay": 0.1}, {"params": ps[2:], "weight_decay": 0.0}],
                   lr=1e-2, betas=(0.9, 0.95), fused=True)
    b = torch.optim.AdamW([{"params": qs[:2], "weight_decay": 0.1}, {"params": qs[2:], "weight_decay": 0.0}],
                          lr=1e-2, betas=(0.9, 0.95))
    for _ in range(3):
        for p, q in zip(ps, qs):
            g = torch.randn_like(p)
            p.grad, q.grad = g.clone(), g.clone()
        a.step()
        b.step()
    for p, q in zip(ps, qs):
        assert rel(p, q) < 1e-6
    sd = a.state_dict()
    assert set(sd["state"][0]) == {"step", "exp_avg", "exp_avg_sq"}


def test_grad_clip_kernels():
    from pluggy_b200.core.grad_helper import clip_grad_norm

    ps = [torch.nn.Parameter(torch.randn(s, device=DEV)) for s in [(100, 30), (5,), (70000,)]]
    for p in ps:
        p.grad = torch.randn_like(p) * 3
    ref = torch.linalg.vector_norm(torch.stack([p.grad.norm() for p in ps]))
    grads0 = [p.grad.clone() for p in ps]
    total = clip_grad_norm(ps, None, 1.0)
    assert abs(total.item() - ref.item()) / ref.item() < 1e-5
    coef = 1.0 / (ref.item() + 1e-6)
    for p, g in zip(ps, grads0):
        assert rel(p.grad, g * coef) < 1e-5


# ----------------------------------------------------------------- attention
ATTN_CASES = [
    # B, S, Hq, Hk, d, causal, window
    (1, 128, 1, 1, 128, True, 0),
    (2, 256, 4, 2, 128, True, 0),
    (1, 384, 2, 2, 64, True, 0),
    (2, 200, 4, 1, 128, True, 0),
    (1, 512, 2, 1, 128, True, 160),
    (1, 256, 2, 2, 64, False, 0),
    (2, 1024, 16, 8, 128, True, 0),
    (2, 200, 4, 1, 64, True, 0),
    (1, 512, 4, 2, 64, True, 160),
    (1, 2048, 8, 2, 64, True, 0),
]


@pytest.mark.parametrize("B,S,Hq,Hk,d,causal,window", ATTN_CASES)
def test_attention_fwd_bwd(B, S, Hq, Hk, d, causal, window):
    from pluggy_b200.ops.attention import attention_reference, flash_attention

    torch.manual_seed(S + d)
    q = torch.randn(B, S, Hq, d, device=DEV).bfloat16().requires_grad_(True)
    k = torch.randn(B, S, Hk, d, device=DEV).bfloat16().requires_grad_(True)
    v = torch.randn(B, S, Hk, d, device=DEV).bfloat16().requires_grad_(True)
    o = flash_attention(q, k, v, causal, window)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    orf = attention_reference(qr, kr, vr, causal, window)
    assert rel(o, orf) < 2e-2, rel(o, orf)
    do = torch.randn_like(orf)
    o.backward(do.bfloat16())
    orf.backward(do)
    assert rel(q.grad, qr.grad) < 3e-2, rel(q.grad, qr.grad)
    assert rel(k.grad, kr.grad) < 3e-2, rel(k.grad, kr.grad)
    assert rel(v.grad, vr.grad) < 3e-2, rel(v.grad, vr.grad)


def test_exp2_poly_error_bound():
    """The FMA-pipe 2^x (a cubic on [-1/2, 1/2] after range reduction) that the attention
    forward uses for part of its softmax stays within 2e-4 relative error of CUDA's exp2f
    over the softmax argument range [-126, 0] (measured maximum 1.44e-4), ten times below
    the 2^-9 rounding of the bf16 P it feeds."""
    from pluggy_b200.ops._ext import ext

    x = torch.cat([torch.linspace(-126.0, 0.0, 1 << 20, device=DEV),
                   torch.rand(1 << 20, device=DEV) * -20.0,
                   torch.arange(-126, 1, device=DEV, dtype=torch.float32)])
    poly, ref = torch.empty_like(x), torch.empty_like(x)
    ext().exp2_poly_eval(x, poly, ref)
    rel = ((poly - ref).abs() / ref).max().item()
    assert rel < 2e-4, rel
    # integers (f = 0 after range reduction): off by the cubic's constant term only
    assert ((poly[-127:] - ref[-127:]).abs() / ref[-127:]).max().item() < 2e-4


@pytest.mark.parametrize("causal", [True])
def test_attention_benchmark_shape_against_fp32(causal):
    """The benchmark's attention shape (S = 4096, 16 q / 8 kv heads, d = 128), B = 2:
    forward output and all three gradients against fp32 math computed head by head."""
    from pluggy_b200.ops.attention import flash_attention

    torch.manual_seed(5)
    B, S, Hq, Hk, d = 2, 4096, 16, 8, 128
    q = torch.randn(B, S, Hq, d, device=DEV).bfloat16().requires_grad_()
    k = torch.randn(B, S, Hk, d, device=DEV).bfloat16().requires_grad_()
    v = torch.randn(B, S, Hk, d, device=DEV).bfloat16().requires_grad_()
    o = flash_attention(q, k, v, causal=causal)
    do = torch.randn_like(o)
    o.backward(do)
    scale = 1.0 / math.sqrt(d)
    mask = torch.ones(S, S, device=DEV, dtype=torch.bool).tril()
    errs = {"o": [0.0, 0.0], "dq": [0.0, 0.0], "dk": [0.0, 0.0], "dv": [0.0, 0.0]}
    dk_ref = torch.zeros(B, S, Hk, d, device=DEV)
    dv_ref = torch.zeros(B, S, Hk, d, device=DEV)
    for b in range(B):
        for h in range(Hq):
            hk = h // (Hq // Hk)
            qf = q[b, :, h].detach().float().requires_grad_()
            kf = k[b, :, hk].detach().float().requires_grad_()
            vf = v[b, :, hk].detach().float().requires_grad_()
            s_ = (qf @ kf.t()) * scale
            p_ = torch.softmax(s_.masked_fill(~mask, float("-inf")), -1)
            of = p_ @ vf
            of.backward(do[b, :, h].float())
            for name, got, want in (("o", o[b, :, h].float(), of.detach()), ("dq", q.grad[b, :, h].float(), qf.grad)):
                errs[name][0] += (got - want).pow(2).sum().item()
                errs[name][1] += want.pow(2).sum().item()
            dk_ref[b, :, hk] += kf.grad
            dv_ref[b, :, hk] += vf.grad
    for name, got, want in (("dk", k.grad.float(), dk_ref), ("dv", v.grad.float(), dv_ref)):
        errs[name] = [(got - want).pow(2).sum().item(), want.pow(2).sum().item()]
    for name, (num, den) in errs.items():
        assert math.sqrt(num / den) < 2e-2, (name, math.sqrt(num / den))


def test_attention_lse():
    from pluggy_b200.ops.attention import attn_fwd

    B, S, H, d = 1, 256, 2, 128
    q = torch.randn(B, S, H, d, device=DEV).bfloat16()
    k = torch.randn(B, S, H, d, device=DEV).bfloat16()
    v = torch.randn(B, S, H, d, device=DEV).bfloat16()
    _, lse = attn_fwd(q, k, v, causal=True)
    s = (q.float().transpose(1, 2) @ k.float().transpose(1, 2).transpose(-1, -2)) / math.sqrt(d)
    mask = torch.ones(S, S, device=DEV, dtype=torch.bool).tril()
    ref = s.masked_fill(~mask, float("-inf")).logsumexp(-1)
    assert (lse - ref).abs().max().item() < 2e-2


# ------------------------------------------------------------- model, fused
@pytest.mark.parametrize("family", ["qwen3", "llama3"])
def test_fused_model_matches_eager(family):
    from pluggy_b200.models.builder import build_model
    from pluggy_b200.objectives.autoregressive import ARObjective

    torch.manual_seed(0)
    cfg = dict(num_layers=2, num_heads=4, num_kv_heads=2, emb_dim=256, head_dim=64 if family == "llama3"
               else 128, vocab_size=2048, ffn_dim=512)
    name = "qwen3_dense" if family == "qwen3" else "llama3_2"
    m = build_model(name, cfg).to(DEV)
    m.init_weights()
    # the fused path runs q/k norms in bf16 (eps = bf16 eps, as the reference under autocast);
    # give the fp32 oracle the same eps so both compute the same function
    for mod in m.modules():
        if isinstance(mod, torch.nn.RMSNorm) and mod.normalized_shape[0] == cfg["head_dim"]:
            mod.eps = torch.finfo(torch.bfloat16).eps
    ids = torch.randint(0, 2048, (2, 256), device=DEV)
    batch = {"input_ids": ids, "labels": ids}
    obj = ARObjective(ce_chunk_size=128)
    loss = obj.compute_loss(m, batch)
    loss.backward()
    grads = {n: p.grad.detach().clone() for n, p in m.named_parameters()}
    m.zero_grad()
    # eager fp32 reference path: same weights, CPU math
    mc = build_model(name, cfg)
    mc.load_state_dict({k: v.cpu() for k, v in m.state_dict().items()})
    for mod in mc.modules():
        if isinstance(mod, torch.nn.RMSNorm) and mod.normalized_shape[0] == cfg["head_dim"]:
            mod.eps = torch.finfo(torch.bfloat16).eps
    lc = obj.compute_loss(mc, {k: v.cpu() for k, v in batch.items()})
    lc.backward()
    assert abs(loss.item() - lc.item()) < 2e-2 * lc.item()
    for n, p in mc.named_parameters():
        r = rel(grads[n].cpu(), p.grad)
        assert r < 6e-2, (n, r)


# --------------------------------------------------------------- grouped GEMM (MoE)
def test_grouped_gemm_modes_match_fp32():
    """Mode 1 (a group per 128-row tile, skipped tiles) and mode 2 (a k range per
    group, empty groups write zeros) against per-group fp32 matmuls."""
    from pluggy_b200.ops._ext import ext
    from pluggy_b200.ops.grouped import expert_layout

    torch.manual_seed(0)
    E, K, N = 6, 192, 320
    counts = torch.tensor([130, 0, 5, 256, 1, 77], device=DEV)
    P = int(counts.sum())
    poff, shift, tg, R = expert_layout(counts, P)
    ex = torch.repeat_interleave(torch.arange(E, device=DEV), counts)
    dst = torch.arange(P, device=DEV) + shift[ex]
    x = torch.randn(P, K, device=DEV).bfloat16()
    x_pad = torch.zeros(R, K, dtype=torch.bfloat16, device=DEV)
    x_pad[dst] = x
    w = (torch.randn(E, N, K, device=DEV) * 0.05).bfloat16()
    # mode 1, K-major B (forward)
    y = torch.empty(R, N, dtype=torch.bfloat16, device=DEV)
    ext().gemm_grouped(x_pad, w.view(E * N, K), False, y, 1, tg, E, N, 1.0, 0.0)
    ref = torch.einsum("pk,pnk->pn", x.float(), w.float()[ex])
    assert rel(y[dst].float(), ref) < 1e-2
    # mode 1, MN-major B (input gradient): dx = dy W_e
    dy = torch.randn(P, N, device=DEV).bfloat16()
    dy_pad = torch.zeros(R, N, dtype=torch.bfloat16, device=DEV)
    dy_pad[dst] = dy
    wt = (torch.randn(E, N, K, device=DEV) * 0.05).bfloat16()  # [E, rows=N(k dim), K(out)]
    dx = torch.empty(R, K, dtype=torch.bfloat16, device=DEV)
    ext().gemm_grouped(dy_pad, wt.view(E * N, K), True, dx, 1, tg, E, N, 1.0, 0.0)
    ref = torch.einsum("pn,pnk->pk", dy.float(), wt.float()[ex])
    assert rel(dx[dst].float(), ref) < 1e-2
    # mode 2 (weight gradient): dW_e = dy_e^T x_e, fp32, empty expert -> 0
    dw = torch.full((E * N, K), float("nan"), device=DEV)
    ext().gemm_grouped(dy_pad, x_pad, True, dw, 2, poff, E, 0, 1.0, 0.0)
    dw = dw.view(E, N, K)
    off = 0
    for e, n in enumerate(counts.tolist()):
        want = dy[off:off + n].float().t() @ x[off:off + n].float()
        if n == 0:
            assert torch.count_nonzero(dw[e]) == 0
        else:
            assert rel(dw[e], want) < 1e-2, e
        off += n
    # mode 2 accumulating into C (beta = 1)
    base = torch.randn(E * N, K, device=DEV)
    acc = base.clone()
    ext().gemm_grouped(dy_pad, x_pad, True, acc, 2, poff, E, 0, 1.0, 1.0)
    assert rel(acc.view(E, N, K) - base.view(E, N, K), dw) < 1e-4


def test_grouped_swiglu_ffn_matches_loop():
    """The one-launch-per-projection grouped FFN against the per-expert loop (fp32
    CPU math), forward and every gradient; includes an expert with no rows."""
    from pluggy_b200.ops.moe import moe_expert_ffn

    torch.manual_seed(1)
    T, H, I, E, k = 200, 256, 128, 8, 2
    h = torch.randn(T, H, device=DEV)
    logits = torch.randn(T, E, device=DEV)
    logits[:, 3] = -1e9  # expert 3 gets nothing
    w, idx = torch.topk(torch.softmax(logits, -1), k, dim=-1)
    gu = (torch.randn(E, 2 * I, H, device=DEV) * 0.05).requires_grad_()
    dn = (torch.randn(E, H, I, device=DEV) * 0.05).requires_grad_()
    hx = h.clone().requires_grad_()
    y = moe_expert_ffn(hx, idx, w, gu, dn)
    gy = torch.randn_like(y)
    (y * gy).sum().backward()
    gc = gu.detach().cpu().requires_grad_()
    dc = dn.detach().cpu().requires_grad_()
    hc = h.cpu().requires_grad_()
    yc = moe_expert_ffn(hc, idx.cpu(), w.cpu(), gc, dc, use_grouped_mm=False)
    (yc * gy.cpu()).sum().backward()
    assert rel(y.cpu(), yc) < 2e-2
    assert rel(hx.grad.cpu(), hc.grad) < 3e-2
    assert rel(gu.grad.cpu(), gc.grad) < 3e-2
    assert rel(dn.grad.cpu(), dc.grad) < 3e-2
    assert torch.count_nonzero(gu.grad[3]) == 0 and torch.count_nonzero(dn.grad[3]) == 0


def test_colsum_matches_torch():
    from pluggy_b200.ops.norm import _colsum

    part = torch.randn(592, 1000, device=DEV)
    assert torch.allclose(_colsum(part), part.sum(0), rtol=1e-5, atol=1e-4)


def test_weight_cache_optimizer_shadows():
    """After optimizer steps, the bf16 copies the GEMMs read equal a fresh cast of
    the fp32 masters although the cache never recast them."""
    from pluggy_b200.ops.linear import WeightCache
    from pluggy_b200.optimizer.fused_adamw import FusedAdamW

    torch.manual_seed(0)
    w1 = torch.nn.Parameter(torch.randn(256, 128, device=DEV))
    w2 = torch.nn.Parameter(torch.randn(64, 128, device=DEV))
    w3 = torch.nn.Parameter(torch.randn(64, 128, device=DEV))
    opt = FusedAdamW([w1, w2, w3], lr=1e-2)
    wc = WeightCache()
    wc.bind_optimizer(opt)
    for _ in range(3):
        a = wc.get(w1)
        cat = wc.get_cat([w2, w3], "w23")
        ref_a, ref_cat = a.clone(), cat.clone()
        loss = (a.float() * w1).sum() + (cat.float() * torch.cat([w2, w3])).sum()
        loss.backward()
        opt.step()
        opt.zero_grad()
        a2 = wc.get(w1)
        cat2 = wc.get_cat([w2, w3], "w23")
        assert a2.data_ptr() == a.data_ptr() and cat2.data_ptr() == cat.data_ptr()
        assert torch.equal(a2, w1.detach().bfloat16())
        assert torch.equal(cat2, torch.cat([w2, w3]).detach().bfloat16())
        assert not torch.equal(a2, ref_a) and not torch.equal(cat2, ref_cat)


def test_peer_store_bounds_are_enforced():
    """A push whose destination offset lies past the buffer is skipped and reported
    (status 8) instead of writing outside the buffer; in-range rows still land."""
    from pluggy_b200.ops import _ext

    st = _ext.status_word()
    st.zero_()
    buf = torch.zeros(64 + 16, 8, dtype=torch.int16, device=DEV)  # 64 rows + a guard band
    flags = torch.zeros(32, dtype=torch.int32, device=DEV)
    src = torch.arange(4 * 8, dtype=torch.int16, device=DEV).view(4, 8)
    cap = 64 * 16  # bytes the kernel may write: the guard band must stay zero
    _ext.ext().ep_exchange("push", src, [flags.data_ptr()], [buf.data_ptr()], 0, 1, 1, [0], [4], [62],
                           0, cap, st)
    torch.cuda.synchronize()
    assert int(st.item()) == 8
    assert torch.equal(buf[62:64], src[:2]) and int(buf[64:].abs().sum()) == 0
    st.zero_()
    _ext.ext().ep_exchange("push", src, [flags.data_ptr()], [buf.data_ptr()], 0, 2, 1, [0], [4], [10],
                           0, cap, st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0 and torch.equal(buf[10:14], src)


def test_peer_wait_times_out_with_status():
    """A collective kernel whose peer never posts its flag gives up after the
    deadline, records status 5 (timed out waiting for a peer) and returns: the
    context stays usable and check_status raises and resets the word. One GPU
    plays rank 0 of two; "rank 1" is a zeroed flag table nobody writes."""
    import time

    from pluggy_b200.ops import _ext

    st = _ext.status_word()
    st.zero_()
    flags = [torch.zeros(4096, dtype=torch.int32, device=DEV) for _ in range(2)]
    bufs = [torch.zeros(64, 8, dtype=torch.int16, device=DEV) for _ in range(2)]
    out = torch.zeros(4, 8, dtype=torch.int16, device=DEV)
    _ext.set_peer_wait_deadline(1e-3)
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _ext.ext().ep_exchange("finish", out, [f.data_ptr() for f in flags],
                               [b.data_ptr() for b in bufs], 0, 1, 0, [0, 0], [0, 0], [0, 0], 4,
                               64 * 16, st)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
    finally:
        _ext.set_peer_wait_deadline(_ext.DEFAULT_PEER_WAIT_S)
    assert int(st.item()) == 5
    assert waited < 1.0  # the 1 ms deadline, not the 2 s default
    with pytest.raises(RuntimeError, match="status 5"):
        _ext.check_status()
    assert int(st.item()) == 0
    # the device still runs work after the timed-out kernel
    x = torch.ones(1024, device=DEV)
    assert float((x * 2).sum()) == 2048.0
    # rank 0's own flag was posted (signal before wait); the missing peer's was not
    assert int(flags[0][0]) == 1 and int(flags[0][1]) == 0


@pytest.mark.parametrize("B,H,S,d,bcast,transposed", [
    (2, 4, 96, 128, True, True), (1, 3, 50, 64, False, False), (2, 2, 33, 256, False, True)])
def test_rope_kernel_fwd_bwd(B, H, S, d, bcast, transposed):
    """The RoPE kernel against fp32 eager math, on transposed [B, S, H, d] views and on
    contiguous [B, H, S, d], with a batch-broadcast or per-batch cos/sin table."""
    from pluggy_b200.ops.elementwise import _rope_kernel_ok, apply_rotary, rotate_half

    torch.manual_seed(d + S)
    pos = torch.arange(S, device=DEV).float()[None].expand(1 if bcast else B, S)
    inv = 1.0 / (10000.0 ** (torch.arange(0, d, 2, device=DEV).float() / d))
    f = pos[:, :, None] * inv
    emb = torch.cat([f, f], -1)
    cos, sin = emb.cos()[:, None], emb.sin()[:, None]
    if transposed:
        x = torch.randn(B, S, H, d, device=DEV).bfloat16().transpose(1, 2)
    else:
        x = torch.randn(B, H, S, d, device=DEV).bfloat16()
    x.requires_grad_(True)
    assert _rope_kernel_ok(x, cos, sin)
    y = apply_rotary(x, cos, sin)
    assert y.stride() == x.stride()  # the input's layout: a transposed view needs no copy
    xf = x.detach().float().requires_grad_(True)
    yf = xf * cos + rotate_half(xf) * sin
    assert rel(y, yf) < 1e-2, rel(y, yf)
    g = torch.randn_like(yf)
    y.backward(g.bfloat16())
    yf.backward(g)
    assert rel(x.grad, xf.grad) < 1e-2, rel(x.grad, xf.grad)


@pytest.mark.parametrize("name,cfg", [
    ("olmo3", dict(num_layers=4, num_heads=4, num_kv_heads=2, emb_dim=256, head_dim=64,
                   vocab_size=2048, ffn_dim=512, sliding_window=64)),
    ("gemma4", dict(num_layers=3, num_heads=4, num_kv_heads=2, emb_dim=256, head_dim=64,
                    global_head_dim=128, vocab_size=2048, ffn_dim=512, sliding_window=64,
                    layer_pattern=3)),
])
def test_composed_model_families_match_fp32(name, cfg):
    """OLMo-3 and Gemma-4 on CUDA (this package's GEMMs, norms, RoPE, GLU, attention and
    fused CE) against the same weights in fp32 on the CPU. Gemma's attention has scale
    1 on per-head-normalised q and k: at the init norm weights (1) the logits have a std
    of ~sqrt(head_dim) and the softmax is so peaked that rounding the weights to bf16
    alone moves the fp32 gradients by ~40 %; the q/k-norm weights are set to 0.3 here
    (1.6 % on the same check), so the comparison measures the kernels, not that."""
    from pluggy_b200.models.builder import build_model
    from pluggy_b200.objectives.autoregressive import ARObjective

    torch.manual_seed(0)
    m = build_model(name, cfg).to(DEV)
    m.init_weights()
    if name == "gemma4":
        with torch.no_grad():
            for b in m.blocks:
                for nm in (b.attn.q_norm, b.attn.k_norm):
                    if nm is not None:
                        nm.weight.fill_(0.3)
    ids = torch.randint(0, 2048, (2, 256), device=DEV)
    batch = {"input_ids": ids, "labels": ids}
    obj = ARObjective(ce_chunk_size=128)
    loss = obj.compute_loss(m, batch)
    loss.backward()
    grads = {n: p.grad.detach().clone() for n, p in m.named_parameters() if p.grad is not None}
    mc = build_model(name, cfg)
    mc.load_state_dict({k: v.cpu() for k, v in m.state_dict().items()})
    lc = obj.compute_loss(mc, {k: v.cpu() for k, v in batch.items()})
    lc.backward()
    assert abs(loss.item() - lc.item()) < 2e-2 * lc.item(), (loss.item(), lc.item())
    for n, p in mc.named_parameters():
        if p.grad is not None and p.grad.abs().max() > 0:
            r = rel(grads[n].cpu(), p.grad)
            assert r < 8e-2, (n, r)


@pytest.mark.parametrize("E,k,renorm,dtype", [(128, 8, True, torch.bfloat16), (64, 4, False, torch.float32),
                                               (512, 2, True, torch.float32)])
def test_router_topk_kernel(E, k, renorm, dtype):
    """The fused router (softmax, top-k, renormalisation, histogram) against the eager
    softmax/topk path, forward and backward."""
    from pluggy_b200.models.qwen3_moe import _RouterTopK
    from pluggy_b200.ops._ext import ext

    torch.manual_seed(E + k)
    T = 1000
    logits = torch.randn(T, E, device=DEV).to(dtype).requires_grad_(True)
    w, idx = _RouterTopK.apply(logits, k, renorm)
    lf = logits.detach().float().requires_grad_(True)
    p = torch.softmax(lf, -1)
    pw, pidx = torch.topk(p, k, dim=-1)
    if renorm:
        pw = pw / pw.sum(-1, keepdim=True)
    assert torch.equal(idx.sort(-1).values, pidx.sort(-1).values)
    assert rel(w.gather(1, idx.argsort(-1)), pw.gather(1, pidx.argsort(-1))) < 1e-5
    # the same upstream gradient per (token, expert) for both selections
    G = torch.randn(T, E, device=DEV)
    (w * G.gather(1, idx)).sum().backward()
    (pw * G.gather(1, pidx)).sum().backward()
    assert rel(logits.grad.float(), lf.grad) < 2e-2
    counts = torch.zeros(E, dtype=torch.int32, device=DEV)
    ww = torch.empty(T, k, device=DEV)
    ii = torch.empty(T, k, dtype=torch.int64, device=DEV)
    ext().router_topk(logits.detach().contiguous(), k, renorm, None, ww, ii, counts)
    assert torch.equal(counts.long(), torch.bincount(ii.view(-1), minlength=E))
