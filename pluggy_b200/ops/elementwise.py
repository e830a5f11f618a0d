"""GLU activations, logit softcap and rotary helpers.

Parity: ``pluggy/kernels/swiglu.py:14-21`` (``swiglu_mul``, ``geglu_mul``),
``pluggy/kernels/softcap.py:13-33`` (``logit_softcap``: cap*tanh(x/cap), analytic
backward), ``pluggy/kernels/rope.py:12-24`` (``apply_rotary``, ``rotate_half``).

On CUDA the GLU forward/backward run in this package's sm_100a kernels over a
packed ``[T, 2F]`` gate|up tensor (what the fused gate/up GEMM produces).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from pluggy_b200.ops._ext import ext

SILU, GELU_TANH = 0, 1


def glu_fwd(gu: torch.Tensor, kind: int = SILU) -> torch.Tensor:
    """``act(gu[..., :F]) * gu[..., F:]`` for a packed gate|up tensor."""
    F2 = gu.shape[-1]
    out = torch.empty((*gu.shape[:-1], F2 // 2), dtype=torch.bfloat16, device=gu.device)
    ext().glu_fwd(gu, out, int(kind))
    return out


def glu_bwd(gu: torch.Tensor, dout: torch.Tensor, kind: int = SILU, out=None) -> torch.Tensor:
    dgu = torch.empty_like(gu) if out is None else out
    ext().glu_bwd(gu, dout.contiguous(), dgu, int(kind))
    return dgu


class _PackedGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate, up, kind):
        gu = torch.cat([gate, up], dim=-1).to(torch.bfloat16).contiguous()
        ctx.save_for_backward(gu)
        ctx.kind = kind
        ctx.dtype = gate.dtype
        return glu_fwd(gu, kind).to(gate.dtype)

    @staticmethod
    def backward(ctx, dout):
        (gu,) = ctx.saved_tensors
        dgu = glu_bwd(gu, dout.to(torch.bfloat16), ctx.kind)
        Fh = gu.shape[-1] // 2
        return dgu[..., :Fh].to(ctx.dtype), dgu[..., Fh:].to(ctx.dtype), None


def swiglu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up."""
    if gate.is_cuda and gate.dtype == torch.bfloat16 and gate.shape[-1] % 2 == 0:
        return _PackedGLU.apply(gate, up, SILU)
    return F.silu(gate) * up


def geglu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """gelu_tanh(gate) * up (Gemma)."""
    if gate.is_cuda and gate.dtype == torch.bfloat16 and gate.shape[-1] % 2 == 0:
        return _PackedGLU.apply(gate, up, GELU_TANH)
    return F.gelu(gate, approximate="tanh") * up


class _LogitSoftcap(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cap):
        t = torch.tanh(x / cap)
        ctx.cap = cap
        ctx.save_for_backward(t)
        return t * cap

    @staticmethod
    def backward(ctx, g):
        (t,) = ctx.saved_tensors
        return g * (1.0 - t * t), None


def logit_softcap(x: torch.Tensor, cap: float | None) -> torch.Tensor:
    """No-op for ``cap`` None or <= 0."""
    if cap is None or cap <= 0:
        return x
    return _LogitSoftcap.apply(x, float(cap))


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class _Rope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin):
        from pluggy_b200.ops._ext import ext

        y = torch.empty_like(x)  # x's layout (a dense transposed view stays transposed)
        ext().rope_apply(x, cos, sin, y, False)
        ctx.save_for_backward(cos, sin)
        return y

    @staticmethod
    def backward(ctx, dy):
        from pluggy_b200.ops._ext import ext

        cos, sin = ctx.saved_tensors
        dy = dy.contiguous() if (dy.stride(-1) != 1 or any(s % 4 for s in dy.stride()[:3])
                                 or dy.data_ptr() % 8) else dy
        dx = torch.empty_like(dy)
        if dx.stride(-1) != 1:
            dx = torch.empty(dy.shape, dtype=dy.dtype, device=dy.device)
        ext().rope_apply(dy, cos, sin, dx, True)
        return dx, None, None


def _rope_kernel_ok(x, cos, sin) -> bool:
    if not (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 4 and x.stride(-1) == 1):
        return False
    B, _, S, d = x.shape
    if d % 8 or any(st % 4 for st in x.stride()[:3]) or x.data_ptr() % 8:
        return False
    if cos.dim() != 4 or cos.dtype != torch.float32 or sin.shape != cos.shape:
        return False
    if cos.shape[1] != 1 or cos.shape[2] != S or cos.shape[3] != d or cos.shape[0] not in (1, B):
        return False
    return (cos.stride() == sin.stride() and cos.stride(-1) == 1 and cos.stride(2) % 4 == 0
            and (cos.shape[0] == 1 or cos.stride(0) % 4 == 0)
            and cos.data_ptr() % 16 == 0 and sin.data_ptr() % 16 == 0)


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x*cos + rotate_half(x)*sin`` with cos/sin broadcast against x (reference layout
    ``[B, H, S, d]``, ``pluggy/kernels/rope.py:12-24``). bf16 CUDA tensors with fp32
    ``[B|1, 1, S, d]`` tables run the sm_100a kernel (fp32 math, any B/H/S strides, so
    transposed views of a projection need no copy); everything else is eager torch with
    the reference's casts."""
    if _rope_kernel_ok(x, cos, sin):
        return _Rope.apply(x, cos.detach(), sin.detach())
    cos = cos.to(x.dtype)
    sin = sin.to(x.dtype)
    return x * cos + rotate_half(x) * sin
