"""bf16 GEMMs on the sm_100a tensor cores (tcgen05 + TMEM + TMA).

One kernel covers the three products of a linear layer ``y = x W^T``:

* ``linear_fwd(x, w)``        y  = x  W^T  (A K-major, B K-major)
* ``linear_dgrad(dy, w)``     dx = dy W    (A K-major, B N-major)
* ``linear_wgrad(dy, x)``     dW = dy^T x  (A M-major, B N-major), fp32 out,
                              split-K with fp32 atomics when the output is small

with an optional addend ``beta * D`` (residual adds, grad accumulation) fused
into the epilogue. CPU tensors take the equivalent ``torch.matmul`` (oracle).
"""

from __future__ import annotations

import torch

from pluggy_b200.ops._ext import ext, status_word


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn_major: bool = False, b_mn_major: bool = False,
         out: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
         addend: torch.Tensor | None = None, alpha: float = 1.0, beta: float = 1.0,
         splits: int = 0, bn: int = 0) -> torch.Tensor:
    """``C = alpha * A' B'^T + beta * addend`` with A' = a (or a^T), B' = b (or b^T).

    ``a`` is [M, K] (``a_mn_major=False``) or [K, M]; ``b`` is [N, K] or [K, N].
    """
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError(f"gemm takes 2-D operands, got {tuple(a.shape)} and {tuple(b.shape)}")
    M = a.shape[1] if a_mn_major else a.shape[0]
    Ka = a.shape[0] if a_mn_major else a.shape[1]
    N = b.shape[1] if b_mn_major else b.shape[0]
    Kb = b.shape[0] if b_mn_major else b.shape[1]
    if Ka != Kb:
        raise ValueError(f"gemm: reduction dims differ ({Ka} vs {Kb}) for a{tuple(a.shape)} "
                         f"(mn_major={a_mn_major}) and b{tuple(b.shape)} (mn_major={b_mn_major})")
    if out is not None and tuple(out.shape) != (M, N):
        raise ValueError(f"gemm: out must be [{M}, {N}], got {tuple(out.shape)}")
    if not a.is_cuda:
        A = (a.t() if a_mn_major else a).float()
        B = (b.t() if b_mn_major else b).float()
        r = alpha * (A @ B.t())
        if addend is not None:
            r = r + beta * addend.float()
        if out is None:
            return r.to(out_dtype)
        out.copy_(r)
        return out
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    ext().gemm(a, a_mn_major, b, b_mn_major, out, addend, float(alpha),
               float(beta) if addend is not None else 0.0, int(splits), int(bn),
               status_word(a.device))
    return out


def linear_fwd(x: torch.Tensor, w: torch.Tensor, *, out=None, out_dtype=torch.bfloat16,
               residual: torch.Tensor | None = None) -> torch.Tensor:
    """``x [T,K] @ w[N,K]^T (+ residual)``."""
    return gemm(x, w, out=out, out_dtype=out_dtype, addend=residual, beta=1.0)


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, *, out=None, out_dtype=torch.bfloat16,
                 addend: torch.Tensor | None = None) -> torch.Tensor:
    """``dy [T,N] @ w [N,K]`` -> [T,K]."""
    return gemm(dy, w, b_mn_major=True, out=out, out_dtype=out_dtype, addend=addend, beta=1.0)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, *, out=None, accumulate: bool = False,
                 scale: float = 1.0) -> torch.Tensor:
    """``dy[T,N]^T @ x[T,K]`` -> fp32 [N,K]; ``accumulate`` adds into ``out``."""
    if accumulate:
        assert out is not None
        return gemm(dy, x, a_mn_major=True, b_mn_major=True, out=out, addend=out, alpha=scale,
                    beta=1.0)
    return gemm(dy, x, a_mn_major=True, b_mn_major=True, out=out, out_dtype=torch.float32,
                alpha=scale)
