"""Tensor-parallel collectives over NVLink peer memory, and the fused
GEMM -> reduce-scatter of the row-parallel linears.

Sequence parallelism moves activations between "each rank holds ``S / n`` of every
sequence" and "every rank holds all of it". Here both directions run on this
package's kernels (``csrc/comm.cu``, ``csrc/gemm_tcgen05.cu``) instead of NCCL:

* reduce-scatter: each rank stores its partial rows straight into the owning
  rank's staging slot with peer stores, then a finishing kernel signals the
  peers, waits (bounded) for theirs and sums the slots in a fixed order;
* fused GEMM -> reduce-scatter (row-parallel ``o_proj`` / ``down_proj``): the
  tcgen05 GEMM's epilogue writes each output row directly into its owner's
  staging slot over NVLink, so the transfer overlaps the GEMM tile by tile and
  the partial product never lands in local memory;
* all-gather: each rank pushes its shard into its slot of every rank's receive
  buffer with peer stores (posted writes beat round-trip loads over NVLink),
  signals, and copies the slots of its own receive buffer into sequence order.

Staging and receive buffers are double-buffered by call parity; a rank cannot start
call ``e + 2`` of a kind before every peer has signalled call ``e + 1``, which each
peer does only after it finished reading call ``e``'s buffer, so two halves
suffice. Flags hold monotonically growing epochs (no reset between calls).
The buffers grow on demand (a collective step: every rank makes the same calls).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from pluggy_b200.comm.symm import SymmetricBuffer
from pluggy_b200.ops._ext import ext, status_word

_RS, _AG = 0, 1
_FLAG_BYTES = 4 * 8 * 4  # kinds x ranks x uint32


class TPComm:
    def __init__(self, mesh, dim: str, capacity_bytes: int = 32 << 20):
        self.mesh, self.dim = mesh, dim
        self.n, self.rank = mesh.size(dim), mesh.coordinate(dim)
        self.flags = SymmetricBuffer(_FLAG_BYTES, mesh, dim)
        self.cap = {_RS: 0, _AG: 0}
        self.buf = {_RS: None, _AG: None}
        self.epoch = {_RS: 0, _AG: 0}
        self._grow(_RS, capacity_bytes)
        self._grow(_AG, capacity_bytes)

    def _grow(self, kind: int, half_bytes: int) -> None:
        half = (int(half_bytes) + 4095) // 4096 * 4096
        if half <= self.cap[kind]:
            return
        old = self.buf[kind]
        if old is not None:
            # peers may still read or write the old buffer: quiesce the axis first
            torch.cuda.synchronize()
            dist.barrier(group=self.mesh.get_group(self.dim))
            old.close()
        self.buf[kind] = SymmetricBuffer(2 * half, self.mesh, self.dim)
        self.cap[kind] = half

    def _args(self, kind: int, need: int):
        self._grow(kind, need)
        self.epoch[kind] += 1
        e = self.epoch[kind]
        off = (e % 2) * self.cap[kind]
        bufs = [p + off for p in self.buf[kind].peers]
        return self.flags.peers, bufs, e, self.cap[kind]

    # ------------------------------------------------------------ collectives
    def reduce_scatter_seq(self, partial: torch.Tensor) -> torch.Tensor:
        """[B, S, W] partial sums (bf16) -> this rank's summed [B, S / n, W]."""
        B, S, W = partial.shape
        p2 = partial.reshape(B * S, W).to(torch.bfloat16).contiguous()
        flags, bufs, e, cap = self._args(_RS, p2.numel() * 2)
        out = torch.empty((B * (S // self.n), W), dtype=torch.bfloat16, device=partial.device)
        st = status_word(partial.device)
        ext().tp_collective("rs_push", p2, flags, bufs, self.rank, e, B, S, cap, st)
        ext().tp_collective("rs_finish", out, flags, bufs, self.rank, e, B, S, cap, st)
        return out.view(B, S // self.n, W)

    def all_gather_seq(self, shard: torch.Tensor) -> torch.Tensor:
        """[B, S / n, W] (bf16) -> [B, S, W] on every rank."""
        B, s, W = shard.shape
        S = s * self.n
        x2 = shard.reshape(B * s, W).to(torch.bfloat16).contiguous()
        flags, bufs, e, cap = self._args(_AG, x2.numel() * 2 * self.n)
        out = torch.empty((B * S, W), dtype=torch.bfloat16, device=shard.device)
        st = status_word(shard.device)
        ext().tp_collective("ag_push", x2, flags, bufs, self.rank, e, B, S, cap, st)
        ext().tp_collective("ag_finish", out, flags, bufs, self.rank, e, B, S, cap, st)
        return out.view(B, S, W)

    def norm_all_gather_seq(self, x: torch.Tensor, w: torch.Tensor | None, eps: float):
        """RMSNorm of this rank's rows fused with the sequence all-gather:
        x [B, S / n, W] (fp32 or bf16) -> (y [B, S, W] bf16 on every rank, rstd [B * S / n])."""
        B, s, W = x.shape
        S = s * self.n
        x2 = x.reshape(B * s, W)
        if x2.dtype not in (torch.float32, torch.bfloat16):
            x2 = x2.float()
        x2 = x2.contiguous()
        flags, bufs, e, cap = self._args(_AG, B * S * W * 2)
        out = torch.empty((B * S, W), dtype=torch.bfloat16, device=x.device)
        rstd = torch.empty(B * s, dtype=torch.float32, device=x.device)
        wf = None if w is None else w.detach().float().contiguous()
        ext().tp_norm_ag(x2, wf, rstd, out, flags, bufs, self.rank, e, B, S, float(eps), cap,
                         status_word(x.device))
        return out.view(B, S, W), rstd

    def gemm_reduce_scatter(self, x: torch.Tensor, w: torch.Tensor, w_mn_major: bool = False) -> torch.Tensor:
        """``(x [B, S, K] @ w [N, K]^T)`` (or ``x @ w`` with ``w`` [K, N] when
        ``w_mn_major``) summed over the axis, sequence-sharded: [B, S / n, N]. One
        tcgen05 GEMM whose epilogue stores into the owners' staging slots, then the
        finishing kernel."""
        B, S, K = x.shape
        N = w.shape[1] if w_mn_major else w.shape[0]
        x2 = x.reshape(B * S, K).to(torch.bfloat16).contiguous()
        flags, bufs, e, cap = self._args(_RS, B * S * N * 2)
        st = status_word(x.device)
        ext().gemm_rs(x2, w, w_mn_major, bufs, self.rank, S, cap, st)
        out = torch.empty((B * (S // self.n), N), dtype=torch.bfloat16, device=x.device)
        ext().tp_collective("rs_finish", out, flags, bufs, self.rank, e, B, S, cap, st)
        return out.view(B, S // self.n, N)

    def close(self) -> None:
        for b in (self.buf[_RS], self.buf[_AG], self.flags):
            if b is not None:
                b.close()


# ------------------------------------------------------------------ autograd
class GatherSeq(torch.autograd.Function):
    """[B, S/n, W] -> [B, S, W] (bf16) forward; reduce-scatter of the grad backward."""

    @staticmethod
    def forward(ctx, x, comm):
        ctx.comm, ctx.dtype = comm, x.dtype
        return comm.all_gather_seq(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.comm.reduce_scatter_seq(g.contiguous()).to(ctx.dtype), None


class ScatterSeq(torch.autograd.Function):
    """Partial [B, S, W] -> this rank's reduced [B, S/n, W]; all-gather backward."""

    @staticmethod
    def forward(ctx, x, comm):
        ctx.comm, ctx.dtype = comm, x.dtype
        return comm.reduce_scatter_seq(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.comm.all_gather_seq(g.contiguous()).to(ctx.dtype), None


class NormGatherSeq(torch.autograd.Function):
    """Pre-norm of a sequence-parallel block fused with the gather of its output:
    x [B, S/n, W] -> RMSNorm(x) * w as bf16 [B, S, W] on every rank.
    backward: reduce-scatter of the gradient, then the norm backward on this rank's rows."""

    @staticmethod
    def forward(ctx, x, weight, comm, eps):
        y, rstd = comm.norm_all_gather_seq(x, weight, eps)
        ctx.comm = comm
        ctx.save_for_backward(x, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, g):
        from pluggy_b200.ops.norm import rmsnorm_bwd

        x, weight, rstd = ctx.saved_tensors
        B, s, W = x.shape
        dy = ctx.comm.reduce_scatter_seq(g.contiguous()).reshape(B * s, W)
        xf = x.reshape(B * s, W)
        if xf.dtype not in (torch.float32, torch.bfloat16):
            xf = xf.float()
        dxf, _, dw = rmsnorm_bwd(dy, xf.contiguous(), None if weight is None else weight.detach().float(),
                                 rstd, want_f32=True, want_dw=weight is not None)
        dx = dxf.view(B, s, W).to(x.dtype)
        return dx, (None if weight is None else dw.to(weight.dtype)), None, None


class TPNormGather(torch.nn.Module):
    """Drop-in for a block's pre-norm under sequence parallelism: returns the
    gathered, normalised activation, so the column-parallel linears that follow
    must not gather again. Keeps the norm's ``weight`` (same parameter, same
    state-dict key)."""

    def __init__(self, norm: torch.nn.Module, comm, eps: float):
        super().__init__()
        self.weight = norm.weight
        self.comm, self.eps = comm, eps

    def forward(self, x):
        return NormGatherSeq.apply(x, self.weight, self.comm, self.eps)


class RowParallelMMRS(torch.autograd.Function):
    """Row-parallel linear with the sequence reduce-scatter fused into the GEMM.

    forward: y[B, S/n, N] = RS(x[B, S, K/n] @ W_shard^T);
    backward: g = AG(dy) [B, S, N]; dx = g @ W_shard; dW = g^T x."""

    @staticmethod
    def forward(ctx, x, weight, comm):
        w = weight.to(torch.bfloat16).contiguous()
        ctx.comm, ctx.x_dtype = comm, x.dtype
        x16 = x.to(torch.bfloat16).contiguous()
        ctx.save_for_backward(x16, w)
        return comm.gemm_reduce_scatter(x16, w)

    @staticmethod
    def backward(ctx, dy):
        from pluggy_b200.ops.gemm import linear_dgrad, linear_wgrad

        x16, w = ctx.saved_tensors
        B, S, K = x16.shape
        g = ctx.comm.all_gather_seq(dy.contiguous()).reshape(B * S, -1)
        dx = linear_dgrad(g, w).view(B, S, K).to(ctx.x_dtype)
        dw = linear_wgrad(g, x16.reshape(B * S, K))
        return dx, dw, None
