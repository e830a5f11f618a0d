"""Context parallelism: ring attention over a zigzag-sharded sequence.

The reference ships this module as an empty file; its design notes describe the
plan implemented here (``notes/ROADMAP.md:380-407`` of the reference):

* zigzag sharding: the sequence is cut into ``2n`` chunks and rank ``i`` owns
  chunks ``i`` and ``2n-1-i``, which balances the causal work;
* forward: the key/value blocks travel around a ring (``ring_send_recv``); each
  rank attends its two query chunks to every block it holds and merges the
  partial results with their log-sum-exps (online softmax);
* backward: a second ring in the same direction carries each key/value block
  together with its dK/dV accumulator; every rank adds its contribution using
  the final output and log-sum-exp, and the accumulator arrives back at the
  block's owner after ``n`` hops;
* overlap: every hop is issued asynchronously before the step's blocks compute
  (forward: the next K/V; backward: the next K/V, and the accumulated dK/dV that
  the neighbour sent at the end of its step is waited for only after this
  step's contribution has been computed into a fresh buffer), so the transfers
  run under the attention kernels instead of between them.

A (query chunk, key chunk) pair is skipped when the key chunk lies after the
query chunk, computed with a causal mask when it is the same chunk, and computed
in full when it lies before. On CUDA each pair runs on this package's flash
attention kernels (forward returning the log-sum-exp, backward given the final
output and log-sum-exp); on CPU on the same math in PyTorch.

Model integration (:func:`parallelize_cp`): every attention module routes to
:func:`ring_attention`, the objective shards ids, labels and RoPE positions with
:func:`zigzag_shard`, and :meth:`ContextParallel.sync_grads` sums the parameter
grads over the axis (each rank holds part of every sequence's loss).
"""

from __future__ import annotations

import math

import torch

from pluggy_b200.core.collective import all_reduce, ring_send_recv


# ------------------------------------------------------------------- sharding
def zigzag_indices(S: int, n: int, r: int, device=None) -> torch.Tensor:
    """Global positions of rank ``r``'s tokens: chunks r and 2n-1-r of 2n chunks."""
    assert S % (2 * n) == 0, f"context parallel: seq_len {S} must divide into {2 * n} chunks"
    c = S // (2 * n)
    a = torch.arange(r * c, (r + 1) * c, device=device)
    b = torch.arange((2 * n - 1 - r) * c, (2 * n - r) * c, device=device)
    return torch.cat([a, b])


def zigzag_shard(x: torch.Tensor, mesh, dim: str, seq_dim: int = 1) -> torch.Tensor:
    n, r = mesh.size(dim), mesh.coordinate(dim)
    idx = zigzag_indices(x.shape[seq_dim], n, r, x.device)
    return x.index_select(seq_dim, idx)


# --------------------------------------------------------------- block math
# (q chunk, key chunk) relation: 0 skip, 1 causal (same chunk), 2 full
def _relation(qi: int, ki: int) -> int:
    return 0 if ki > qi else (1 if ki == qi else 2)


def _block_fwd(q, k, v, causal: bool, scale: float):
    """[B, c, H, d] blocks -> (o [B, c, Hq, d] fp32, lse [B, Hq, c] fp32)."""
    if q.is_cuda and q.shape[-1] in (64, 128):
        from pluggy_b200.ops.attention import attn_fwd

        o, lse = attn_fwd(q.bfloat16().contiguous(), k.bfloat16().contiguous(),
                          v.bfloat16().contiguous(), causal=causal, scale=scale)
        return o.float(), lse
    Hq, Hk = q.shape[2], k.shape[2]
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    if Hk != Hq:
        kf, vf = kf.repeat_interleave(Hq // Hk, 1), vf.repeat_interleave(Hq // Hk, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        c = s.shape[-1]
        s = s.masked_fill(torch.ones(c, c, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ vf
    return o.transpose(1, 2), lse


def _block_bwd(q, k, v, o, lse, do, causal: bool, scale: float):
    """Contributions of one block given the FINAL o and lse: (dq, dk, dv) fp32."""
    if q.is_cuda and q.shape[-1] in (64, 128):
        from pluggy_b200.ops.attention import attn_bwd

        dq, dk, dv = attn_bwd(q.bfloat16().contiguous(), k.bfloat16().contiguous(),
                              v.bfloat16().contiguous(), o.bfloat16().contiguous(),
                              lse.contiguous(), do.bfloat16().contiguous(), causal=causal,
                              scale=scale)
        return dq.float(), dk.float(), dv.float()
    Hq, Hk = q.shape[2], k.shape[2]
    G = Hq // Hk
    qf, kf, vf, of, dof = (t.float().transpose(1, 2) for t in (q, k, v, o, do))
    if G > 1:
        kf, vf = kf.repeat_interleave(G, 1), vf.repeat_interleave(G, 1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        c = s.shape[-1]
        s = s.masked_fill(torch.ones(c, c, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    p = torch.exp(s - lse[..., None])
    delta = (dof * of).sum(-1, keepdim=True)
    dp = dof @ vf.transpose(-1, -2)
    ds = p * (dp - delta)
    dq = (ds @ kf) * scale
    dk = (ds.transpose(-1, -2) @ qf) * scale
    dv = p.transpose(-1, -2) @ dof
    if G > 1:
        B, _, c, d = dk.shape
        dk = dk.view(B, Hk, G, c, d).sum(2)
        dv = dv.view(B, Hk, G, c, d).sum(2)
    return dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)


def _merge(o1, lse1, o2, lse2):
    """Combine two partial softmax results over disjoint key sets."""
    lse = torch.logaddexp(lse1, lse2)
    w1 = torch.exp(lse1 - lse).transpose(1, 2)[..., None]
    w2 = torch.exp(lse2 - lse).transpose(1, 2)[..., None]
    return o1 * w1 + o2 * w2, lse


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, mesh, dim, scale):
        n, r = mesh.size(dim), mesh.coordinate(dim)
        B, S2, Hq, d = q.shape
        c = S2 // 2
        qc = (q[:, :c], q[:, c:])
        q_ids = (r, 2 * n - 1 - r)
        o = [None, None]
        lse = [None, None]
        kv = torch.stack([k, v])
        for step in range(n):
            src = (r - step) % n
            k_ids = (src, 2 * n - 1 - src)
            # the next hop's K/V are in flight while this step's blocks compute
            work = None
            if step + 1 < n:
                kv_next, work = ring_send_recv(kv, mesh, dim, async_op=True)
            kb, vb = kv[0], kv[1]
            for a in range(2):
                for b in range(2):
                    rel = _relation(q_ids[a], k_ids[b])
                    if rel == 0:
                        continue
                    ob, lb = _block_fwd(qc[a], kb[:, b * c:(b + 1) * c], vb[:, b * c:(b + 1) * c],
                                        rel == 1, scale)
                    if o[a] is None:
                        o[a], lse[a] = ob, lb
                    else:
                        o[a], lse[a] = _merge(o[a], lse[a], ob, lb)
            if work is not None:
                work.wait()
                kv = kv_next
        out = torch.cat(o, dim=1)
        lse_all = torch.cat(lse, dim=2)
        ctx.save_for_backward(q, k, v, out, lse_all)
        ctx.mesh, ctx.dim, ctx.scale = mesh, dim, scale
        return out.to(q.dtype)

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse = ctx.saved_tensors
        mesh, dim, scale = ctx.mesh, ctx.dim, ctx.scale
        n, r = mesh.size(dim), mesh.coordinate(dim)
        c = q.shape[1] // 2
        q_ids = (r, 2 * n - 1 - r)
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        kv = torch.stack([k, v])
        dkv_in, dkv_work = None, None
        for step in range(n):
            src = (r - step) % n
            k_ids = (src, 2 * n - 1 - src)
            # prefetch the next hop's K/V while this step computes
            kv_work = None
            if step + 1 < n:
                kv_next, kv_work = ring_send_recv(kv, mesh, dim, async_op=True)
            # this step's contribution to the travelling block's dK/dV, in a fresh buffer
            part = torch.zeros(kv.shape, dtype=torch.float32, device=q.device)
            for a in range(2):
                qs = slice(a * c, (a + 1) * c)
                for b in range(2):
                    rel = _relation(q_ids[a], k_ids[b])
                    if rel == 0:
                        continue
                    ks = slice(b * c, (b + 1) * c)
                    g_q, g_k, g_v = _block_bwd(q[:, qs], kv[0][:, ks], kv[1][:, ks], out[:, qs],
                                               lse[:, :, qs], do[:, qs], rel == 1, scale)
                    dq[:, qs] += g_q
                    part[0][:, ks] += g_k
                    part[1][:, ks] += g_v
            # the block's accumulated dK/dV from the ranks that saw it before (sent at the
            # end of their previous step, so the transfer overlapped this step's compute)
            if dkv_work is not None:
                dkv_work.wait()
                part += dkv_in
            # accumulator and block move on together; after n hops both are home
            dkv_in, dkv_work = ring_send_recv(part, mesh, dim, async_op=True)
            if kv_work is not None:
                kv_work.wait()
                kv = kv_next
        if dkv_work is not None:
            dkv_work.wait()
        dkv = dkv_in
        return dq.to(q.dtype), dkv[0].to(k.dtype), dkv[1].to(v.dtype), None, None, None


def ring_attention(q, k, v, mesh, dim: str, scale: float | None = None):
    """Causal GQA attention of zigzag-sharded ``[B, 2c, H, d]`` q/k/v over the axis."""
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    return _RingAttention.apply(q, k, v, mesh, dim, float(scale))


# -------------------------------------------------------------- model plumbing
class ContextParallel:
    """Handle returned by :func:`parallelize_cp`."""

    def __init__(self, model, mesh, dim):
        self.model, self.mesh, self.dim = model, mesh, dim

    def shard_batch(self, ids: torch.Tensor, labels: torch.Tensor):
        """(local ids, local labels, local positions) for already-shifted labels."""
        n, r = self.mesh.size(self.dim), self.mesh.coordinate(self.dim)
        idx = zigzag_indices(ids.shape[1], n, r, ids.device)
        pos = idx.unsqueeze(0).expand(ids.shape[0], -1)
        return ids.index_select(1, idx), labels.index_select(1, idx), pos

    @torch.no_grad()
    def sync_grads(self) -> None:
        """Sum every parameter grad over the axis (one flat all-reduce)."""
        if self.mesh.size(self.dim) == 1:
            return
        grads = [p.grad for p in self.model.parameters() if p.grad is not None]
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        all_reduce(flat, self.mesh, self.dim, "sum")
        off = 0
        for g in grads:
            g.copy_(flat[off:off + g.numel()].view_as(g))
            off += g.numel()


def parallelize_cp(model, mesh, dim: str = "cp") -> ContextParallel:
    """Route every attention module of ``model`` through :func:`ring_attention`."""
    cp = ContextParallel(model, mesh, dim)
    for blk in model.blocks:
        for name in ("gqa", "attn", "attention"):
            att = getattr(blk, name, None)
            if att is not None and hasattr(att, "q_proj"):
                att.cp = cp
                break
    model.cp = cp
    return cp


__all__ = ["zigzag_indices", "zigzag_shard", "ring_attention", "ContextParallel", "parallelize_cp"]
