"""Tensor parallelism with optional sequence parallelism over one mesh axis.

The reference has no tensor parallelism; its design notes describe the plan this
module implements (``notes/ROADMAP.md:327-378`` of the reference):

* autograd-aware collective pairs: copy-to (identity forward, all-reduce backward),
  reduce-from (all-reduce forward, identity backward), and with sequence
  parallelism gather-seq (all-gather forward, reduce-scatter backward) and
  scatter-seq (reduce-scatter forward, all-gather backward);
* attention: q/k/v column-parallel by head, o row-parallel;
* MLP: gate/up column-parallel, down row-parallel;
* vocabulary-parallel embedding and LM head, and a vocabulary-parallel chunked
  linear cross-entropy that never materialises the full-vocabulary logits;
* sequence parallelism on the norms and the residual stream: between sublayers
  every rank holds ``S / tp`` of the tokens.

On CUDA with sequence parallelism the sequence collectives run on this package's
peer-memory kernels (:mod:`pluggy_b200.comm.tp_fused`): the row-parallel linears
are one tcgen05 GEMM whose epilogue reduce-scatters into the owners' staging
buffers over NVLink, and the column-parallel inputs are gathered with peer loads.
All projections use the sm_100a GEMMs (:func:`pluggy_b200.ops.linear.linear`).

Weights are initialised full on every rank (same seed) and sliced here, so a TP
run starts from the same model as a single-GPU run. Parameters that stay
replicated across the axis (norm weights, per-head q/k norms) get their gradients
summed over the axis by :meth:`TensorParallel.sync_replicated_grads`, which the
trainer calls before the data-parallel reduction.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from pluggy_b200.core.collective import all_gather, all_reduce, reduce_scatter
from pluggy_b200.ops.linear import linear


# ------------------------------------------------------------------ collectives
class _CopyTo(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mesh, dim):
        ctx.mesh, ctx.dim = mesh, dim
        return x

    @staticmethod
    def backward(ctx, g):
        return all_reduce(g.contiguous(), ctx.mesh, ctx.dim, "sum"), None, None


class _ReduceFrom(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mesh, dim):
        return all_reduce(x.contiguous(), mesh, dim, "sum")

    @staticmethod
    def backward(ctx, g):
        return g, None, None


class _GatherSeq(torch.autograd.Function):
    """[B, S/tp, ...] -> [B, S, ...] forward; reduce-scatter of the grad backward."""

    @staticmethod
    def forward(ctx, x, mesh, dim):
        ctx.mesh, ctx.dim = mesh, dim
        return all_gather(x.contiguous(), mesh, dim, gather_dim=1)

    @staticmethod
    def backward(ctx, g):
        return reduce_scatter(g.contiguous(), ctx.mesh, ctx.dim, "sum", scatter_dim=1), None, None


class _ScatterSeq(torch.autograd.Function):
    """Partial sums [B, S, ...] -> this rank's reduced [B, S/tp, ...]."""

    @staticmethod
    def forward(ctx, x, mesh, dim):
        ctx.mesh, ctx.dim = mesh, dim
        return reduce_scatter(x.contiguous(), mesh, dim, "sum", scatter_dim=1)

    @staticmethod
    def backward(ctx, g):
        return all_gather(g.contiguous(), ctx.mesh, ctx.dim, gather_dim=1), None, None


# ---------------------------------------------------------------------- layers
class _SharedInput:
    """The axis-entry collective of several column-parallel linears that read the
    same activation (q/k/v, gate/up): applied once per distinct input tensor, so the
    forward gathers once and autograd sums the branches' grads before the single
    backward reduction."""

    def __init__(self, mesh, dim: str, sequence_parallel: bool, comm=None, pre_gathered: bool = False):
        self.mesh, self.dim, self.sp, self.comm = mesh, dim, sequence_parallel, comm
        self.pre_gathered = pre_gathered  # the preceding norm already gathered its output
        self._src = None
        self._out = None

    def __call__(self, x):
        if self.pre_gathered:
            return x
        if x is not self._src:
            if self.sp and self.comm is not None:
                from pluggy_b200.comm.tp_fused import GatherSeq

                self._out = GatherSeq.apply(x, self.comm)
            elif self.sp:
                self._out = _GatherSeq.apply(x, self.mesh, self.dim)
            else:
                self._out = _CopyTo.apply(x, self.mesh, self.dim)
            self._src = x
        return self._out


class ColumnParallelLinear(nn.Module):
    """y[..., out/tp] = x W_shard^T; with SP the input is gathered along the sequence."""

    def __init__(self, full: nn.Linear, mesh, dim: str, sequence_parallel: bool,
                 shared: _SharedInput | None = None):
        super().__init__()
        n, r = mesh.size(dim), mesh.coordinate(dim)
        out = full.weight.shape[0]
        assert out % n == 0, f"column-parallel: {out} outputs not divisible by tp={n}"
        k = out // n
        self.weight = nn.Parameter(full.weight.detach()[r * k:(r + 1) * k].clone())
        self.mesh, self.dim, self.sp = mesh, dim, sequence_parallel
        self._enter = shared if shared is not None else _SharedInput(mesh, dim, sequence_parallel)

    def forward(self, x):
        return linear(self._enter(x), self.weight)


class RowParallelLinear(nn.Module):
    """Partial x[..., in/tp] W_shard^T summed over the axis (reduce-scatter with SP)."""

    def __init__(self, full: nn.Linear, mesh, dim: str, sequence_parallel: bool, comm=None):
        super().__init__()
        n, r = mesh.size(dim), mesh.coordinate(dim)
        inp = full.weight.shape[1]
        assert inp % n == 0, f"row-parallel: {inp} inputs not divisible by tp={n}"
        k = inp // n
        self.weight = nn.Parameter(full.weight.detach()[:, r * k:(r + 1) * k].clone())
        self.mesh, self.dim, self.sp = mesh, dim, sequence_parallel
        self.comm = comm

    def forward(self, x):
        if self.sp and self.comm is not None and x.dim() == 3:
            from pluggy_b200.comm.tp_fused import RowParallelMMRS

            return RowParallelMMRS.apply(x, self.weight, self.comm)
        y = linear(x, self.weight)
        return _ScatterSeq.apply(y, self.mesh, self.dim) if self.sp else _ReduceFrom.apply(y, self.mesh, self.dim)


class VocabParallelEmbedding(nn.Module):
    """Rows [vstart, vstart + V/tp) of the table on each rank; the lookup is summed
    over the axis (reduce-scattered along the sequence with SP)."""

    def __init__(self, full: nn.Embedding, mesh, dim: str, sequence_parallel: bool):
        super().__init__()
        n, r = mesh.size(dim), mesh.coordinate(dim)
        V = full.weight.shape[0]
        assert V % n == 0, f"vocab-parallel: vocab {V} not divisible by tp={n}"
        k = V // n
        self.vstart, self.vlocal = r * k, k
        self.weight = nn.Parameter(full.weight.detach()[r * k:(r + 1) * k].clone())
        self.mesh, self.dim, self.sp = mesh, dim, sequence_parallel
        self.num_embeddings, self.embedding_dim = V, full.weight.shape[1]

    def forward(self, ids):
        local = ids - self.vstart
        hit = (local >= 0) & (local < self.vlocal)
        out = F.embedding(local.clamp(0, self.vlocal - 1), self.weight) * hit.unsqueeze(-1)
        return _ScatterSeq.apply(out, self.mesh, self.dim) if self.sp else _ReduceFrom.apply(out, self.mesh, self.dim)


# ---------------------------------------------------------- vocab-parallel CE
class _VocabParallelCE(torch.autograd.Function):
    """Chunked linear + cross-entropy with the vocabulary sharded over the axis.

    Per chunk of rows: local logits [c, V/tp] (fp32), global row max and sum of
    exponentials by all-reduce, the target logit from the rank that owns it, then
    grad_logits = softmax - onehot on the local slice; grad_hidden is summed over
    the axis by the collective the hidden entered through (see
    :func:`tp_hidden_for_head`), grad_W stays local. Gradients are computed in
    forward and scaled by grad_out / n_valid in backward, the contract of the
    single-GPU fused CE.
    """

    @staticmethod
    def forward(ctx, hidden, w_local, labels, vstart, mesh, dim, ignore_index, chunk, w_lowp=None):
        if hidden.is_cuda:
            return _VocabParallelCE._forward_cuda(ctx, hidden, w_local, labels, vstart, mesh, dim,
                                                  ignore_index, chunk, w_lowp)
        T = hidden.shape[0]
        Vl = w_local.shape[0]
        gh = torch.empty(hidden.shape, dtype=torch.float32, device=hidden.device)
        gw = torch.zeros(w_local.shape, dtype=torch.float32, device=hidden.device)
        loss_sum = torch.zeros((), dtype=torch.float32, device=hidden.device)
        wf = w_local.float()
        valid_all = labels != ignore_index
        for s in range(0, T, chunk):
            h = hidden[s:s + chunk].float()
            y = labels[s:s + chunk]
            valid = valid_all[s:s + chunk]
            logits = h @ wf.t()
            m = logits.max(dim=-1).values
            all_reduce(m, mesh, dim, "max")
            se = (logits - m[:, None]).exp().sum(-1)
            all_reduce(se, mesh, dim, "sum")
            lse = m + se.log()
            loc = y - vstart
            own = (loc >= 0) & (loc < Vl) & valid
            tgt = torch.where(own, logits.gather(1, loc.clamp(0, Vl - 1)[:, None]).squeeze(1),
                              torch.zeros_like(lse))
            all_reduce(tgt, mesh, dim, "sum")
            loss_sum += ((lse - tgt) * valid).sum()
            g = (logits - lse[:, None]).exp()
            g[own, loc.clamp(0, Vl - 1)[own]] -= 1.0
            g *= valid[:, None]
            # this rank's share of grad_hidden; the caller's entry collective sums it
            gh[s:s + chunk] = g @ wf
            gw += g.t() @ h
        n_valid = valid_all.sum().clamp(min=1).float()
        ctx.save_for_backward(gh, gw, n_valid)
        ctx.h_dtype, ctx.w_dtype = hidden.dtype, w_local.dtype
        return loss_sum / n_valid

    @staticmethod
    def _forward_cuda(ctx, hidden, w_local, labels, vstart, mesh, dim, ignore_index, chunk, w_lowp):
        """The same algorithm on the sm_100a kernels: per chunk, the local bf16 logits
        (tcgen05 GEMM), this shard's (max, sum of exp, owned target logit) per row
        (``ce_rows`` statistics pass), ONE all-gather of those three numbers per row,
        the full-vocabulary lse combined locally, the gradient written in place over
        the logits (``ce_rows`` gradient pass), then grad_hidden and grad_W GEMMs."""
        from pluggy_b200.ops._ext import ext
        from pluggy_b200.ops.gemm import gemm

        T, D = hidden.shape
        Vl = w_local.shape[0]
        dev = hidden.device
        n = mesh.size(dim)
        h = hidden.to(torch.bfloat16).contiguous()
        w = w_lowp if w_lowp is not None else w_local.detach().to(torch.bfloat16)
        lab = labels.contiguous()
        valid_all = lab != ignore_index
        gh = torch.empty((T, D), dtype=torch.float32, device=dev)
        gw = torch.empty(w_local.shape, dtype=torch.float32, device=dev)
        row_loss = torch.empty(T, dtype=torch.float32, device=dev)
        logits = torch.empty((min(chunk, T), Vl), dtype=torch.bfloat16, device=dev)
        for s in range(0, T, chunk):
            e = min(s + chunk, T)
            c = e - s
            lg = logits[:c]
            gemm(h[s:e], w, out=lg)
            st = torch.empty((c, 3), dtype=torch.float32, device=dev)
            ext().ce_rows(lg, lab[s:e], int(ignore_index), 1.0, 0.0, None, None, None, None, st,
                          None, int(vstart))
            allst = all_gather(st, mesh, dim, gather_dim=0).view(n, c, 3)
            m_all, s_all, t_all = allst[..., 0], allst[..., 1], allst[..., 2]
            M = m_all.max(dim=0).values
            lse = M + (s_all * torch.exp(m_all - M)).sum(0).log()
            tgt = t_all.sum(0)
            valid = valid_all[s:e]
            row_loss[s:e] = torch.where(valid, lse - tgt, torch.zeros_like(lse))
            ext().ce_rows(lg, lab[s:e], int(ignore_index), 1.0, 0.0, None, None, None, None, None,
                          lse.contiguous(), int(vstart))
            # this rank's share of grad_hidden; the caller's entry collective sums it
            gemm(lg, w, b_mn_major=True, out=gh[s:e], out_dtype=torch.float32)
            gemm(lg, h[s:e], a_mn_major=True, b_mn_major=True, out=gw,
                 addend=gw if s > 0 else None, beta=1.0)
        if T == 0:
            gw.zero_()
        n_valid = valid_all.sum().clamp(min=1).float()
        ctx.save_for_backward(gh, gw, n_valid)
        ctx.h_dtype, ctx.w_dtype = hidden.dtype, w_local.dtype
        return row_loss.sum() / n_valid

    @staticmethod
    def backward(ctx, grad_out):
        gh, gw, n_valid = ctx.saved_tensors
        s = grad_out / n_valid
        return (gh * s).to(ctx.h_dtype), (gw * s).to(ctx.w_dtype), None, None, None, None, None, None, None


def vocab_parallel_cross_entropy(hidden, w_local, labels, vstart, mesh, dim, ignore_index=-100,
                                 chunk=4096, w_lowp=None):
    """Mean CE over valid rows of ``hidden [T, D] @ W^T`` with W's rows sharded over ``dim``.
    ``w_lowp``: a bf16 copy of ``w_local`` (CUDA; else it is cast here)."""
    return _VocabParallelCE.apply(hidden, w_local, labels, int(vstart), mesh, dim, int(ignore_index),
                                  int(chunk), w_lowp)


# ------------------------------------------------------------------ the plan
class TensorParallel:
    """Handle returned by :func:`parallelize_tp`: the axis, the replicated params
    and the vocab shard of the LM head."""

    def __init__(self, model, mesh, dim, sequence_parallel):
        self.model, self.mesh, self.dim, self.sp = model, mesh, dim, sequence_parallel
        self.sharded: list[nn.Parameter] = []
        self.replicated: list[nn.Parameter] = []  # replicated params with partial grads
        self.vstart = 0
        self.comm = None  # peer-memory collectives (CUDA + sequence parallel)

    def close(self) -> None:
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    @torch.no_grad()
    def sync_replicated_grads(self) -> None:
        """Sum the grads of params replicated over the axis (one flat all-reduce)."""
        if self.mesh.size(self.dim) == 1:
            return
        grads = [p.grad for p in self.replicated if p.grad is not None]
        if not grads:
            return
        flat = torch.cat([g.reshape(-1).float() for g in grads])
        all_reduce(flat, self.mesh, self.dim, "sum")
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[off:off + n].view_as(g))
            off += n

    def sharded_param_ids(self) -> set[int]:
        return {id(p) for p in self.sharded}

    @torch.no_grad()
    def full_state_dict(self) -> dict[str, torch.Tensor]:
        """The unsharded state dict (collective over the axis; every rank gets it)."""
        out = {}
        for name, t in self.model.state_dict().items():
            mod_name, _, pname = name.rpartition(".")
            mod = self.model.get_submodule(mod_name) if mod_name else self.model
            if isinstance(mod, (ColumnParallelLinear, VocabParallelEmbedding)) or name == "lm_head.weight":
                out[name] = all_gather(t.contiguous(), self.mesh, self.dim, gather_dim=0)
            elif isinstance(mod, RowParallelLinear):
                out[name] = all_gather(t.contiguous(), self.mesh, self.dim, gather_dim=1)
            else:
                out[name] = t
        return out

    @torch.no_grad()
    def load_full_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        n, r = self.mesh.size(self.dim), self.mesh.coordinate(self.dim)
        local = {}
        for name, t in self.model.state_dict().items():
            full = sd[name]
            mod_name, _, _ = name.rpartition(".")
            mod = self.model.get_submodule(mod_name) if mod_name else self.model
            if isinstance(mod, (ColumnParallelLinear, VocabParallelEmbedding)) or name == "lm_head.weight":
                k = full.shape[0] // n
                local[name] = full[r * k:(r + 1) * k]
            elif isinstance(mod, RowParallelLinear):
                k = full.shape[1] // n
                local[name] = full[:, r * k:(r + 1) * k]
            else:
                local[name] = full
        self.model.load_state_dict(local)


def _prenorm_forward():
    """The pre-norm block forward (``x + attn(norm1(x))``, ``x + ffn(norm2(x))``) whose
    norms may be fused with the sequence gather."""
    from pluggy_b200.models.qwen3 import Qwen3TransformerBlock

    return Qwen3TransformerBlock.forward


def _attention_modules(block):
    for name in ("gqa", "attn", "attention"):
        mod = getattr(block, name, None)
        if isinstance(mod, nn.Module) and hasattr(mod, "q_proj"):
            return name, mod
    raise ValueError(f"no attention module with q_proj in {type(block).__name__}")


def parallelize_tp(model: nn.Module, mesh, dim: str = "tp", sequence_parallel: bool = True,
                   fused: bool | None = None) -> TensorParallel:
    """Shard ``model`` (a decoder with ``token_emb``, ``blocks``, ``norm``, ``lm_head``)
    over mesh axis ``dim``; returns the :class:`TensorParallel` handle (also stored
    as ``model.tp``). Heads, FFN width and vocabulary must divide by the axis size.
    ``fused`` (default: on CUDA with sequence parallelism) selects the peer-memory
    collectives and the fused GEMM -> reduce-scatter."""
    n = mesh.size(dim)
    tp = TensorParallel(model, mesh, dim, sequence_parallel)
    on_cuda = next(model.parameters()).is_cuda
    if fused is None:
        fused = on_cuda and sequence_parallel and n > 1
    comm = None
    if fused and n > 1:
        if not (on_cuda and sequence_parallel):
            raise ValueError("fused tensor-parallel collectives need CUDA and sequence parallelism")
        from pluggy_b200.comm.tp_fused import TPComm

        comm = TPComm(mesh, dim)
    tp.comm = comm
    if n == 1:
        model.tp = tp
        tp.replicated = []
        tp.sharded = list(model.parameters())
        return tp
    tied = model.lm_head.weight is model.token_emb.weight
    for blk in model.blocks:
        _, att = _attention_modules(blk)
        assert att.num_heads % n == 0 and att.num_kv_heads % n == 0, \
            f"tp={n} must divide the query ({att.num_heads}) and KV ({att.num_kv_heads}) heads"
        # pre-norms fused with the sequence gather (peer-memory path, RMSNorm pre-norms)
        fuse_norm = (comm is not None and isinstance(getattr(blk, "norm1", None), nn.RMSNorm)
                     and isinstance(getattr(blk, "norm2", None), nn.RMSNorm)
                     and type(blk).forward is _prenorm_forward())
        if fuse_norm:
            from pluggy_b200.comm.tp_fused import TPNormGather
            from pluggy_b200.models.common import norm_eps

            blk.norm1 = TPNormGather(blk.norm1, comm, norm_eps(blk.norm1))
            blk.norm2 = TPNormGather(blk.norm2, comm, norm_eps(blk.norm2))
        qkv_in = _SharedInput(mesh, dim, sequence_parallel, comm, pre_gathered=fuse_norm)
        att.q_proj = ColumnParallelLinear(att.q_proj, mesh, dim, sequence_parallel, qkv_in)
        att.k_proj = ColumnParallelLinear(att.k_proj, mesh, dim, sequence_parallel, qkv_in)
        att.v_proj = ColumnParallelLinear(att.v_proj, mesh, dim, sequence_parallel, qkv_in)
        att.o_proj = RowParallelLinear(att.o_proj, mesh, dim, sequence_parallel, comm)
        att.num_heads //= n
        att.num_kv_heads //= n
        ffn = blk.ffn
        gu_in = _SharedInput(mesh, dim, sequence_parallel, comm, pre_gathered=fuse_norm)
        ffn.gate_proj = ColumnParallelLinear(ffn.gate_proj, mesh, dim, sequence_parallel, gu_in)
        ffn.up_proj = ColumnParallelLinear(ffn.up_proj, mesh, dim, sequence_parallel, gu_in)
        ffn.down_proj = RowParallelLinear(ffn.down_proj, mesh, dim, sequence_parallel, comm)
    emb = VocabParallelEmbedding(model.token_emb, mesh, dim, sequence_parallel)
    model.token_emb = emb
    if tied:
        model.lm_head.weight = emb.weight
    else:
        V = model.lm_head.weight.shape[0]
        k = V // n
        r = mesh.coordinate(dim)
        model.lm_head.weight = nn.Parameter(model.lm_head.weight.detach()[r * k:(r + 1) * k].clone())
    tp.vstart = emb.vstart
    sharded_ids = set()
    for mod in model.modules():
        if isinstance(mod, (ColumnParallelLinear, RowParallelLinear, VocabParallelEmbedding)):
            sharded_ids.add(id(mod.weight))
    sharded_ids.add(id(model.lm_head.weight))
    tp.sharded = [p for p in model.parameters() if id(p) in sharded_ids]
    # replicated params whose grads are partial over the axis: every one of them
    # with SP (norms see this rank's tokens); without SP only the per-head q/k norms
    # (they see this rank's heads), the block and final norms already get the full grad
    head_norm_ids = set()
    for blk in model.blocks:
        _, att = _attention_modules(blk)
        for nm in ("q_norm", "k_norm"):
            mod = getattr(att, nm, None)
            if mod is not None and getattr(mod, "weight", None) is not None:
                head_norm_ids.add(id(mod.weight))
    tp.replicated = [p for p in model.parameters() if id(p) not in sharded_ids
                     and (sequence_parallel or id(p) in head_norm_ids)]
    model.tp = tp
    if hasattr(model, "weight_cache"):
        model.weight_cache.clear()
    return tp


def tp_hidden_for_head(model, hidden: torch.Tensor) -> torch.Tensor:
    """The final hidden of a TP model entering the vocabulary-parallel head: gathered
    to the full sequence with SP (the partial grads reduce-scatter back), else passed
    through an all-reduce-on-backward copy."""
    tp = getattr(model, "tp", None)
    if tp is None or tp.mesh.size(tp.dim) == 1:
        return hidden
    if tp.sp:
        return _GatherSeq.apply(hidden, tp.mesh, tp.dim)
    return _CopyTo.apply(hidden, tp.mesh, tp.dim)


__all__ = ["ColumnParallelLinear", "RowParallelLinear", "VocabParallelEmbedding", "TensorParallel",
           "parallelize_tp", "vocab_parallel_cross_entropy", "tp_hidden_for_head"]
