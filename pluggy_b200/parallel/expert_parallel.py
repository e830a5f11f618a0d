"""Expert parallelism for the Qwen3-MoE sparse MLP.

The reference has no expert parallelism; its design notes describe the plan this
module implements (``notes/ROADMAP.md:409-433`` of the reference): the experts of
every sparse layer are split evenly over one mesh axis, tokens travel to the rank
that owns their expert and back with an all-to-all of uneven splits, and the
expert parameters are kept out of the data-parallel all-reduce.

Per sparse layer and microbatch (``EPExperts.forward``):

1. the (token, expert) pairs are ordered by destination rank, then by expert;
2. the per-destination pair counts are exchanged (an even all-to-all of one
   integer per rank) so every rank knows how many rows it receives;
3. dispatch: the hidden rows of the pairs are exchanged with an uneven
   all-to-all; the local expert ids ride along;
4. the local experts run as one dropless grouped SwiGLU FFN over the received
   rows (the same op as the single-GPU path);
5. combine: the outputs return with the reverse all-to-all, are scaled by the
   routing weights and scatter-added into the token rows.

Both exchanges are autograd functions whose backward is the reverse exchange. On
CUDA the count exchange, dispatch and combine run on this package's peer-memory
kernels (:mod:`pluggy_b200.comm.ep_fused`: each rank stores its rows straight into
the owners' receive buffers over NVLink) instead of NCCL all-to-alls.
When the expert axis is also the data-parallel axis (the usual EP = DP layout),
each expert's gradient already holds the contributions of every rank's tokens;
:meth:`ExpertParallel.finish_grads` divides it by the axis size so it matches the
average the data-parallel all-reduce gives the replicated parameters.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from pluggy_b200.core.collective import all_gather, all_to_all
from pluggy_b200.ops.moe import expert_histogram, moe_expert_ffn


class _AllToAllV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send, recv, mesh, dim):
        ctx.send, ctx.recv, ctx.mesh, ctx.dim = send, recv, mesh, dim
        return all_to_all(x, mesh, dim, input_splits=send, output_splits=recv)

    @staticmethod
    def backward(ctx, g):
        return (all_to_all(g.contiguous(), ctx.mesh, ctx.dim, input_splits=ctx.recv,
                           output_splits=ctx.send), None, None, None, None)


class EPExperts(nn.Module):
    """This rank's share ``[E/ep]`` of a packed expert bank, with token dispatch and
    combine over the ``dim`` axis. Drop-in for ``Qwen3MoeExperts``."""

    def __init__(self, full: nn.Module, mesh, dim: str):
        super().__init__()
        n, r = mesh.size(dim), mesh.coordinate(dim)
        E = full.num_experts
        assert E % n == 0, f"expert parallelism: {E} experts not divisible by ep={n}"
        el = E // n
        self.num_experts, self.local_experts, self.first = E, el, r * el
        self.emb_dim, self.moe_ffn_dim = full.emb_dim, full.moe_ffn_dim
        self.gate_up_proj = nn.Parameter(full.gate_up_proj.detach()[r * el:(r + 1) * el].clone())
        self.down_proj = nn.Parameter(full.down_proj.detach()[r * el:(r + 1) * el].clone())
        for p in (self.gate_up_proj, self.down_proj):
            p._plg_expert_sharded = True  # kept out of the data-parallel all-reduce
        self.mesh, self.dim = mesh, dim
        self.comm = None  # peer-memory exchange (set by parallelize_ep on CUDA)

    def forward(self, h, top_indices, top_weights):
        T, H = h.shape
        K = top_indices.shape[1]
        n = self.mesh.size(self.dim)
        tok = torch.arange(T, device=h.device).repeat_interleave(K)
        exp = top_indices.reshape(-1)
        w = top_weights.reshape(-1)
        dest = torch.div(exp, self.local_experts, rounding_mode="floor")
        order = torch.argsort(dest * self.num_experts + exp, stable=True)
        s_tok, s_exp, s_w, s_dest = tok[order], exp[order], w[order], dest[order]
        if self.comm is not None:
            from pluggy_b200.comm.ep_fused import ToOwners, ToSources

            C = self.comm.exchange_counts(expert_histogram(exp, self.num_experts))
            pl = self.comm.plan(C)
            lc = torch.as_tensor(pl["local_counts"].reshape(-1), dtype=torch.int64)
            r_exp = torch.repeat_interleave(torch.arange(self.local_experts).repeat(n), lc).to(h.device)
            x = ToOwners.apply(h[s_tok].contiguous(), self.comm, pl)
            back_fn = lambda y: ToSources.apply(y, self.comm, pl)  # noqa: E731
        else:
            send_counts = expert_histogram(s_dest, n)
            recv_counts = all_to_all(send_counts.clone(), self.mesh, self.dim)
            send, recv = send_counts.tolist(), recv_counts.tolist()
            # local expert ids of the pairs this rank will receive (no gradient)
            rel = (s_exp - s_dest * self.local_experts).to(torch.int64)
            r_exp = all_to_all(rel, self.mesh, self.dim, input_splits=send, output_splits=recv)
            x = _AllToAllV.apply(h[s_tok].contiguous(), send, recv, self.mesh, self.dim)
            back_fn = lambda y: _AllToAllV.apply(y, recv, send, self.mesh, self.dim)  # noqa: E731
        if x.shape[0] > 0:
            ones = torch.ones(x.shape[0], 1, device=h.device, dtype=h.dtype)
            gu_lp = dn_lp = None
            cache = getattr(self, "weight_cache", None)
            if cache is not None and h.is_cuda:
                gu_lp, dn_lp = cache.get(self.gate_up_proj), cache.get(self.down_proj)
            y = moe_expert_ffn(x, r_exp.view(-1, 1), ones, self.gate_up_proj, self.down_proj,
                               gu_lowp=gu_lp, dn_lowp=dn_lp)
        else:
            # no rows for this rank's experts: keep the expert params in the graph
            y = x + 0.0 * (self.gate_up_proj.sum() + self.down_proj.sum()).to(x.dtype)
        back = back_fn(y.to(h.dtype))
        out = torch.zeros(T, H, device=h.device, dtype=back.dtype)
        out.index_add_(0, s_tok, back * s_w.unsqueeze(1).to(back.dtype))
        return out.to(h.dtype)


class ExpertParallel:
    """Handle returned by :func:`parallelize_ep`."""

    def __init__(self, model, mesh, dim):
        self.model, self.mesh, self.dim = model, mesh, dim
        self.expert_params: list[nn.Parameter] = []
        self.comm = None

    def close(self) -> None:
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    def expert_param_ids(self) -> set[int]:
        return {id(p) for p in self.expert_params}

    @torch.no_grad()
    def finish_grads(self, average_over_dim: bool) -> None:
        """Average the expert grads over the axis when it doubles as the dp axis."""
        n = self.mesh.size(self.dim)
        if not average_over_dim or n == 1:
            return
        for p in self.expert_params:
            if p.grad is not None:
                p.grad.div_(n)

    @torch.no_grad()
    def full_state_dict(self) -> dict[str, torch.Tensor]:
        """The unsharded state dict (collective over the axis; every rank gets it)."""
        out = {}
        for name, t in self.model.state_dict().items():
            mod_name, _, _ = name.rpartition(".")
            mod = self.model.get_submodule(mod_name) if mod_name else self.model
            out[name] = (all_gather(t.contiguous(), self.mesh, self.dim, gather_dim=0)
                         if isinstance(mod, EPExperts) else t)
        return out

    @torch.no_grad()
    def load_full_state_dict(self, sd: dict[str, torch.Tensor]) -> None:
        local = {}
        for name, t in self.model.state_dict().items():
            mod_name, _, _ = name.rpartition(".")
            mod = self.model.get_submodule(mod_name) if mod_name else self.model
            full = sd[name]
            if isinstance(mod, EPExperts):
                full = full[mod.first:mod.first + mod.local_experts]
            local[name] = full
        self.model.load_state_dict(local)


def parallelize_ep(model: nn.Module, mesh, dim: str = "dp", fused: bool | None = None) -> ExpertParallel:
    """Replace the packed experts of every sparse block by :class:`EPExperts` over
    ``dim``; returns the handle (also stored as ``model.ep``). ``fused`` (default: on
    CUDA) exchanges tokens over peer memory instead of NCCL all-to-alls."""
    ep = ExpertParallel(model, mesh, dim)
    if fused is None:
        fused = next(model.parameters()).is_cuda and mesh.size(dim) > 1
    for blk in model.blocks:
        ffn = getattr(blk, "ffn", None)
        experts = getattr(ffn, "experts", None)
        if experts is None or not hasattr(experts, "gate_up_proj"):
            continue
        ffn.experts = EPExperts(experts, mesh, dim)
        ffn.experts.weight_cache = getattr(model, "weight_cache", None)
        ep.expert_params += [ffn.experts.gate_up_proj, ffn.experts.down_proj]
        if fused and mesh.size(dim) > 1:
            if ep.comm is None:
                from pluggy_b200.comm.ep_fused import EPComm

                ep.comm = EPComm(mesh, dim, ffn.experts.num_experts, ffn.experts.emb_dim)
            ffn.experts.comm = ep.comm
    model.ep = ep
    if hasattr(model, "weight_cache"):
        model.weight_cache.clear()
    return ep


__all__ = ["EPExperts", "ExpertParallel", "parallelize_ep"]
