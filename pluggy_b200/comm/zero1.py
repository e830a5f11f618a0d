"""ZeRO-1 inside data parallelism: reduce-scatter, AdamW on the owned slice,
all-gather of the updated parameters.

``DDP(..., reducer="zero1")`` keeps the reference's DDP bucket contract
(``pluggy/parallelism/data_parallel.py:89-147``: reverse-order 25 MB buckets
launched from post-accumulate hooks while backward runs, ``sync()`` before the
optimizer) but splits the all-reduce of each bucket around the optimizer, so each
rank updates only 1/N of the parameters and holds only 1/N of the AdamW state
(the reference runs ``torch.optim.AdamW(fused=True)`` over every parameter on
every rank, ``pluggy/optimizer/builder.py:20-46``):

* backward, per bucket (``csrc/comm.cu`` ``zero1_rs_kernel``): the rank's slice
  of the bucket is averaged over the ranks with peer loads into its own grad
  arena, and the sum of squares of the averaged slice (the clip's global norm)
  is published to every rank -- half the NVLink bytes of an all-reduce;
* optimizer step, per bucket (``zero1_adamw_ag_kernel``): AdamW with the folded
  clip coefficient on the owned slice, the new fp32 values stored into every
  rank's parameter arena with peer stores, in forward order (embedding and
  first layers first);
* next forward: each block waits only for the bucket that holds its
  parameters (:class:`ParamGate`), so the all-gather of later layers overlaps the
  compute of earlier ones; the bf16 weight copies the GEMMs read are recast from
  the updated fp32 parameters on first use.

Parameters live in a symmetric (peer-mapped) fp32 arena laid out like the
gradient buckets, so a replica is bitwise identical on every rank after each
step (DDP semantics are kept: checkpoints of rank 0 hold the full model).

On CPU (gloo) the same slicing and update run with torch collectives (an
all-reduce then the slice, an all-gather of the slices): the oracle for the
host-side logic.
"""

from __future__ import annotations

import math
import os

import torch
import torch.distributed as dist

_ALIGN = 64  # elements: every bucket starts 256-byte aligned
_KINDS = 3   # flag kinds of the kernels: RS ready, RS done, AG done
_FLAG_BYTES = _KINDS * 8 * 128 * 4
_SLOT_BYTES = 8 * 128 * 4


def owned_slice(numel: int, n: int, r: int) -> tuple[int, int]:
    """Elements [s0, s1) of a bucket that rank r of n updates (the kernels' rule)."""
    seg = ((numel + n - 1) // n + 3) // 4 * 4
    s0 = min(numel, r * seg)
    return s0, min(numel, s0 + seg)


class _Work:
    def __init__(self, event):
        self.event = event

    def wait(self) -> None:
        if self.event is not None:
            torch.cuda.current_stream().wait_event(self.event)


class Zero1Reducer:
    """Owns the grad and parameter arenas of the DDP buckets and the RS launches."""

    def __init__(self, mesh, dim: str, buckets, chunks: int | None = None):
        self.mesh, self.dim = mesh, dim
        self.n, self.rank = mesh.size(dim), mesh.coordinate(dim)
        self.buckets = buckets
        self.device = buckets[0].params[0].device
        self.cuda = self.device.type == "cuda"
        offs, total = [], 0
        for b in buckets:
            offs.append(total)
            total += (self._numel(b) + _ALIGN - 1) // _ALIGN * _ALIGN
        total = max(total, _ALIGN)
        if self.cuda:
            from pluggy_b200.comm.symm import SymmetricBuffer

            self.grad_buf = SymmetricBuffer(total * 4, mesh, dim)
            self.param_buf = SymmetricBuffer(total * 4, mesh, dim)
            self.flags = SymmetricBuffer(_FLAG_BYTES, mesh, dim)
            self.slots = SymmetricBuffer(_SLOT_BYTES, mesh, dim)
            grad_arena = self.grad_buf.tensor(0, [total])
            param_arena = self.param_buf.tensor(0, [total])
        else:
            grad_arena = torch.zeros(total, dtype=torch.float32)
            param_arena = torch.zeros(total, dtype=torch.float32)
        self.grad_arena, self.param_arena = grad_arena, param_arena
        self.offset: dict[int, tuple[int, int]] = {}
        self.slice: dict[int, tuple[int, int]] = {}
        with torch.no_grad():
            for b, off in zip(buckets, offs, strict=True):
                numel = self._numel(b)
                flat = grad_arena[off:off + numel]
                b.flat, b.views, o = flat, [], 0
                for p in b.params:
                    b.views.append(flat[o:o + p.numel()].view_as(p))
                    # the parameter moves into the arena: peers' stores update it in place
                    pv = param_arena[off + o:off + o + p.numel()].view_as(p)
                    pv.copy_(p.data)
                    p.data = pv
                    o += p.numel()
                self.offset[b.index] = (off, numel)
                self.slice[b.index] = owned_slice(numel, self.n, self.rank)
        # CTAs per bucket kernel (PLG_COMM_CTAS overrides the default for measurements)
        self.chunks = chunks or int(os.environ.get("PLG_COMM_CTAS", "128"))
        self.rs_epoch = 0
        self.ag_epoch = 0
        self.norm_sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._first = True
        # high priority: at each kernel boundary the block scheduler places the
        # collective's CTAs before pending compute CTAs
        self.stream = torch.cuda.Stream(self.device, priority=-1) if self.cuda else None

    @staticmethod
    def _numel(b) -> int:
        return sum(p.numel() for p in b.params)

    # ------------------------------------------------------------- backward
    def launch(self, b) -> _Work:
        """Average this rank's slice of bucket ``b`` over the ranks (grads in the arena)."""
        off, numel = self.offset[b.index]
        if len(b.params) == 1 and b.params[0].grad is not b.views[0]:
            b.views[0].copy_(b.params[0].grad)
            b.params[0].grad = b.views[0]
        if not self.cuda:
            return self._launch_cpu(b)
        from pluggy_b200.ops._ext import ext, status_word

        ready = torch.cuda.Event()
        ready.record()
        self.stream.wait_event(ready)
        self.rs_epoch += 1
        with torch.cuda.stream(self.stream):
            ext().zero1_rs(self.grad_buf.peers, self.param_buf.peers, self.flags.peers,
                           self.slots.peers, off, numel, self.rank, self.rs_epoch, self.chunks,
                           self.norm_sq, not self._first, status_word(self.device))
        self._first = False
        done = torch.cuda.Event()
        done.record(self.stream)
        return _Work(done)

    def _launch_cpu(self, b) -> _Work:
        g = b.flat
        s0, s1 = self.slice[b.index]
        red = g.clone()
        dist.all_reduce(red, group=self.mesh.get_group(self.dim))
        red /= self.n
        g[s0:s1] = red[s0:s1]
        # every rank's slice sum of squares, summed over the ranks (the kernel's slot table)
        sq = torch.zeros(self.n, dtype=torch.float64)
        sq[self.rank] = float(red[s0:s1].double().pow(2).sum())
        dist.all_reduce(sq, group=self.mesh.get_group(self.dim))
        tot = torch.tensor([float(sq.sum())], dtype=torch.float32)
        if self._first:
            self.norm_sq.copy_(tot)
        else:
            self.norm_sq += tot
        self._first = False
        return _Work(None)

    def finish(self) -> None:
        self._first = True

    def reduced_norm_sq(self) -> torch.Tensor:
        return self.norm_sq[0]

    def close(self) -> None:
        if self.cuda:
            for buf in (self.grad_buf, self.param_buf, self.flags, self.slots):
                buf.close()


class ParamGate:
    """Orders the next forward after the parameter all-gather, bucket by bucket.

    ``enter(key)`` (``"emb"``, a block index, or ``"all"``) makes the current
    stream wait for the all-gather of the buckets that hold that part's
    parameters; the all-gathers are issued in forward order, so waiting for the
    last of them covers the earlier ones."""

    def __init__(self, model, bucket_of: dict):
        self._key_bucket: dict = {}

        def low(params):
            idx = [bucket_of[p].index for p in params if p in bucket_of]
            return min(idx) if idx else None

        emb = getattr(model, "token_emb", None)
        if emb is not None:
            self._key_bucket["emb"] = low(list(emb.parameters()))
        for i, blk in enumerate(getattr(model, "blocks", [])):
            self._key_bucket[i] = low(list(blk.parameters()))
        self._key_bucket["all"] = min((b.index for b in bucket_of.values()), default=None)
        self._events: dict[int, torch.cuda.Event] = {}
        self._waited: set[int] = set()

    def arm(self, events: dict[int, torch.cuda.Event]) -> None:
        self._events = events
        self._waited = set()

    def enter(self, key) -> None:
        if not self._events:
            return
        b = self._key_bucket.get(key)
        if b is None:
            b = self._key_bucket["all"]
        if b is None or b in self._waited:
            return
        ev = self._events.get(b)
        if ev is not None:
            torch.cuda.current_stream().wait_event(ev)
        # buckets launched before b are covered by the same wait
        self._waited.update(k for k in self._events if k >= b)
        if b == self._key_bucket["all"]:
            self._events = {}


class Zero1AdamW(torch.optim.Optimizer):
    """AdamW over the slices a :class:`Zero1Reducer` owns (see the module docstring).

    Built from the param groups and hyper-parameters of an AdamW built by the
    optimizer builder (two groups: decay on >= 2-D tensors). ``state_dict`` holds
    this rank's slices only: checkpoints save one optimizer file per rank."""

    def __init__(self, base: torch.optim.Optimizer, reducer: Zero1Reducer, gate: ParamGate | None,
                 gate_used_by_model: bool):
        defaults = dict(base.defaults)
        groups = [{k: v for k, v in g.items()} for g in base.param_groups]
        super().__init__(groups, defaults)
        assert len(self.param_groups) <= 4, "zero1: at most 4 param groups"
        self.reducer = reducer
        self.gate = gate
        self.gate_used = gate_used_by_model
        self._grad_scale = None
        self._step = 0
        group_of = {}
        for gi, g in enumerate(self.param_groups):
            for p in g["params"]:
                group_of[p] = gi
        r = reducer
        self._rows: dict[int, torch.Tensor] = {}
        self._m: dict[int, torch.Tensor] = {}
        self._v: dict[int, torch.Tensor] = {}
        for b in r.buckets:
            rows, o = [], 0
            for p in b.params:
                if p not in group_of:
                    raise ValueError("zero1: every bucketed parameter must be in an optimizer group")
                rows.append([o, o + p.numel(), group_of[p]])
                o += p.numel()
            self._rows[b.index] = torch.tensor(rows, dtype=torch.int64, device=r.device)
            s0, s1 = r.slice[b.index]
            self._m[b.index] = torch.zeros(max(s1 - s0, 4), dtype=torch.float32, device=r.device)
            self._v[b.index] = torch.zeros(max(s1 - s0, 4), dtype=torch.float32, device=r.device)

    def set_grad_scale(self, coef: torch.Tensor | None) -> None:
        self._grad_scale = coef

    def zero_grad(self, set_to_none: bool = True) -> None:
        for g in self.param_groups:
            for p in g["params"]:
                p.grad = None

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._step += 1
        b1, b2 = self.param_groups[0]["betas"]
        eps = self.param_groups[0]["eps"]
        lrs = [float(g["lr"]) for g in self.param_groups]
        wds = [float(g["weight_decay"]) for g in self.param_groups]
        bc1, bc2 = 1 - b1 ** self._step, 1 - b2 ** self._step
        scale = self._grad_scale
        self._grad_scale = None
        r = self.reducer
        order = sorted(r.buckets, key=lambda b: -b.index)  # forward order: embedding first
        if not r.cuda:
            self._step_cpu(order, lrs, wds, b1, b2, eps, bc1, bc2, scale)
            return loss
        from pluggy_b200.ops._ext import ext, status_word

        ready = torch.cuda.Event()
        ready.record()
        r.stream.wait_event(ready)
        if scale is not None:
            scale.record_stream(r.stream)
        events = {}
        gs = None if scale is None else scale.reshape(1).float()
        with torch.cuda.stream(r.stream):
            for b in order:
                off, numel = r.offset[b.index]
                r.ag_epoch += 1
                ext().zero1_adamw_ag(r.grad_buf.peers, r.param_buf.peers, r.flags.peers,
                                     r.slots.peers, off, numel, r.rank, r.ag_epoch, r.chunks,
                                     lrs, wds, b1, b2, eps, bc1, bc2, gs, self._rows[b.index],
                                     self._m[b.index], self._v[b.index], status_word(r.device))
                ev = torch.cuda.Event()
                ev.record(r.stream)
                events[b.index] = ev
        # the kernels wrote the params through raw pointers: bump their versions so
        # the bf16 weight caches recast them on first use
        torch.autograd.graph.increment_version([p for b in order for p in b.params])
        if self.gate is not None and self.gate_used:
            self.gate.arm(events)
        else:
            torch.cuda.current_stream().wait_event(events[order[-1].index])
        return loss

    def _step_cpu(self, order, lrs, wds, b1, b2, eps, bc1, bc2, scale):
        r = self.reducer
        grp = r.mesh.get_group(r.dim)
        for b in order:
            off, numel = r.offset[b.index]
            s0, s1 = r.slice[b.index]
            seg = ((numel + r.n - 1) // r.n + 3) // 4 * 4
            p_all = r.param_arena[off:off + numel]
            g = r.grad_arena[off + s0:off + s1]
            if scale is not None:
                g = g * scale
            m, v = self._m[b.index][:s1 - s0], self._v[b.index][:s1 - s0]
            p = p_all[s0:s1].clone()
            rows = self._rows[b.index].tolist()
            for start, end, gi in rows:
                lo, hi = max(start, s0), min(end, s1)
                if lo >= hi:
                    continue
                sl = slice(lo - s0, hi - s0)
                lr, wd = lrs[gi], wds[gi]
                p[sl].mul_(1 - lr * wd)
                m[sl].lerp_(g[sl], 1 - b1)
                v[sl].mul_(b2).addcmul_(g[sl], g[sl], value=1 - b2)
                denom = (v[sl].sqrt() / math.sqrt(bc2)).add_(eps)
                p[sl].addcdiv_(m[sl], denom, value=-lr / bc1)
            # all-gather of the slices (padded to the common slice length)
            pad = torch.zeros(seg, dtype=torch.float32)
            pad[:s1 - s0] = p
            out = [torch.zeros(seg, dtype=torch.float32) for _ in range(r.n)]
            dist.all_gather(out, pad, group=grp)
            for q in range(r.n):
                q0, q1 = owned_slice(numel, r.n, q)
                p_all[q0:q1] = out[q][:q1 - q0]
        torch.autograd.graph.increment_version([p for b in order for p in b.params])

    def wait_params(self) -> None:
        """Make the current stream wait until every updated parameter has landed."""
        if self.gate is not None:
            self.gate.enter("all")

    # --------------------------------------------------------- checkpoints
    def state_dict(self) -> dict:
        r = self.reducer
        return {
            "zero1": {"rank": r.rank, "nranks": r.n, "step": self._step,
                      "slices": {k: list(v) for k, v in r.slice.items()}},
            "exp_avg": {k: v.detach().cpu() for k, v in self._m.items()},
            "exp_avg_sq": {k: v.detach().cpu() for k, v in self._v.items()},
            "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups],
        }

    def load_state_dict(self, sd: dict) -> None:
        z = sd["zero1"]
        r = self.reducer
        assert z["nranks"] == r.n and z["rank"] == r.rank, (
            "zero1 optimizer state is per rank: resume on the same data-parallel layout")
        self._step = int(z["step"])
        for k in self._m:
            self._m[k].copy_(sd["exp_avg"][k])
            self._v[k].copy_(sd["exp_avg_sq"][k])
        for g, s in zip(self.param_groups, sd["param_groups"], strict=True):
            for k, v in s.items():
                g[k] = v
