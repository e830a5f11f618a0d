"""FSDP2: per-parameter ``Shard(0)`` of params, grads and optimizer state.

Parity: reference ``pluggy/parallelism/fsdp2.py:75-261``:

* units = one per ``model.blocks[i]`` plus a root unit (embedding, head, final
  norm) that stays gathered after forward because the fused linear-CE reads
  ``lm_head.weight`` after ``forward`` returns;
* pre-forward hook gathers the unit, post-forward hook frees the full storage
  (``resize_(0)``, so a use-after-reshard fails loudly), pre-backward hook
  re-gathers;
* the post-accumulate-grad hook reduce-scatters (avg) each full grad into an
  fp32 shard accumulator every microbatch; once a unit's last grad has
  arrived its params point back at their shards;
* ``sync()`` publishes the shard grads as ``p.grad``; the optimizer and the
  clip (``shard_dims=("dp",)``) see only shards.

B200 differences (same observable contract):

* every shard of a unit lives in ONE flat fp32 buffer and every gather of a
  unit is one coalesced collective (one NCCL group) instead of a synchronous
  call per parameter;
* on CUDA the gathers run on a dedicated comm stream and the NEXT unit is
  prefetched while the current one computes (forward: i+1, backward: i-1);
  the compute stream waits on an event only when it needs the weights;
* grad reduce-scatters are also issued on the comm stream and coalesced per
  unit once the unit's last grad arrives;
* a unit's full parameters are views of one flat storage, so on CUDA the gather is
  one peer-memory push (every rank stores its shards into every rank's staging
  buffer over NVLink, :mod:`pluggy_b200.comm.fsdp_fused`) plus one finishing copy,
  instead of an NCCL all-gather (``gather="nccl"`` keeps NCCL). Gradient
  reduce-scatters stay on NCCL;
* ``reduce="peer"``: the gradient reduce-scatter is one peer-memory kernel per unit
  (``fsdp_rs_kernel``: each rank stages its full unit gradient in symmetric memory, sums
  its shards over the ranks' copies and writes or accumulates them straight into a flat
  fp32 grad-shard buffer) instead of NCCL;
* for the fused-engine models (their GEMMs read bf16 weights through the weight
  cache) the block units are gathered in low precision: each rank casts its shards
  to bf16 while pushing them into a slot of symmetric memory that the GEMMs then
  read in place (half the bytes, no finishing copy, no cast pass, and no
  full-size copy of the unit kept anywhere: during a block only the slot and the
  gradients hold full-size data). Norm weights travel as fp32. While a block unit is
  in use its matrix parameters are zero-byte placeholders of the full shape, so
  autograd accumulates full-shape gradients for the reduce-scatter.
"""

from __future__ import annotations

import contextlib

import torch
import torch._dynamo
import torch.distributed as dist
import torch.nn as nn

from pluggy_b200.core.collective import MeshLike, broadcast


class _ParamState:
    def __init__(self, param: nn.Parameter, n: int, coord: int):
        assert param.shape[0] % n == 0, (
            f"param dim 0 ({param.shape[0]}) not divisible by the dp size {n} (even shards only)"
        )
        self.param = param
        self.full_shape = tuple(param.shape)
        self.full_numel = param.numel()
        rows = param.shape[0] // n
        self.shard_shape = (rows, *param.shape[1:])
        self.shard_numel = param.numel() // n
        self.full: torch.Tensor | None = None  # a view of the unit's flat full storage
        self._init_shard = param.data.narrow(0, coord * rows, rows).clone()
        self.sharded: torch.Tensor | None = None
        self.grad_shard: torch.Tensor | None = None


class _Unit:
    def __init__(self, name: str, states: list[_ParamState], reshard_after_forward: bool):
        self.name = name
        self.params = states
        self.reshard_after_forward = reshard_after_forward
        self.n_grads = sum(1 for s in states if s.param.requires_grad)
        self.pending = self.n_grads
        numel = sum(s.shard_numel for s in states)
        dev = states[0].param.device if states else torch.device("cpu")
        dt = states[0].param.dtype if states else torch.float32
        self.flat_shard = torch.empty(numel, dtype=dt, device=dev)
        off = 0
        for s in states:
            v = self.flat_shard[off: off + s.shard_numel].view(s.shard_shape)
            v.copy_(s._init_shard)
            s._init_shard = None
            s.sharded = v
            s.param.data = v
            off += s.shard_numel
        # every full parameter of the unit is a view of one flat storage, allocated
        # while the unit is gathered and resized to 0 bytes otherwise (a use after
        # resharding fails loudly)
        full_numel = sum(s.full_numel for s in states)
        self.full_flat = torch.empty(full_numel, dtype=dt, device=dev)
        self.full_nbytes = self.full_flat.untyped_storage().nbytes()
        off = 0
        for s in states:
            s.full = self.full_flat[off: off + s.full_numel].view(s.full_shape)
            off += s.full_numel
        self.full_flat.untyped_storage().resize_(0)
        self.gathered = False
        self.gather_event = None
        self.ready_grads: list[_ParamState] = []
        self.peer_table = None  # peer-gather parameter table (device), built on first use

    def alloc_full(self) -> None:
        st = self.full_flat.untyped_storage()
        if st.nbytes() != self.full_nbytes:
            st.resize_(self.full_nbytes)

    def free_full(self) -> None:
        self.full_flat.untyped_storage().resize_(0)


class FSDP2:
    def __init__(self, model: nn.Module, mesh: MeshLike, dim: str = "dp", *, prefetch: bool = True,
                 gather: str = "auto", lowp_gather: bool = True, reduce: str = "nccl"):
        self.mesh = mesh
        self.dim = dim
        self.group_size = mesh.size(dim)
        self.requires_sync = True  # API parity with DDP; FSDP2 reduces every microbatch
        if self.group_size == 1:
            return
        assert hasattr(model, "blocks"), "fsdp2 units are per transformer block (model.blocks)"
        for t in [*model.parameters(), *model.buffers()]:
            broadcast(t.detach(), mesh, dim, src=0)
        n, coord = self.group_size, mesh.coordinate(dim)
        block_ids = {id(p) for b in model.blocks for p in b.parameters()}
        self._units: list[_Unit] = []
        for i, block in enumerate(model.blocks):
            u = _Unit(f"block{i}", [_ParamState(p, n, coord) for p in block.parameters()], True)
            self._units.append(u)
            self._install(block, u)
        root = [_ParamState(p, n, coord) for p in model.parameters() if id(p) not in block_ids]
        self._root = _Unit("root", root, False)
        self._units.append(self._root)
        self._install(model, self._root)
        dev = self._root.flat_shard.device
        self._cuda = dev.type == "cuda"
        self._prefetch = prefetch and self._cuda
        self._comm_stream = torch.cuda.Stream(device=dev) if self._cuda else None
        self._block_units = self._units[:-1]
        self._pending_work: list = []
        # parameter all-gathers over peer memory ("peer") or NCCL ("nccl"); "auto" picks
        # peer on CUDA when every parameter splits into whole 16-byte pieces
        self._peer = None
        aligned = all(s.full_numel % (4 * n) == 0 for u in self._units for s in u.params)
        if gather not in ("auto", "peer", "nccl"):
            raise ValueError(f"gather must be 'auto', 'peer' or 'nccl', got {gather!r}")
        if gather == "peer" and not (self._cuda and aligned and dev.type == "cuda"):
            raise ValueError("peer gathers need CUDA and parameters of whole 16-byte shards")
        if gather == "peer" or (gather == "auto" and self._cuda and aligned):
            from pluggy_b200.comm.fsdp_fused import PeerGather

            self._peer = PeerGather(mesh, dim, max(u.full_nbytes for u in self._units))
        # gradient reduce-scatter: NCCL, or the peer-memory kernel that accumulates into
        # a flat fp32 grad-shard buffer per unit
        self._peer_rs = None
        if reduce not in ("nccl", "peer"):
            raise ValueError(f"reduce must be 'nccl' or 'peer', got {reduce!r}")
        if reduce == "peer":
            if not (self._cuda and aligned):
                raise ValueError("peer reduce-scatters need CUDA and parameters of whole 16-byte shards")
            from pluggy_b200.comm.fsdp_fused import PeerReduceScatter

            for u in self._units:
                u.rs_states = [st for st in u.params if st.param.requires_grad]
                u.rs_table, u.rs_offsets = PeerReduceScatter.plan(u.rs_states, dev)
                u.grad_flat = torch.zeros(sum(st.shard_numel for st in u.rs_states),
                                          dtype=torch.float32, device=dev)
                off = 0
                for st in u.rs_states:
                    st.rs_view = u.grad_flat[off:off + st.shard_numel].view(st.shard_shape)
                    off += st.shard_numel
                u.grad_acc = False
            self._peer_rs = PeerReduceScatter(
                mesh, dim, max(4 * sum(st.full_numel for st in u.rs_states) for u in self._units))
        # low-precision slot gathers for the block units of fused-engine models
        self._slots = None
        self._slot_views: dict[int, torch.Tensor] = {}
        for u in self._units:
            u.slot = None
        if (self._peer is not None and lowp_gather and getattr(type(model), "fused_engine", False)
                and hasattr(model, "weight_cache")):
            from pluggy_b200.comm.fsdp_fused import SlotGather, SlotLayout

            layouts = [SlotLayout(u.params, n) for u in self._block_units]
            if layouts and all(lay.ok for lay in layouts):
                self._slots = SlotGather(mesh, dim, max(lay.nbytes for lay in layouts))
                for i, (u, lay) in enumerate(zip(self._block_units, layouts, strict=True)):
                    u.slot = i % 2
                    u.slot_table, u.slot_groups = lay.table(u.params, dev)
                    views = self._slots.views(lay, u.slot)
                    u.slot_views = views
                    self._slot_views.update(views)
                    # zero-byte stand-ins of the full shape (the GEMMs read the slot)
                    u.placeholders = {id(st.param): torch.empty(1, dtype=st.param.dtype, device=dev)
                                      .expand(st.full_shape) for st in u.params if len(st.full_shape) >= 2}
                model.weight_cache.provider = self._lowp_view
        # the models' fused CUDA path runs blocks through ``fused_forward`` (not the
        # module call, so the module hooks do not fire): it calls these instead
        model._plg_fsdp = self
        if hasattr(model, "weight_cache"):
            model.weight_cache.always_recast = True
            model.weight_cache.clear()

    # --------------------------------------------------------------- plumbing
    def _install(self, module: nn.Module, unit: _Unit) -> None:
        module.register_forward_pre_hook(lambda m, a, u=unit: self._pre_forward(u))
        if unit.reshard_after_forward:
            module.register_forward_hook(lambda m, a, o, u=unit: self._reshard(u))
            module.register_full_backward_pre_hook(lambda m, g, u=unit: self._pre_backward(u))
        for s in unit.params:
            if s.param.requires_grad:
                s.param.register_post_accumulate_grad_hook(
                    lambda p, s=s, u=unit: self._on_grad_ready(s, u))

    def _group(self):
        return self.mesh.get_group(self.dim)

    @staticmethod
    def _coalesced(group, unit):
        """One NCCL group launch per unit; gloo has no coalescing, so plain calls there."""
        if dist.get_backend(group) == "nccl":
            return dist._coalescing_manager(group=group, device=unit.flat_shard.device)
        return contextlib.nullcontext()

    def _lowp_view(self, params) -> torch.Tensor | None:
        """The weight cache's source of bf16 weights: the slot views of block-unit
        matrices (one view over consecutive parameters for a concatenation), else None."""
        views = [self._slot_views.get(id(p)) for p in params]
        if not views or any(v is None or v.dtype != torch.bfloat16 for v in views):
            return None
        if len(views) == 1:
            return views[0]
        for a, b in zip(views, views[1:]):
            if b.data_ptr() != a.data_ptr() + a.numel() * 2 or b.shape[1:] != a.shape[1:]:
                return None
        from pluggy_b200.ops._ext import ext

        rows = sum(v.shape[0] for v in views)
        return ext().tensor_from_ptr(views[0].data_ptr(), [rows, *views[0].shape[1:]], torch.bfloat16,
                                     views[0].device.index)

    def _issue_gather(self, unit: _Unit) -> None:
        """Launch the coalesced all-gather of ``unit`` (on the comm stream on CUDA)."""
        if unit.gathered:
            return
        if unit.slot is not None:
            self._comm_stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self._comm_stream):
                self._slots.gather(unit, unit.slot)
                unit.gather_event = torch.cuda.Event()
                unit.gather_event.record(self._comm_stream)
            unit.gathered = True
            return
        unit.alloc_full()
        ctx = torch.cuda.stream(self._comm_stream) if self._cuda else contextlib.nullcontext()
        if self._cuda:
            self._comm_stream.wait_stream(torch.cuda.current_stream())
        with ctx:
            if self._peer is not None:
                self._peer.gather(unit)
            else:
                group = self._group()
                with self._coalesced(group, unit):
                    for s in unit.params:
                        dist.all_gather_into_tensor(s.full, s.sharded, group=group)
            if self._cuda:
                unit.gather_event = torch.cuda.Event()
                unit.gather_event.record(self._comm_stream)
                unit.full_flat.record_stream(torch.cuda.current_stream())
        unit.gathered = True

    def _use(self, unit: _Unit) -> None:
        if unit.gather_event is not None:
            torch.cuda.current_stream().wait_event(unit.gather_event)
            unit.gather_event = None
        if unit.slot is not None:
            for s in unit.params:
                ph = unit.placeholders.get(id(s.param))
                s.param.data = ph if ph is not None else unit.slot_views[id(s.param)]
            return
        for s in unit.params:
            s.param.data = s.full

    def _neighbor(self, unit: _Unit, step: int) -> _Unit | None:
        if unit is self._root:
            return self._block_units[0] if step > 0 and self._block_units else None
        i = self._block_units.index(unit) + step
        return self._block_units[i] if 0 <= i < len(self._block_units) else None

    # ------------------------------------------------------------------ hooks
    @torch._dynamo.disable
    def _pre_forward(self, unit: _Unit) -> None:
        self._issue_gather(unit)
        self._use(unit)
        if self._prefetch:
            nxt = self._neighbor(unit, +1)
            if nxt is not None:
                self._issue_gather(nxt)

    @torch._dynamo.disable
    def _reshard(self, unit: _Unit) -> None:
        unit.free_full()
        unit.gathered = False

    @torch._dynamo.disable
    def _pre_backward(self, unit: _Unit) -> None:
        self._issue_gather(unit)
        self._use(unit)
        if self._prefetch:
            prv = self._neighbor(unit, -1)
            if prv is not None and prv is not self._root:
                self._issue_gather(prv)

    @torch._dynamo.disable
    def _on_grad_ready(self, s: _ParamState, unit: _Unit) -> None:
        unit.ready_grads.append(s)
        unit.pending -= 1
        if unit.pending == 0:
            unit.pending = unit.n_grads
            self._reduce_unit(unit)
            for st in unit.params:
                st.param.data = st.sharded
            unit.free_full()
            unit.gathered = False

    def _reduce_unit(self, unit: _Unit) -> None:
        """Average each full grad of ``unit`` into its fp32 shard accumulator."""
        if self._peer_rs is not None:
            ready = {id(s) for s in unit.ready_grads}
            assert all(id(s) in ready for s in unit.rs_states), f"unit {unit.name}: missing grads"
            grads = [s.param.grad for s in unit.rs_states]
            self._comm_stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self._comm_stream):
                self._peer_rs.reduce(unit, grads, accumulate=unit.grad_acc)
                for g in grads:
                    g.record_stream(self._comm_stream)
            unit.grad_acc = True
            for s in unit.rs_states:
                s.grad_shard = s.rs_view
                s.param.grad = None
            unit.ready_grads = []
            return
        group = self._group()
        n = self.group_size
        nccl = dist.get_backend(group) == "nccl"
        outs = []
        grads = [s.param.grad for s in unit.ready_grads]
        if self._cuda:
            self._comm_stream.wait_stream(torch.cuda.current_stream())
        ctx = torch.cuda.stream(self._comm_stream) if self._cuda else contextlib.nullcontext()
        with ctx:
            for s, g in zip(unit.ready_grads, grads, strict=True):
                outs.append(torch.empty(s.shard_shape, dtype=g.dtype, device=g.device))
            op = dist.ReduceOp.AVG if nccl else dist.ReduceOp.SUM
            with self._coalesced(group, unit):
                for g, o in zip(grads, outs, strict=True):
                    dist.reduce_scatter_tensor(o, g.contiguous(), op=op, group=group)
            for s, o in zip(unit.ready_grads, outs, strict=True):
                if not nccl:
                    o.div_(n)
                if s.grad_shard is None:
                    s.grad_shard = o
                else:
                    s.grad_shard.add_(o)
            if self._cuda:
                for g in grads:
                    g.record_stream(self._comm_stream)
        for s in unit.ready_grads:
            s.param.grad = None
        unit.ready_grads = []

    def sync(self) -> None:
        if self.group_size == 1:
            return
        if self._cuda:
            torch.cuda.current_stream().wait_stream(self._comm_stream)
        for unit in self._units:
            assert unit.pending == unit.n_grads, (
                f"unit {unit.name}: only {unit.n_grads - unit.pending}/{unit.n_grads} grads "
                "arrived -- a param got no grad this backward"
            )
            for s in unit.params:
                assert s.full.untyped_storage().nbytes() == 0, (
                    f"unit {unit.name}: full param storage still allocated at sync"
                )
                if s.param.requires_grad:
                    assert s.grad_shard is not None, f"unit {unit.name}: no reduced grad to publish"
                    s.param.grad = s.grad_shard
                    s.grad_shard = None
            # peer reduce-scatter: the next step's first microbatch overwrites the shards
            unit.grad_acc = False

    @torch._dynamo.disable
    def fused_block_enter(self, i: int) -> None:
        """Before block ``i`` of a fused forward: gather it (and prefetch the next)."""
        self._pre_forward(self._block_units[i])

    @torch._dynamo.disable
    def fused_block_exit(self, i: int, out: torch.Tensor) -> None:
        """After block ``i``: reshard it; when the gradient of its output arrives,
        re-gather it for its backward (what the module's backward pre-hook does)."""
        unit = self._block_units[i]
        self._reshard(unit)
        if out.requires_grad:
            out.register_hook(lambda g, u=unit: self._pre_backward(u))

    def close(self) -> None:
        """Release the peer-gather buffers (collective over the axis)."""
        if getattr(self, "_peer", None) is not None:
            torch.cuda.synchronize()
            self._peer.close()
            self._peer = None
        if getattr(self, "_slots", None) is not None:
            torch.cuda.synchronize()
            self._slots.close()
            self._slots = None
        if getattr(self, "_peer_rs", None) is not None:
            torch.cuda.synchronize()
            self._peer_rs.close()
            self._peer_rs = None

    # ------------------------------------------------------------- inspection
    @property
    def units(self) -> list[_Unit]:
        return getattr(self, "_units", [])
