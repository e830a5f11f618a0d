"""Mesh-aware collectives: the only module that calls torch.distributed comm ops.

Parity: reference ``pluggy/core/collective.py:87-363``. Same contract:

* callers name a mesh axis, never a ProcessGroup (``MeshLike`` protocol);
* ``op`` is a string; ``"avg"`` is native on NCCL and emulated on other
  backends by dividing before a ``"sum"`` (so an async avg needs no fix-up);
* ``all_reduce`` / ``broadcast`` work in place and return their input;
  ``all_gather`` / ``reduce_scatter`` / ``all_to_all`` / ``ring_send_recv``
  return a new tensor (or a caller-owned ``output_tensor``);
* ``async_op=True`` returns ``(tensor, work)``.

Additions over the reference: ``all_to_all`` accepts uneven ``input_splits`` /
``output_splits`` (expert-parallel dispatch needs them), and ``ring_send_recv``
can run asynchronously (context-parallel ring attention overlaps it).

These NCCL/gloo calls are the baseline and the oracle. The fused sm_100a
collectives live in ``pluggy_b200.comm`` and are checked against these.
"""

from __future__ import annotations

from typing import Literal, Protocol, Sequence

import torch
import torch.distributed as dist

ReduceOpName = Literal["sum", "avg", "max", "min"]

_OPS = {
    "sum": dist.ReduceOp.SUM,
    "avg": dist.ReduceOp.AVG,
    "max": dist.ReduceOp.MAX,
    "min": dist.ReduceOp.MIN,
}


class MeshLike(Protocol):
    def size(self, dim: str) -> int: ...

    def get_group(self, dim: str) -> dist.ProcessGroup: ...

    def coordinate(self, dim: str) -> int: ...


def _native_avg(group) -> bool:
    return dist.get_backend(group) == "nccl"


def _check_out(out: torch.Tensor, shape, like: torch.Tensor, dim_arg: int, what: str) -> None:
    assert dim_arg == 0, (
        f"caller-provided output_tensor needs {what}=0 (the buffer is stacked along dim 0), "
        f"got {dim_arg}"
    )
    assert tuple(out.shape) == tuple(shape), f"output_tensor shape {tuple(out.shape)} != {tuple(shape)}"
    assert out.dtype == like.dtype, f"output_tensor dtype {out.dtype} != {like.dtype}"
    assert out.device == like.device, f"output_tensor device {out.device} != {like.device}"
    assert out.is_contiguous(), "output_tensor must be contiguous"


def all_reduce(tensor: torch.Tensor, mesh: MeshLike, dim: str, op: ReduceOpName = "sum", *,
               async_op: bool = False):
    """Reduce ``tensor`` over the ``dim`` group in place; returns ``tensor``."""
    group = mesh.get_group(dim)
    if op == "avg" and not _native_avg(group):
        tensor.div_(mesh.size(dim))
        op = "sum"
    work = dist.all_reduce(tensor, _OPS[op], group=group, async_op=async_op)
    return (tensor, work) if async_op else tensor


def broadcast(tensor: torch.Tensor, mesh: MeshLike, dim: str, src: int = 0, *,
              async_op: bool = False):
    """Copy from the rank at group COORDINATE ``src`` to the group, in place."""
    group = mesh.get_group(dim)
    work = dist.broadcast(tensor, src=None, group=group, async_op=async_op, group_src=src)
    return (tensor, work) if async_op else tensor


def all_gather(tensor: torch.Tensor, mesh: MeshLike, dim: str, gather_dim: int = 0, *,
               async_op: bool = False, output_tensor: torch.Tensor | None = None):
    """Concatenate every rank's ``tensor`` along ``gather_dim`` in coordinate order."""
    group = mesh.get_group(dim)
    n = mesh.size(dim)
    inp = tensor.movedim(gather_dim, 0).contiguous()
    shape = (n * inp.shape[0], *inp.shape[1:])
    if output_tensor is None:
        output_tensor = torch.empty(shape, dtype=tensor.dtype, device=tensor.device)
    else:
        _check_out(output_tensor, shape, tensor, gather_dim, "gather_dim")
    work = dist.all_gather_into_tensor(output_tensor, inp, group=group, async_op=async_op)
    out = output_tensor.movedim(0, gather_dim)
    return (out, work) if async_op else out


def reduce_scatter(tensor: torch.Tensor, mesh: MeshLike, dim: str, op: ReduceOpName = "sum",
                   scatter_dim: int = 0, *, async_op: bool = False,
                   output_tensor: torch.Tensor | None = None):
    """Reduce over the group; keep this coordinate's even slice of ``scatter_dim``."""
    group = mesh.get_group(dim)
    n = mesh.size(dim)
    assert tensor.shape[scatter_dim] % n == 0, (
        f"shape[{scatter_dim}]={tensor.shape[scatter_dim]} not divisible by group size {n}"
    )
    inp = tensor.movedim(scatter_dim, 0).contiguous()
    shape = (inp.shape[0] // n, *inp.shape[1:])
    if output_tensor is None:
        output_tensor = torch.empty(shape, dtype=tensor.dtype, device=tensor.device)
    else:
        _check_out(output_tensor, shape, tensor, scatter_dim, "scatter_dim")
    if op == "avg" and not _native_avg(group):
        assert not async_op, "async 'avg' reduce_scatter needs a backend with ReduceOp.AVG"
        dist.reduce_scatter_tensor(output_tensor, inp, op=_OPS["sum"], group=group)
        out = output_tensor.movedim(0, scatter_dim)
        out.div_(n)
        return out
    work = dist.reduce_scatter_tensor(output_tensor, inp, op=_OPS[op], group=group,
                                      async_op=async_op)
    out = output_tensor.movedim(0, scatter_dim)
    return (out, work) if async_op else out


def all_to_all(tensor: torch.Tensor, mesh: MeshLike, dim: str, split_dim: int = 0,
               concat_dim: int = 0, *, input_splits: Sequence[int] | None = None,
               output_splits: Sequence[int] | None = None, async_op: bool = False):
    """Chunk ``j`` of ``split_dim`` goes to coordinate ``j``; received chunks are
    concatenated along ``concat_dim`` in sender order.

    Even splits reproduce the reference (``Shard(i)->Shard(j)``). With
    ``input_splits``/``output_splits`` (row counts along dim 0, ``split_dim``
    and ``concat_dim`` must then be 0) this is the uneven exchange used by
    expert-parallel token dispatch.
    """
    group = mesh.get_group(dim)
    n = mesh.size(dim)
    if input_splits is not None or output_splits is not None:
        assert split_dim == 0 and concat_dim == 0, "uneven all_to_all works along dim 0"
        assert input_splits is not None and output_splits is not None
        assert len(input_splits) == n and len(output_splits) == n
        assert sum(input_splits) == tensor.shape[0]
        inp = tensor.contiguous()
        out = torch.empty((sum(output_splits), *inp.shape[1:]), dtype=inp.dtype, device=inp.device)
        work = dist.all_to_all_single(out, inp, list(output_splits), list(input_splits),
                                      group=group, async_op=async_op)
        return (out, work) if async_op else out
    assert tensor.shape[split_dim] % n == 0, (
        f"shape[{split_dim}]={tensor.shape[split_dim]} not divisible by group size {n}"
    )
    assert not async_op, "even-split all_to_all is synchronous"
    inp = tensor.movedim(split_dim, 0).contiguous()
    out = torch.empty_like(inp)
    dist.all_to_all_single(out, inp, group=group)
    pieces = [c.movedim(0, split_dim) for c in out.chunk(n, dim=0)]
    return torch.cat(pieces, dim=concat_dim)


def ring_send_recv(tensor: torch.Tensor, mesh: MeshLike, dim: str, *, async_op: bool = False):
    """Send to coordinate+1 and receive from coordinate-1 (mod size) at once."""
    group = mesh.get_group(dim)
    n = mesh.size(dim)
    if n == 1:
        out = tensor.clone()
        return (out, None) if async_op else out
    me = mesh.coordinate(dim)
    dst = dist.get_global_rank(group, (me + 1) % n)
    src = dist.get_global_rank(group, (me - 1) % n)
    send = tensor.contiguous()
    recv = torch.empty_like(send)
    reqs = dist.batch_isend_irecv([
        dist.P2POp(dist.isend, send, dst, group=group),
        dist.P2POp(dist.irecv, recv, src, group=group),
    ])
    if async_op:
        return recv, _MultiWork(reqs, keep=send)
    for r in reqs:
        r.wait()
    return recv


class _MultiWork:
    """Waits on a list of P2P requests; keeps the send buffer alive until then."""

    def __init__(self, reqs, keep=None):
        self.reqs = reqs
        self.keep = keep

    def wait(self):
        for r in self.reqs:
            r.wait()
        self.keep = None
        return True


def barrier(mesh: MeshLike | None = None, dim: str | None = None) -> None:
    """Block until every rank of the ``dim`` group (or the world) arrives."""
    dist.barrier(group=None if mesh is None else mesh.get_group(dim))
