"""Symmetric (peer-mapped) device buffers over one mesh axis.

Every rank of the axis allocates the same number of bytes on its GPU; the CUDA IPC
handles are exchanged with an all-gather over the axis and each rank opens its
peers' buffers, so this package's kernels can load from and store to any rank's
copy over NVLink. Used by the fused collectives (:mod:`pluggy_b200.comm.fused_ddp`).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from pluggy_b200.ops._ext import ext


class SymmetricBuffer:
    def __init__(self, nbytes: int, mesh, dim: str):
        self.nbytes = int(nbytes)
        self.mesh, self.dim = mesh, dim
        self.n = mesh.size(dim)
        self.rank = mesh.coordinate(dim)
        self.device = torch.cuda.current_device()
        self.ptr, handle = ext().symm_malloc(self.nbytes)
        group = mesh.get_group(dim)
        h = handle.to(f"cuda:{self.device}")
        out = torch.empty(self.n * 64, dtype=torch.uint8, device=h.device)
        dist.all_gather_into_tensor(out, h, group=group)
        hs = out.cpu().view(self.n, 64)
        self.peers = [self.ptr if j == self.rank else ext().symm_open(hs[j].clone())
                      for j in range(self.n)]

    def tensor(self, offset_bytes: int, shape, dtype=torch.float32) -> torch.Tensor:
        """A view of this rank's copy starting ``offset_bytes`` in."""
        return ext().tensor_from_ptr(self.ptr + int(offset_bytes), list(shape), dtype, self.device)

    def close(self) -> None:
        if self.ptr is None:
            return
        for j, p in enumerate(self.peers):
            if j != self.rank:
                ext().symm_close(p)
        ext().symm_free(self.ptr)
        self.ptr = None
