"""Loader for the in-tree sm_100a extension ``pluggy_b200._C``.

On a CUDA device every op in ``pluggy_b200.ops`` runs through this extension;
if it is missing the op raises immediately instead of falling back to eager
PyTorch, so a GPU run can never silently measure a library path. The extension
is built in-tree by ``python setup.py build_ext --inplace`` (or
``__graft_entry__.build()``).

A per-device int32 status word is shared by every kernel that has bounded
waits; ``check_status()`` raises if any of them timed out. The deadline of the
collective kernels' waits on a peer's flag is 2 s by default and is set per
device with ``set_peer_wait_deadline()``.
"""

from __future__ import annotations

import importlib

import torch

_C = None
_ERR: Exception | None = None
_STATUS: dict[int, torch.Tensor] = {}

_STATUS_NAMES = {
    1: "MMA warp timed out waiting for a TMA stage",
    2: "TMA producer timed out waiting for a free shared-memory stage",
    3: "epilogue timed out waiting for an accumulator",
    4: "MMA warp timed out waiting for the epilogue",
    5: "fused collective timed out waiting for a peer",
    6: "kernel unwinding timed out waiting for its in-flight copies",
    7: "bad kernel argument",
    8: "a peer-memory store was outside its destination buffer and was skipped",
}


def ext():
    """Return the compiled extension module or raise with the build hint."""
    global _C, _ERR
    if _C is not None:
        return _C
    if _ERR is None:
        try:
            _C = importlib.import_module("pluggy_b200._C")
            return _C
        except Exception as e:  # pragma: no cover - depends on the build
            _ERR = e
    raise RuntimeError(
        "pluggy_b200._C (the sm_100a kernels) is not built or failed to load: "
        f"{_ERR!r}. Run `python setup.py build_ext --inplace` in the repository root."
    )


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def status_word(device: torch.device | None = None) -> torch.Tensor:
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def check_status(device: torch.device | None = None, reset: bool = True) -> None:
    """Raise if any bounded wait in a kernel on ``device`` gave up (synchronises)."""
    t = status_word(device)
    code = int(t.item())
    if code:
        if reset:
            t.zero_()
        raise RuntimeError(f"sm_100a kernel reported status {code}: "
                           f"{_STATUS_NAMES.get(code, 'unknown')}")


DEFAULT_PEER_WAIT_S = 2.0


def set_peer_wait_deadline(seconds: float, device: torch.device | None = None) -> None:
    """Deadline of every wait on a peer's flag in the collective kernels of ``device``
    (kernels launched after the call on the current stream use it)."""
    ns = int(seconds * 1e9)
    if ns <= 0:
        raise ValueError("the deadline must be positive")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        ext().set_peer_wait_deadline(ns)
