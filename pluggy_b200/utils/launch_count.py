"""Counts this package's kernel launches (for the benchmark's ``gpu_launches`` claim).

Wraps the extension module so every binding call adds the number of kernels
that binding launches (fixed per binding; GEMM adds its split-K memset, the
attention backward its pre/post passes).
"""

from __future__ import annotations

import contextlib

from pluggy_b200.ops import _ext

# kernels launched per binding call (memsets included)
KERNELS_PER_CALL = {
    "gemm": 1, "rmsnorm_fwd": 1, "rmsnorm_bwd": 1, "qk_norm_rope_fwd": 1, "qk_norm_rope_bwd": 1,
    "glu_fwd": 1, "glu_bwd": 1, "cast_f32_bf16": 1, "embedding_fwd": 1, "embedding_bwd": 1,
    "softcap": 1, "ce_rows": 1, "multi_sumsq": 2, "multi_scale": 1, "adamw_multi": 1,
    "attn_fwd": 1, "attn_bwd": 4,
}


class _Counting:
    def __init__(self, mod):
        self._mod = mod
        self.count = 0
        self.by_name: dict[str, int] = {}

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def wrapped(*a, **k):
            n = KERNELS_PER_CALL.get(name, 1)
            self.count += n
            self.by_name[name] = self.by_name.get(name, 0) + n
            return fn(*a, **k)

        return wrapped


@contextlib.contextmanager
def count_launches():
    real = _ext.ext()
    counter = _Counting(real)
    _ext._C = counter
    try:
        yield counter
    finally:
        _ext._C = real
