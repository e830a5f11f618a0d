"""The allocation-free C entry point (csrc/plg_noalloc.h) against the regular
multi-tensor sum of squares; collected last so it also runs after every other test."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_CHUNKS = 65536


def _lib():
    import pluggy_b200._C as ext_mod

    lib = ctypes.CDLL(ext_mod.__file__)
    fn = lib.plg_multi_sumsq_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _table(tensors):
    from pluggy_b200.ops.optim import _table

    return _table([[t.data_ptr(), 0, 0, 0, 0] for t in tensors], [t.numel() for t in tensors],
                  tensors[0].device)


def test_noalloc_sumsq_matches_entry_point():
    from pluggy_b200.ops.optim import multi_tensor_sumsq

    torch.manual_seed(0)
    ts = [torch.randn(n, device="cuda") for n in (1, 1000, 65536, 65537, 3 * 65536 + 5, 4096 * 7)]
    table, chunks = _table(ts)
    ref = multi_tensor_sumsq(ts)
    fn = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):  # two consecutive calls reuse the same scratch
        out = torch.full((1,), float("nan"), device="cuda")
        assert fn(table.data_ptr(), len(ts), chunks, out.data_ptr(), stream) == 0
        outs.append(out)
    torch.cuda.synchronize()
    exact = sum(float(t.double().pow(2).sum()) for t in ts)
    for out in outs:
        assert torch.allclose(out[0], ref, rtol=1e-5, atol=0)
        assert abs(float(out[0]) - exact) / exact < 1e-5


def test_noalloc_sumsq_rejects_oversize():
    fn = _lib()
    out = torch.full((1,), 7.0, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert fn(0, 1, MAX_CHUNKS + 1, out.data_ptr(), stream) == 1
    assert fn(0, 1, -1, out.data_ptr(), stream) == 1
    torch.cuda.synchronize()
    assert float(out[0]) == 7.0  # nothing was enqueued


def test_noalloc_sumsq_zero_chunks_writes_zero():
    """No chunks: the total is written as 0 (the NaN fill must not survive)."""
    fn = _lib()
    out = torch.full((1,), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert fn(0, 0, 0, out.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    assert float(out[0]) == 0.0


def test_noalloc_sumsq_at_scratch_limit():
    """Exactly PLG_NOALLOC_MAX_CHUNKS chunks (every scratch slot used): 1024 table
    rows share one 64-chunk storage, so the table reaches the limit with 16 MB."""
    from pluggy_b200.ops.optim import multi_tensor_sumsq

    torch.manual_seed(1)
    base = torch.randn(64 * 65536, device="cuda")
    ts = [base] * (MAX_CHUNKS // 64)
    table, chunks = _table(ts)
    assert chunks == MAX_CHUNKS
    ref = multi_tensor_sumsq(ts)
    fn = _lib()
    out = torch.full((1,), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert fn(table.data_ptr(), len(ts), chunks, out.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    assert torch.allclose(out[0], ref, rtol=1e-5, atol=0)
    exact = len(ts) * float(base.double().pow(2).sum())
    assert abs(float(out[0]) - exact) / exact < 1e-5


def test_noalloc_sumsq_rejects_empty_table():
    fn = _lib()
    out = torch.full((1,), 7.0, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert fn(0, 0, 5, out.data_ptr(), stream) == 1
    torch.cuda.synchronize()
    assert float(out[0]) == 7.0
