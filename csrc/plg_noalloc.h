// C entry point of pluggy_b200 that allocates no device memory.
//
// This interface has no counterpart in the reference (which computes gradient
// norms with torch._foreach_norm and lets the caching allocator hold every
// temporary). It exists for callers that must not allocate device memory: a C or
// C++ host runtime that drives the framework's kernels without owning an
// allocator, and an out-of-memory recovery path that still has to measure the
// gradient norm after the allocator has refused a request.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest supported total_chunks (one 64K-element chunk of the input tensors per
// slot of the file-scope scratch array): 65536 chunks = 4.29e9 elements; the
// scratch is 256 KiB of device memory reserved when the library is loaded.
#define PLG_NOALLOC_MAX_CHUNKS 65536

// Sum of squares of every element of a list of fp32 tensors, written as one fp32
// value to *total_out (device memory owned by the caller).
//
// table:        device int64 [ntensors][7], rows (ptr, 0, 0, 0, 0, numel, first
//               chunk) in the layout of the framework's multi-tensor optimizer
//               table (chunks of 65536 elements, first chunk = running sum of
//               ceil(numel / 65536) over the preceding rows).
// total_chunks: sum of ceil(numel / 65536) over all rows.
// stream:       a cudaStream_t (passed as void*); the call only enqueues work.
//
// Per-chunk partial sums go to a file-scope __device__ scratch array; every slot
// that is read is written by the same call first, so nothing in it has to start
// at zero and total_out need not be cleared. Because the scratch is shared,
// calls that overlap on the device (other streams, other host threads, without
// ordering between them) race on it: serialize them on one stream.
// The first call on each device looks up the scratch address with
// cudaGetSymbolAddress (no allocation); make that first call before any
// work on the device that must not see a runtime setup call.
//
// Returns 0 on success; 1 if total_chunks exceeds PLG_NOALLOC_MAX_CHUNKS, is
// negative, or is positive with ntensors < 1 (nothing enqueued); 2 on a CUDA
// runtime error. A CUDA error that is already pending on the calling thread when
// the call starts is reported as 2 and left pending (cudaPeekAtLastError), with
// nothing enqueued. A nonzero return also prints one line naming the problem to
// stderr.
int plg_multi_sumsq_noalloc(const int64_t* table, int ntensors, long long total_chunks,
                            float* total_out, void* stream);

#ifdef __cplusplus
}
#endif
