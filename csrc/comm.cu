// Collectives as sm_100a kernels over NVLink peer memory.
//
// Symmetric memory: every rank allocates the same-size buffer with cudaMalloc and
// exports a CUDA IPC handle; the Python side exchanges the handles over the
// process group and opens the peers' buffers here, so a kernel can load and store
// any rank's buffer directly (NVLink 5 / NVSwitch P2P).
//
// Fused data-parallel gradient reduction (replaces the reference's
// all_reduce(op="avg") of each DDP bucket, pluggy/parallelism/data_parallel.py:120-130,
// plus the grad-norm pass of pluggy/core/grad_helper.py:17-33): the bucket lives in
// the symmetric buffer; the range is split into n segments (one per owning rank)
// of C chunks (one per CTA). CTA c of rank r
//   1. tells every peer its copy of the bucket is ready (flag store, release, system scope),
//      then waits (bounded) until every peer's CTA c said the same;
//   2. sums chunk c of segment r over all ranks' copies (P2P loads), scales by
//      1/n, accumulates the sum of squares of the result;
//   3. stores the averaged chunk into every rank's copy (P2P stores) and its
//      sum of squares into every rank's slot table, then signals "done";
//   4. waits (bounded) for every peer's "done" of chunk c, i.e. until chunk c of
//      every segment has been written into this rank's copy.
// A CTA only ever waits for the CTA of the same index on other GPUs, and signals
// before it waits, so no scheduling order can deadlock. Flags hold a monotonically
// increasing epoch (no reset between launches). A wait that runs out of time
// records a status code and returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <type_traits>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "ops.h"

namespace plg {
namespace comm {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Deadline of every wait on a peer's flag, per device (default 2 s). The host
// changes it with set_peer_wait_deadline_ns(): a test shortens it to make a wait
// whose flag is never posted run out quickly; a job with very uneven ranks can
// lengthen it.
__device__ uint64_t g_peer_wait_deadline_ns = kWaitDeadlineNs;

// wait until *p >= want (flags only grow); false after the deadline
__device__ __forceinline__ bool wait_flag(const uint32_t* p, uint32_t want) {
  if (static_cast<int32_t>(ld_acquire_sys(p) - want) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t deadline = *reinterpret_cast<volatile uint64_t*>(&g_peer_wait_deadline_ns);
  uint32_t spins = 0;
  while (true) {
    if (static_cast<int32_t>(ld_acquire_sys(p) - want) >= 0) return true;
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > deadline) return false;
  }
}

__global__ void __launch_bounds__(512) allreduce_avg_kernel(SymmAllReduceArgs a) {
  const int c = blockIdx.x, n = a.nranks, me = a.rank;
  const uint32_t e_ready = 2u * a.epoch + 1u, e_done = 2u * a.epoch + 2u;
  __shared__ int s_ok;
  // 1. ready handshake with CTA c of every peer
  if (threadIdx.x < n) {
    const int p = threadIdx.x;
    st_release_sys(a.flags[p] + (0 * kSymmMaxRanks + me) * kSymmMaxChunks + c, e_ready);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int p = 0; p < n && ok; ++p)
      ok = wait_flag(a.flags[me] + (0 * kSymmMaxRanks + p) * kSymmMaxChunks + c, e_ready);
    if (!ok) record_status(a.status, kTimeoutPeerFlag);
    s_ok = ok;
  }
  __syncthreads();
  float ss = 0.f;
  if (s_ok) {
    // 2./3. reduce chunk c of my segment over all copies; write it back everywhere
    const long long seg = (a.numel + n - 1) / n;
    const long long s0 = me * seg, s1 = min(a.numel, s0 + seg);
    const long long per = ((s1 - s0 + a.chunks - 1) / a.chunks + 3) & ~3LL;  // multiple of 4
    const long long c0 = s0 + c * per, c1 = min(s1, c0 + per);
    const float inv = 1.f / n;
    const long long v0 = (c0 + 3) & ~3LL;  // float4-aligned interior (buffers are 16B aligned)
    const long long v1 = max(v0, c1 & ~3LL);
    for (long long i = c0 + threadIdx.x; i < min(v0, c1); i += blockDim.x) {
      float acc = 0.f;
      for (int p = 0; p < n; ++p) acc += a.data[p][a.offset + i];
      acc *= inv;
      ss += acc * acc;
      for (int p = 0; p < n; ++p) a.data[p][a.offset + i] = acc;
    }
    for (long long i = v0 + 4LL * threadIdx.x; i < v1; i += 4LL * blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int p = 0; p < n; ++p) {
        const float4 x = *reinterpret_cast<const float4*>(a.data[p] + a.offset + i);
        acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
      }
      acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
      ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
#pragma unroll 8
      for (int p = 0; p < n; ++p) *reinterpret_cast<float4*>(a.data[p] + a.offset + i) = acc;
    }
    for (long long i = v1 + threadIdx.x; i < c1; i += blockDim.x) {
      float acc = 0.f;
      for (int p = 0; p < n; ++p) acc += a.data[p][a.offset + i];
      acc *= inv;
      ss += acc * acc;
      for (int p = 0; p < n; ++p) a.data[p][a.offset + i] = acc;
    }
  }
  // chunk sum of squares into every rank's slot table
  ss = warp_sum(ss);
  __shared__ float s_red[16];
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_red[w];
    for (int p = 0; p < n; ++p) a.sumsq[p][me * kSymmMaxChunks + c] = t;
  }
  __syncthreads();
  // 3. done: my chunk c of segment `me` is in every copy
  if (threadIdx.x == 0) __threadfence_system();
  __syncthreads();
  if (threadIdx.x < n) {
    const int p = threadIdx.x;
    st_release_sys(a.flags[p] + (1 * kSymmMaxRanks + me) * kSymmMaxChunks + c, e_done);
  }
  // 4. chunk c of every segment has arrived here
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int p = 0; p < n && ok; ++p)
      ok = wait_flag(a.flags[me] + (1 * kSymmMaxRanks + p) * kSymmMaxChunks + c, e_done);
    if (!ok) record_status(a.status, kTimeoutPeerFlag);
  }
}

// ------------------------------------------------------------------- ZeRO-1
// Data parallelism with the optimizer state sharded (ZeRO stage 1) and the two
// halves of the gradient all-reduce split around the optimizer:
//   zero1_rs_kernel (per bucket, during backward): CTA c of rank r averages chunk
//     c of r's slice over every rank's grad arena (peer loads) into r's own arena,
//     sums the squares of the result (the clip's norm) into every rank's slot table;
//   zero1_adamw_ag_kernel (per bucket, after the global norm is known): AdamW on
//     r's slice with r's optimizer state, the new fp32 params stored into every
//     rank's param arena (peer stores).
// Both follow the allreduce_avg_kernel protocol: CTA c signals before it waits and
// only ever waits for CTA c of the peers; flags carry per-kind epochs.
__device__ __forceinline__ void zero1_slice(long long numel, int n, int r, long long& s0,
                                            long long& s1) {
  const long long seg = ((numel + n - 1) / n + 3) & ~3LL;
  s0 = min(numel, static_cast<long long>(r) * seg);
  s1 = min(numel, s0 + seg);
}

__device__ __forceinline__ uint32_t* zero1_flag(const Zero1Args& a, int table, int kind, int src, int c) {
  return a.flags[table] + (kind * kSymmMaxRanks + src) * kSymmMaxChunks + c;
}

// signal kind `kind` of chunk c to every rank, then wait for every rank's; false on timeout
__device__ bool zero1_handshake(const Zero1Args& a, int kind) {
  __shared__ int s_ok;
  const int c = blockIdx.x;
  if (threadIdx.x < a.nranks) st_release_sys(zero1_flag(a, threadIdx.x, kind, a.rank, c), a.epoch);
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int p = 0; p < a.nranks && ok; ++p) ok = wait_flag(zero1_flag(a, a.rank, kind, p, c), a.epoch);
    if (!ok) record_status(a.status, kTimeoutPeerFlag);
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

__device__ __forceinline__ void zero1_chunk(const Zero1Args& a, long long& c0, long long& c1,
                                            long long& s0) {
  long long s1;
  zero1_slice(a.numel, a.nranks, a.rank, s0, s1);
  const long long per = ((s1 - s0 + a.chunks - 1) / a.chunks + 3) & ~3LL;
  c0 = min(s1, s0 + blockIdx.x * per);
  c1 = min(s1, c0 + per);
}

__global__ void __launch_bounds__(1024) zero1_rs_kernel(Zero1Args a) {
  const int n = a.nranks, me = a.rank, c = blockIdx.x;
  const bool ok = zero1_handshake(a, 0);
  float ss = 0.f;
  if (ok) {
    long long c0, c1, s0;
    zero1_chunk(a, c0, c1, s0);
    const float inv = 1.f / n;
    const long long v1 = c0 + ((c1 - c0) & ~3LL);  // c0 is a multiple of 4: float4 body
    float* mine = a.grads[me] + a.offset;
    for (long long i = c0 + 4LL * threadIdx.x; i < v1; i += 4LL * blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int p = 0; p < n; ++p) {  // fixed rank order: deterministic sums
        const float4 x = *reinterpret_cast<const float4*>(a.grads[p] + a.offset + i);
        acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
      }
      acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
      ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
      *reinterpret_cast<float4*>(mine + i) = acc;
    }
    for (long long i = v1 + threadIdx.x; i < c1; i += blockDim.x) {
      float acc = 0.f;
      for (int p = 0; p < n; ++p) acc += a.grads[p][a.offset + i];
      acc *= inv;
      ss += acc * acc;
      mine[i] = acc;
    }
  }
  ss = warp_sum(ss);
  __shared__ float s_red[32];
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_red[w];
    for (int p = 0; p < n; ++p) a.sumsq[p][me * kSymmMaxChunks + c] = t;
    __threadfence_system();
  }
  __syncthreads();
  // done: this CTA has read chunk c of its slice from every copy (peers may reuse
  // their grad arenas) and published its sum of squares
  zero1_handshake(a, 1);
}

__device__ __forceinline__ int zero1_group(const int64_t* rows, int nrows, long long i, int& r) {
  while (r + 1 < nrows && rows[3 * r + 1] <= i) ++r;
  return static_cast<int>(rows[3 * r + 2]);
}

__global__ void __launch_bounds__(1024) zero1_adamw_ag_kernel(Zero1Args a, Zero1Adam h) {
  const int n = a.nranks, me = a.rank;
  long long c0, c1, s0;
  zero1_chunk(a, c0, c1, s0);
  const float scale = h.grad_scale ? *h.grad_scale : 1.f;
  const float b1 = h.beta1, b2 = h.beta2, eps = h.eps;
  const float rbc2 = rsqrtf(h.bc2);
  const float* g = a.grads[me] + a.offset;
  const float* pin = a.params[me] + a.offset;
  int r = 0;
  const long long v1 = c0 + ((c1 - c0) & ~3LL);
  for (long long i = c0 + 4LL * threadIdx.x; i < v1; i += 4LL * blockDim.x) {
    float4 pp = *reinterpret_cast<const float4*>(pin + i);
    const float4 gg = *reinterpret_cast<const float4*>(g + i);
    float* const mp = h.exp_avg + (i - s0);  // slice state is indexed from the slice start
    float* const vp = h.exp_avg_sq + (i - s0);
    float4 mm = *reinterpret_cast<const float4*>(mp);
    float4 vv = *reinterpret_cast<const float4*>(vp);
    float* P = &pp.x; const float* G = &gg.x; float* M = &mm.x; float* W = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // a param boundary may fall inside the vector
      const int grp = zero1_group(h.rows, h.nrows, i + j, r);
      const float lr = h.lr[grp];
      adamw_update(P[j], M[j], W[j], G[j] * scale, 1.f - lr * h.wd[grp], b1, b2, lr / h.bc1, rbc2, eps);
    }
    *reinterpret_cast<float4*>(mp) = mm;
    *reinterpret_cast<float4*>(vp) = vv;
    for (int k = 0; k < n; ++k) {  // rotated: rank r starts with itself
      int q = me + k;
      q = q >= n ? q - n : q;
      *reinterpret_cast<float4*>(a.params[q] + a.offset + i) = pp;
    }
  }
  for (long long i = v1 + threadIdx.x; i < c1; i += blockDim.x) {
    float pj = pin[i], mj = h.exp_avg[i - s0], vj = h.exp_avg_sq[i - s0];
    const int grp = zero1_group(h.rows, h.nrows, i, r);
    const float lr = h.lr[grp];
    adamw_update(pj, mj, vj, g[i] * scale, 1.f - lr * h.wd[grp], b1, b2, lr / h.bc1, rbc2, eps);
    h.exp_avg[i - s0] = mj;
    h.exp_avg_sq[i - s0] = vj;
    for (int q = 0; q < n; ++q) a.params[q][a.offset + i] = pj;
  }
  __threadfence_system();
  __syncthreads();
  // done: chunk c of this rank's slice is in every arena; wait for the peers' chunk c
  zero1_handshake(a, 2);
}

// total = sum of the [nranks][chunks] slot table (fixed order: deterministic)
__global__ void sumsq_total_kernel(const float* __restrict__ slots, int nranks, int chunks,
                                   float* __restrict__ out, int accumulate) {
  __shared__ double s[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < nranks * chunks; i += blockDim.x)
    acc += slots[(i / chunks) * kSymmMaxChunks + (i % chunks)];
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s[w];
    out[0] = (accumulate ? out[0] : 0.f) + static_cast<float>(t);
  }
}

// ------------------------------------------------------------ tensor parallel
// Rows are [B, S] flattened; with n ranks each owns seg = S / n positions of every
// sequence. Row (b, s) -> owner s / seg, local row b * seg + s % seg.
struct TpMap {
  long long S, seg, rows;  // rows = B * seg per rank
  __device__ __forceinline__ void split(long long row, int& owner, long long& lrow) const {
    const long long b = row / S, s = row - b * S;
    owner = static_cast<int>(s / seg);
    lrow = b * seg + (s - owner * seg);
  }
  __device__ __forceinline__ long long join(int owner, long long lrow) const {
    const long long b = lrow / seg;
    return b * S + owner * seg + (lrow - b * seg);
  }
};

__device__ __forceinline__ const void* tp_buf(const TpArgs& a, int j) {
  const void* p = a.bufs[0];
#pragma unroll
  for (int i = 1; i < kSymmMaxRanks; ++i)
    if (j == i) p = a.bufs[i];
  return p;
}

// 16-byte store into a peer's buffer at index `i16` (16-byte units), skipped (and
// reported) when it would leave the buffer
__device__ __forceinline__ void peer_store16(const TpArgs& a, int p, long long i16, uint4 v) {
  if (i16 < 0 || i16 >= a.cap16) {
    record_status(a.status, kOutOfBounds);
    return;
  }
  reinterpret_cast<uint4*>(const_cast<void*>(tp_buf(a, p)))[i16] = v;
}

__device__ __forceinline__ uint32_t* tp_flag(const TpArgs& a, int j) {
  uint32_t* p = a.flags[0];
#pragma unroll
  for (int i = 1; i < kSymmMaxRanks; ++i)
    if (j == i) p = a.flags[i];
  return p;
}

// every CTA: publish "this rank's part of call `epoch` is in place" to each peer
// (idempotent), then wait for every peer's; false (status recorded) on timeout
__device__ bool tp_handshake(const TpArgs& a, int kind) {
  __shared__ int s_ok;
  if (threadIdx.x < a.n) {
    __threadfence_system();
    st_release_sys(tp_flag(a, threadIdx.x) + kind * kSymmMaxRanks + a.rank, a.epoch);
  }
  if (threadIdx.x == 0) {
    int ok = 1;
    uint32_t* mine = tp_flag(a, a.rank) + kind * kSymmMaxRanks;
    for (int p = 0; p < a.n && ok; ++p) ok = wait_flag(mine + p, a.epoch);
    if (!ok) record_status(a.status, kTimeoutPeerFlag);
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

__global__ void __launch_bounds__(256) tp_rs_push_kernel(TpArgs a, const __nv_bfloat16* __restrict__ part,
                                                         long long ld) {
  const TpMap m{a.S, a.S / a.n, a.B * (a.S / a.n)};
  const long long g8 = a.W / 8, per = m.rows * g8, total = a.n * per;
  // owners in rotated order (rank r starts with owner r): the ranks' writes spread
  // over all links instead of all converging on one owner at a time
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(g / per);
    const int owner = (a.rank + i) % a.n;
    const long long rem = g - i * per;
    const long long lrow = rem / g8, c = (rem - lrow * g8) * 8;
    const long long row = m.join(owner, lrow);
    const uint4 v = *reinterpret_cast<const uint4*>(part + row * ld + c);
    peer_store16(a, owner, ((a.rank * m.rows + lrow) * a.W + c) / 8, v);
  }
  __threadfence_system();
}

__global__ void __launch_bounds__(256) tp_rs_finish_kernel(TpArgs a, __nv_bfloat16* __restrict__ out,
                                                           long long ld_out) {
  if (!tp_handshake(a, 0)) return;
  const long long rows = a.B * (a.S / a.n), g8 = a.W / 8, total = rows * g8;
  const __nv_bfloat16* st = reinterpret_cast<const __nv_bfloat16*>(tp_buf(a, a.rank));
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = g / g8;
    const long long c = (g - r * g8) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int p = 0; p < a.n; ++p) {  // fixed order: deterministic
      const uint4 v = *reinterpret_cast<const uint4*>(st + (p * rows + r) * a.W + c);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(u[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + r * ld_out + c) = o;
  }
}

// AG: this rank's shard rows go into slot `rank` of EVERY rank's receive buffer
// (peer stores are posted over NVLink: pushing beats pulling with loads)
__global__ void __launch_bounds__(256) tp_ag_push_kernel(TpArgs a, const __nv_bfloat16* __restrict__ shard,
                                                         long long ld) {
  const long long rows = a.B * (a.S / a.n), g8 = a.W / 8, total = rows * g8;
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = g / g8;
    const long long c = (g - r * g8) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(shard + r * ld + c);
    for (int p = 0; p < a.n; ++p)
      peer_store16(a, (a.rank + p) % a.n, ((a.rank * rows + r) * a.W + c) / 8, v);
  }
  __threadfence_system();
}

// AG: signal, wait for every peer's push, then copy the n slots into [B, S] order
__global__ void __launch_bounds__(256) tp_ag_finish_kernel(TpArgs a, __nv_bfloat16* __restrict__ out,
                                                           long long ld_out) {
  if (!tp_handshake(a, 1)) return;
  const TpMap m{a.S, a.S / a.n, a.B * (a.S / a.n)};
  const long long g8 = a.W / 8, per = m.rows * g8, total = a.n * per;
  const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(tp_buf(a, a.rank));
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(g / per);
    const long long rem = g - p * per;
    const long long lrow = rem / g8, c = (rem - lrow * g8) * 8;
    *reinterpret_cast<uint4*>(out + m.join(p, lrow) * ld_out + c) =
        *reinterpret_cast<const uint4*>(rb + (p * m.rows + lrow) * a.W + c);
  }
}

// ------------------------------------------------ RMSNorm fused with the AG push
// One CTA per row at a time, W / 8 threads, 8 channels (one 16-byte bf16 chunk) per
// thread: the norm's output never lands in local memory, each thread stores its
// chunk into every rank's receive slot (a warp writes 512 contiguous bytes).
template <typename TX>
__global__ void __launch_bounds__(1024) tp_norm_ag_push_kernel(TpArgs a, const TX* __restrict__ x,
                                                               long long ld, const float* __restrict__ w,
                                                               float eps, float* __restrict__ rstd_out) {
  __shared__ float s_red[32];
  const long long rows = a.B * (a.S / a.n);
  const int c0 = threadIdx.x * 8;
  float wv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) wv[k] = w ? w[c0 + k] : 1.f;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    float v[8];
    if constexpr (std::is_same<TX, float>::value) {
      const float4 u0 = *reinterpret_cast<const float4*>(x + r * ld + c0);
      const float4 u1 = *reinterpret_cast<const float4*>(x + r * ld + c0 + 4);
      v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
      v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
    } else {
      const uint4 u = *reinterpret_cast<const uint4*>(x + r * ld + c0);
      const uint32_t* uu = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(uu[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += v[k] * v[k];
    ss = warp_sum(ss);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    if (warp == 0) {
      float t = lane < nw ? s_red[lane] : 0.f;
      t = warp_sum(t);
      if (lane == 0) s_red[0] = t;
    }
    __syncthreads();
    const float rs = rsqrtf(s_red[0] / a.W + eps);
    __syncthreads();  // s_red is reused by the next row
    if (threadIdx.x == 0 && rstd_out) rstd_out[r] = rs;
    uint4 o;
    o.x = pack_bf16x2(v[0] * rs * wv[0], v[1] * rs * wv[1]);
    o.y = pack_bf16x2(v[2] * rs * wv[2], v[3] * rs * wv[3]);
    o.z = pack_bf16x2(v[4] * rs * wv[4], v[5] * rs * wv[5]);
    o.w = pack_bf16x2(v[6] * rs * wv[6], v[7] * rs * wv[7]);
    const long long dst16 = ((a.rank * rows + r) * a.W + c0) / 8;
    for (int p = 0; p < a.n; ++p) peer_store16(a, (a.rank + p) % a.n, dst16, o);
  }
  __threadfence_system();
}

// ------------------------------------------------------------- expert parallel
__global__ void __launch_bounds__(256) ep_push_kernel(TpArgs a, EpSegs sg, const __nv_bfloat16* __restrict__ src,
                                                      long long ld) {
  const long long g8 = a.W / 8;
  long long total = 0;
  for (int p = 0; p < a.n; ++p) total += sg.count[p] * g8;
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    // segments in rotated order (rank r starts with peer r), so the ranks' writes
    // spread over all links instead of converging on one peer at a time
    long long rem = g;
    int p = -1;
    long long start = 0, off = 0;
#pragma unroll
    for (int i = 0; i < kSymmMaxRanks; ++i) {
      if (i < a.n && p < 0) {
        int q = a.rank + i;
        q = q >= a.n ? q - a.n : q;
        long long cnt = 0, st0 = 0, of0 = 0;
#pragma unroll
        for (int j = 0; j < kSymmMaxRanks; ++j)  // static indices: no local-memory copy
          if (j == q) {
            cnt = sg.count[j];
            st0 = sg.src_start[j];
            of0 = sg.dst_off[j];
          }
        const long long seg = cnt * g8;
        if (rem < seg) {
          p = q;
          start = st0;
          off = of0;
        } else {
          rem -= seg;
        }
      }
    }
    const long long k = rem / g8, c = (rem - k * g8) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(src + (start + k) * ld + c);
    peer_store16(a, p, ((off + k) * a.W + c) / 8, v);
  }
  __threadfence_system();
}

__global__ void __launch_bounds__(256) ep_finish_kernel(TpArgs a, int kind, __nv_bfloat16* __restrict__ out,
                                                        long long rows, long long ld_out) {
  if (!tp_handshake(a, kind)) return;
  const long long g8 = a.W / 8, total = rows * g8;
  const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(tp_buf(a, a.rank));
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = g / g8, c = (g - r * g8) * 8;
    *reinterpret_cast<uint4*>(out + r * ld_out + c) = *reinterpret_cast<const uint4*>(rb + r * a.W + c);
  }
}

// ------------------------------------------------------------------ FSDP gather
// FSDP gradient reduce-scatter (see ops.h): CTA c reduces chunk c of the rank's flat
// shard after a ready handshake with CTA c of every peer, then signals done (peers
// may refill their staging slot) and waits for the peers' done.
__device__ bool fsdp_rs_handshake(const FsdpRsArgs& a, int kind) {
  __shared__ int s_ok;
  const int c = blockIdx.x;
  if (threadIdx.x < a.nranks)
    st_release_sys(a.flags[threadIdx.x] + (kind * kSymmMaxRanks + a.rank) * kSymmMaxChunks + c, a.epoch);
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int p = 0; p < a.nranks && ok; ++p)
      ok = wait_flag(a.flags[a.rank] + (kind * kSymmMaxRanks + p) * kSymmMaxChunks + c, a.epoch);
    if (!ok) record_status(a.status, kTimeoutPeerFlag);
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

__global__ void __launch_bounds__(1024) fsdp_rs_kernel(FsdpRsArgs a) {
  if (fsdp_rs_handshake(a, 0)) {
    const long long per = ((a.shard_numel + a.chunks - 1) / a.chunks + 3) & ~3LL;
    const long long c0 = min(a.shard_numel, blockIdx.x * per), c1 = min(a.shard_numel, c0 + per);
    int r = 0;
    for (long long s4 = c0 + 4LL * threadIdx.x; s4 < c1; s4 += 4LL * blockDim.x) {
      while (r + 1 < a.k && a.table[3 * (r + 1)] <= s4) ++r;
      const int64_t* row = a.table + 3 * r;
      const long long full = row[1] + a.rank * row[2] + (s4 - row[0]);  // 4-aligned: one row
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int p = 0; p < a.nranks; ++p) {  // fixed rank order: deterministic
        const float4 v = *reinterpret_cast<const float4*>(a.stage[p] + full);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      float4* o = reinterpret_cast<float4*>(a.out + s4);
      float4 prev = a.accumulate ? *o : make_float4(0.f, 0.f, 0.f, 0.f);
      prev.x += acc.x * a.scale; prev.y += acc.y * a.scale;
      prev.z += acc.z * a.scale; prev.w += acc.w * a.scale;
      *o = prev;
    }
  }
  __syncthreads();
  fsdp_rs_handshake(a, 1);
}

// Low-precision unit gather: every rank pushes its fp32 parameter shards into every
// rank's slot of the unit, matrices cast to bf16 on the way (half the NVLink bytes),
// vectors kept fp32. table [k][5] int64: first 16-byte destination group of the row
// (running sum), source offset in the fp32 shard (elements), destination offset of
// the parameter in the slot (16-byte units), this rank's shard length (16-byte
// destination units), kind (0: bf16, 1: fp32). The rank's shard of parameter i lands
// at dst_off16_i + rank * len16_i.
__global__ void __launch_bounds__(256) fsdp_push_lowp_kernel(TpArgs a, const int64_t* __restrict__ table,
                                                             int k, long long total16,
                                                             const float* __restrict__ shard) {
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < total16;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    int i = 0;
    while (i + 1 < k && table[5 * (i + 1)] <= g) ++i;
    const int64_t* r = table + 5 * i;
    const long long local = g - r[0];
    uint4 v;
    if (r[4] == 0) {
      const float4* src = reinterpret_cast<const float4*>(shard + r[1] + local * 8);
      const float4 x0 = src[0], x1 = src[1];
      v = make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w), pack_bf16x2(x1.x, x1.y),
                     pack_bf16x2(x1.z, x1.w));
    } else {
      v = *reinterpret_cast<const uint4*>(shard + r[1] + local * 4);
    }
    const long long dst = r[2] + a.rank * r[3] + local;
    for (int p = 0; p < a.n; ++p) {
      int q = a.rank + p;
      q = q >= a.n ? q - a.n : q;
      peer_store16(a, q, dst, v);
    }
  }
  __threadfence_system();
}

__global__ void __launch_bounds__(256) fsdp_push_kernel(TpArgs a, const int64_t* __restrict__ table, int k,
                                                        long long total16, const uint4* __restrict__ shard) {
  for (long long g = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; g < total16;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    // parameter of this 16-byte group (a unit has a handful of parameters)
    int i = 0;
    while (i + 1 < k && table[3 * (i + 1)] <= g) ++i;
    const long long local = g - table[3 * i];
    const long long dst = table[3 * i + 1] + a.rank * table[3 * i + 2] + local;
    const uint4 v = shard[g];
    for (int p = 0; p < a.n; ++p) {
      int q = a.rank + p;
      q = q >= a.n ? q - a.n : q;
      peer_store16(a, q, dst, v);
    }
  }
  __threadfence_system();
}

}  // namespace comm

void* symm_malloc(size_t bytes, void* ipc_handle_out) {
  void* p = nullptr;
  PLG_CUDA_CHECK(cudaMalloc(&p, bytes));
  PLG_CUDA_CHECK(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t h;
  PLG_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  return p;
}

void* symm_open(const void* ipc_handle) {
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  PLG_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}

void symm_close(void* peer_ptr) { PLG_CUDA_CHECK(cudaIpcCloseMemHandle(peer_ptr)); }

void symm_free(void* p) { PLG_CUDA_CHECK(cudaFree(p)); }

void symm_allreduce_avg(const SymmAllReduceArgs& a, float* norm_sq, bool accumulate_norm,
                        cudaStream_t st) {
  if (a.nranks < 1 || a.nranks > kSymmMaxRanks)
    throw std::invalid_argument("symm_allreduce_avg: 1..8 ranks");
  if (a.chunks < 1 || a.chunks > kSymmMaxChunks)
    throw std::invalid_argument("symm_allreduce_avg: chunks must be in 1..kSymmMaxChunks");
  if (a.offset % 4) throw std::invalid_argument("symm_allreduce_avg: offset must be a multiple of 4");
  if (a.numel > 0) {
    comm::allreduce_avg_kernel<<<a.chunks, 512, 0, st>>>(a);
    PLG_CUDA_CHECK(cudaGetLastError());
  }
  if (norm_sq != nullptr) {
    comm::sumsq_total_kernel<<<1, 256, 0, st>>>(a.sumsq[a.rank], a.nranks, a.chunks, norm_sq,
                                                accumulate_norm ? 1 : 0);
    PLG_CUDA_CHECK(cudaGetLastError());
  }
}

static void zero1_check(const Zero1Args& a, const char* what) {
  if (a.nranks < 1 || a.nranks > kSymmMaxRanks || a.rank < 0 || a.rank >= a.nranks)
    throw std::invalid_argument(std::string(what) + ": 1..8 ranks");
  if (a.chunks < 1 || a.chunks > kSymmMaxChunks)
    throw std::invalid_argument(std::string(what) + ": chunks must be in 1..kSymmMaxChunks");
  if (a.offset % 4 || a.numel < 0) throw std::invalid_argument(std::string(what) + ": offset must be a multiple of 4");
  for (int p = 0; p < a.nranks; ++p)
    if (a.grads[p] == nullptr || a.params[p] == nullptr || a.flags[p] == nullptr || a.sumsq[p] == nullptr ||
        (reinterpret_cast<uintptr_t>(a.grads[p]) & 15) || (reinterpret_cast<uintptr_t>(a.params[p]) & 15))
      throw std::invalid_argument(std::string(what) + ": every rank's 16-byte aligned arenas and tables");
}

void zero1_reduce_scatter(const Zero1Args& a, float* norm_sq, bool accumulate, cudaStream_t st) {
  zero1_check(a, "zero1_reduce_scatter");
  // launched also for an empty bucket: the handshakes keep the ranks' epochs in step
  comm::zero1_rs_kernel<<<a.chunks, 1024, 0, st>>>(a);
  PLG_CUDA_CHECK(cudaGetLastError());
  if (norm_sq != nullptr) {
    comm::sumsq_total_kernel<<<1, 256, 0, st>>>(a.sumsq[a.rank], a.nranks, a.chunks, norm_sq,
                                                accumulate ? 1 : 0);
    PLG_CUDA_CHECK(cudaGetLastError());
  }
}

void zero1_adamw_allgather(const Zero1Args& a, const Zero1Adam& h, cudaStream_t st) {
  zero1_check(a, "zero1_adamw_allgather");
  if (h.nrows < 1 || h.rows == nullptr || h.exp_avg == nullptr || h.exp_avg_sq == nullptr ||
      (reinterpret_cast<uintptr_t>(h.exp_avg) & 15) || (reinterpret_cast<uintptr_t>(h.exp_avg_sq) & 15))
    throw std::invalid_argument("zero1_adamw_allgather: a row table and 16-byte aligned slice state");
  comm::zero1_adamw_ag_kernel<<<a.chunks, 1024, 0, st>>>(a, h);
  PLG_CUDA_CHECK(cudaGetLastError());
}

static void tp_check(const TpArgs& a, long long ld, const void* p, const char* what) {
  if (a.n < 1 || a.n > kSymmMaxRanks || a.rank < 0 || a.rank >= a.n)
    throw std::invalid_argument(std::string(what) + ": 1..8 ranks");
  if (a.S % a.n || a.W % 8 || ld % 8 || (reinterpret_cast<uintptr_t>(p) & 15))
    throw std::invalid_argument(std::string(what) +
                                ": S divisible by ranks, width and row stride multiples of 8, 16-byte rows");
  for (int j = 0; j < a.n; ++j)
    if (a.flags[j] == nullptr || a.bufs[j] == nullptr || (reinterpret_cast<uintptr_t>(a.bufs[j]) & 15))
      throw std::invalid_argument(std::string(what) + ": every rank's flags and 16-byte aligned buffer");
}

static unsigned tp_grid(long long groups, int cap) {
  long long g = (groups + 255) / 256;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return static_cast<unsigned>(g);
}

void tp_rs_push(const TpArgs& a, const void* partial, long long ld, cudaStream_t st) {
  tp_check(a, ld, partial, "tp_rs_push");
  comm::tp_rs_push_kernel<<<tp_grid(a.B * a.S * (a.W / 8), 148 * 8), 256, 0, st>>>(
      a, reinterpret_cast<const __nv_bfloat16*>(partial), ld);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void tp_rs_finish(const TpArgs& a, void* out, long long ld_out, cudaStream_t st) {
  tp_check(a, ld_out, out, "tp_rs_finish");
  if (a.B * a.S * a.W / 8 > a.cap16)
    throw std::invalid_argument("tp_rs_finish: the staging buffer is smaller than the partial");
  comm::tp_rs_finish_kernel<<<tp_grid(a.B * (a.S / a.n) * (a.W / 8), 148 * 4), 256, 0, st>>>(
      a, reinterpret_cast<__nv_bfloat16*>(out), ld_out);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void tp_ag_push(const TpArgs& a, const void* shard, long long ld, cudaStream_t st) {
  tp_check(a, ld, shard, "tp_ag_push");
  comm::tp_ag_push_kernel<<<tp_grid(a.B * (a.S / a.n) * (a.W / 8), 148 * 4), 256, 0, st>>>(
      a, reinterpret_cast<const __nv_bfloat16*>(shard), ld);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void tp_ag_finish(const TpArgs& a, void* out, long long ld_out, cudaStream_t st) {
  tp_check(a, ld_out, out, "tp_ag_finish");
  if (a.B * a.S * a.W / 8 > a.cap16)
    throw std::invalid_argument("tp_ag_finish: the receive buffer is smaller than the gathered rows");
  comm::tp_ag_finish_kernel<<<tp_grid(a.B * a.S * (a.W / 8), 148 * 8), 256, 0, st>>>(
      a, reinterpret_cast<__nv_bfloat16*>(out), ld_out);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void ep_push(const TpArgs& a, const EpSegs& sg, const void* src, long long ld, cudaStream_t st) {
  if (a.n < 1 || a.n > kSymmMaxRanks || a.rank < 0 || a.rank >= a.n || a.W % 8 || ld % 8 ||
      (reinterpret_cast<uintptr_t>(src) & 15))
    throw std::invalid_argument("ep_push: 1..8 ranks, row width and stride multiples of 8, 16-byte rows");
  long long rows = 0;
  for (int p = 0; p < a.n; ++p) {
    if (sg.count[p] < 0 || sg.src_start[p] < 0 || sg.dst_off[p] < 0)
      throw std::invalid_argument("ep_push: negative segment");
    if (sg.count[p] > 0 && (a.bufs[p] == nullptr || (reinterpret_cast<uintptr_t>(a.bufs[p]) & 15)))
      throw std::invalid_argument("ep_push: every destination needs a 16-byte aligned buffer");
    rows += sg.count[p];
  }
  if (rows == 0) return;
  comm::ep_push_kernel<<<tp_grid(rows * (a.W / 8), 148 * 4), 256, 0, st>>>(
      a, sg, reinterpret_cast<const __nv_bfloat16*>(src), ld);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void ep_finish(const TpArgs& a, int kind, void* out, long long rows, long long ld_out, cudaStream_t st) {
  if (kind < 0 || kind >= kTpKinds) throw std::invalid_argument("ep_finish: flag kind out of range");
  if (rows > 0 && (ld_out % 8 || (reinterpret_cast<uintptr_t>(out) & 15)))
    throw std::invalid_argument("ep_finish: 16-byte aligned output rows");
  if (rows * a.W / 8 > a.cap16)
    throw std::invalid_argument("ep_finish: the receive buffer is smaller than the requested rows");
  for (int p = 0; p < a.n; ++p)
    if (a.flags[p] == nullptr) throw std::invalid_argument("ep_finish: every rank's flag table");
  // always launched, also with no rows to copy: the handshake keeps the ranks in step
  comm::ep_finish_kernel<<<tp_grid(rows * (a.W / 8), 148 * 4), 256, 0, st>>>(
      a, kind, reinterpret_cast<__nv_bfloat16*>(out), rows, ld_out);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void fsdp_reduce_scatter(const FsdpRsArgs& a, cudaStream_t st) {
  if (a.nranks < 1 || a.nranks > kSymmMaxRanks || a.rank < 0 || a.rank >= a.nranks)
    throw std::invalid_argument("fsdp_reduce_scatter: 1..8 ranks");
  if (a.chunks < 1 || a.chunks > kSymmMaxChunks || a.k < 1 || a.table == nullptr || a.out == nullptr ||
      a.shard_numel % 4 || (reinterpret_cast<uintptr_t>(a.out) & 15))
    throw std::invalid_argument("fsdp_reduce_scatter: chunks in 1..128, a table, a 16-byte aligned "
                                "shard of whole float4 groups");
  for (int p = 0; p < a.nranks; ++p)
    if (a.stage[p] == nullptr || a.flags[p] == nullptr || (reinterpret_cast<uintptr_t>(a.stage[p]) & 15))
      throw std::invalid_argument("fsdp_reduce_scatter: every rank's 16-byte aligned staging and flags");
  comm::fsdp_rs_kernel<<<a.chunks, 1024, 0, st>>>(a);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void fsdp_push_lowp(const TpArgs& a, const int64_t* table, int k, long long total16, const float* shard,
                    cudaStream_t st) {
  if (a.n < 1 || a.n > kSymmMaxRanks || a.rank < 0 || a.rank >= a.n || k < 1 ||
      (reinterpret_cast<uintptr_t>(shard) & 15))
    throw std::invalid_argument("fsdp_push_lowp: 1..8 ranks, a parameter table, 16-byte aligned shard");
  for (int p = 0; p < a.n; ++p)
    if (a.bufs[p] == nullptr || (reinterpret_cast<uintptr_t>(a.bufs[p]) & 15))
      throw std::invalid_argument("fsdp_push_lowp: every rank's 16-byte aligned slot");
  if (total16 <= 0) return;
  comm::fsdp_push_lowp_kernel<<<tp_grid(total16, 148 * 4), 256, 0, st>>>(a, table, k, total16, shard);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void fsdp_push(const TpArgs& a, const int64_t* table, int k, long long total16, const void* shard,
               cudaStream_t st) {
  if (a.n < 1 || a.n > kSymmMaxRanks || a.rank < 0 || a.rank >= a.n || k < 1 ||
      (reinterpret_cast<uintptr_t>(shard) & 15))
    throw std::invalid_argument("fsdp_push: 1..8 ranks, a parameter table, 16-byte aligned shard");
  for (int p = 0; p < a.n; ++p)
    if (a.bufs[p] == nullptr || (reinterpret_cast<uintptr_t>(a.bufs[p]) & 15))
      throw std::invalid_argument("fsdp_push: every rank's 16-byte aligned buffer");
  if (total16 <= 0) return;
  comm::fsdp_push_kernel<<<tp_grid(total16, 148 * 4), 256, 0, st>>>(
      a, table, k, total16, reinterpret_cast<const uint4*>(shard));
  PLG_CUDA_CHECK(cudaGetLastError());
}

void tp_norm_ag_push(const TpArgs& a, const void* x, bool x_fp32, long long ld, const float* w,
                     float eps, float* rstd, cudaStream_t st) {
  tp_check(a, ld, x, "tp_norm_ag_push");
  if (a.W % 256 || a.W > 8192)
    throw std::invalid_argument("tp_norm_ag_push: width must be a multiple of 256, at most 8192");
  const long long rows = a.B * (a.S / a.n);
  if (rows <= 0) return;
  const unsigned grid = static_cast<unsigned>(std::min<long long>(rows, 148LL * 8));
  const unsigned threads = static_cast<unsigned>(a.W / 8);
  if (x_fp32)
    comm::tp_norm_ag_push_kernel<float><<<grid, threads, 0, st>>>(a, reinterpret_cast<const float*>(x), ld,
                                                                  w, eps, rstd);
  else
    comm::tp_norm_ag_push_kernel<__nv_bfloat16><<<grid, threads, 0, st>>>(
        a, reinterpret_cast<const __nv_bfloat16*>(x), ld, w, eps, rstd);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void set_peer_wait_deadline_ns(unsigned long long ns, cudaStream_t st) {
  if (ns == 0) throw std::invalid_argument("set_peer_wait_deadline_ns: the deadline must be positive");
  const uint64_t v = ns;
  // ordered on the stream: kernels launched before the call keep the old deadline
  PLG_CUDA_CHECK(cudaMemcpyToSymbolAsync(comm::g_peer_wait_deadline_ns, &v, sizeof(v), 0,
                                         cudaMemcpyHostToDevice, st));
  PLG_CUDA_CHECK(cudaStreamSynchronize(st));
}

}  // namespace plg
