// Memory-bound sm_100a kernels: GLU activations, casts, embedding, softcap,
// cross-entropy rows, and the multi-tensor optimizer / grad-norm kernels.
//
// Parity:
//   glu          pluggy/kernels/swiglu.py:14-21 (silu(g)*u, gelu_tanh(g)*u)
//   embedding    nn.Embedding in pluggy/models/qwen3/qwen3.py:318 (+ Gemma's sqrt(d) scale)
//   softcap      pluggy/kernels/softcap.py:13-33
//   ce_rows      the per-chunk math of pluggy/loss/fused_linear_ce.py:31-58
//                (lse, target gather, softmax - onehot masked by ignore_index)
//   adamw/sumsq  torch.optim.AdamW(fused=True) and pluggy/core/grad_helper.py:8-34
#include <cstdio>
#include <mutex>
#include <stdexcept>

#include <cstdlib>

#include "common.cuh"
#include "ops.h"
#include "plg_noalloc.h"

namespace plg {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

// tanh-approximated GELU and its derivative (Hendrycks & Gimpel 2016, eq. for
// the tanh form): g(x) = 0.5 x (1 + tanh(k0 (x + k1 x^3))), k0 = sqrt(2/pi), k1 = 0.044715
__device__ __forceinline__ void gelu_tanh(float x, float& y, float& dy) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float inner = k0 * (x + k1 * x * x * x);
  const float t = tanhf(inner);
  y = 0.5f * x * (1.f + t);
  dy = 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x * x);
}

// GLU kernels: one block per group of rows, 8 channels (16 bytes) per thread
// access; needs F % 8 == 0 and 16-byte aligned rows (checked by the launchers).
__device__ __forceinline__ void glu_act(float g, float u, int kind, float& a) {
  if (kind == 0) {
    a = __fdividef(g, 1.f + fast_exp2(-g * kLog2e)) * u;
  } else {
    float y, dy;
    gelu_tanh(g, y, dy);
    a = y * u;
  }
}

__global__ void __launch_bounds__(256) glu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, long long ld,
                                                      __nv_bfloat16* __restrict__ out, long long rows,
                                                      int F, int kind) {
  const int c8 = F / 8;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* grow = gu + r * ld;
    for (int c = threadIdx.x; c < c8; c += blockDim.x) {
      const uint4 gv = *reinterpret_cast<const uint4*>(grow + c * 8);
      const uint4 uv = *reinterpret_cast<const uint4*>(grow + F + c * 8);
      const uint32_t* gp = reinterpret_cast<const uint32_t*>(&gv);
      const uint32_t* up = reinterpret_cast<const uint32_t*>(&uv);
      uint4 ov;
      uint32_t* op = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 g = unpack_bf16x2(gp[k]), u = unpack_bf16x2(up[k]);
        float a0, a1;
        glu_act(g.x, u.x, kind, a0);
        glu_act(g.y, u.y, kind, a1);
        op[k] = pack_bf16x2(a0, a1);
      }
      *reinterpret_cast<uint4*>(out + r * F + c * 8) = ov;
    }
  }
}

__device__ __forceinline__ void glu_grad(float g, float u, float d, int kind, float& dg, float& du) {
  if (kind == 0) {
    const float sg = __fdividef(1.f, 1.f + fast_exp2(-g * kLog2e));
    du = d * g * sg;
    dg = d * u * sg * (1.f + g * (1.f - sg));
  } else {
    float y, e;
    gelu_tanh(g, y, e);
    du = d * y;
    dg = d * u * e;
  }
}

__global__ void __launch_bounds__(256) glu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, long long ld,
                                                      const __nv_bfloat16* __restrict__ dout,
                                                      __nv_bfloat16* __restrict__ dgu, long long rows,
                                                      int F, int kind) {
  const int c8 = F / 8;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* grow = gu + r * ld;
    __nv_bfloat16* drow = dgu + r * ld;
    for (int c = threadIdx.x; c < c8; c += blockDim.x) {
      const uint4 gv = *reinterpret_cast<const uint4*>(grow + c * 8);
      const uint4 uv = *reinterpret_cast<const uint4*>(grow + F + c * 8);
      const uint4 dv = *reinterpret_cast<const uint4*>(dout + r * F + c * 8);
      const uint32_t* gp = reinterpret_cast<const uint32_t*>(&gv);
      const uint32_t* up = reinterpret_cast<const uint32_t*>(&uv);
      const uint32_t* dp = reinterpret_cast<const uint32_t*>(&dv);
      uint4 og, ou;
      uint32_t* ogp = reinterpret_cast<uint32_t*>(&og);
      uint32_t* oup = reinterpret_cast<uint32_t*>(&ou);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 g = unpack_bf16x2(gp[k]), u = unpack_bf16x2(up[k]), d = unpack_bf16x2(dp[k]);
        float dg0, du0, dg1, du1;
        glu_grad(g.x, u.x, d.x, kind, dg0, du0);
        glu_grad(g.y, u.y, d.y, kind, dg1, du1);
        ogp[k] = pack_bf16x2(dg0, dg1);
        oup[k] = pack_bf16x2(du0, du1);
      }
      *reinterpret_cast<uint4*>(drow + c * 8) = og;
      *reinterpret_cast<uint4*>(drow + F + c * 8) = ou;
    }
  }
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                     long long n) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(x)[i];
    uint2 o;
    o.x = pack_bf16x2(v.x, v.y);
    o.y = pack_bf16x2(v.z, v.w);
    reinterpret_cast<uint2*>(y)[i] = o;
  }
  for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16(x[i]);
}

__global__ void cast_bf16_f32_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ y,
                                     long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ w,
                                     float* __restrict__ out, long long T, int D, float scale) {
  const long long t = blockIdx.x;
  if (t >= T) return;
  const float4* src = reinterpret_cast<const float4*>(w + ids[t] * (long long)D);
  float4* dst = reinterpret_cast<float4*>(out + t * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) {
    float4 v = src[i];
    v.x *= scale; v.y *= scale; v.z *= scale; v.w *= scale;
    dst[i] = v;
  }
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids,
                                     const float* __restrict__ dout, float* __restrict__ dw,
                                     long long T, int D, float scale) {
  const long long t = blockIdx.x;
  if (t >= T) return;
  float* dst = dw + ids[t] * (long long)D;
  const float* src = dout + t * D;
  for (int i = threadIdx.x * 4; i < D; i += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(src + i);
    atomicAdd(reinterpret_cast<float4*>(dst + i),
              make_float4(v.x * scale, v.y * scale, v.z * scale, v.w * scale));
  }
}

// Deterministic embedding backward over ids sorted ascending (stable). The sorted
// positions are cut into pieces: a piece starts at the first position of an id's run
// and at every multiple of kEmbPiece, so a frequent id (Zipf: one id can own 10% of
// the tokens) is spread over many CTAs. Pass 1: the CTA of each piece sums the
// piece's dout rows in sorted (= token) order; a run that is one piece adds its sum
// into dw[id] directly, a longer run's pieces are written to a scratch row at the
// piece's first position. Pass 2: the CTA at the start of each multi-piece run adds
// its pieces in order into dw[id]. Every id has exactly one writer and every sum has
// a fixed order: no atomics, bitwise reproducible.
constexpr int kEmbPiece = 64;

__device__ __forceinline__ long long emb_run_end(const int64_t* ids, long long i, long long T,
                                                 long long limit) {
  // first position > i with a different id, scanning at most up to `limit`
  __shared__ long long s_end;
  if (threadIdx.x == 0) s_end = limit;
  __syncthreads();
  const int64_t id = ids[i];
  for (long long base = i + 1; base < limit; base += blockDim.x) {
    const long long j = base + threadIdx.x;
    const bool stop = j < limit && ids[j] != id;
    if (stop) atomicMin(reinterpret_cast<unsigned long long*>(&s_end), static_cast<unsigned long long>(j));
    if (__syncthreads_or(stop || base + blockDim.x >= limit)) break;
  }
  const long long e = s_end;
  __syncthreads();
  return e;
}

__global__ void __launch_bounds__(256) embedding_bwd_pieces_kernel(
    const int64_t* __restrict__ ids_sorted, const int64_t* __restrict__ pos_sorted,
    const float* __restrict__ dout, float* __restrict__ dw, float* __restrict__ scratch, long long T,
    int D, float scale) {
  const long long i = blockIdx.x;
  if (i >= T) return;
  const int64_t id = ids_sorted[i];
  const bool run_start = i == 0 || ids_sorted[i - 1] != id;
  if (!run_start && i % kEmbPiece != 0) return;  // not the first position of a piece
  const long long window_end = min(T, (i / kEmbPiece + 1) * kEmbPiece);
  const long long end = emb_run_end(ids_sorted, i, T, window_end);
  // a single-piece run starts here and ends before the window does (or at T)
  const bool whole = run_start && (end < window_end || end == T ||
                                   ids_sorted[window_end] != id);
  float* dst = whole ? dw + id * (long long)D : scratch + i * (long long)D;
  for (int c = threadIdx.x * 4; c < D; c += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (long long j = i; j < end; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(dout + pos_sorted[j] * D + c);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (whole) {
      float4 d = *reinterpret_cast<float4*>(dst + c);
      d.x += acc.x * scale; d.y += acc.y * scale; d.z += acc.z * scale; d.w += acc.w * scale;
      *reinterpret_cast<float4*>(dst + c) = d;
    } else {
      *reinterpret_cast<float4*>(dst + c) = acc;
    }
  }
}

__global__ void __launch_bounds__(256) embedding_bwd_combine_kernel(
    const int64_t* __restrict__ ids_sorted, const float* __restrict__ scratch, float* __restrict__ dw,
    long long T, int D, float scale) {
  const long long i = blockIdx.x;
  if (i >= T) return;
  const int64_t id = ids_sorted[i];
  if (i > 0 && ids_sorted[i - 1] == id) return;  // not a run start
  const long long window_end = min(T, (i / kEmbPiece + 1) * kEmbPiece);
  if (window_end >= T || ids_sorted[window_end] != id) return;  // single-piece run: done in pass 1
  const long long end = emb_run_end(ids_sorted, window_end - 1, T, T);
  float* dst = dw + id * (long long)D;
  for (int c = threadIdx.x * 4; c < D; c += blockDim.x * 4) {
    float4 acc = *reinterpret_cast<const float4*>(scratch + i * (long long)D + c);  // first piece
    for (long long p = window_end; p < end; p += kEmbPiece) {
      const float4 v = *reinterpret_cast<const float4*>(scratch + p * (long long)D + c);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    float4 d = *reinterpret_cast<float4*>(dst + c);
    d.x += acc.x * scale; d.y += acc.y * scale; d.z += acc.z * scale; d.w += acc.w * scale;
    *reinterpret_cast<float4*>(dst + c) = d;
  }
}

template <typename T>
__global__ void softcap_kernel(const T* __restrict__ x, T* __restrict__ y, long long n, float cap) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float v = static_cast<float>(x[i]);
    y[i] = static_cast<T>(cap * tanhf(v / cap));
  }
}

// ------------------------------------------------------------ cross entropy
// One CTA per row of bf16 logits. Pass 1: online max / sum of exp (8 bf16 per
// 16-byte load). Pass 2: gradient (softmax - onehot) * scale written in place.
// 1024 threads, 2 CTAs per SM: about 300 rows (~90 MB of bf16 logits at V = 152k) are
// in flight at once, so pass 2 re-reads the row from L2 instead of DRAM.
constexpr int kCeThreads = 1024;

// kCeBatch: row loads in flight per thread before their math (1: at 32 registers for
// two resident 1024-thread blocks per SM; 2 loads, or 4 loads at one block per SM,
// measured 4 % and 8 % slower)
constexpr int kCeBatch = 1;

__global__ void __launch_bounds__(kCeThreads, 2) ce_rows_kernel(
    __nv_bfloat16* __restrict__ logits, long long ld, const int64_t* __restrict__ labels, int V,
    int ignore_index, float grad_scale, float softcap, float* __restrict__ lse_out,
    float* __restrict__ loss_sum, int* __restrict__ n_valid, float* __restrict__ row_loss,
    float* __restrict__ stats_out, const float* __restrict__ lse_in, long long label_offset) {
  const long long row = blockIdx.x;
  __nv_bfloat16* x = logits + row * ld;
  const int64_t lab_g = labels[row];
  const bool valid = lab_g != ignore_index;
  // vocabulary-parallel rows hold the columns [label_offset, label_offset + V) of the
  // full vocabulary: the target is on this row only when its label falls inside
  const long long lab = valid ? lab_g - label_offset : -1;
  const bool owned = valid && lab >= 0 && lab < V;
  const bool cap = softcap > 0.f;
  __shared__ float s_m[kCeThreads / 32], s_s[kCeThreads / 32];
  float m = -INFINITY, s = 0.f;
  const int nvec = V / 8;
  float lse;
  if (lse_in != nullptr) {
    // gradient pass of a vocabulary-parallel row: the lse over the full vocabulary is given
    lse = lse_in[row];
  } else {
  // kCeBatch row loads in flight per thread before their math (the same elements in
  // the same order as a one-load loop, so the result is unchanged)
  for (int i0 = threadIdx.x; i0 < nvec; i0 += kCeBatch * blockDim.x) {
  uint4 ub[kCeBatch];
#pragma unroll
  for (int q = 0; q < kCeBatch; ++q) {
    const int i = i0 + q * blockDim.x;
    if (i < nvec) ub[q] = reinterpret_cast<const uint4*>(x)[i];
  }
#pragma unroll
  for (int q = 0; q < kCeBatch; ++q) {
    if (i0 + q * static_cast<int>(blockDim.x) >= nvec) break;
    const uint4 u = ub[q];
    float f[8];
    float2 t;
    t = unpack_bf16x2(u.x); f[0] = t.x; f[1] = t.y;
    t = unpack_bf16x2(u.y); f[2] = t.x; f[3] = t.y;
    t = unpack_bf16x2(u.z); f[4] = t.x; f[5] = t.y;
    t = unpack_bf16x2(u.w); f[6] = t.x; f[7] = t.y;
    float lm = m;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (cap) f[j] = softcap * tanhf(f[j] / softcap);
      lm = fmaxf(lm, f[j]);
    }
    float acc = s * fast_exp2((m - lm) * kLog2e);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += fast_exp2((f[j] - lm) * kLog2e);
    m = lm;
    s = acc;
  }
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    float f = __bfloat162float(x[i]);
    if (cap) f = softcap * tanhf(f / softcap);
    const float lm = fmaxf(m, f);
    s = s * fast_exp2((m - lm) * kLog2e) + fast_exp2((f - lm) * kLog2e);
    m = lm;
  }
  // block reduction of (m, s)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * fast_exp2((m - nm) * kLog2e)) +
        (om == -INFINITY ? 0.f : os * fast_exp2((om - nm) * kLog2e));
    m = nm;
  }
  if (lane == 0) { s_m[warp] = m; s_s[warp] = s; }
  __syncthreads();
  if (warp == 0) {
    m = lane < kCeThreads / 32 ? s_m[lane] : -INFINITY;
    s = lane < kCeThreads / 32 ? s_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * fast_exp2((m - nm) * kLog2e)) +
          (om == -INFINITY ? 0.f : os * fast_exp2((om - nm) * kLog2e));
      m = nm;
    }
    if (lane == 0) { s_m[0] = m; s_s[0] = s; }
  }
  __syncthreads();
  lse = s_m[0] + logf(s_s[0]);
  if (stats_out != nullptr) {
    // statistics pass of a vocabulary-parallel row: (max, sum of exp relative to the
    // max, target logit or 0) of this shard; the caller combines the shards
    if (threadIdx.x == 0) {
      float tgt = 0.f;
      if (owned) {
        tgt = __bfloat162float(x[lab]);
        if (cap) tgt = softcap * tanhf(tgt / softcap);
      }
      stats_out[3 * row] = s_m[0];
      stats_out[3 * row + 1] = s_s[0];
      stats_out[3 * row + 2] = tgt;
    }
    return;
  }
  if (threadIdx.x == 0) {
    if (lse_out) lse_out[row] = lse;
    float loss = 0.f;
    if (valid) {
      float tgt = __bfloat162float(x[lab]);
      if (cap) tgt = softcap * tanhf(tgt / softcap);
      loss = lse - tgt;
      if (n_valid) atomicAdd(n_valid, 1);
    }
    // per-row losses (summed later in a fixed order) or an fp32 atomic sum
    if (row_loss) row_loss[row] = loss;
    else if (valid && loss_sum) atomicAdd(loss_sum, loss);
  }
  __syncthreads();  // the target logit is read before pass 2 overwrites it
  }
  // pass 2: gradient in place
  const float gs = valid ? grad_scale : 0.f;
  for (int i0 = threadIdx.x; i0 < nvec; i0 += kCeBatch * blockDim.x) {
  uint4 ub[kCeBatch];
#pragma unroll
  for (int q = 0; q < kCeBatch; ++q) {
    const int i = i0 + q * blockDim.x;
    if (i < nvec) ub[q] = reinterpret_cast<const uint4*>(x)[i];
  }
#pragma unroll
  for (int q = 0; q < kCeBatch; ++q) {
    const int i = i0 + q * blockDim.x;
    if (i >= nvec) break;
    uint4 u = ub[q];
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 t = unpack_bf16x2(w[j]);
      float a = t.x, b = t.y;
      float ca = 1.f, cb = 1.f;
      if (cap) {
        const float ta = tanhf(a / softcap), tb = tanhf(b / softcap);
        a = softcap * ta; b = softcap * tb;
        ca = 1.f - ta * ta; cb = 1.f - tb * tb;
      }
      float pa = fast_exp2((a - lse) * kLog2e), pb = fast_exp2((b - lse) * kLog2e);
      const int c = i * 8 + j * 2;
      if (c == lab) pa -= 1.f;
      if (c + 1 == lab) pb -= 1.f;
      w[j] = pack_bf16x2(pa * gs * ca, pb * gs * cb);
    }
    reinterpret_cast<uint4*>(x)[i] = u;
  }
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    float a = __bfloat162float(x[i]);
    float ca = 1.f;
    if (cap) {
      const float ta = tanhf(a / softcap);
      a = softcap * ta;
      ca = 1.f - ta * ta;
    }
    float p = fast_exp2((a - lse) * kLog2e);
    if (i == lab) p -= 1.f;
    x[i] = __float2bfloat16(p * gs * ca);
  }
}

// ------------------------------------------------------------ multi-tensor
// table row (int64): [p0, p1, p2, p3, p4, numel, chunk_start]; chunk_start is
// the global index of the tensor's first kOptChunk-element chunk.
constexpr int kRow = 7;

__device__ __forceinline__ int find_tensor(const int64_t* table, int ntensors, long long chunk) {
  int lo = 0, hi = ntensors - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (table[mid * kRow + 6] <= chunk) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void multi_sumsq_kernel(const int64_t* __restrict__ table, int ntensors,
                                   long long total_chunks, float* __restrict__ partial) {
  __shared__ float s_red[32];
  for (long long ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    const int ti = find_tensor(table, ntensors, ch);
    const float* g = reinterpret_cast<const float*>(table[ti * kRow + 0]);
    const long long n = table[ti * kRow + 5];
    const long long off = (ch - table[ti * kRow + 6]) * kOptChunk;
    const long long end = min(n, off + kOptChunk);
    float acc = 0.f;
    if ((reinterpret_cast<uintptr_t>(g + off) & 15) == 0) {
      const long long n4 = (end - off) / 4;
      const float4* g4 = reinterpret_cast<const float4*>(g + off);
      for (long long i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 v = g4[i];
        acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      for (long long i = off + n4 * 4 + threadIdx.x; i < end; i += blockDim.x) acc += g[i] * g[i];
    } else {
      for (long long i = off + threadIdx.x; i < end; i += blockDim.x) acc += g[i] * g[i];
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? s_red[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) partial[ch] = v;
    }
    __syncthreads();
  }
}

// out[c] = sum_r part[r, c] for a [R, D] fp32 matrix of per-block partial sums,
// in a fixed order (deterministic): a block owns 32 columns, its 8 warps sum
// strided row groups, then the warps' sums are added in shared memory.
__global__ void __launch_bounds__(256) colsum_kernel(const float* __restrict__ part, int R, int D,
                                                     float* __restrict__ out) {
  __shared__ float acc[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (c < D)
    for (int r = warp; r < R; r += 8) s += part[static_cast<long long>(r) * D + c];
  acc[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && c < D) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += acc[w][lane];
    out[c] = t;
  }
}

// deterministic final reduction of the per-chunk partials (one block)
__global__ void reduce_partials_kernel(const float* __restrict__ partial, long long n,
                                       float* __restrict__ out) {
  __shared__ double s_red[32];
  double acc = 0.0;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < (blockDim.x >> 5) ? s_red[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) out[0] = static_cast<float>(v);
  }
}

__global__ void multi_scale_kernel(const int64_t* __restrict__ table, int ntensors,
                                   long long total_chunks, const float* __restrict__ coef) {
  const float c = *coef;
  for (long long ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    const int ti = find_tensor(table, ntensors, ch);
    float* g = reinterpret_cast<float*>(table[ti * kRow + 0]);
    const long long n = table[ti * kRow + 5];
    const long long off = (ch - table[ti * kRow + 6]) * kOptChunk;
    const long long end = min(n, off + kOptChunk);
    for (long long i = off + threadIdx.x; i < end; i += blockDim.x) g[i] *= c;
  }
}

__global__ void __launch_bounds__(512) adamw_kernel(const int64_t* __restrict__ table,
                                                    int ntensors, long long total_chunks,
                                                    float lr, float b1, float b2, float eps,
                                                    float wd, float bc1, float bc2,
                                                    const float* __restrict__ gscale,
                                                    const float* __restrict__ hyper) {
  const float scale = gscale ? *gscale : 1.f;
  // device-resident (lr, bc1, bc2) when given: a step replayed from a CUDA graph reads
  // the values the host wrote for this step instead of the ones baked into the launch
  if (hyper != nullptr) {
    lr = hyper[0];
    bc1 = hyper[1];
    bc2 = hyper[2];
  }
  const float step = lr / bc1;
  const float rbc2 = rsqrtf(bc2);
  const float decay = 1.f - lr * wd;
  for (long long ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    const int ti = find_tensor(table, ntensors, ch);
    const int64_t* r = table + ti * kRow;
    float* p = reinterpret_cast<float*>(r[0]);
    const float* g = reinterpret_cast<const float*>(r[1]);
    float* m = reinterpret_cast<float*>(r[2]);
    float* v = reinterpret_cast<float*>(r[3]);
    __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(r[4]);
    const long long n = r[5];
    const long long off = (ch - r[6]) * kOptChunk;
    const long long end = min(n, off + kOptChunk);
    const bool vec = ((reinterpret_cast<uintptr_t>(p + off) | reinterpret_cast<uintptr_t>(g + off) |
                       reinterpret_cast<uintptr_t>(m + off) | reinterpret_cast<uintptr_t>(v + off)) &
                      15) == 0 &&
                     (sh == nullptr || (reinterpret_cast<uintptr_t>(sh + off) & 7) == 0);
    long long i0 = off;
    if (vec) {
      const long long n4 = (end - off) / 4;
      for (long long i = threadIdx.x; i < n4; i += blockDim.x) {
        const long long e = off + i * 4;
        float4 pp = *reinterpret_cast<float4*>(p + e);
        float4 gg = *reinterpret_cast<const float4*>(g + e);
        float4 mm = *reinterpret_cast<float4*>(m + e);
        float4 vv = *reinterpret_cast<float4*>(v + e);
        float* P = &pp.x; float* G = &gg.x; float* M = &mm.x; float* W = &vv.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          adamw_update(P[j], M[j], W[j], G[j] * scale, decay, b1, b2, step, rbc2, eps);
        }
        *reinterpret_cast<float4*>(p + e) = pp;
        *reinterpret_cast<float4*>(m + e) = mm;
        *reinterpret_cast<float4*>(v + e) = vv;
        if (sh) {
          uint2 o;
          o.x = pack_bf16x2(pp.x, pp.y);
          o.y = pack_bf16x2(pp.z, pp.w);
          *reinterpret_cast<uint2*>(sh + e) = o;
        }
      }
      i0 = off + n4 * 4;
    }
    for (long long e = i0 + threadIdx.x; e < end; e += blockDim.x) {
      float pj = p[e], mj = m[e], vj = v[e];
      adamw_update(pj, mj, vj, g[e] * scale, decay, b1, b2, step, rbc2, eps);
      p[e] = pj; m[e] = mj; v[e] = vj;
      if (sh) sh[e] = __float2bfloat16(pj);
    }
  }
}

// 2^x by the FMA-pipe cubic the attention kernels use for part of their softmax
// (exp2_poly2) and by CUDA's exp2f, side by side, for the error-bound test.
__global__ void exp2_poly_eval_kernel(const float* __restrict__ x, float* __restrict__ poly,
                                      float* __restrict__ ref, long long n) {
  const long long i = 2 * (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x);
  if (i >= n) return;
  const float x0 = x[i], x1 = i + 1 < n ? x[i + 1] : 0.f;
  float p0, p1;
  exp2_poly2(x0, x1, p0, p1);
  poly[i] = p0;
  ref[i] = exp2f(x0);
  if (i + 1 < n) {
    poly[i + 1] = p1;
    ref[i + 1] = exp2f(x1);
  }
}

int grid_for(long long work, int per_block) {
  long long b = (work + per_block - 1) / per_block;
  if (b > 148 * 16) b = 148 * 16;
  if (b < 1) b = 1;
  return static_cast<int>(b);
}

}  // namespace

static void check_glu(const void* gu, long long ld_gu, const void* out, int F) {
  if (F % 8 || ld_gu % 8 || (reinterpret_cast<uintptr_t>(gu) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15))
    throw std::invalid_argument("glu: F and the row stride must be multiples of 8, buffers 16B aligned");
}

static unsigned glu_blocks(long long rows) {
  const long long cap = 148LL * 16;
  return static_cast<unsigned>(rows < cap ? rows : cap);
}

void glu_fwd(const void* gu, long long ld_gu, void* out, long long rows, int F, int kind,
             cudaStream_t st) {
  if (rows <= 0) return;
  check_glu(gu, ld_gu, out, F);
  glu_fwd_kernel<<<glu_blocks(rows), 128, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu), ld_gu, reinterpret_cast<__nv_bfloat16*>(out),
      rows, F, kind);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void glu_bwd(const void* gu, long long ld_gu, const void* dout, void* dgu, long long rows, int F,
             int kind, cudaStream_t st) {
  if (rows <= 0) return;
  check_glu(gu, ld_gu, dgu, F);
  check_glu(dout, F, dout, F);
  glu_bwd_kernel<<<glu_blocks(rows), 128, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(gu), ld_gu,
      reinterpret_cast<const __nv_bfloat16*>(dout), reinterpret_cast<__nv_bfloat16*>(dgu), rows,
      F, kind);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void colsum(const float* part, int R, int D, float* out, cudaStream_t st) {
  if (D <= 0) return;
  colsum_kernel<<<(D + 31) / 32, 256, 0, st>>>(part, R, D, out);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void cast_f32_bf16(const float* x, void* y, long long n, cudaStream_t st) {
  if (n <= 0) return;
  cast_f32_bf16_kernel<<<grid_for(n / 4 + 1, 256), 256, 0, st>>>(
      x, reinterpret_cast<__nv_bfloat16*>(y), n);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void cast_bf16_f32(const void* x, float* y, long long n, cudaStream_t st) {
  if (n <= 0) return;
  cast_bf16_f32_kernel<<<grid_for(n, 256), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), y, n);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void embedding_fwd(const int64_t* ids, const float* w, float* out, long long T, int D, float scale,
                   cudaStream_t st) {
  if (T <= 0) return;
  if (D % 4) throw std::invalid_argument("embedding: D must be a multiple of 4");
  embedding_fwd_kernel<<<T, 256, 0, st>>>(ids, w, out, T, D, scale);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void embedding_bwd(const int64_t* ids, const float* dout, float* dw, long long T, int D,
                   float scale, cudaStream_t st) {
  if (T <= 0) return;
  embedding_bwd_kernel<<<T, 256, 0, st>>>(ids, dout, dw, T, D, scale);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void embedding_bwd_sorted(const int64_t* ids_sorted, const int64_t* pos_sorted, const float* dout,
                          float* dw, float* scratch, long long T, int D, float scale, cudaStream_t st) {
  if (T <= 0) return;
  if (D % 4 || (reinterpret_cast<uintptr_t>(dout) & 15) || (reinterpret_cast<uintptr_t>(dw) & 15) ||
      (reinterpret_cast<uintptr_t>(scratch) & 15))
    throw std::invalid_argument("embedding_bwd_sorted: D a multiple of 4, 16-byte aligned rows");
  embedding_bwd_pieces_kernel<<<T, 256, 0, st>>>(ids_sorted, pos_sorted, dout, dw, scratch, T, D, scale);
  embedding_bwd_combine_kernel<<<T, 256, 0, st>>>(ids_sorted, scratch, dw, T, D, scale);
  PLG_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ MoE router
// One warp per token: fp32 softmax over the E router logits, the top k (largest
// probability first, the lower expert index on ties, as a sort would give), the
// weights renormalised over the k when asked, and the per-expert histogram of the
// choices (int32 atomics: exact). kE = E / 32 logits per lane.
template <int kE, typename T>
__global__ void __launch_bounds__(256) router_topk_kernel(const T* __restrict__ logits, long long T_,
                                                          int k, int renorm, float* __restrict__ probs,
                                                          float* __restrict__ w_out,
                                                          int64_t* __restrict__ idx_out,
                                                          int* __restrict__ counts) {
  constexpr int E = kE * 32;
  const long long tok = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (tok >= T_) return;
  float v[kE];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kE; ++j) {
    v[j] = static_cast<float>(logits[tok * E + j * 32 + lane]);
    m = fmaxf(m, v[j]);
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kE; ++j) {
    v[j] = expf(v[j] - m);
    s += v[j];
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int j = 0; j < kE; ++j) {
    v[j] *= inv;
    if (probs != nullptr) probs[tok * E + j * 32 + lane] = v[j];
  }
  unsigned taken = 0;
  float wsum = 0.f, wmine = 0.f;
  int mine = -1;  // lane r < k keeps the r-th choice
  for (int r = 0; r < k; ++r) {
    float bv = -1.f;
    int bi = E;
#pragma unroll
    for (int j = 0; j < kE; ++j)
      if (!((taken >> j) & 1u) && v[j] > bv) {
        bv = v[j];
        bi = j * 32 + lane;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    wsum += bv;
    if (lane == r) {
      mine = bi;
      wmine = bv;
    }
  }
  if (lane < k) {
    idx_out[tok * k + lane] = mine;
    w_out[tok * k + lane] = renorm ? wmine / wsum : wmine;
    if (counts != nullptr) atomicAdd(counts + mine, 1);
  }
}

void router_topk(const void* logits, bool bf16, long long T, int E, int k, bool renorm, float* probs,
                 float* w, int64_t* idx, int* counts, cudaStream_t st) {
  if (E % 32 || E > 512 || k < 1 || k > 32 || k > E)
    throw std::invalid_argument("router_topk: E a multiple of 32 up to 512, 1 <= k <= min(32, E)");
  if (T <= 0) return;
  const unsigned blocks = static_cast<unsigned>((T * 32 + 255) / 256);
#define PLG_ROUTER(KE)                                                                              \
  if (E == KE * 32) {                                                                               \
    if (bf16)                                                                                       \
      router_topk_kernel<KE, __nv_bfloat16><<<blocks, 256, 0, st>>>(                                \
          static_cast<const __nv_bfloat16*>(logits), T, k, renorm, probs, w, idx, counts);          \
    else                                                                                            \
      router_topk_kernel<KE, float><<<blocks, 256, 0, st>>>(static_cast<const float*>(logits), T,   \
                                                            k, renorm, probs, w, idx, counts);      \
    PLG_CUDA_CHECK(cudaGetLastError());                                                             \
    return;                                                                                         \
  }
  PLG_ROUTER(1) PLG_ROUTER(2) PLG_ROUTER(4) PLG_ROUTER(8) PLG_ROUTER(16)
#undef PLG_ROUTER
  throw std::invalid_argument("router_topk: E must be 32, 64, 128, 256 or 512");
}

void exp2_poly_eval(const float* x, float* poly, float* ref, long long n, cudaStream_t st) {
  if (n <= 0) return;
  const long long pairs = (n + 1) / 2;
  exp2_poly_eval_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, st>>>(x, poly, ref, n);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void softcap_fwd(const void* x, void* y, long long n, float cap, bool bf16, cudaStream_t st) {
  if (n <= 0) return;
  if (bf16)
    softcap_kernel<__nv_bfloat16><<<grid_for(n, 256), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<__nv_bfloat16*>(y), n, cap);
  else
    softcap_kernel<float><<<grid_for(n, 256), 256, 0, st>>>(
        reinterpret_cast<const float*>(x), reinterpret_cast<float*>(y), n, cap);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void ce_rows(void* logits, long long ld, const int64_t* labels, long long rows, int V,
             int ignore_index, float grad_scale, float softcap, float* lse_out, float* loss_sum,
             int* n_valid, cudaStream_t st, float* row_loss, float* stats_out,
             const float* lse_in, long long label_offset) {
  if (rows <= 0) return;
  if ((ld % 8) || (reinterpret_cast<uintptr_t>(logits) & 15))
    throw std::invalid_argument("ce_rows: logits rows must be 16-byte aligned");
  ce_rows_kernel<<<rows, kCeThreads, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(logits), ld, labels,
                                              V, ignore_index, grad_scale, softcap, lse_out,
                                              loss_sum, n_valid, row_loss, stats_out, lse_in,
                                              label_offset);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void multi_sumsq(const int64_t* table, int ntensors, long long total_chunks, float* out,
                 cudaStream_t st) {
  // out: [1 + total_chunks]; out[0] receives the total, out[1:] the partials
  if (total_chunks <= 0) return;
  multi_sumsq_kernel<<<grid_for(total_chunks, 1), 512, 0, st>>>(table, ntensors, total_chunks,
                                                                out + 1);
  reduce_partials_kernel<<<1, 1024, 0, st>>>(out + 1, total_chunks, out);
  PLG_CUDA_CHECK(cudaGetLastError());
}

}  // namespace plg

// ---------------------------------------------------------------------------
// Allocation-free variant of multi_sumsq (declared in plg_noalloc.h): the
// per-chunk partials live in a file-scope device array instead of a buffer the
// caller allocates, for callers that cannot allocate device memory.
static __device__ __align__(256) float g_noalloc_sumsq_scratch[PLG_NOALLOC_MAX_CHUNKS];

extern "C" __attribute__((visibility("default"))) int plg_multi_sumsq_noalloc(
    const int64_t* table, int ntensors, long long total_chunks, float* total_out, void* stream) {
  if (total_chunks < 0 || total_chunks > PLG_NOALLOC_MAX_CHUNKS) {
    std::fprintf(stderr,
                 "plg_multi_sumsq_noalloc: total_chunks %lld outside [0, %d] (the scratch holds "
                 "one partial sum per 65536-element chunk)\n",
                 total_chunks, PLG_NOALLOC_MAX_CHUNKS);
    return 1;
  }
  if (total_chunks > 0 && (ntensors < 1 || table == nullptr)) {
    std::fprintf(stderr, "plg_multi_sumsq_noalloc: %lld chunks but an empty tensor table\n",
                 total_chunks);
    return 1;
  }
  // an error already pending on this thread belongs to the caller: report it
  // without consuming it, and enqueue nothing
  cudaError_t pending = cudaPeekAtLastError();
  if (pending != cudaSuccess) {
    std::fprintf(stderr, "plg_multi_sumsq_noalloc: a CUDA error was already pending (%s)\n",
                 cudaGetErrorString(pending));
    return 2;
  }
  // scratch address per device, looked up once (cudaGetSymbolAddress allocates nothing)
  static std::mutex mu;
  static float* scratch[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    std::fprintf(stderr, "plg_multi_sumsq_noalloc: cudaGetDevice failed (%s)\n",
                 cudaGetErrorString(e));
    return 2;
  }
  float* part = nullptr;
  {
    std::lock_guard<std::mutex> g(mu);
    if (scratch[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_sumsq_scratch);
      if (e != cudaSuccess) {
        std::fprintf(stderr, "plg_multi_sumsq_noalloc: cudaGetSymbolAddress failed (%s)\n",
                     cudaGetErrorString(e));
        return 2;
      }
      scratch[dev] = static_cast<float*>(p);
    }
    part = scratch[dev];
  }
  if (total_chunks == 0) {
    e = cudaMemsetAsync(total_out, 0, sizeof(float), static_cast<cudaStream_t>(stream));
  } else {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    plg::multi_sumsq_kernel<<<plg::grid_for(total_chunks, 1), 512, 0, st>>>(table, ntensors,
                                                                          total_chunks, part);
    // nothing was pending before the launch, so an error now is this launch's
    e = cudaGetLastError();
    if (e == cudaSuccess) {
      plg::reduce_partials_kernel<<<1, 1024, 0, st>>>(part, total_chunks, total_out);
      e = cudaGetLastError();
    }
  }
  if (e != cudaSuccess) {
    std::fprintf(stderr, "plg_multi_sumsq_noalloc: launch failed (%s)\n", cudaGetErrorString(e));
    return 2;
  }
  return 0;
}

namespace plg {

void multi_scale(const int64_t* table, int ntensors, long long total_chunks, const float* coef,
                 cudaStream_t st) {
  if (total_chunks <= 0) return;
  multi_scale_kernel<<<grid_for(total_chunks, 1), 512, 0, st>>>(table, ntensors, total_chunks,
                                                                coef);
  PLG_CUDA_CHECK(cudaGetLastError());
}

void adamw_multi(const int64_t* table, int ntensors, long long total_chunks, float lr, float beta1,
                 float beta2, float eps, float weight_decay, float bc1, float bc2,
                 const float* grad_scale, const float* hyper, cudaStream_t st) {
  if (total_chunks <= 0) return;
  adamw_kernel<<<grid_for(total_chunks, 1), 512, 0, st>>>(table, ntensors, total_chunks, lr, beta1,
                                                         beta2, eps, weight_decay, bc1, bc2,
                                                         grad_scale, hyper);
  PLG_CUDA_CHECK(cudaGetLastError());
}

}  // namespace plg
