// RMSNorm (fwd/bwd) and fused QK-norm + RoPE (fwd/bwd) for sm_100a.
//
// Parity:
//   RMSNorm       pluggy/kernels/rms_norm.py:13-29 and nn.RMSNorm in
//                 pluggy/models/qwen3/qwen3.py:99-100,229-230,269 (fp32 math,
//                 fp32 weight)
//   QK-norm+RoPE  qwen3.py:190-195 (q_norm/k_norm per head, then apply_rotary
//                 from pluggy/kernels/rope.py:18-24: x*cos + rotate_half(x)*sin)
// These are memory-bound: one warp per row (or per token-head), 16-byte
// vector loads where alignment allows, fp32 accumulation, bf16/fp32 stores.
#include <algorithm>
#include <stdexcept>

#include <type_traits>

#include <cstdlib>

#include "common.cuh"
#include "ops.h"

namespace plg {
namespace {

// load 4 consecutive elements starting at p (16B or 8B aligned)
__device__ __forceinline__ void ld4(const float* p, float (&v)[4]) {
  float4 t = *reinterpret_cast<const float4*>(p);
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
__device__ __forceinline__ void ld4(const __nv_bfloat16* p, float (&v)[4]) {
  uint2 t = *reinterpret_cast<const uint2*>(p);
  float2 a = unpack_bf16x2(t.x), b = unpack_bf16x2(t.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void st4(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(__nv_bfloat16* p, const float (&v)[4]) {
  uint2 t;
  t.x = pack_bf16x2(v[0], v[1]);
  t.y = pack_bf16x2(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = t;
}

// ------------------------------------------------------------------ RMSNorm fwd
// one warp per row; D % 128 == 0; the row is kept in registers (D / 128 vectors of 4)

template <typename TX, typename TY, int NV>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const TX* __restrict__ x,
                                                          const float* __restrict__ w,
                                                          TY* __restrict__ y,
                                                          float* __restrict__ rstd,
                                                          long long rows, int D, float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const TX* xr = x + row * D;
  float v[NV][4];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = j * 128 + lane * 4;
    ld4(xr + c, v[j]);
    ss += v[j][0] * v[j][0] + v[j][1] * v[j][1] + v[j][2] * v[j][2] + v[j][3] * v[j][3];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  if (lane == 0 && rstd) rstd[row] = r;
  TY* yr = y + row * D;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = j * 128 + lane * 4;
    float o[4];
    if (w) {
      float wv[4];
      ld4(w + c, wv);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = v[j][i] * r * wv[i];
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = v[j][i] * r;
    }
    st4(yr + c, o);
  }
}

template <typename TX, typename TY>
void rmsnorm_fwd_t(const void* x, const float* w, void* y, float* rstd, long long rows, int D,
                   float eps, cudaStream_t st) {
  const int warps = 8;
  dim3 grid((rows + warps - 1) / warps);
  const int nv = D / 128;
#define PLG_RMS_CASE(NV)                                                                    \
  case NV:                                                                                  \
    rmsnorm_fwd_kernel<TX, TY, NV><<<grid, warps * 32, 0, st>>>(                            \
        reinterpret_cast<const TX*>(x), w, reinterpret_cast<TY*>(y), rstd, rows, D, eps); \
    break;
  switch (nv) {
    PLG_RMS_CASE(1) PLG_RMS_CASE(2) PLG_RMS_CASE(4) PLG_RMS_CASE(8) PLG_RMS_CASE(16)
    PLG_RMS_CASE(20) PLG_RMS_CASE(24) PLG_RMS_CASE(32) PLG_RMS_CASE(6) PLG_RMS_CASE(12)
    PLG_RMS_CASE(3) PLG_RMS_CASE(5) PLG_RMS_CASE(10) PLG_RMS_CASE(18) PLG_RMS_CASE(28)
    default:
      throw std::invalid_argument("rmsnorm: unsupported D (need a supported multiple of 128)");
  }
#undef PLG_RMS_CASE
  PLG_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------------ RMSNorm bwd
// dx = rstd * (w*dy - xh * mean(w*dy*xh)) (+ dres),  xh = x * rstd
// dw_partial[block, :] = sum over the block's rows of dy * xh, in a fixed order:
// each warp owns a slice of shared memory ([warps][D], lane-owned columns, rows
// in the warp's order) and the slices are summed warp by warp at the end, so the
// partials are bitwise reproducible (no atomics)
template <typename TDY, typename TX, int NV>
// 128 threads and at most 128 registers: the caller's DW_BLOCKS (4 per SM) must all
// be resident at once, or the grid-strided rows run in several waves
__global__ void __launch_bounds__(128, 4) rmsnorm_bwd_kernel(
    const TDY* __restrict__ dy, const TX* __restrict__ x, const float* __restrict__ w,
    const float* __restrict__ rstd, const float* __restrict__ dres, float* __restrict__ dx_f32,
    __nv_bfloat16* __restrict__ dx_bf16, float* __restrict__ dw_partial, long long rows, int D) {
  extern __shared__ float s_dw_all[];  // [warps][D]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  float* s_dw = s_dw_all + warp * D;  // this warp's slice
  if (dw_partial)
    for (int i = threadIdx.x; i < nwarps * D; i += blockDim.x) s_dw_all[i] = 0.f;
  __syncthreads();
  // small D: dw accumulates in registers (lane-owned channels) and is reduced
  // across warps once; large D: straight into shared memory
  constexpr bool kRegDw = NV <= 8;
  float dw_acc[kRegDw ? NV : 1][4];
#pragma unroll
  for (int j = 0; j < (kRegDw ? NV : 1); ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) dw_acc[j][i] = 0.f;
  for (long long row = (long long)blockIdx.x * nwarps + warp; row < rows;
       row += (long long)gridDim.x * nwarps) {
    const float r = rstd[row];
    // the raw row stays in registers between the two passes (bf16 dy packed, w
    // re-read from L1)
    constexpr bool kDyBf16 = std::is_same_v<TDY, __nv_bfloat16>;
    uint2 dpk[kDyBf16 ? NV : 1];
    float dvf[kDyBf16 ? 1 : NV][4];
    auto dy_at = [&](int j, float (&v)[4]) {
      if constexpr (kDyBf16) {
        const float2 a = unpack_bf16x2(dpk[j].x), b = unpack_bf16x2(dpk[j].y);
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = dvf[j][i];
      }
    };
    float xvs[NV][4];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = j * 128 + lane * 4;
      if constexpr (kDyBf16) dpk[j] = *reinterpret_cast<const uint2*>(dy + row * D + c);
      else ld4(dy + row * D + c, dvf[j]);
      float dvs_j[4];
      dy_at(j, dvs_j);
      ld4(x + row * D + c, xvs[j]);
      float wv[4] = {1.f, 1.f, 1.f, 1.f};
      if (w) ld4(w + c, wv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float xh = xvs[j][i] * r;
        dot += dvs_j[i] * wv[i] * xh;
        if constexpr (kRegDw) dw_acc[j][i] += dvs_j[i] * xh;
        else if (dw_partial) s_dw[c + i] += dvs_j[i] * xh;  // lane-owned column of this warp
      }
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = j * 128 + lane * 4;
      float wv[4] = {1.f, 1.f, 1.f, 1.f};
      if (w) ld4(w + c, wv);
      float dvs_j[4];
      dy_at(j, dvs_j);
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = r * (dvs_j[i] * wv[i] - xvs[j][i] * r * dot);
      if (dres) {
        float rv[4];
        ld4(dres + row * D + c, rv);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] += rv[i];
      }
      if (dx_f32) st4(dx_f32 + row * D + c, o);
      if (dx_bf16) st4(dx_bf16 + row * D + c, o);
    }
  }
  if (dw_partial) {
    if constexpr (kRegDw) {
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) s_dw[j * 128 + lane * 4 + i] = dw_acc[j][i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      float t = 0.f;
      for (int w2 = 0; w2 < nwarps; ++w2) t += s_dw_all[w2 * D + i];
      dw_partial[(long long)blockIdx.x * D + i] = t;
    }
  }
}

template <typename TDY, typename TX>
void rmsnorm_bwd_t(const void* dy, const void* x, const float* w, const float* rstd,
                   const float* dres, float* dx_f32, void* dx_bf16, float* dw_partial,
                   int dw_blocks, long long rows, int D, cudaStream_t st) {
  const int threads = 128;
  const int nv = D / 128;
  const size_t sm = dw_partial ? (threads / 32) * D * sizeof(float) : 0;
#define PLG_RMSB_CASE(NV)                                                                      \
  case NV:                                                                                     \
    if (sm > 48 * 1024)                                                                        \
      PLG_CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bwd_kernel<TDY, TX, NV>,                     \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                                          static_cast<int>(sm)));                              \
    rmsnorm_bwd_kernel<TDY, TX, NV><<<dw_blocks, threads, sm, st>>>(                           \
        reinterpret_cast<const TDY*>(dy), reinterpret_cast<const TX*>(x), w, rstd, dres,       \
        dx_f32, reinterpret_cast<__nv_bfloat16*>(dx_bf16), dw_partial, rows, D);               \
    break;
  switch (nv) {
    PLG_RMSB_CASE(1) PLG_RMSB_CASE(2) PLG_RMSB_CASE(4) PLG_RMSB_CASE(8) PLG_RMSB_CASE(16)
    PLG_RMSB_CASE(20) PLG_RMSB_CASE(24) PLG_RMSB_CASE(32) PLG_RMSB_CASE(6) PLG_RMSB_CASE(12)
    PLG_RMSB_CASE(3) PLG_RMSB_CASE(5) PLG_RMSB_CASE(10) PLG_RMSB_CASE(18) PLG_RMSB_CASE(28)
    default:
      throw std::invalid_argument("rmsnorm_bwd: unsupported D");
  }
#undef PLG_RMSB_CASE
  PLG_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------ QK-norm + RoPE
// Lane layout: a head row of d channels is spread over LPH = d / NV lanes of NV
// consecutive channels each (NV = 8: one 16-byte access per lane; NV = 16 for
// d = 512), so one warp instruction covers HPW = 32 / LPH heads. A work item is
// (token, kRounds * HPW consecutive heads); all of its rows are loaded before any
// is used, which keeps enough bytes in flight for the memory system.
// RoPE is rotate-half over the first rot_dim channels: channel i < rot_dim/2
// pairs with i + rot_dim/2, a lane shuffle away inside the head's lane group.
template <int D>
struct RopeLayout {
  static constexpr int NV = D >= 512 ? 16 : 8;
  static constexpr int LPH = D / NV;
  static constexpr int HPW = 32 / LPH;
  static constexpr int kRounds = D >= 512 ? 1 : (D >= 256 ? 2 : 4);
};

template <int NV>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&v)[NV]) {
#pragma unroll
  for (int q = 0; q < NV / 8; ++q) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p + q * 8);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = unpack_bf16x2(u[k]);
      v[q * 8 + 2 * k] = f.x;
      v[q * 8 + 2 * k + 1] = f.y;
    }
  }
}

template <int NV>
__device__ __forceinline__ void store_row(__nv_bfloat16* p, const float (&v)[NV]) {
#pragma unroll
  for (int q = 0; q < NV / 8; ++q) {
    uint4 raw;
    uint32_t* u = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
    for (int k = 0; k < 4; ++k) u[k] = pack_bf16x2(v[q * 8 + 2 * k], v[q * 8 + 2 * k + 1]);
    *reinterpret_cast<uint4*>(p + q * 8) = raw;
  }
}

// sum over the LPH lanes of one head group (aligned power-of-two groups)
template <int LPH>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// cos/sin of this lane's channels for position pos (c0 = first channel of the lane)
template <int NV>
__device__ __forceinline__ void rope_angles(const QkRopeArgs& a, int pos, int c0, float (&cs)[NV],
                                            float (&sn)[NV]) {
  const int rh = a.rot_dim / 2;
  const int f0 = c0 < rh ? c0 : c0 - rh;
  if (a.rope_table != nullptr) {
    // a lane's NV channels lie in one half of the rotated prefix (rh % NV == 0)
    const float* row = a.rope_table + static_cast<long long>(pos) * a.rot_dim;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const bool rot = c0 + k < a.rot_dim;
      cs[k] = rot ? row[f0 + k] : 1.f;
      sn[k] = rot ? row[rh + f0 + k] : 0.f;
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    if (c0 + k < a.rot_dim) {
      sincosf(static_cast<float>(pos) * a.inv_freq[f0 + k], &sn[k], &cs[k]);
    } else {
      cs[k] = 1.f;
      sn[k] = 0.f;
    }
  }
}

// One work item's inputs, loaded one item ahead of use: the warp issues the next
// item's loads before it computes the current one, so every warp keeps two items'
// rows in flight and the memory latency hides behind the arithmetic.
// The backward holds twice the rows per head (x and dq/dk) plus the norm-weight
// accumulators, so its items cover half as many heads; d = 512 rows are too wide
// to hold two items in registers and are loaded at the top of each iteration.
template <int D, bool kBwd>
struct RopeItem {
  using L = RopeLayout<D>;
  static constexpr int NQ = L::NV / 8;
  static constexpr int R = kBwd && L::kRounds > 1 ? L::kRounds / 2 : L::kRounds;
  static constexpr int HPI = L::HPW * R;
  static constexpr bool kPrefetch = D < 512;
  uint4 x[R][NQ];               // pre-norm q/k rows (raw bf16)
  uint4 g[kBwd ? R : 1][NQ];    // backward: dq/dk rows
  float rs[kBwd ? R : 1];       // backward: saved rstd
  float cs[L::NV], sn[L::NV];
};

template <int NV>
__device__ __forceinline__ void unpack_row(const uint4 (&raw)[NV / 8], float (&v)[NV]) {
#pragma unroll
  for (int q = 0; q < NV / 8; ++q) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&raw[q]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = unpack_bf16x2(u[k]);
      v[q * 8 + 2 * k] = f.x;
      v[q * 8 + 2 * k + 1] = f.y;
    }
  }
}

template <int D, bool kBwd>
__device__ __forceinline__ void rope_fetch(const QkRopeArgs& a, const __nv_bfloat16* dq,
                                           const __nv_bfloat16* dk, long long it, int nch, int sub,
                                           int c0, RopeItem<D, kBwd>& f) {
  using L = RopeLayout<D>;
  using I = RopeItem<D, kBwd>;
  constexpr int NQ = L::NV / 8;
  const int H = a.Hq + a.Hk;
  const long long t = it / nch;
  const int h0 = static_cast<int>(it - t * nch) * I::HPI;
  const int pos = a.positions ? a.positions[t] : static_cast<int>(t % a.S);
  const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + t * a.ld_qkv;
#pragma unroll
  for (int rr = 0; rr < I::R; ++rr) {
    const int h = h0 + rr * L::HPW + sub;
    const bool is_q = h < a.Hq;
    if (h < H) {
      const int col = is_q ? h * D : a.k_offset * D + (h - a.Hq) * D;
#pragma unroll
      for (int q = 0; q < NQ; ++q) f.x[rr][q] = *reinterpret_cast<const uint4*>(row + col + c0 + q * 8);
      if constexpr (kBwd) {
        const __nv_bfloat16* gp = is_q ? dq + (t * a.Hq + h) * D : dk + (t * a.Hk + (h - a.Hq)) * D;
#pragma unroll
        for (int q = 0; q < NQ; ++q) f.g[rr][q] = *reinterpret_cast<const uint4*>(gp + c0 + q * 8);
        f.rs[rr] = (is_q ? a.norm_q : a.norm_k) ? a.rstd[t * H + h] : 1.f;
      }
    } else {
#pragma unroll
      for (int q = 0; q < NQ; ++q) f.x[rr][q] = make_uint4(0u, 0u, 0u, 0u);
      if constexpr (kBwd) {
#pragma unroll
        for (int q = 0; q < NQ; ++q) f.g[rr][q] = make_uint4(0u, 0u, 0u, 0u);
        f.rs[rr] = 1.f;
      }
    }
  }
  rope_angles<L::NV>(a, pos, c0, f.cs, f.sn);
}

// 256 threads, 2 CTAs per SM, a persistent grid: each warp walks work items
// (token, 8 heads for d=128) with the next item's loads in flight.
template <int D>
__global__ void __launch_bounds__(256, 2) qk_rope_fwd_kernel(QkRopeArgs a) {
  using L = RopeLayout<D>;
  using I = RopeItem<D, false>;
  constexpr int NV = L::NV, HPI = I::HPI;
  const int lane = threadIdx.x & 31;
  const int sub = lane / L::LPH, ll = lane % L::LPH, c0 = ll * NV;
  const int H = a.Hq + a.Hk;
  const int nch = (H + HPI - 1) / HPI;
  const int rh = a.rot_dim / 2;
  const int off = rh / NV;
  const int pl = c0 < rh ? ll + off : (c0 < a.rot_dim ? ll - off : ll);
  const int partner = sub * L::LPH + pl;
  const float sgn = c0 < rh ? -1.f : 1.f;
  float wq[NV], wk[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    wq[k] = a.norm_q ? a.wq[c0 + k] : 1.f;
    wk[k] = a.norm_k ? a.wk[c0 + k] : 1.f;
  }
  const long long items = a.T * nch;
  const long long stride = (long long)gridDim.x * (blockDim.x >> 5);
  long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  I cur;
  if (I::kPrefetch && it < items) rope_fetch<D, false>(a, nullptr, nullptr, it, nch, sub, c0, cur);
  for (; it < items; it += stride) {
    I nxt;
    if (!I::kPrefetch) rope_fetch<D, false>(a, nullptr, nullptr, it, nch, sub, c0, cur);
    else if (it + stride < items) rope_fetch<D, false>(a, nullptr, nullptr, it + stride, nch, sub, c0, nxt);
    const long long t = it / nch;
    const int h0 = static_cast<int>(it - t * nch) * HPI;
#pragma unroll
    for (int rr = 0; rr < I::R; ++rr) {
      const int h = h0 + rr * L::HPW + sub;
      const bool is_q = h < a.Hq;
      const bool do_norm = is_q ? a.norm_q : a.norm_k;
      float v[NV];
      unpack_row<NV>(cur.x[rr], v);
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < NV; ++k) ss += v[k] * v[k];
      ss = group_sum<L::LPH>(ss);
      const float r = do_norm ? rsqrtf(ss / D + a.eps) : 1.f;
#pragma unroll
      for (int k = 0; k < NV; ++k) v[k] *= do_norm ? r * (is_q ? wq[k] : wk[k]) : 1.f;
      float o[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const float p = __shfl_sync(0xffffffffu, v[k], partner);
        o[k] = v[k] * cur.cs[k] + sgn * p * cur.sn[k];
      }
      if (h < H) {
        if (ll == 0 && a.rstd) a.rstd[t * H + h] = r;
        __nv_bfloat16* dst = is_q ? reinterpret_cast<__nv_bfloat16*>(a.q) + (t * a.Hq + h) * D
                                  : reinterpret_cast<__nv_bfloat16*>(a.k) + (t * a.Hk + (h - a.Hq)) * D;
        store_row<NV>(dst + c0, o);
      }
    }
    if (I::kPrefetch) cur = nxt;
  }
}

// 128 threads, at most 128 registers: all DW_BLOCKS (4 per SM) resident at once
template <int D>
__global__ void __launch_bounds__(128, 4) qk_rope_bwd_kernel(QkRopeArgs a, const __nv_bfloat16* dq,
                                                             const __nv_bfloat16* dk,
                                                             __nv_bfloat16* dqkv, long long ld_dqkv,
                                                             float* dwq_part, float* dwk_part) {
  using L = RopeLayout<D>;
  using I = RopeItem<D, true>;
  constexpr int NV = L::NV, HPI = I::HPI;
  extern __shared__ float s_dw[];  // [2 * D]: q weights then k weights
  const int lane = threadIdx.x & 31;
  const int sub = lane / L::LPH, ll = lane % L::LPH, c0 = ll * NV;
  for (int i = threadIdx.x; i < 2 * D; i += blockDim.x) s_dw[i] = 0.f;
  __syncthreads();
  const int H = a.Hq + a.Hk;
  const int nch = (H + HPI - 1) / HPI;
  const int rh = a.rot_dim / 2;
  const int off = rh / NV;
  const int pl = c0 < rh ? ll + off : (c0 < a.rot_dim ? ll - off : ll);
  const int partner = sub * L::LPH + pl;
  // transpose of the rotation: d_lo = g_lo c + g_hi s, d_hi = g_hi c - g_lo s
  const float sgn = c0 < rh ? 1.f : -1.f;
  float accq[NV], acck[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) accq[k] = acck[k] = 0.f;
  const long long items = a.T * nch;
  const long long stride = (long long)gridDim.x * (blockDim.x >> 5);
  long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  I cur;
  if (I::kPrefetch && it < items) rope_fetch<D, true>(a, dq, dk, it, nch, sub, c0, cur);
  for (; it < items; it += stride) {
    I nxt;
    if (!I::kPrefetch) rope_fetch<D, true>(a, dq, dk, it, nch, sub, c0, cur);
    else if (it + stride < items) rope_fetch<D, true>(a, dq, dk, it + stride, nch, sub, c0, nxt);
    const long long t = it / nch;
    const int h0 = static_cast<int>(it - t * nch) * HPI;
    __nv_bfloat16* orow = dqkv + t * ld_dqkv;
#pragma unroll
    for (int rr = 0; rr < I::R; ++rr) {
      const int h = h0 + rr * L::HPW + sub;
      const bool is_q = h < a.Hq;
      const bool do_norm = (is_q ? a.norm_q : a.norm_k) && h < H;
      const float* wp = is_q ? a.wq : a.wk;
      float g[NV], x[NV];
      unpack_row<NV>(cur.g[rr], g);
      unpack_row<NV>(cur.x[rr], x);
      float gr[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        const float p = __shfl_sync(0xffffffffu, g[k], partner);
        gr[k] = g[k] * cur.cs[k] + sgn * p * cur.sn[k];
      }
      const float r = cur.rs[rr];
      float dot = 0.f;
      float wv[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        wv[k] = do_norm ? wp[c0 + k] : 1.f;
        dot += gr[k] * wv[k] * x[k] * r;
      }
      dot = group_sum<L::LPH>(dot) / D;
      float o[NV];
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        if (do_norm) {
          const float xh = x[k] * r;
          if (is_q) accq[k] += gr[k] * xh;
          else acck[k] += gr[k] * xh;
          o[k] = r * (gr[k] * wv[k] - xh * dot);
        } else {
          o[k] = gr[k];
        }
      }
      if (h < H) {
        const int col = is_q ? h * D : a.k_offset * D + (h - a.Hq) * D;
        store_row<NV>(orow + col + c0, o);
      }
    }
    if (I::kPrefetch) cur = nxt;
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    atomicAdd(&s_dw[c0 + k], accq[k]);
    atomicAdd(&s_dw[D + c0 + k], acck[k]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    if (dwq_part) dwq_part[(long long)blockIdx.x * D + i] = s_dw[i];
    if (dwk_part) dwk_part[(long long)blockIdx.x * D + i] = s_dw[D + i];
  }
}

// ---------------------------------------------------- QK-norm + RoPE, TMA-fed
// The same math as the kernels above with the loads moved onto the bulk-copy
// engine: each CTA walks tiles of `tt` tokens; thread 0 issues cp.async.bulk
// copies of a tile's q/k rows (and, in the backward, its dq/dk rows, saved rstd
// and the cos/sin table row) into a ring of shared-memory stages, so up to
// `nst - 1` tiles per CTA are in flight while the warps work on the current one.
// Work per stage: one (token, head) row per LPH lanes, read from shared memory.
struct RopeTma {
  const __nv_bfloat16* dq; const __nv_bfloat16* dk; __nv_bfloat16* dqkv; long long ld_dqkv;
  float* dwq_part; float* dwk_part;
  int tt;          // tokens per stage
  int nst;         // stages (2..4)
  int tok_bytes;   // shared bytes per token slot (16-byte multiple)
  int off_g;       // backward: dq|dk rows
  int off_rs;      // backward: rstd row (when rs_bulk)
  int off_tab;     // cos|sin row (when a.rope_table)
  int rs_bulk;     // rstd rows are bulk-copied (H % 4 == 0)
};
constexpr int kRopeTmaThreads = 128;
constexpr int kRopeTmaMaxStages = 4;

// Channel layout of a lane. Unpaired: NV consecutive channels (the rotation
// partner sits a shuffle away). Paired (rot_dim == d): NV/2 channels of the lower
// half and the same NV/2 channels of the upper half, so the rotation is local to
// the lane and every cos/sin value is used twice.
template <int D, bool kPaired>
struct RopeLanes {
  static constexpr int NV = RopeLayout<D>::NV;
  static constexpr int LPH = RopeLayout<D>::LPH;
  __device__ static int chan(int ll, int k) {
    if constexpr (kPaired) return k < NV / 2 ? ll * (NV / 2) + k : D / 2 + ll * (NV / 2) + (k - NV / 2);
    else return ll * NV + k;
  }
  // load NV bf16 channels of a row at `base` (shared or global) into floats
  __device__ static void load(const uint8_t* base, int ll, float (&v)[NV]) {
    if constexpr (kPaired) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint8_t* p = base + (half * (D / 2) + ll * (NV / 2)) * 2;
#pragma unroll
        for (int q = 0; q < NV / 8; ++q) {
          const uint2 raw = *reinterpret_cast<const uint2*>(p + q * 8);
          const float2 f0 = unpack_bf16x2(raw.x), f1 = unpack_bf16x2(raw.y);
          v[half * (NV / 2) + q * 4 + 0] = f0.x;
          v[half * (NV / 2) + q * 4 + 1] = f0.y;
          v[half * (NV / 2) + q * 4 + 2] = f1.x;
          v[half * (NV / 2) + q * 4 + 3] = f1.y;
        }
      }
    } else {
      uint4 raw[NV / 8];
#pragma unroll
      for (int q = 0; q < NV / 8; ++q) raw[q] = *reinterpret_cast<const uint4*>(base + (ll * NV + q * 8) * 2);
      unpack_row<NV>(raw, v);
    }
  }
  __device__ static void store(__nv_bfloat16* row, int ll, const float (&v)[NV]) {
    if constexpr (kPaired) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        __nv_bfloat16* p = row + half * (D / 2) + ll * (NV / 2);
#pragma unroll
        for (int q = 0; q < NV / 8; ++q) {
          uint2 raw;
          raw.x = pack_bf16x2(v[half * (NV / 2) + q * 4 + 0], v[half * (NV / 2) + q * 4 + 1]);
          raw.y = pack_bf16x2(v[half * (NV / 2) + q * 4 + 2], v[half * (NV / 2) + q * 4 + 3]);
          *reinterpret_cast<uint2*>(p + q * 4) = raw;
        }
      }
    } else {
      store_row<NV>(row + ll * NV, v);
    }
  }
};

template <int D, bool kBwd, bool kPaired>
__global__ void __launch_bounds__(kRopeTmaThreads, 4) qk_rope_tma_kernel(QkRopeArgs a, RopeTma b) {
  using L = RopeLayout<D>;
  using C = RopeLanes<D, kPaired>;
  constexpr int NV = L::NV, HPW = L::HPW, NH = NV / 2;
  constexpr int kWarps = kRopeTmaThreads / 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const int H = a.Hq + a.Hk;
  uint8_t* slots = smem;
  int* s_pos = reinterpret_cast<int*>(smem + b.nst * b.tt * b.tok_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(s_pos + b.nst * b.tt) + 7) & ~uintptr_t(7));
  float* s_dw = reinterpret_cast<float*>(full + kRopeTmaMaxStages);  // [2 * D] (backward)
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sub = lane / L::LPH, ll = lane % L::LPH;
  // unpaired layout: rotation partner lane and sign
  const int c0 = ll * NV;
  const int rh = a.rot_dim / 2;
  const int off = rh / NV;
  const int pl = c0 < rh ? ll + off : (c0 < a.rot_dim ? ll - off : ll);
  const int partner = sub * L::LPH + pl;
  const float sgn_f = c0 < rh ? -1.f : 1.f;   // forward rotation
  const float sgn_b = -sgn_f;                 // its transpose
  const int f0 = c0 < rh ? c0 : c0 - rh;
  const bool rot_lane = c0 < a.rot_dim;
  if (tid == 0) {
    for (int s2 = 0; s2 < b.nst; ++s2) mbar_init(&full[s2], 1);
    fence_barrier_init();
    s_abort = 0;
  }
  if (kBwd)
    for (int i = tid; i < 2 * D; i += blockDim.x) s_dw[i] = 0.f;
  float wq[NV], wk[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    wq[k] = a.norm_q ? a.wq[C::chan(ll, k)] : 1.f;
    wk[k] = a.norm_k ? a.wk[C::chan(ll, k)] : 1.f;
  }
  float accq[kBwd ? NV : 1], acck[kBwd ? NV : 1];
#pragma unroll
  for (int k = 0; k < (kBwd ? NV : 1); ++k) accq[k] = acck[k] = 0.f;
  __syncthreads();

  const long long ntiles = (a.T + b.tt - 1) / b.tt;
  const uint32_t qbytes = a.Hq * D * 2, kbytes = a.Hk * D * 2;
  const __nv_bfloat16* qkv = reinterpret_cast<const __nv_bfloat16*>(a.qkv);
  // thread 0: positions of the tile, then every copy of the tile on one barrier
  auto issue = [&](long long tile, int st) {
    const long long t0 = tile * b.tt;
    const int n = static_cast<int>(a.T - t0 < b.tt ? a.T - t0 : b.tt);
    uint32_t per = qbytes + kbytes;
    if (kBwd) per += qbytes + kbytes + (b.rs_bulk ? H * 4 : 0);
    if (a.rope_table) per += a.rot_dim * 4;
    for (int j = 0; j < n; ++j) {
      const long long t = t0 + j;
      s_pos[st * b.tt + j] = a.positions ? a.positions[t] : static_cast<int>(t % a.S);
    }
    mbar_arrive_expect_tx(&full[st], per * n);
    for (int j = 0; j < n; ++j) {
      const long long t = t0 + j;
      uint8_t* slot = slots + (st * b.tt + j) * b.tok_bytes;
      bulk_load(slot, qkv + t * a.ld_qkv, qbytes, &full[st]);
      bulk_load(slot + qbytes, qkv + t * a.ld_qkv + static_cast<long long>(a.k_offset) * D, kbytes,
                &full[st]);
      if (kBwd) {
        bulk_load(slot + b.off_g, b.dq + t * a.Hq * D, qbytes, &full[st]);
        bulk_load(slot + b.off_g + qbytes, b.dk + t * a.Hk * D, kbytes, &full[st]);
        if (b.rs_bulk) bulk_load(slot + b.off_rs, a.rstd + t * H, H * 4, &full[st]);
      }
      if (a.rope_table)
        bulk_load(slot + b.off_tab, a.rope_table + static_cast<long long>(s_pos[st * b.tt + j]) * a.rot_dim,
                  a.rot_dim * 4, &full[st]);
    }
  };
  const long long first = blockIdx.x, stride = gridDim.x;
  if (tid == 0)
    for (int s2 = 0; s2 < b.nst - 1; ++s2)
      if (first + s2 * stride < ntiles) issue(first + s2 * stride, s2);

  int it = 0;
  for (long long tile = first; tile < ntiles; tile += stride, ++it) {
    const int st = it % b.nst;
    if (tid == 0) {
      const long long nt = tile + (b.nst - 1) * stride;
      if (nt < ntiles) issue(nt, (it + b.nst - 1) % b.nst);
    }
    if (!mbar_wait_bounded(&full[st], (it / b.nst) & 1, &s_abort)) {
      s_abort = 1;
      record_status(a.status, kTimeoutTmaFull);
    }
    __syncthreads();
    if (s_abort) break;
    const long long t0 = tile * b.tt;
    const int n = static_cast<int>(a.T - t0 < b.tt ? a.T - t0 : b.tt);
    for (int j = 0; j < n; ++j) {
      const long long t = t0 + j;
      const uint8_t* slot = slots + (st * b.tt + j) * b.tok_bytes;
      // cos / sin of this lane's channels (per token)
      float cs[kPaired ? NH : NV], sn[kPaired ? NH : NV];
      if constexpr (kPaired) {
        if (a.rope_table) {
          const float* tab = reinterpret_cast<const float*>(slot + b.off_tab);
#pragma unroll
          for (int k = 0; k < NH; ++k) {
            cs[k] = tab[ll * NH + k];
            sn[k] = tab[rh + ll * NH + k];
          }
        } else {
          const float pos = static_cast<float>(s_pos[st * b.tt + j]);
#pragma unroll
          for (int k = 0; k < NH; ++k) sincosf(pos * a.inv_freq[ll * NH + k], &sn[k], &cs[k]);
        }
      } else if (a.rope_table) {
        const float* tab = reinterpret_cast<const float*>(slot + b.off_tab);
#pragma unroll
        for (int k = 0; k < NV; ++k) {
          cs[k] = rot_lane ? tab[f0 + k] : 1.f;
          sn[k] = rot_lane ? tab[rh + f0 + k] : 0.f;
        }
      } else {
        rope_angles<NV>(a, s_pos[st * b.tt + j], c0, cs, sn);
      }
      for (int hb = warp * HPW; hb < H; hb += kWarps * HPW) {
        const int h = hb + sub;
        const bool live = h < H;
        const int hh = live ? h : 0;
        const bool is_q = hh < a.Hq;
        const bool do_norm = is_q ? a.norm_q : a.norm_k;
        float x[NV];
        C::load(slot + hh * D * 2, ll, x);
        if constexpr (!kBwd) {
          float ss = 0.f;
#pragma unroll
          for (int k = 0; k < NV; ++k) ss += x[k] * x[k];
          ss = group_sum<L::LPH>(ss);
          const float rr = do_norm ? rsqrtf(ss / D + a.eps) : 1.f;
#pragma unroll
          for (int k = 0; k < NV; ++k) x[k] *= rr * (is_q ? wq[k] : wk[k]);
          float o[NV];
          if constexpr (kPaired) {
#pragma unroll
            for (int k = 0; k < NH; ++k) {
              o[k] = x[k] * cs[k] - x[NH + k] * sn[k];
              o[NH + k] = x[NH + k] * cs[k] + x[k] * sn[k];
            }
          } else {
#pragma unroll
            for (int k = 0; k < NV; ++k) {
              const float p = __shfl_sync(0xffffffffu, x[k], partner);
              o[k] = x[k] * cs[k] + sgn_f * p * sn[k];
            }
          }
          if (live) {
            if (ll == 0 && a.rstd) a.rstd[t * H + h] = rr;
            __nv_bfloat16* dst = is_q ? reinterpret_cast<__nv_bfloat16*>(a.q) + (t * a.Hq + h) * D
                                      : reinterpret_cast<__nv_bfloat16*>(a.k) + (t * a.Hk + (h - a.Hq)) * D;
            C::store(dst, ll, o);
          }
        } else {
          float g[NV];
          C::load(slot + b.off_g + hh * D * 2, ll, g);
          float gr[NV];
          if constexpr (kPaired) {
#pragma unroll
            for (int k = 0; k < NH; ++k) {
              gr[k] = g[k] * cs[k] + g[NH + k] * sn[k];
              gr[NH + k] = g[NH + k] * cs[k] - g[k] * sn[k];
            }
          } else {
#pragma unroll
            for (int k = 0; k < NV; ++k) {
              const float p = __shfl_sync(0xffffffffu, g[k], partner);
              gr[k] = g[k] * cs[k] + sgn_b * p * sn[k];
            }
          }
          const bool norm_row = do_norm && live;
          const float rr = !norm_row ? 1.f
                           : (b.rs_bulk ? reinterpret_cast<const float*>(slot + b.off_rs)[h] : a.rstd[t * H + h]);
          float dot = 0.f;
#pragma unroll
          for (int k = 0; k < NV; ++k) dot += gr[k] * (is_q ? wq[k] : wk[k]) * x[k];
          dot = group_sum<L::LPH>(dot) * rr / D;
          float o[NV];
#pragma unroll
          for (int k = 0; k < NV; ++k) {
            if (norm_row) {
              const float xh = x[k] * rr;
              if (is_q) accq[k] += gr[k] * xh;
              else acck[k] += gr[k] * xh;
              o[k] = rr * (gr[k] * (is_q ? wq[k] : wk[k]) - xh * dot);
            } else {
              o[k] = gr[k];
            }
          }
          if (live) {
            const int col = is_q ? h * D : a.k_offset * D + (h - a.Hq) * D;
            C::store(b.dqkv + t * b.ld_dqkv + col, ll, o);
          }
        }
      }
    }
    __syncthreads();  // stage st is free for the refill issued next iteration
  }
  if (s_abort) {
    // wait (bounded) for copies still in flight into the stages before exiting
    for (int s2 = 0; s2 < b.nst; ++s2) {
      volatile int none = 0;
      mbar_wait_bounded(&full[s2], 0, &none, 1000000ull);
      mbar_wait_bounded(&full[s2], 1, &none, 1000000ull);
    }
    return;
  }
  if constexpr (kBwd) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      atomicAdd(&s_dw[C::chan(ll, k)], accq[k]);
      atomicAdd(&s_dw[D + C::chan(ll, k)], acck[k]);
    }
    __syncthreads();
    for (int i = tid; i < D; i += blockDim.x) {
      if (b.dwq_part) b.dwq_part[(long long)blockIdx.x * D + i] = s_dw[i];
      if (b.dwk_part) b.dwk_part[(long long)blockIdx.x * D + i] = s_dw[D + i];
    }
  }
}

}  // namespace

void rmsnorm_fwd(const void* x, bool x_fp32, const float* w, void* y, bool y_fp32, float* rstd,
                 long long rows, int D, float eps, cudaStream_t st) {
  if (rows <= 0) return;
  if (D % 128) throw std::invalid_argument("rmsnorm: D must be a multiple of 128");
  if (x_fp32 && y_fp32) rmsnorm_fwd_t<float, float>(x, w, y, rstd, rows, D, eps, st);
  else if (x_fp32) rmsnorm_fwd_t<float, __nv_bfloat16>(x, w, y, rstd, rows, D, eps, st);
  else if (y_fp32) rmsnorm_fwd_t<__nv_bfloat16, float>(x, w, y, rstd, rows, D, eps, st);
  else rmsnorm_fwd_t<__nv_bfloat16, __nv_bfloat16>(x, w, y, rstd, rows, D, eps, st);
}

void rmsnorm_bwd(const void* dy, bool dy_fp32, const void* x, bool x_fp32, const float* w,
                 const float* rstd, const float* dres, float* dx_f32, void* dx_bf16,
                 float* dw_partial, int dw_blocks, long long rows, int D, cudaStream_t st) {
  if (rows <= 0) return;
  if (D % 128) throw std::invalid_argument("rmsnorm_bwd: D must be a multiple of 128");
  if (dy_fp32 && x_fp32)
    rmsnorm_bwd_t<float, float>(dy, x, w, rstd, dres, dx_f32, dx_bf16, dw_partial, dw_blocks, rows, D, st);
  else if (dy_fp32)
    rmsnorm_bwd_t<float, __nv_bfloat16>(dy, x, w, rstd, dres, dx_f32, dx_bf16, dw_partial, dw_blocks, rows, D, st);
  else if (x_fp32)
    rmsnorm_bwd_t<__nv_bfloat16, float>(dy, x, w, rstd, dres, dx_f32, dx_bf16, dw_partial, dw_blocks, rows, D, st);
  else
    rmsnorm_bwd_t<__nv_bfloat16, __nv_bfloat16>(dy, x, w, rstd, dres, dx_f32, dx_bf16, dw_partial, dw_blocks, rows, D, st);
}

static void check_rope_args(const QkRopeArgs& a) {
  const int nv = a.d >= 512 ? 16 : 8;
  if (a.rot_dim < 0 || a.rot_dim > a.d || (a.rot_dim % (2 * nv)) != 0)
    throw std::invalid_argument("qk_norm_rope: rot_dim must be a multiple of 2*(d>=512 ? 16 : 8)");
  if ((a.ld_qkv % 8) != 0 || (reinterpret_cast<uintptr_t>(a.qkv) & 15) ||
      (a.q && (reinterpret_cast<uintptr_t>(a.q) & 15)) || (a.k && (reinterpret_cast<uintptr_t>(a.k) & 15)))
    throw std::invalid_argument("qk_norm_rope: rows must be 16-byte aligned");
}

template <int D>
static long long rope_items(const QkRopeArgs& a) {
  constexpr int hpi = RopeItem<D, false>::HPI;
  return a.T * ((a.Hq + a.Hk + hpi - 1) / hpi);
}

template <int D>
static void rope_fwd_t(const QkRopeArgs& a, cudaStream_t st) {
  long long blocks = (rope_items<D>(a) + 7) / 8;
  if (blocks > 148 * 2) blocks = 148 * 2;  // persistent: the resident CTAs (2 per SM)
  qk_rope_fwd_kernel<D><<<static_cast<unsigned>(blocks), 256, 0, st>>>(a);
}

// Shared-memory plan of the TMA-fed kernels: token slot layout, tokens per stage
// and stage count, sized for 4 CTAs per SM (<= ~54 KB each) where possible.
static RopeTma rope_tma_plan(const QkRopeArgs& a, bool bwd) {
  RopeTma b{};
  const int H = a.Hq + a.Hk;
  auto up16 = [](int x) { return (x + 15) & ~15; };
  int off = H * a.d * 2;  // x rows
  if (bwd) {
    b.off_g = off;
    off += H * a.d * 2;
    b.rs_bulk = (H % 4) == 0;
    if (b.rs_bulk) {
      b.off_rs = off;
      off = up16(off + H * 4);
    }
  }
  if (a.rope_table) {
    b.off_tab = off;
    off += a.rot_dim * 4;
  }
  b.tok_bytes = up16(off);
  // shared-memory budgets (KB) of one tile and of all stages of a CTA; four CTAs per SM
  // (PLG_ROPE_TILE_KB / PLG_ROPE_STAGES_KB override them for tuning). Measured at the
  // Qwen3-0.6B shape (T = 32768, 16q/8kv x 128), forward / backward ms: tile 7 KB
  // 0.123 / 0.176, 13 KB 0.104 / 0.176, 26 KB 0.094 / 0.156, 40 KB 0.136 / 0.215.
  static const int tile_kb = [] {
    const char* e = std::getenv("PLG_ROPE_TILE_KB");
    const int v = e ? std::atoi(e) : 26;
    return v >= 4 && v <= 48 ? v : 26;
  }();
  static const int stages_kb = [] {
    const char* e = std::getenv("PLG_ROPE_STAGES_KB");
    const int v = e ? std::atoi(e) : 54;
    return v >= 16 && v <= 54 ? v : 54;
  }();
  b.tt = std::max(1, (tile_kb * 1024) / b.tok_bytes);
  b.nst = std::min(kRopeTmaMaxStages, std::max(2, (stages_kb * 1024) / (b.tt * b.tok_bytes)));
  return b;
}

static size_t rope_tma_smem(const RopeTma& b, int d, bool bwd) {
  size_t bytes = static_cast<size_t>(b.nst) * b.tt * b.tok_bytes + b.nst * b.tt * sizeof(int) + 8;
  bytes += kRopeTmaMaxStages * sizeof(uint64_t) + (bwd ? 2 * d * sizeof(float) : 0);
  return bytes;
}

// The TMA path needs 16-byte-aligned rows and offsets (checked by check_rope_args)
// and a rotated prefix the lane layout supports; d = 512 keeps the register path.
static bool rope_tma_ok(const QkRopeArgs& a) {
  return a.d == 64 || a.d == 128 || a.d == 256;
}

template <int D, bool kBwd, bool kPaired>
static void rope_tma_launch_t(const QkRopeArgs& a, RopeTma b, int grid, cudaStream_t st) {
  const size_t sm = rope_tma_smem(b, D, kBwd);
  // the plan's size varies with the head counts: raise the limit once to what the
  // device allows beside the kernel's static shared memory
  static int limit[64] = {0};
  int dev = 0;
  PLG_CUDA_CHECK(cudaGetDevice(&dev));
  if (limit[dev & 63] == 0) {
    int optin = 0;
    PLG_CUDA_CHECK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    cudaFuncAttributes fa{};
    PLG_CUDA_CHECK(cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(&qk_rope_tma_kernel<D, kBwd, kPaired>)));
    limit[dev & 63] = optin - static_cast<int>(fa.sharedSizeBytes);
  }
  if (sm > static_cast<size_t>(limit[dev & 63]))
    throw std::invalid_argument("qk_norm_rope: a token's rows exceed shared memory");
  set_max_smem_once(reinterpret_cast<const void*>(&qk_rope_tma_kernel<D, kBwd, kPaired>), limit[dev & 63]);
  qk_rope_tma_kernel<D, kBwd, kPaired><<<grid, kRopeTmaThreads, sm, st>>>(a, b);
}

// full rotary uses the paired lane layout (no rotation shuffles)
template <int D, bool kBwd>
static void rope_tma_launch(const QkRopeArgs& a, RopeTma b, int grid, cudaStream_t st) {
  if (a.rot_dim == D) rope_tma_launch_t<D, kBwd, true>(a, b, grid, st);
  else rope_tma_launch_t<D, kBwd, false>(a, b, grid, st);
}

void qk_norm_rope_fwd(const QkRopeArgs& a, cudaStream_t st) {
  if (a.T <= 0) return;
  check_rope_args(a);
  if (rope_tma_ok(a)) {
    const RopeTma b = rope_tma_plan(a, false);
    const long long tiles = (a.T + b.tt - 1) / b.tt;
    const int grid = static_cast<int>(std::min<long long>(tiles, 148LL * 4));
    switch (a.d) {
      case 64: rope_tma_launch<64, false>(a, b, grid, st); break;
      case 128: rope_tma_launch<128, false>(a, b, grid, st); break;
      default: rope_tma_launch<256, false>(a, b, grid, st); break;
    }
    PLG_CUDA_CHECK(cudaGetLastError());
    return;
  }
  switch (a.d) {
    case 64: rope_fwd_t<64>(a, st); break;
    case 128: rope_fwd_t<128>(a, st); break;
    case 256: rope_fwd_t<256>(a, st); break;
    case 512: rope_fwd_t<512>(a, st); break;
    default: throw std::invalid_argument("qk_norm_rope: head_dim must be 64/128/256/512");
  }
  PLG_CUDA_CHECK(cudaGetLastError());
}

void qk_norm_rope_bwd(const QkRopeArgs& a, const void* dq, const void* dk, void* dqkv,
                      long long ld_dqkv, float* dwq_partial, float* dwk_partial, int dw_blocks,
                      cudaStream_t st) {
  if (a.T <= 0) return;
  check_rope_args(a);
  if ((ld_dqkv % 8) || (reinterpret_cast<uintptr_t>(dqkv) & 15) ||
      (reinterpret_cast<uintptr_t>(dq) & 15) || (reinterpret_cast<uintptr_t>(dk) & 15))
    throw std::invalid_argument("qk_norm_rope_bwd: rows must be 16-byte aligned");
  if (rope_tma_ok(a)) {
    RopeTma b = rope_tma_plan(a, true);
    b.dq = reinterpret_cast<const __nv_bfloat16*>(dq);
    b.dk = reinterpret_cast<const __nv_bfloat16*>(dk);
    b.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv);
    b.ld_dqkv = ld_dqkv;
    b.dwq_part = dwq_partial;
    b.dwk_part = dwk_partial;
    // one partial dw row per CTA: the grid is exactly dw_blocks
    switch (a.d) {
      case 64: rope_tma_launch<64, true>(a, b, dw_blocks, st); break;
      case 128: rope_tma_launch<128, true>(a, b, dw_blocks, st); break;
      default: rope_tma_launch<256, true>(a, b, dw_blocks, st); break;
    }
    PLG_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const size_t sm = 2 * a.d * sizeof(float);
  auto q = reinterpret_cast<const __nv_bfloat16*>(dq);
  auto k = reinterpret_cast<const __nv_bfloat16*>(dk);
  auto o = reinterpret_cast<__nv_bfloat16*>(dqkv);
  switch (a.d) {
    case 64: qk_rope_bwd_kernel<64><<<dw_blocks, 128, sm, st>>>(a, q, k, o, ld_dqkv, dwq_partial, dwk_partial); break;
    case 128: qk_rope_bwd_kernel<128><<<dw_blocks, 128, sm, st>>>(a, q, k, o, ld_dqkv, dwq_partial, dwk_partial); break;
    case 256: qk_rope_bwd_kernel<256><<<dw_blocks, 128, sm, st>>>(a, q, k, o, ld_dqkv, dwq_partial, dwk_partial); break;
    case 512: qk_rope_bwd_kernel<512><<<dw_blocks, 128, sm, st>>>(a, q, k, o, ld_dqkv, dwq_partial, dwk_partial); break;
    default: throw std::invalid_argument("qk_norm_rope_bwd: head_dim must be 64/128/256/512");
  }
  PLG_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------------------------------------ RoPE on [B, H, S, d]
// (x and y with any B/H/S strides: a transposed view of a projection in, the same
// layout out, so neither side needs a copy)
// y = x * cos + rotate_half(x) * sin (rotate_half(x) = [-x2, x1] over the two halves of
// d), the reference's apply_rotary, for x of any B/H/S strides and a cos/sin table
// [Bc, S, d] (Bc = 1 broadcasts). Backward (the transpose): dx1 = dy1 cos1 + dy2 sin2,
// dx2 = dy2 cos2 - dy1 sin1. fp32 math on bf16 data.
__global__ void __launch_bounds__(256) rope_apply_kernel(
    const __nv_bfloat16* __restrict__ x, long long xs_b, long long xs_h, long long xs_s,
    const float* __restrict__ cs, const float* __restrict__ sn, long long cs_b, long long cs_s,
    __nv_bfloat16* __restrict__ y, long long ys_b, long long ys_h, long long ys_s, int B, int H,
    int S, int d, int backward) {
  // four adjacent pairs per thread: 8-byte data accesses, 16-byte table reads
  const int hd = d / 2, q = d / 8;
  const long long n = static_cast<long long>(B) * H * S * q;
  for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; t < n;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = t / q;
    const int i = static_cast<int>(t - row * q) * 4;
    const int s = static_cast<int>(row % S);
    const long long bh = row / S;
    const int h = static_cast<int>(bh % H), b = static_cast<int>(bh / H);
    const __nv_bfloat16* xr = x + b * xs_b + h * xs_h + s * xs_s;
    const uint2 u1 = *reinterpret_cast<const uint2*>(xr + i);
    const uint2 u2 = *reinterpret_cast<const uint2*>(xr + hd + i);
    const long long co = b * cs_b + s * cs_s;
    const float4 c1 = *reinterpret_cast<const float4*>(cs + co + i);
    const float4 c2 = *reinterpret_cast<const float4*>(cs + co + hd + i);
    const float4 s1 = *reinterpret_cast<const float4*>(sn + co + i);
    const float4 s2 = *reinterpret_cast<const float4*>(sn + co + hd + i);
    const float2 a0 = unpack_bf16x2(u1.x), a1 = unpack_bf16x2(u1.y);
    const float2 b0 = unpack_bf16x2(u2.x), b1 = unpack_bf16x2(u2.y);
    const float x1[4] = {a0.x, a0.y, a1.x, a1.y}, x2[4] = {b0.x, b0.y, b1.x, b1.y};
    const float cc1[4] = {c1.x, c1.y, c1.z, c1.w}, cc2[4] = {c2.x, c2.y, c2.z, c2.w};
    const float ss1[4] = {s1.x, s1.y, s1.z, s1.w}, ss2[4] = {s2.x, s2.y, s2.z, s2.w};
    float y1[4], y2[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (backward) {
        y1[e] = fmaf(x1[e], cc1[e], x2[e] * ss2[e]);
        y2[e] = fmaf(x2[e], cc2[e], -x1[e] * ss1[e]);
      } else {
        y1[e] = fmaf(x1[e], cc1[e], -x2[e] * ss1[e]);
        y2[e] = fmaf(x2[e], cc2[e], x1[e] * ss2[e]);
      }
    }
    __nv_bfloat16* yr = y + b * ys_b + h * ys_h + s * ys_s;
    *reinterpret_cast<uint2*>(yr + i) = make_uint2(pack_bf16x2(y1[0], y1[1]), pack_bf16x2(y1[2], y1[3]));
    *reinterpret_cast<uint2*>(yr + hd + i) =
        make_uint2(pack_bf16x2(y2[0], y2[1]), pack_bf16x2(y2[2], y2[3]));
  }
}

void rope_apply(const void* x, long long xs_b, long long xs_h, long long xs_s, const float* cos,
                const float* sin, long long cs_b, long long cs_s, void* y, long long ys_b,
                long long ys_h, long long ys_s, int B, int H, int S, int d, bool backward,
                cudaStream_t st) {
  if (d % 8 != 0 || (xs_b | xs_h | xs_s) % 4 != 0 || (cs_b | cs_s) % 4 != 0 ||
      (ys_b | ys_h | ys_s) % 4 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 7) || (reinterpret_cast<uintptr_t>(cos) & 15) ||
      (reinterpret_cast<uintptr_t>(sin) & 15) || (reinterpret_cast<uintptr_t>(y) & 7))
    throw std::invalid_argument(
        "rope_apply: head_dim % 8, strides in multiples of 4 elements and 8/16-byte aligned bases");
  const long long n = static_cast<long long>(B) * H * S * (d / 8);
  if (n == 0) return;
  const long long blocks = std::min<long long>((n + 255) / 256, 148LL * 16);
  rope_apply_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), xs_b, xs_h, xs_s, cos, sin, cs_b, cs_s,
      static_cast<__nv_bfloat16*>(y), ys_b, ys_h, ys_s, B, H, S, d, backward ? 1 : 0);
  PLG_CUDA_CHECK(cudaGetLastError());
}

}  // namespace plg
