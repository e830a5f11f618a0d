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
#include <stdexcept>

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
// dw_partial[block, :] = sum over the block's rows of dy * xh
template <typename TDY, typename TX, int NV>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(
    const TDY* __restrict__ dy, const TX* __restrict__ x, const float* __restrict__ w,
    const float* __restrict__ rstd, const float* __restrict__ dres, float* __restrict__ dx_f32,
    __nv_bfloat16* __restrict__ dx_bf16, float* __restrict__ dw_partial, long long rows, int D) {
  extern __shared__ float s_dw[];  // [D]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  if (dw_partial)
    for (int i = threadIdx.x; i < D; i += blockDim.x) s_dw[i] = 0.f;
  __syncthreads();
  for (long long row = (long long)blockIdx.x * nwarps + warp; row < rows;
       row += (long long)gridDim.x * nwarps) {
    const float r = rstd[row];
    float g[NV][4], xh[NV][4];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = j * 128 + lane * 4;
      float dv[4], xv[4];
      ld4(dy + row * D + c, dv);
      ld4(x + row * D + c, xv);
      float wv[4] = {1.f, 1.f, 1.f, 1.f};
      if (w) ld4(w + c, wv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xh[j][i] = xv[i] * r;
        g[j][i] = dv[i] * wv[i];
        dot += g[j][i] * xh[j][i];
        if (dw_partial) atomicAdd(&s_dw[c + i], dv[i] * xh[j][i]);
      }
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = j * 128 + lane * 4;
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = r * (g[j][i] - xh[j][i] * dot);
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
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x)
      dw_partial[(long long)blockIdx.x * D + i] = s_dw[i];
  }
}

template <typename TDY, typename TX>
void rmsnorm_bwd_t(const void* dy, const void* x, const float* w, const float* rstd,
                   const float* dres, float* dx_f32, void* dx_bf16, float* dw_partial,
                   int dw_blocks, long long rows, int D, cudaStream_t st) {
  const int threads = 256;
  const int nv = D / 128;
  const size_t sm = dw_partial ? D * sizeof(float) : 0;
#define PLG_RMSB_CASE(NV)                                                                      \
  case NV:                                                                                     \
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
// One warp per (token, head). Lane l owns first-half channels i = l + 32*j
// (j < d/64) and their RoPE partners i + d/2.
template <int NJ>
__global__ void __launch_bounds__(256) qk_rope_fwd_kernel(QkRopeArgs a) {
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int H = a.Hq + a.Hk;
  if (gw >= a.T * H) return;
  const long long t = gw / H;
  const int h = static_cast<int>(gw - t * H);
  const bool is_q = h < a.Hq;
  const int d = a.d, half = d / 2;
  const int col = is_q ? h * d : a.k_offset * d + (h - a.Hq) * d;
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + t * a.ld_qkv + col;
  float lo[NJ], hi[NJ];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    lo[j] = __bfloat162float(src[lane + 32 * j]);
    hi[j] = __bfloat162float(src[lane + 32 * j + half]);
    ss += lo[j] * lo[j] + hi[j] * hi[j];
  }
  const bool do_norm = is_q ? a.norm_q : a.norm_k;
  float r = 1.f;
  if (do_norm) {
    ss = warp_sum(ss);
    r = rsqrtf(ss / d + a.eps);
    const float* w = is_q ? a.wq : a.wk;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      lo[j] *= r * w[lane + 32 * j];
      hi[j] *= r * w[lane + 32 * j + half];
    }
  }
  if (lane == 0 && a.rstd) a.rstd[t * H + h] = r;
  const int pos = a.positions ? a.positions[t] : static_cast<int>(t % a.S);
  const int rhalf = a.rot_dim / 2;
  __nv_bfloat16* dst = is_q ? reinterpret_cast<__nv_bfloat16*>(a.q) + (t * a.Hq + h) * d
                            : reinterpret_cast<__nv_bfloat16*>(a.k) + (t * a.Hk + (h - a.Hq)) * d;
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int i = lane + 32 * j;
    float o_lo = lo[j], o_hi = hi[j];
    if (i < rhalf) {
      // rotate-half pairs (i, i + rot_dim/2) inside the rotated prefix; for
      // full rotation rot_dim == d and the partner is i + d/2.
      float s, c;
      sincosf(static_cast<float>(pos) * a.inv_freq[i], &s, &c);
      if (rhalf == half) {
        o_lo = lo[j] * c - hi[j] * s;
        o_hi = hi[j] * c + lo[j] * s;
      }
    }
    dst[i] = __float2bfloat16(o_lo);
    dst[i + half] = __float2bfloat16(o_hi);
  }
}

template <int NJ>
__global__ void __launch_bounds__(256) qk_rope_bwd_kernel(QkRopeArgs a, const __nv_bfloat16* dq,
                                                          const __nv_bfloat16* dk,
                                                          __nv_bfloat16* dqkv, long long ld_dqkv,
                                                          float* dwq_part, float* dwk_part) {
  extern __shared__ float s_dw[];  // [2 * d]: q weights then k weights
  const int lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int d = a.d, half = d / 2;
  for (int i = threadIdx.x; i < 2 * d; i += blockDim.x) s_dw[i] = 0.f;
  __syncthreads();
  const int H = a.Hq + a.Hk;
  const int rhalf = a.rot_dim / 2;
  float accq_lo[NJ], accq_hi[NJ], acck_lo[NJ], acck_hi[NJ];
#pragma unroll
  for (int j = 0; j < NJ; ++j) accq_lo[j] = accq_hi[j] = acck_lo[j] = acck_hi[j] = 0.f;
  for (long long gw = (long long)blockIdx.x * nwarps + (threadIdx.x >> 5); gw < a.T * H;
       gw += (long long)gridDim.x * nwarps) {
    const long long t = gw / H;
    const int h = static_cast<int>(gw - t * H);
    const bool is_q = h < a.Hq;
    const int col = is_q ? h * d : a.k_offset * d + (h - a.Hq) * d;
    const __nv_bfloat16* g = is_q ? dq + (t * a.Hq + h) * d : dk + (t * a.Hk + (h - a.Hq)) * d;
    const __nv_bfloat16* xs = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + t * a.ld_qkv + col;
    const int pos = a.positions ? a.positions[t] : static_cast<int>(t % a.S);
    float glo[NJ], ghi[NJ], xlo[NJ], xhi[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int i = lane + 32 * j;
      float gl = __bfloat162float(g[i]), gh = __bfloat162float(g[i + half]);
      if (i < rhalf && rhalf == half) {
        float s, c;
        sincosf(static_cast<float>(pos) * a.inv_freq[i], &s, &c);
        // transpose of the rotation
        glo[j] = gl * c + gh * s;
        ghi[j] = gh * c - gl * s;
      } else {
        glo[j] = gl;
        ghi[j] = gh;
      }
      xlo[j] = __bfloat162float(xs[i]);
      xhi[j] = __bfloat162float(xs[i + half]);
    }
    const bool do_norm = is_q ? a.norm_q : a.norm_k;
    __nv_bfloat16* out = dqkv + t * ld_dqkv + col;
    if (do_norm) {
      const float r = a.rstd[t * H + h];
      const float* w = is_q ? a.wq : a.wk;
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int i = lane + 32 * j;
        const float xl = xlo[j] * r, xh = xhi[j] * r;
        const float wl = w[i], wh = w[i + half];
        dot += glo[j] * wl * xl + ghi[j] * wh * xh;
        if (is_q) { accq_lo[j] += glo[j] * xl; accq_hi[j] += ghi[j] * xh; }
        else { acck_lo[j] += glo[j] * xl; acck_hi[j] += ghi[j] * xh; }
      }
      dot = warp_sum(dot) / d;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int i = lane + 32 * j;
        out[i] = __float2bfloat16(r * (glo[j] * w[i] - xlo[j] * r * dot));
        out[i + half] = __float2bfloat16(r * (ghi[j] * w[i + half] - xhi[j] * r * dot));
      }
    } else {
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int i = lane + 32 * j;
        out[i] = __float2bfloat16(glo[j]);
        out[i + half] = __float2bfloat16(ghi[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    const int i = lane + 32 * j;
    atomicAdd(&s_dw[i], accq_lo[j]);
    atomicAdd(&s_dw[i + half], accq_hi[j]);
    atomicAdd(&s_dw[d + i], acck_lo[j]);
    atomicAdd(&s_dw[d + i + half], acck_hi[j]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    if (dwq_part) dwq_part[(long long)blockIdx.x * d + i] = s_dw[i];
    if (dwk_part) dwk_part[(long long)blockIdx.x * d + i] = s_dw[d + i];
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

void qk_norm_rope_fwd(const QkRopeArgs& a, cudaStream_t st) {
  if (a.T <= 0) return;
  const long long warps = a.T * (a.Hq + a.Hk);
  dim3 grid((warps + 7) / 8);
  switch (a.d) {
    case 64: qk_rope_fwd_kernel<1><<<grid, 256, 0, st>>>(a); break;
    case 128: qk_rope_fwd_kernel<2><<<grid, 256, 0, st>>>(a); break;
    case 256: qk_rope_fwd_kernel<4><<<grid, 256, 0, st>>>(a); break;
    case 512: qk_rope_fwd_kernel<8><<<grid, 256, 0, st>>>(a); break;
    default: throw std::invalid_argument("qk_norm_rope: head_dim must be 64/128/256/512");
  }
  PLG_CUDA_CHECK(cudaGetLastError());
}

void qk_norm_rope_bwd(const QkRopeArgs& a, const void* dq, const void* dk, void* dqkv,
                      long long ld_dqkv, float* dwq_partial, float* dwk_partial, int dw_blocks,
                      cudaStream_t st) {
  if (a.T <= 0) return;
  const size_t sm = 2 * a.d * sizeof(float);
  auto q = reinterpret_cast<const __nv_bfloat16*>(dq);
  auto k = reinterpret_cast<const __nv_bfloat16*>(dk);
  auto o = reinterpret_cast<__nv_bfloat16*>(dqkv);
  switch (a.d) {
    case 64: qk_rope_bwd_kernel<1><<<dw_blocks, 256, sm, st>>>(a, q, k, o, ld_dqkv, dwq_partial, dwk_partial); break;
    case 128: qk_rope_bwd_kernel<2><<<dw_blocks, 256, sm, st>>>(a, q, k, o, ld_dqkv, dwq_partial, dwk_partial); break;
    case 256: qk_rope_bwd_kernel<4><<<dw_blocks, 256, sm, st>>>(a, q, k, o, ld_dqkv, dwq_partial, dwk_partial); break;
    case 512: qk_rope_bwd_kernel<8><<<dw_blocks, 256, sm, st>>>(a, q, k, o, ld_dqkv, dwq_partial, dwk_partial); break;
    default: throw std::invalid_argument("qk_norm_rope_bwd: head_dim must be 64/128/256/512");
  }
  PLG_CUDA_CHECK(cudaGetLastError());
}

}  // namespace plg
