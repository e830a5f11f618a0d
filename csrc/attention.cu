// Causal / sliding-window GQA flash attention, forward and backward, on the
// sm_100a tensor cores (tcgen05 MMA with TMEM accumulators, TMA tile loads).
//
// Replaces F.scaled_dot_product_attention(is_causal=True, enable_gqa=True)
// (pluggy/models/qwen3/qwen3.py:166-181) and the dense S x S band mask used for
// sliding windows (pluggy/models/olmo3/olmo3.py:109-143,
// pluggy/models/gemma4/gemma4.py:187-217): the window is applied in-kernel.
//
// Layouts: q [B, S, Hq, d], k/v [B, S, Hk, d] (heads packed, any token stride,
// so K and V may be column slices of the fused QKV projection), o [B, S, Hq, d],
// lse [B, Hq, S] in natural log. d in {64, 128}.
//
// Forward, one CTA per (128-query tile, q head, batch), heavy causal tiles first:
//   warp 0      TMA: Q once, then K_j / V_j into two stages
//   warp 1      TMEM owner + MMA issuer: S_j = Q K_j^T into one of two S
//               buffers (so S_{j+1} overlaps the softmax of S_j), O += P_j V_j
//   warps 2..5  one query row per thread: online softmax in the log2 domain,
//               P_j (bf16) written to a 128-byte-swizzled smem tile, O rescaled
//               in TMEM when the row max grows, final O / l and LSE stored.
// Backward, one CTA per (128-key tile, kv head, batch), looping over the q
// heads of the GQA group and the q tiles that see the keys:
//   S^T = K Q^T and dP^T = V dO^T into TMEM; per key row: P^T = exp2(S^T - lse),
//   dS^T = P^T (dP^T - delta) * scale, both written to smem; then
//   dV += P^T dO, dK += dS^T Q (TMEM accumulators for the whole loop) and
//   dQ_i = dS K (TMEM, then fp32 vector atomics into a workspace).
// delta = rowsum(dO * O) comes from a small pre-pass; a post-pass casts dQ.
#include <cudaTypedefs.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "ops.h"

namespace plg {
namespace attn {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int kThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kBox = 128 * 128;  // bytes of one [128 rows x 64 bf16] swizzled box

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// K-major SW128 descriptor for k-step kk (16 elements) of a [128 rows x (64*nbox)] tile
// stored as nbox boxes of [128 rows x 64].
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int kk) {
  return make_smem_desc(base + (kk >> 2) * kBox + (kk & 3) * 32, 16, 1024, kLayoutSW128);
}
// MN-major SW128 descriptor for k-step kk (16 rows) of the same storage read with
// rows as the K dimension and the 64-wide boxes as MN atoms.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int kk) {
  return make_smem_desc(base + kk * 2048, kBox, 1024, kLayoutSW128);
}

// byte offset of 16-byte chunk `c16` (8 bf16) of row `r` in a [128 x 128] tile made of
// two swizzled boxes
__device__ __forceinline__ uint32_t swz_off(int r, int c16) {
  return (c16 >> 3) * kBox + r * 128 + (((c16 & 7) ^ (r & 7)) << 4);
}

__device__ __forceinline__ bool key_ok(int qi, int ki, int S, int causal, int window) {
  return ki < S && qi < S && (!causal || ki <= qi) && (window <= 0 || qi - ki < window);
}

// --------------------------------------------------------------------- forward
template <int D>
struct FwdCfg {
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kQ = 0;
  static constexpr int kK = kTile;          // 2 stages
  static constexpr int kV = 3 * kTile;      // 2 stages
  static constexpr int kP = 5 * kTile;      // [128 x 128] bf16
  static constexpr int kBar = kP + 128 * 128 * 2;
  static constexpr int kSmem = kBar + 256 + 1024;
  static constexpr int kTmemO = 256;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  using C = FwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2]
  uint64_t* s_free = bars + 9;    // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* o_done = bars + 12;
  uint64_t* mma_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;  // heavy causal tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.Hq / a.Hk);
  const int q0 = qt * BQ;
  const int n_kv = (a.S + BKV - 1) / BKV;
  const int j_hi = a.causal ? min(qt, n_kv - 1) : n_kv - 1;
  int j_lo = 0;
  if (a.window > 0) {
    const int lo_key = q0 - a.window + 1;
    j_lo = lo_key > 0 ? lo_key / BKV : 0;
  }
  const int n = j_hi - j_lo + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  uint8_t* sQ = smem + C::kQ;
  uint8_t* sK = smem + C::kK;
  uint8_t* sV = smem + C::kV;
  uint8_t* sP = smem + C::kP;

  if (warp == 0) {
    if (lane == 0 && n > 0) {
      uint32_t issued = 0, par = 0;  // bit i: stage i in flight; its parity
      bool ok = true;
      mbar_arrive_expect_tx(q_full, C::kTile);
#pragma unroll
      for (int x = 0; x < D / 64; ++x) tma_load_4d(sQ + x * kBox, &tmQ, q_full, x * 64, h, q0, b);
      for (int t = 0; t < n && ok; ++t) {
        const int st = t & 1;
        if (t >= 2 && !mbar_wait_bounded(&kv_empty[st], ((t >> 1) - 1) & 1, abort_flag)) {
          record_status(a.status, kTimeoutSmemEmpty);
          *abort_flag = 1;
          ok = false;
          break;
        }
        const int kv0 = (j_lo + t) * BKV;
        mbar_arrive_expect_tx(&k_full[st], C::kTile);
#pragma unroll
        for (int x = 0; x < D / 64; ++x)
          tma_load_4d(sK + st * C::kTile + x * kBox, &tmK, &k_full[st], x * 64, hk, kv0, b);
        mbar_arrive_expect_tx(&v_full[st], C::kTile);
#pragma unroll
        for (int x = 0; x < D / 64; ++x)
          tma_load_4d(sV + st * C::kTile + x * kBox, &tmV, &v_full[st], x * 64, hk, kv0, b);
        issued |= 1u << st;
        par = (par & ~(1u << st)) | (((t >> 1) & 1u) << st);
      }
      if (!ok) {
        mbar_wait_bounded(q_full, 0, nullptr);
        for (int st = 0; st < 2; ++st)
          if ((issued >> st) & 1u) {
            if (!mbar_wait_bounded(&k_full[st], (par >> st) & 1u, nullptr) ||
                !mbar_wait_bounded(&v_full[st], (par >> st) & 1u, nullptr))
              record_status(a.status, kTimeoutDrain);
          }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, D, false, true);
      const uint32_t aQ = smem_u32(sQ), aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP);
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag);
      auto issue_s = [&](int t) -> bool {
        const int st = t & 1;
        if (!mbar_wait_bounded(&k_full[st], (t >> 1) & 1, abort_flag)) return false;
        if (t >= 2 && !mbar_wait_bounded(&s_free[st], ((t >> 1) - 1) & 1, abort_flag)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_ss(tmem + st * 128, desc_kmajor(aQ, kk), desc_kmajor(aK + st * C::kTile, kk),
                    idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int t = 0; t < n && ok; ++t) {
        if (t + 1 < n && !(ok = issue_s(t + 1))) break;
        if (!mbar_wait_bounded(p_full, t & 1, abort_flag) ||
            !mbar_wait_bounded(&v_full[t & 1], (t >> 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          tc_mma_ss(tmem + C::kTmemO, desc_kmajor(aP, kk), desc_mnmajor(aV + (t & 1) * C::kTile, kk),
                    idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
        tc_commit(o_done);
        tc_commit(&kv_empty[t & 1]);
      }
      if (!ok) {
        record_status(a.status, kTimeoutTmaFull);
        *abort_flag = 1;
      }
      tc_commit(mma_done);
      if (!mbar_wait_bounded(mma_done, 0, nullptr)) record_status(a.status, kTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------ softmax warps
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qi = q0 + r;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float scale2 = a.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = n > 0;
    for (int t = 0; t < n && ok; ++t) {
      const int buf = t & 1;
      if (!mbar_wait_bounded(&s_full[buf], (t >> 1) & 1, abort_flag)) {
        record_status(a.status, kTimeoutAccFull);
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      float s[BKV];
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c) {
        uint32_t u[32];
        __syncwarp();
        tmem_ld_32x32b_x32(trow + buf * 128 + c * 32, u);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(u[e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[buf]);

      const int kv0 = (j_lo + t) * BKV;
      const bool need_mask = (a.causal && kv0 + BKV - 1 > q0) || (kv0 + BKV > a.S) ||
                             (a.window > 0 && q0 + BQ - 1 - kv0 >= a.window);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BKV; ++c) {
        float v = s[c] * scale2;
        if (need_mask && !key_ok(qi, kv0 + c, a.S, a.causal, a.window)) v = -INFINITY;
        s[c] = v;
        mx = fmaxf(mx, v);
      }
      const float m_new = fmaxf(m, mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(m - m_use);
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < BKV; ++c) {
        s[c] = exp2f(s[c] - m_use);
        rs += s[c];
      }
      l = l * alpha + rs;
      m = m_new;
      if (t > 0) {
        if (!mbar_wait_bounded(o_done, (t - 1) & 1, abort_flag)) {
          record_status(a.status, kTimeoutAccFull);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t u[32];
            tmem_ld_32x32b_x32(trow + C::kTmemO + c * 32, u);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
            tmem_st_32x32b_x32(trow + C::kTmemO + c * 32, u);
          }
          tmem_st_wait();
        }
      }
      // P (bf16) into the swizzled K-major tile, row r
#pragma unroll
      for (int c16 = 0; c16 < BKV / 8; ++c16) {
        uint4 w;
        w.x = pack_bf16x2(s[c16 * 8 + 0], s[c16 * 8 + 1]);
        w.y = pack_bf16x2(s[c16 * 8 + 2], s[c16 * 8 + 3]);
        w.z = pack_bf16x2(s[c16 * 8 + 4], s[c16 * 8 + 5]);
        w.w = pack_bf16x2(s[c16 * 8 + 6], s[c16 * 8 + 7]);
        *reinterpret_cast<uint4*>(sP + swz_off(r, c16)) = w;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && mbar_wait_bounded(o_done, (n - 1) & 1, abort_flag)) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.o) +
                            (static_cast<long long>(b) * a.S + qi) * a.o_row + h * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t u[32];
        __syncwarp();
        tmem_ld_32x32b_x32(trow + C::kTmemO + c * 32, u);
        tmem_ld_wait();
        if (qi < a.S) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(u[e]) * inv_l, __uint_as_float(u[e + 1]) * inv_l);
            w.y = pack_bf16x2(__uint_as_float(u[e + 2]) * inv_l, __uint_as_float(u[e + 3]) * inv_l);
            w.z = pack_bf16x2(__uint_as_float(u[e + 4]) * inv_l, __uint_as_float(u[e + 5]) * inv_l);
            w.w = pack_bf16x2(__uint_as_float(u[e + 6]) * inv_l, __uint_as_float(u[e + 7]) * inv_l);
            *reinterpret_cast<uint4*>(orow + c * 32 + e) = w;
          }
        }
      }
      if (qi < a.S)
        a.lse[(static_cast<long long>(b) * a.Hq + h) * a.S + qi] =
            (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
    } else if (ok) {
      record_status(a.status, kTimeoutAccFull);
      *abort_flag = 1;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// -------------------------------------------------------------------- backward
template <int D>
struct BwdCfg {
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kK = 0;
  static constexpr int kV = kTile;
  static constexpr int kQ = 2 * kTile;
  static constexpr int kDO = 3 * kTile;
  static constexpr int kPt = 4 * kTile;               // [128 kv x 128 q] bf16
  static constexpr int kDSt = kPt + 128 * 128 * 2;    // [128 kv x 128 q] bf16
  static constexpr int kLse = kDSt + 128 * 128 * 2;   // float [2][128]
  static constexpr int kDelta = kLse + 2 * 128 * 4;   // float [2][128]
  static constexpr int kBar = kDelta + 2 * 128 * 4;
  static constexpr int kSmem = kBar + 256 + 1024;
  static constexpr int kTS = 0, kTdP = 128, kTdV = 256, kTdK = 256 + D;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    AttnBwdArgs g) {
  using C = BwdCfg<D>;
  const AttnArgs& a = g.f;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;
  uint64_t* qd_empty = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* s_free = bars + 4;
  uint64_t* p_full = bars + 5;
  uint64_t* dq_full = bars + 6;
  uint64_t* dq_free = bars + 7;
  uint64_t* mma_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_lse = reinterpret_cast<float*>(smem + C::kLse);
  float* s_delta = reinterpret_cast<float*>(smem + C::kDelta);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int jt = blockIdx.x;  // key tile; small j has the most causal work: scheduled first
  const int hk = blockIdx.y, b = blockIdx.z;
  const int G = a.Hq / a.Hk;
  const int kv0 = jt * BKV;
  const int n_q = (a.S + BQ - 1) / BQ;
  const int i_lo = a.causal ? jt : 0;
  int i_hi = n_q - 1;
  if (a.window > 0) i_hi = min(i_hi, (kv0 + BKV - 1 + a.window - 1) / BQ);
  const int n_i = i_hi >= i_lo ? i_hi - i_lo + 1 : 0;
  const int n_it = n_i * G;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(qd_full, 1);
    mbar_init(qd_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint8_t* sK = smem + C::kK;
  uint8_t* sV = smem + C::kV;
  uint8_t* sQ = smem + C::kQ;
  uint8_t* sDO = smem + C::kDO;
  uint8_t* sPt = smem + C::kPt;
  uint8_t* sDSt = smem + C::kDSt;

  auto it_head = [&](int it) { return hk * G + it % G; };
  auto it_q0 = [&](int it) { return (i_lo + it / G) * BQ; };

  if (warp == 0) {
    if (lane == 0 && n_it > 0) {
      bool ok = true;
      bool q_inflight = false;
      uint32_t q_par = 0;
      mbar_arrive_expect_tx(kv_full, 2 * C::kTile);
#pragma unroll
      for (int x = 0; x < D / 64; ++x) {
        tma_load_4d(sK + x * kBox, &tmK, kv_full, x * 64, hk, kv0, b);
        tma_load_4d(sV + x * kBox, &tmV, kv_full, x * 64, hk, kv0, b);
      }
      for (int it = 0; it < n_it && ok; ++it) {
        if (it > 0 && !mbar_wait_bounded(qd_empty, (it - 1) & 1, abort_flag)) {
          record_status(a.status, kTimeoutSmemEmpty);
          *abort_flag = 1;
          ok = false;
          break;
        }
        const int h = it_head(it), q0 = it_q0(it);
        mbar_arrive_expect_tx(qd_full, 2 * C::kTile);
#pragma unroll
        for (int x = 0; x < D / 64; ++x) {
          tma_load_4d(sQ + x * kBox, &tmQ, qd_full, x * 64, h, q0, b);
          tma_load_4d(sDO + x * kBox, &tmDO, qd_full, x * 64, h, q0, b);
        }
        q_inflight = true;
        q_par = it & 1;
      }
      if (!ok) {
        if (!mbar_wait_bounded(kv_full, 0, nullptr)) record_status(a.status, kTimeoutDrain);
        if (q_inflight && !mbar_wait_bounded(qd_full, q_par, nullptr))
          record_status(a.status, kTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_it > 0) {
      constexpr uint32_t id_sq = make_idesc_bf16_f32(128, 128, false, false);  // S^T, dP^T
      constexpr uint32_t id_kv = make_idesc_bf16_f32(128, D, false, true);     // dV, dK
      constexpr uint32_t id_dq = make_idesc_bf16_f32(128, D, true, true);      // dQ
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aQ = smem_u32(sQ), aDO = smem_u32(sDO);
      const uint32_t aPt = smem_u32(sPt), aDS = smem_u32(sDSt);
      bool ok = mbar_wait_bounded(kv_full, 0, abort_flag);
      for (int it = 0; it < n_it && ok; ++it) {
        const uint32_t par = it & 1, ppar = (it - 1) & 1;
        if (!mbar_wait_bounded(qd_full, par, abort_flag) ||
            (it > 0 && !mbar_wait_bounded(s_free, ppar, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_ss(tmem + C::kTS, desc_kmajor(aK, kk), desc_kmajor(aQ, kk), id_sq, kk > 0);
        if (it > 0 && !mbar_wait_bounded(dq_free, ppar, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_ss(tmem + C::kTdP, desc_kmajor(aV, kk), desc_kmajor(aDO, kk), id_sq, kk > 0);
        tc_commit(s_full);
        if (!mbar_wait_bounded(p_full, par, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          tc_mma_ss(tmem + C::kTdV, desc_kmajor(aPt, kk), desc_mnmajor(aDO, kk), id_kv,
                    (it > 0 || kk > 0) ? 1u : 0u);
          tc_mma_ss(tmem + C::kTdK, desc_kmajor(aDS, kk), desc_mnmajor(aQ, kk), id_kv,
                    (it > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          tc_mma_ss(tmem + C::kTdP, desc_mnmajor(aDS, kk), desc_mnmajor(aK, kk), id_dq, kk > 0);
        tc_commit(dq_full);
        tc_commit(qd_empty);
      }
      if (!ok) {
        record_status(a.status, kTimeoutTmaFull);
        *abort_flag = 1;
      }
      tc_commit(mma_done);
      if (!mbar_wait_bounded(mma_done, 0, nullptr)) record_status(a.status, kTimeoutDrain);
    }
  } else {
    // -------------------------------------------------- softmax-grad warps
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // key row (S^T, dP^T) / query row (dQ)
    const int ki = kv0 + r;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float scale2 = a.scale * kLog2e;
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      const int h = it_head(it), q0 = it_q0(it);
      const int buf = it & 1;
      {
        const int qrow = q0 + r;
        const long long li = (static_cast<long long>(b) * a.Hq + h) * a.S + qrow;
        s_lse[buf * 128 + r] = qrow < a.S ? a.lse[li] * kLog2e : INFINITY;
        s_delta[buf * 128 + r] = qrow < a.S ? g.delta[li] : 0.f;
      }
      named_bar_sync(1, 128);
      if (!mbar_wait_bounded(s_full, it & 1, abort_flag)) {
        record_status(a.status, kTimeoutAccFull);
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const bool need_mask = (a.causal && q0 < kv0 + BKV - 1) || (kv0 + BKV > a.S) ||
                             (q0 + BQ > a.S) || (a.window > 0 && q0 + BQ - 1 - kv0 >= a.window);
#pragma unroll 1
      for (int c = 0; c < BQ / 32; ++c) {
        uint32_t us[32], ud[32];
        __syncwarp();
        tmem_ld_32x32b_x32(trow + C::kTS + c * 32, us);
        tmem_ld_32x32b_x32(trow + C::kTdP + c * 32, ud);
        tmem_ld_wait();
        float p[32], ds[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int qc = c * 32 + e;
          float pv = exp2f(__uint_as_float(us[e]) * scale2 - s_lse[buf * 128 + qc]);
          if (need_mask && !key_ok(q0 + qc, ki, a.S, a.causal, a.window)) pv = 0.f;
          p[e] = pv;
          ds[e] = pv * (__uint_as_float(ud[e]) - s_delta[buf * 128 + qc]) * a.scale;
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int c16 = c * 4 + w;
          uint4 pp, dd;
          pp.x = pack_bf16x2(p[w * 8 + 0], p[w * 8 + 1]);
          pp.y = pack_bf16x2(p[w * 8 + 2], p[w * 8 + 3]);
          pp.z = pack_bf16x2(p[w * 8 + 4], p[w * 8 + 5]);
          pp.w = pack_bf16x2(p[w * 8 + 6], p[w * 8 + 7]);
          dd.x = pack_bf16x2(ds[w * 8 + 0], ds[w * 8 + 1]);
          dd.y = pack_bf16x2(ds[w * 8 + 2], ds[w * 8 + 3]);
          dd.z = pack_bf16x2(ds[w * 8 + 4], ds[w * 8 + 5]);
          dd.w = pack_bf16x2(ds[w * 8 + 6], ds[w * 8 + 7]);
          *reinterpret_cast<uint4*>(sPt + swz_off(r, c16)) = pp;
          *reinterpret_cast<uint4*>(sDSt + swz_off(r, c16)) = dd;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // dQ_i readout: TMEM lane r is query row q0 + r
      if (!mbar_wait_bounded(dq_full, it & 1, abort_flag)) {
        record_status(a.status, kTimeoutAccFull);
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const int qrow = q0 + r;
      float* dqr = g.dq_acc + ((static_cast<long long>(b) * a.S + qrow) * a.Hq + h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t u[32];
        __syncwarp();
        tmem_ld_32x32b_x32(trow + C::kTdP + c * 32, u);
        tmem_ld_wait();
        if (qrow < a.S) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            atomicAdd(reinterpret_cast<float4*>(dqr + c * 32 + e),
                      make_float4(__uint_as_float(u[e]), __uint_as_float(u[e + 1]),
                                  __uint_as_float(u[e + 2]), __uint_as_float(u[e + 3])));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
    }
    // dK, dV for this key tile (all MMAs finished: the last dq_full was observed)
    if (ok && n_it > 0) {
      __nv_bfloat16* dkr = reinterpret_cast<__nv_bfloat16*>(g.dk) +
                           (static_cast<long long>(b) * a.S + ki) * g.dk_row + hk * D;
      __nv_bfloat16* dvr = reinterpret_cast<__nv_bfloat16*>(g.dv) +
                           (static_cast<long long>(b) * a.S + ki) * g.dv_row + hk * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t u[32], w32[32];
        __syncwarp();
        tmem_ld_32x32b_x32(trow + C::kTdV + c * 32, u);
        tmem_ld_32x32b_x32(trow + C::kTdK + c * 32, w32);
        tmem_ld_wait();
        if (ki < a.S) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 vv, kk4;
            vv.x = pack_bf16x2(__uint_as_float(u[e]), __uint_as_float(u[e + 1]));
            vv.y = pack_bf16x2(__uint_as_float(u[e + 2]), __uint_as_float(u[e + 3]));
            vv.z = pack_bf16x2(__uint_as_float(u[e + 4]), __uint_as_float(u[e + 5]));
            vv.w = pack_bf16x2(__uint_as_float(u[e + 6]), __uint_as_float(u[e + 7]));
            kk4.x = pack_bf16x2(__uint_as_float(w32[e]), __uint_as_float(w32[e + 1]));
            kk4.y = pack_bf16x2(__uint_as_float(w32[e + 2]), __uint_as_float(w32[e + 3]));
            kk4.z = pack_bf16x2(__uint_as_float(w32[e + 4]), __uint_as_float(w32[e + 5]));
            kk4.w = pack_bf16x2(__uint_as_float(w32[e + 6]), __uint_as_float(w32[e + 7]));
            *reinterpret_cast<uint4*>(dvr + c * 32 + e) = vv;
            *reinterpret_cast<uint4*>(dkr + c * 32 + e) = kk4;
          }
        }
      }
    } else if (n_it == 0 && ki < a.S) {
      // keys no query attends to (only possible with a window / non-causal edge cases)
      __nv_bfloat16* dkr = reinterpret_cast<__nv_bfloat16*>(g.dk) +
                           (static_cast<long long>(b) * a.S + ki) * g.dk_row + hk * D;
      __nv_bfloat16* dvr = reinterpret_cast<__nv_bfloat16*>(g.dv) +
                           (static_cast<long long>(b) * a.S + ki) * g.dv_row + hk * D;
      for (int c = 0; c < D; ++c) {
        dkr[c] = __float2bfloat16(0.f);
        dvr[c] = __float2bfloat16(0.f);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b, h, s] = sum_d dO * O
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, long long o_row,
                                  const __nv_bfloat16* __restrict__ dout, long long do_row,
                                  float* __restrict__ delta, int B, int S, int H, int D) {
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(B) * S * H;
  if (wid >= total) return;
  const int h = static_cast<int>(wid % H);
  const long long bs = wid / H;  // b*S + s
  const __nv_bfloat16* orow = o + bs * o_row + h * D;
  const __nv_bfloat16* drow = dout + bs * do_row + h * D;
  float acc = 0.f;
  for (int c = lane * 2; c < D; c += 64) {
    const float2 x = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(orow + c));
    const float2 y = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(drow + c));
    acc += x.x * y.x + x.y * y.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const long long b = bs / S, s = bs % S;
    delta[(b * H + h) * S + s] = acc;
  }
}

__global__ void attn_dq_cast_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                                    long long dq_row, int B, int S, int H, int D) {
  const long long n = static_cast<long long>(B) * S * H * D;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long tok = i / (static_cast<long long>(H) * D);
    const long long rem = i - tok * H * D;
    dq[tok * dq_row + rem] = __float2bfloat16(acc[i]);
  }
}

// ------------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    PLG_CUDA_CHECK(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                                    cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not found");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// [B, S, H, d] bf16 with token stride `row` (elements); box = 64 x 1 x 128 x 1
static CUtensorMap map_bshd(const void* base, int B, int S, int H, int d, long long row) {
  if (reinterpret_cast<uintptr_t>(base) & 15) throw std::invalid_argument("attention: base not 16B aligned");
  if ((row * 2) % 16) throw std::invalid_argument("attention: token stride must be a multiple of 8");
  CUtensorMap m;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(row) * 2,
                           static_cast<cuuint64_t>(row) * 2 * S};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                           strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("attention: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return m;
}

template <int D>
static void fwd_launch(const AttnArgs& a, cudaStream_t st) {
  using C = FwdCfg<D>;
  CUtensorMap tq = map_bshd(a.q, a.B, a.S, a.Hq, D, a.q_row);
  CUtensorMap tk = map_bshd(a.k, a.B, a.S, a.Hk, D, a.k_row);
  CUtensorMap tv = map_bshd(a.v, a.B, a.S, a.Hk, D, a.v_row);
  static bool set = false;
  if (!set) {
    PLG_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel<D>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    set = true;
  }
  dim3 grid((a.S + BQ - 1) / BQ, a.Hq, a.B);
  attn_fwd_kernel<D><<<grid, kThreads, C::kSmem, st>>>(tq, tk, tv, a);
  PLG_CUDA_CHECK(cudaGetLastError());
}

template <int D>
static void bwd_launch(const AttnBwdArgs& g, cudaStream_t st) {
  using C = BwdCfg<D>;
  const AttnArgs& a = g.f;
  CUtensorMap tq = map_bshd(a.q, a.B, a.S, a.Hq, D, a.q_row);
  CUtensorMap tk = map_bshd(a.k, a.B, a.S, a.Hk, D, a.k_row);
  CUtensorMap tv = map_bshd(a.v, a.B, a.S, a.Hk, D, a.v_row);
  CUtensorMap td = map_bshd(g.dout, a.B, a.S, a.Hq, D, g.do_row);
  static bool set = false;
  if (!set) {
    PLG_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel<D>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem));
    set = true;
  }
  const long long rows = static_cast<long long>(a.B) * a.S * a.Hq;
  attn_delta_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.o), a.o_row,
      reinterpret_cast<const __nv_bfloat16*>(g.dout), g.do_row, g.delta, a.B, a.S, a.Hq, D);
  PLG_CUDA_CHECK(cudaMemsetAsync(g.dq_acc, 0, sizeof(float) * rows * D, st));
  dim3 grid((a.S + BKV - 1) / BKV, a.Hk, a.B);
  attn_bwd_kernel<D><<<grid, kThreads, C::kSmem, st>>>(tq, tk, tv, td, g);
  PLG_CUDA_CHECK(cudaGetLastError());
  const long long n = rows * D;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  attn_dq_cast_kernel<<<blocks, 256, 0, st>>>(g.dq_acc, reinterpret_cast<__nv_bfloat16*>(g.dq),
                                              g.dq_row, a.B, a.S, a.Hq, D);
  PLG_CUDA_CHECK(cudaGetLastError());
}

}  // namespace attn

void attn_fwd(const AttnArgs& a, cudaStream_t st) {
  if (a.Hq % a.Hk) throw std::invalid_argument("attention: Hq must be a multiple of Hk");
  if (a.d == 128) return attn::fwd_launch<128>(a, st);
  if (a.d == 64) return attn::fwd_launch<64>(a, st);
  throw std::invalid_argument("attention: head_dim must be 64 or 128");
}

void attn_bwd(const AttnBwdArgs& g, cudaStream_t st) {
  const AttnArgs& a = g.f;
  if (a.Hq % a.Hk) throw std::invalid_argument("attention: Hq must be a multiple of Hk");
  if (a.d == 128) return attn::bwd_launch<128>(g, st);
  if (a.d == 64) return attn::bwd_launch<64>(g, st);
  throw std::invalid_argument("attention: head_dim must be 64 or 128");
}

}  // namespace plg
