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
// Forward: two query tiles per CTA with one softmax warpgroup each (see the
// comment above attn_fwd_kernel); P stays in TMEM.
// Backward, one CTA per (128-key tile, kv head, batch), looping over the q
// heads of the GQA group and the q tiles that see the keys:
//   S^T = K Q^T and dP^T = V dO^T into TMEM; per key row: P^T = exp2(S^T - lse),
//   dS^T = P^T (dP^T - delta) * scale, both written to smem; then
//   dV += P^T dO, dK += dS^T Q (TMEM accumulators for the whole loop) and
//   dQ_i = dS K (TMEM, then fp32 vector atomics into a workspace).
// delta = rowsum(dO * O) comes from a small pre-pass; a post-pass casts dQ.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <algorithm>
#include <stdexcept>
#include <string>

#include <type_traits>

#include "common.cuh"
#include "ops.h"

namespace plg {
namespace attn {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kBox = 128 * 128;  // bytes of one [128 rows x 64 bf16] swizzled box

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

// Bounded wait whose outcome is the same on every lane of the warp: a lane that
// gave up makes the whole warp give up, so the tcgen05 .sync.aligned loads and
// stores that follow never execute on a partial warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag)) != 0;
}

__device__ __forceinline__ bool key_ok(int qi, int ki, int S, int causal, int window) {
  return ki < S && qi < S && (!causal || ki <= qi) && (window <= 0 || qi - ki < window);
}

// --------------------------------------------------------------------- forward
// Two 128-row query tiles per CTA, one softmax warpgroup each, so that one
// group's softmax overlaps the tensor core working on the other group:
//   warps 0..3   softmax group 0 (query tile 0), warps 4..7 group 1
//   warp 8       TMA: Q tiles once, then K_t / V_t (two stages each, released
//                separately: K after the S MMAs, V after the PV MMAs)
//   warp 9       TMEM owner + MMA issuer, per tile t in the order
//                PV_0(t), S_0(t+1), PV_1(t), S_1(t+1)
//   warps 10,11  idle; with 8 and 9 they form the warpgroup whose registers
//                are handed to the softmax groups (setmaxnreg is per warpgroup)
// S_w lives in TMEM; the softmax group overwrites it in place with P (bf16,
// two per 32-bit column) and the PV MMA reads P straight from TMEM (A operand
// in tensor memory), so P never touches shared memory. O_w stays in TMEM; it
// is rescaled only when a row max grows by more than 2^8 (stale maxima keep
// p <= 256, safe in bf16/fp32). Masks are applied only on edge tiles, without
// branches.
// The two query tiles are two heads of one GQA group (same keys, same range)
// when the group size is even, else two consecutive row tiles of one head.
constexpr int kFwdThreads = 384;
constexpr int kFwdTmaWarp = 8, kFwdMmaWarp = 9;  // warps 10, 11 only lend registers
// Register split (setmaxnreg): launched at 168 per thread (the most 384 threads
// can hold), the control warpgroup drops to 80 and the softmax warpgroups rise
// to 208: 8*32*208 + 4*32*80 = 63488 <= 384*168 = 64512 registers, and each
// SM sub-partition (one warp of every warpgroup) needs 208+208+80 <= 512 per lane.
// Neither role spills at these limits.
constexpr int kFwdRegsSoftmax = 208, kFwdRegsCtl = 80, kFwdRegsLaunch = 168;
static_assert(8 * 32 * kFwdRegsSoftmax + 4 * 32 * kFwdRegsCtl <= kFwdThreads * kFwdRegsLaunch,
              "register split exceeds the launch allocation");
constexpr float kRescale = 8.0f;

template <int D>
struct Fwd {
  static constexpr int kTile = 128 * D * 2;
  static constexpr int kQ = 0;            // Q0, Q1
  static constexpr int kK = 2 * kTile;    // two stages
  static constexpr int kV = 4 * kTile;    // two stages
  static constexpr int kBar = 6 * kTile;
  static constexpr int kSmem = kBar + 256;
  static constexpr int kTO = 256;         // O_w at kTO + w * D
};

struct QTile {
  int h, qt, lo, hi;
};

__device__ __forceinline__ QTile make_qtile(const AttnArgs& a, int h, int qt) {
  QTile t;
  t.h = h;
  t.qt = qt;
  const int n_kv = (a.S + BKV - 1) / BKV;
  const int n_q = (a.S + BQ - 1) / BQ;
  if (qt >= n_q) {
    t.lo = 1;
    t.hi = 0;  // empty
    return t;
  }
  t.hi = a.causal ? min(qt, n_kv - 1) : n_kv - 1;
  t.lo = 0;
  if (a.window > 0) {
    const int lo_key = qt * BQ - a.window + 1;
    t.lo = lo_key > 0 ? lo_key / BKV : 0;
  }
  return t;
}

// One softmax row of a 128-key tile, in place: v holds raw scores (fp32 bits,
// masked entries already -inf); P, packed two bf16 per word, overwrites v[0, 64)
// (word j is written after scores 2j and 2j+1 were consumed); m/l are
// the running max (base 2, scaled) and sum. alpha is the factor the O row must
// be multiplied by (1 when the max did not move by more than 2^kRescale).
// kPolyMask selects which pairs of every eight pairs of exponentials run on the
// FMA pipe (exp2_poly2) instead of the SFU; it is used only on tiles without
// masked entries (0 on edge tiles).
template <int kPolyMask>
__device__ __forceinline__ void softmax_row(uint32_t (&v)[BKV], float scale2,
                                            float& m, float& l, float& alpha, float& rs) {
  float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
  for (int e = 0; e < BKV; e += 8) {
    m0 = fmax3(m0, __uint_as_float(v[e]), __uint_as_float(v[e + 1]));
    m1 = fmax3(m1, __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3]));
    m2 = fmax3(m2, __uint_as_float(v[e + 4]), __uint_as_float(v[e + 5]));
    m3 = fmax3(m3, __uint_as_float(v[e + 6]), __uint_as_float(v[e + 7]));
  }
  const float mx2 = fmax3(m0, m1, fmaxf(m2, m3)) * scale2;
  float m_new = m;
  if (mx2 > m + kRescale) m_new = mx2;  // also taken on the first tile (m = -inf)
  const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
  alpha = (m_new == m) ? 1.f : fast_exp2(m - m_use);
  const float nm = -m_use;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int e = 0; e < BKV; e += 2) {
    float x0, x1, p0, p1;
    ffma2(x0, x1, __uint_as_float(v[e]), __uint_as_float(v[e + 1]), scale2, scale2, nm, nm);
    if (kPolyMask != 0 && ((kPolyMask >> ((e >> 1) & 7)) & 1)) {
      exp2_poly2(x0, x1, p0, p1);
    } else {
      p0 = fast_exp2(x0);
      p1 = fast_exp2(x1);
    }
    const int q = ((e >> 1) & 3) * 2;
    fadd2(acc[q], acc[q + 1], acc[q], acc[q + 1], p0, p1);
    v[e >> 1] = pack_bf16x2(p0, p1);
  }
  rs = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
  l = l * alpha + rs;
  m = m_new;
}

template <int D, int kPolyMask>
__global__ void __launch_bounds__(kFwdThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnArgs a, int pair_heads) {
  using C = Fwd<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023) {
    if (threadIdx.x == 0) record_status(a.status, kBadArgument);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* k_empty = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2] per group
  uint64_t* p_full = bars + 11;   // [2] per group
  uint64_t* o_done = bars + 13;   // [2] per group
  uint64_t* mma_done = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.Hq / a.Hk;
  // 1-D grid ordered heaviest query tiles first across all heads and batches, so
  // that the causal tail is made of short CTAs (longest-first list scheduling)
  const int n_q = (a.S + BQ - 1) / BQ;
  const int units = pair_heads ? n_q : (n_q + 1) / 2;
  const int slots = pair_heads ? a.Hq / 2 : a.Hq;
  const int rank = blockIdx.x / (slots * a.B);
  const int rest = blockIdx.x - rank * slots * a.B;
  const int slot = rest % slots;
  const int b = rest / slots;
  const int unit = units - 1 - rank;
  QTile qtl[2];
  if (pair_heads) {
    qtl[0] = make_qtile(a, 2 * slot, unit);
    qtl[1] = make_qtile(a, 2 * slot + 1, unit);
  } else {
    qtl[0] = make_qtile(a, slot, 2 * unit);
    qtl[1] = make_qtile(a, slot, 2 * unit + 1);
  }
  const int hk = qtl[0].h / G;
  const bool live0 = qtl[0].hi >= qtl[0].lo, live1 = qtl[1].hi >= qtl[1].lo;
  const int t_lo = live1 && (!live0 || qtl[1].lo < qtl[0].lo) ? qtl[1].lo : qtl[0].lo;
  const int t_hi = live1 && (!live0 || qtl[1].hi > qtl[0].hi) ? qtl[1].hi : qtl[0].hi;
  const int n = (live0 || live1) ? t_hi - t_lo + 1 : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kFwdMmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  uint8_t* sQ = smem + C::kQ;
  uint8_t* sK = smem + C::kK;
  uint8_t* sV = smem + C::kV;

  // registers move from the TMA/MMA warpgroup to the two softmax warpgroups;
  // each setmaxnreg heads the branch of its warpgroup so the compiler applies
  // the matching register limit to all code of that role
  if (warp >= 8) {
  setmaxnreg_dec<kFwdRegsCtl>();
  if (warp == kFwdTmaWarp) {
    if (lane == 0 && n > 0) {
      bool ok = true;
      uint32_t kin = 0, vin = 0, kpar = 0, vpar = 0;  // stages in flight and their parity
      mbar_arrive_expect_tx(q_full, (live0 + live1) * C::kTile);
      for (int w = 0; w < 2; ++w) {
        if (w == 0 ? !live0 : !live1) continue;
#pragma unroll
        for (int x = 0; x < D / 64; ++x)
          tma_load_4d(sQ + w * C::kTile + x * kBox, &tmQ, q_full, x * 64, qtl[w].h, qtl[w].qt * BQ, b);
      }
      for (int i = 0; i < n && ok; ++i) {
        const int st = i & 1;
        const uint32_t par = ((i >> 1) - 1) & 1;
        const int kv0 = (t_lo + i) * BKV;
        if (i >= 2 && !mbar_wait_bounded(&k_empty[st], par, abort_flag)) { record_status(a.status, 17); ok = false; break; }
        mbar_arrive_expect_tx(&k_full[st], C::kTile);
#pragma unroll
        for (int x = 0; x < D / 64; ++x)
          tma_load_4d(sK + st * C::kTile + x * kBox, &tmK, &k_full[st], x * 64, hk, kv0, b);
        kin |= 1u << st;
        kpar = (kpar & ~(1u << st)) | (((i >> 1) & 1u) << st);
        if (i >= 2 && !mbar_wait_bounded(&v_empty[st], par, abort_flag)) { record_status(a.status, 18); ok = false; break; }
        mbar_arrive_expect_tx(&v_full[st], C::kTile);
#pragma unroll
        for (int x = 0; x < D / 64; ++x)
          tma_load_4d(sV + st * C::kTile + x * kBox, &tmV, &v_full[st], x * 64, hk, kv0, b);
        vin |= 1u << st;
        vpar = (vpar & ~(1u << st)) | (((i >> 1) & 1u) << st);
      }
      if (!ok) {
        record_status(a.status, kTimeoutSmemEmpty);
        *abort_flag = 1;
        mbar_wait_bounded(q_full, 0, nullptr);
        for (int st = 0; st < 2; ++st) {
          if (((kin >> st) & 1u) && !mbar_wait_bounded(&k_full[st], (kpar >> st) & 1u, nullptr))
            record_status(a.status, kTimeoutDrain);
          if (((vin >> st) & 1u) && !mbar_wait_bounded(&v_full[st], (vpar >> st) & 1u, nullptr))
            record_status(a.status, kTimeoutDrain);
        }
      }
    }
  } else if (warp == kFwdMmaWarp && n > 0) {
    // the whole warp walks the loop (warp-uniform descriptors); one lane issues
    const bool leader = elect_one_sync();
    constexpr uint32_t id_s = make_idesc_bf16_f32(128, 128, false, false);
    constexpr uint32_t id_o = make_idesc_bf16_f32(128, D, false, true);
    const uint64_t dQ0 = make_smem_desc(smem_u32(sQ), 16, 1024, kLayoutSW128);
    const uint64_t dK0 = make_smem_desc(smem_u32(sK), 16, 1024, kLayoutSW128);
    const uint64_t dV0 = make_smem_desc(smem_u32(sV), kBox, 1024, kLayoutSW128);
    const int lo0 = qtl[0].lo, hi0 = qtl[0].hi, lo1 = qtl[1].lo, hi1 = qtl[1].hi;
    auto issue_s = [&](int w, int i) {
      const int st = i & 1;
      if (leader) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc_mma_ss(tmem + w * 128, desc_advance(dQ0, w * C::kTile + (kk >> 2) * kBox + (kk & 3) * 32),
                    desc_advance(dK0, st * C::kTile + (kk >> 2) * kBox + (kk & 3) * 32), id_s,
                    kk > 0 ? 1u : 0u);
        tc_commit(&s_full[w]);
      }
      __syncwarp();
    };
    bool ok = warp_wait(q_full, 0, abort_flag) && warp_wait(&k_full[0], 0, abort_flag);
    if (ok) {
      tc_fence_after();
      if (t_lo >= lo0 && t_lo <= hi0) issue_s(0, 0);
      if (t_lo >= lo1 && t_lo <= hi1) issue_s(1, 0);
      if (leader) tc_commit(&k_empty[0]);
      __syncwarp();
    }
    for (int i = 0; i < n && ok; ++i) {
      const int t = t_lo + i, st = i & 1;
      if (!warp_wait(&v_full[st], (i >> 1) & 1, abort_flag)) {
        if (leader) record_status(a.status, 12);
        ok = false;
        break;
      }
      bool k_next = false;
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        const int lo = w == 0 ? lo0 : lo1, hi = w == 0 ? hi0 : hi1;
        if (ok && t >= lo && t <= hi) {
          const int u = t - lo;
          if (!warp_wait(&p_full[w], u & 1, abort_flag)) {
            if (leader) record_status(a.status, 13);
            ok = false;
          } else {
            tc_fence_after();
            if (leader) {
#pragma unroll
              for (int kk = 0; kk < BKV / 16; ++kk)
                tc_mma_ts(tmem + C::kTO + w * D, tmem + w * 128 + kk * 8,
                          desc_advance(dV0, st * C::kTile + kk * 2048), id_o,
                          (u > 0 || kk > 0) ? 1u : 0u);
            }
            __syncwarp();
          }
        }
        if (ok && i + 1 < n && t + 1 >= lo && t + 1 <= hi) {
          if (!k_next) {
            if (!warp_wait(&k_full[(i + 1) & 1], ((i + 1) >> 1) & 1, abort_flag)) {
              if (leader) record_status(a.status, 14);
              ok = false;
            } else {
              tc_fence_after();
              k_next = true;
            }
          }
          if (ok) issue_s(w, i + 1);
        }
      }
      if (!ok) break;
      if (leader) {
        tc_commit(&v_empty[st]);
        if (i + 1 < n) tc_commit(&k_empty[(i + 1) & 1]);
      }
      __syncwarp();
    }
    if (!ok) {
      if (leader) record_status(a.status, kTimeoutTmaFull);
      *abort_flag = 1;
    }
    if (leader) {
      tc_commit(&o_done[0]);
      tc_commit(&o_done[1]);
      tc_commit(mma_done);
    }
    __syncwarp();
    if (!warp_wait(mma_done, 0, nullptr) && leader) record_status(a.status, kTimeoutDrain);
  }
  } else {
    setmaxnreg_inc<kFwdRegsSoftmax>();
    // ------------------------------------------------------ softmax groups
    const int w = warp >> 2;
    const QTile me = qtl[w];
    const int nw = me.hi - me.lo + 1;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int q0 = me.qt * BQ;
    const int qi = q0 + r;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t tS = lane_base + w * 128;
    const uint32_t tO = lane_base + C::kTO + w * D;
    const float scale2 = a.scale * kLog2e;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int u = 0; u < nw && ok; ++u) {
      const int t = me.lo + u;
      if (!warp_wait(&s_full[w], u & 1, abort_flag)) {
        record_status(a.status, 15);
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const int kv0 = t * BKV;
      const bool edge = (a.causal && kv0 + BKV - 1 > q0) | (kv0 + BKV > a.S) |
                        (a.window > 0 && q0 + BQ - 1 - kv0 >= a.window);
      // the whole 128-column row of S in registers (one TMEM round trip)
      uint32_t v[BKV];
#pragma unroll
      for (int c = 0; c < BKV / 32; ++c)
        tmem_ld_32x32b_x32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v + c * 32));
      tmem_ld_wait();
      float alpha, rs;
      if (edge) {
        // valid key columns of this row form the range [c_lo, c_hi]
        int c_hi = (a.causal ? min(qi, a.S - 1) : a.S - 1) - kv0;
        const int c_lo = a.window > 0 ? qi - a.window + 1 - kv0 : 0;
        if (qi >= a.S) c_hi = -1;
#pragma unroll
        for (int e = 0; e < BKV; ++e)
          v[e] = (e >= c_lo && e <= c_hi) ? v[e] : 0xff800000u;  // -inf
        softmax_row<0>(v, scale2, m, l, alpha, rs);
      } else {
        softmax_row<kPolyMask>(v, scale2, m, l, alpha, rs);
      }
      tmem_st_32x32b_x32(tS, *reinterpret_cast<const uint32_t(*)[32]>(v));
      tmem_st_32x32b_x32(tS + 32, *reinterpret_cast<const uint32_t(*)[32]>(v + 32));
      if (u > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tO + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          tmem_st_32x32b_x32(tO + c * 32, v);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[w]);
    }
    if (ok && nw > 0) {
      if (warp_wait(&o_done[w], 0, abort_flag)) {
        tc_fence_after();
        const float inv_l = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.o) +
                              (static_cast<long long>(b) * a.S + qi) * a.o_row + me.h * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tO + c * 32, v);
          tmem_ld_wait();
          if (qi < a.S) {
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
              uint4 q4;
              q4.x = pack_bf16x2(__uint_as_float(v[e]) * inv_l, __uint_as_float(v[e + 1]) * inv_l);
              q4.y = pack_bf16x2(__uint_as_float(v[e + 2]) * inv_l, __uint_as_float(v[e + 3]) * inv_l);
              q4.z = pack_bf16x2(__uint_as_float(v[e + 4]) * inv_l, __uint_as_float(v[e + 5]) * inv_l);
              q4.w = pack_bf16x2(__uint_as_float(v[e + 6]) * inv_l, __uint_as_float(v[e + 7]) * inv_l);
              *reinterpret_cast<uint4*>(orow + c * 32 + e) = q4;
            }
          }
        }
        if (qi < a.S)
          a.lse[(static_cast<long long>(b) * a.Hq + me.h) * a.S + qi] =
              (l > 0.f) ? (m + log2f(l)) * kLn2 : -INFINITY;
      } else {
        record_status(a.status, 16);
        *abort_flag = 1;
      }
    }
  }
  __syncthreads();
  if (warp == kFwdMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// -------------------------------------------------------------------- backward
constexpr int kBwdThreads = 192;

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
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    AttnBwdArgs g) {
  using C = BwdCfg<D>;
  const AttnArgs& a = g.f;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
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
  uint64_t* stats_ready = bars + 9;  // lse/delta of an iteration staged in smem (4 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
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
    mbar_init(stats_ready, 4);
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
      __syncwarp();
      if (lane == 0) mbar_arrive(stats_ready);
      if (!warp_wait(stats_ready, it & 1, abort_flag)) {
        record_status(a.status, 25);
        *abort_flag = 1;
        ok = false;
        break;
      }
      if (!warp_wait(s_full, it & 1, abort_flag)) {
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
          float pv = fast_exp2(__uint_as_float(us[e]) * scale2 - s_lse[buf * 128 + qc]);
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
      if (!warp_wait(dq_full, it & 1, abort_flag)) {
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

// ------------------------------------------------ backward, head_dim 64 and 128
// One CTA per (128-key tile, kv head, batch), heaviest causal key tiles first.
// The loop runs over steps of 64 query rows (all q heads of the GQA group and
// every query block that sees the keys). Per step j, with buffers b = j & 1:
//   S^T_j  = K Q_j^T   -> TMEM S_b   (128 keys x 64 queries, fp32)
//   dP^T_j = V dO_j^T  -> TMEM dP_b
//   compute warps: P^T = exp2(S^T * scale*log2e - lse*log2e) -> bf16 into S_b,
//                  dS^T = P^T (dP^T * scale - delta * scale) -> bf16 into S_b
//                  and into smem
//   dV += P^T dO_j, dK += dS^T Q_j  (A operands from TMEM)
//   dQ^T_j = K^T dS^T_j -> TMEM dP_b (d x 64 queries), read out by the drain
//   warps, staged in smem and added into the fp32 dQ workspace with one bulk
//   tensor reduce-add per warp (red.global from registers measured 1.3x slower).
// The A operands that can come from TMEM do (P^T, dS^T), which spares shared
// memory the operand reads of dV and dK.
// The MMA warp issues S/dP of step j+1 before dV/dK/dQ of step j, so the
// compute warps work on step j+1 while the tensor core finishes step j.
// TMEM: dV [0,128), dK [128,256), S_b at 256+128b, dP_b at 320+128b. After the
// P / dS warps of query half h (queries 32h..32h+31) have read S_b, they overwrite
// S_b columns 32h..32h+15 with P^T and 32h+16..32h+31 with dS^T (bf16 pairs).
// lse*log2e and delta*scale come pre-negated from a pre-pass, padded to a
// multiple of 64 queries ([B*Hq][2][S64]) so each step fetches them with two
// 256-byte bulk copies; padded queries carry -inf / 0 and contribute nothing.
// head_dim 64 runs the same pipeline with half-width K/V/Q/dO tiles, dV/dK MMAs of
// N = 64 and a dQ^T MMA that keeps M = 128: its A operand (K^T, MN-major) spans two
// 64-row atoms and the second one is V's tile, which sits right after K's, so TMEM
// lanes 64..127 of dQ^T hold V^T dS^T and the drain warps of those lanes skip them.
// The P / dS work (exp2 and the dS products of 128 keys x 64 queries per step) is
// split over two warpgroups, one per 32-query half of the step: with one warpgroup
// the math of a step took longer than the step's five MMAs (SM-clock timeline of the
// pipeline), so the tensor core waited on it.
constexpr int kB3Threads = 512;
// warps 0..7 P / dS (warp w: key rows 32 * (w & 3).., queries 32 * (w >> 2)..),
// 8..11 dQ drain, 12 TMA producer, 13 MMA issuer
constexpr int kB3TmaWarp = 12, kB3MmaWarp = 13;
// setmaxnreg split of the 512 x 128 launch allocation: 256 * 152 + 128 * (112 + 96)
// = 65536, and 152 + 152 + 112 + 96 = 512 per lane of each SM sub-partition.
constexpr int kB3RegsComp = 152, kB3RegsDrain = 112, kB3RegsCtl = 96, kB3RegsLaunch = 128;
static_assert(256 * kB3RegsComp + 128 * (kB3RegsDrain + kB3RegsCtl) <= kB3Threads * kB3RegsLaunch,
              "register split exceeds the launch allocation");
static_assert(2 * kB3RegsComp + kB3RegsDrain + kB3RegsCtl <= 512,
              "register split exceeds a sub-partition's registers per lane");
constexpr int kBQ3 = 64;

template <int kD>
struct Bwd3 {
  static_assert(kD == 64 || kD == 128, "backward head_dim");
  static constexpr int D = kD;
  static constexpr int kKVTile = 128 * D * 2;  // 32 KB
  static constexpr int kQTile = kBQ3 * D * 2;  // 16 KB, two [64 x 64] boxes
  static constexpr int kQBox = kBQ3 * 128;     // bytes of one [64 rows x 64] box
  static constexpr int kStages = 3;
  static constexpr int kK = 0;
  static constexpr int kV = kKVTile;
  static constexpr int kQ = 2 * kKVTile;                      // [stage] Q, dO
  static constexpr int kDS = kQ + kStages * 2 * kQTile;       // [2] dS^T [128 x 64] bf16
  static constexpr int kDQ = kDS + 2 * 128 * kBQ3 * 2;        // [4 warps] dQ [64 q x 32 d] fp32
  static constexpr int kStats = kDQ + 4 * kBQ3 * 32 * 4;      // [stage] 2 x 64 floats
  static constexpr int kBar = kStats + kStages * 512;
  static constexpr int kSmem = kBar + 256 + 1024;             // + manual 1024 alignment
  static_assert(kSmem <= 232448, "backward shared memory exceeds the per-CTA limit");
  static constexpr int kTdV = 0, kTdK = 128;
  static constexpr int kTS0 = 256, kTdP0 = 320;               // + 128 * b
};

// Per-step timeline of CTA 0 (SM clock), recorded only when a trace buffer is
// given: 0 producer issued Q/dO, 1 MMA issued S/dP(j), 2 MMA saw P(j) ready,
// 3 MMA issued dQ(j), 4 compute saw S/dP(j), 5 compute released P(j), 6 drain saw
// dQ(j), 7 drain released the TMEM columns, 8 drain issued the reductions,
// 9 compute has S/dP in registers, 10 compute finished the math, 11 compute's
// P / dS stores completed.
__device__ __forceinline__ void trace_ev(long long* trace, int ev, int j) {
  if (trace != nullptr && blockIdx.x == 0 && j < kAttnTraceSteps)
    trace[ev * kAttnTraceSteps + j] = clock64();
}

template <int kD>
__global__ void __launch_bounds__(kB3Threads, 1)
    attn_bwd3_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                     const __grid_constant__ CUtensorMap tmDQ, AttnBwdArgs g) {
  using C = Bwd3<kD>;
  constexpr int D = C::D;
  static_assert(kD != 64 || C::kV == C::kK + kBox, "dQ^T's second A atom must be V's tile");
  const AttnArgs& a = g.f;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBar);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;    // [kStages]
  uint64_t* qd_empty = bars + 4;   // [kStages]
  uint64_t* s_full = bars + 7;     // [2]
  uint64_t* p_full = bars + 9;     // [2]
  uint64_t* dq_full = bars + 11;   // [2]
  uint64_t* dq_free = bars + 13;   // [2]
  uint64_t* mma_done = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_tile = a.Hk * a.B;
  const int jt = blockIdx.x / per_tile;
  const int rest = blockIdx.x - jt * per_tile;
  const int hk = rest % a.Hk, b = rest / a.Hk;
  const int G = a.Hq / a.Hk;
  const int kv0 = jt * BKV;
  const int n_qb = (a.S + kBQ3 - 1) / kBQ3;
  const int S64 = n_qb * kBQ3;
  const int qb_lo = a.causal ? kv0 / kBQ3 : 0;
  int qb_hi = n_qb - 1;
  if (a.window > 0) qb_hi = min(qb_hi, (kv0 + BKV - 1 + a.window - 1) / kBQ3);
  const int n = qb_hi >= qb_lo ? (qb_hi - qb_lo + 1) * G : 0;
  // step j: query block qb_lo + j / G, head hk * G + j % G

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&qd_full[s], 1);
      mbar_init(&qd_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_free[i], 4);
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kB3MmaWarp) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint8_t* sK = smem + C::kK;
  uint8_t* sV = smem + C::kV;
  auto sQ = [&](int s) { return smem + C::kQ + s * 2 * C::kQTile; };
  auto sDO = [&](int s) { return smem + C::kQ + s * 2 * C::kQTile + C::kQTile; };
  auto sDS = [&](int bb) { return smem + C::kDS + bb * 128 * kBQ3 * 2; };
  auto sStats = [&](int s) { return reinterpret_cast<float*>(smem + C::kStats + s * 512); };

  if (warp >= 12) {
    setmaxnreg_dec<kB3RegsCtl>();
    if (warp == kB3TmaWarp && lane == 0 && n > 0) {
      // ------------------------------------------------------------ producer
      bool ok = true;
      int last = -1;  // last step whose loads were issued
      mbar_arrive_expect_tx(kv_full, 2 * C::kKVTile);
#pragma unroll
      for (int x = 0; x < D / 64; ++x) {
        tma_load_4d(sK + x * kBox, &tmK, kv_full, x * 64, hk, kv0, b);
        tma_load_4d(sV + x * kBox, &tmV, kv_full, x * 64, hk, kv0, b);
      }
      for (int j = 0; j < n; ++j) {
        const int s = j % C::kStages, u = j / C::kStages;
        if (u > 0 && !mbar_wait_bounded(&qd_empty[s], (u - 1) & 1, abort_flag)) {
          record_status(a.status, 30);
          ok = false;
          break;
        }
        const int h = hk * G + j % G, q0 = (qb_lo + j / G) * kBQ3;
        mbar_arrive_expect_tx(&qd_full[s], 2 * C::kQTile + 512);
#pragma unroll
        for (int x = 0; x < D / 64; ++x) {
          tma_load_4d(sQ(s) + x * C::kQBox, &tmQ, &qd_full[s], x * 64, h, q0, b);
          tma_load_4d(sDO(s) + x * C::kQBox, &tmDO, &qd_full[s], x * 64, h, q0, b);
        }
        const float* st = g.delta + (static_cast<long long>(b) * a.Hq + h) * 2 * S64 + q0;
        bulk_load(sStats(s), st, 256, &qd_full[s]);
        bulk_load(sStats(s) + 64, st + S64, 256, &qd_full[s]);
        trace_ev(g.trace, 0, j);
        last = j;
      }
      if (!ok) {
        *abort_flag = 1;
        // let every copy still in flight land before the CTA can exit
        if (!mbar_wait_bounded(kv_full, 0, nullptr)) record_status(a.status, kTimeoutDrain);
        for (int j = last - C::kStages + 1; j <= last; ++j)
          if (j >= 0 && !mbar_wait_bounded(&qd_full[j % C::kStages], (j / C::kStages) & 1, nullptr))
            record_status(a.status, kTimeoutDrain);
      }
    } else if (warp == kB3MmaWarp && n > 0) {
      // ------------------------------------------------------------ MMA issuer
      // The whole warp walks the loop (descriptors stay warp-uniform); the
      // elected lane issues the MMAs and commits.
      const bool leader = elect_one_sync();
      constexpr uint32_t id_s = make_idesc_bf16_f32(128, kBQ3, false, false);  // S^T, dP^T
      constexpr uint32_t id_kv = make_idesc_bf16_f32(128, D, false, true);     // dV, dK
      constexpr uint32_t id_dq = make_idesc_bf16_f32(128, kBQ3, true, true);   // dQ^T
      const uint64_t kK = make_smem_desc(smem_u32(sK), 16, 1024, kLayoutSW128);
      const uint64_t kV = make_smem_desc(smem_u32(sV), 16, 1024, kLayoutSW128);
      const uint64_t mK = make_smem_desc(smem_u32(sK), kBox, 1024, kLayoutSW128);
      bool ok = warp_wait(kv_full, 0, abort_flag);
      if (!ok && leader) record_status(a.status, 31);
      auto issue_sdp = [&](int j) -> bool {
        const int s = j % C::kStages, bj = j & 1;
        if (!warp_wait(&qd_full[s], (j / C::kStages) & 1, abort_flag)) {
          if (leader) record_status(a.status, 32);
          return false;
        }
        tc_fence_after();
        const uint64_t kQ = make_smem_desc(smem_u32(sQ(s)), 16, 1024, kLayoutSW128);
        const uint64_t kDO = make_smem_desc(smem_u32(sDO(s)), 16, 1024, kLayoutSW128);
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            tc_mma_ss(tmem + C::kTS0 + 128 * bj, desc_advance(kK, (kk >> 2) * kBox + (kk & 3) * 32),
                      desc_advance(kQ, (kk >> 2) * C::kQBox + (kk & 3) * 32), id_s, kk > 0 ? 1u : 0u);
        }
        __syncwarp();
        // dP_b still holds dQ^T of step j-2 until the drain warps have read it
        if (j >= 2 && !warp_wait(&dq_free[bj], ((j - 2) >> 1) & 1, abort_flag)) {
          if (leader) record_status(a.status, 33);
          return false;
        }
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            tc_mma_ss(tmem + C::kTdP0 + 128 * bj, desc_advance(kV, (kk >> 2) * kBox + (kk & 3) * 32),
                      desc_advance(kDO, (kk >> 2) * C::kQBox + (kk & 3) * 32), id_s,
                      kk > 0 ? 1u : 0u);
          tc_commit(&s_full[bj]);
          trace_ev(g.trace, 1, j);
        }
        __syncwarp();
        return true;
      };
      if (ok) ok = issue_sdp(0);
      for (int j = 0; j < n && ok; ++j) {
        if (j + 1 < n && !issue_sdp(j + 1)) {
          ok = false;
          break;
        }
        const int s = j % C::kStages, bj = j & 1;
        if (!warp_wait(&p_full[bj], (j >> 1) & 1, abort_flag)) {
          if (leader) record_status(a.status, 34);
          ok = false;
          break;
        }
        if (leader) trace_ev(g.trace, 2, j);
        tc_fence_after();
        const uint64_t mQ = make_smem_desc(smem_u32(sQ(s)), C::kQBox, 1024, kLayoutSW128);
        const uint64_t mDO = make_smem_desc(smem_u32(sDO(s)), C::kQBox, 1024, kLayoutSW128);
        const uint64_t mDS = make_smem_desc(smem_u32(sDS(bj)), kBox, 1024, kLayoutSW128);
        const uint32_t acc0 = j > 0 ? 1u : 0u;
        if (leader) {
          // A operands from TMEM: P^T and dS^T of query half h (16 queries per k-step,
          // 8 packed columns) sit at S_b columns 32h.. and 32h + 16..
#pragma unroll
          for (int kk = 0; kk < kBQ3 / 16; ++kk)
            tc_mma_ts(tmem + C::kTdV, tmem + C::kTS0 + 128 * bj + (kk >> 1) * 32 + (kk & 1) * 8,
                      desc_advance(mDO, kk * 2048), id_kv, kk > 0 ? 1u : acc0);
#pragma unroll
          for (int kk = 0; kk < kBQ3 / 16; ++kk)
            tc_mma_ts(tmem + C::kTdK, tmem + C::kTS0 + 128 * bj + (kk >> 1) * 32 + 16 + (kk & 1) * 8,
                      desc_advance(mQ, kk * 2048), id_kv, kk > 0 ? 1u : acc0);
          tc_commit(&qd_empty[s]);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            tc_mma_ss(tmem + C::kTdP0 + 128 * bj, desc_advance(mK, kk * 2048),
                      desc_advance(mDS, kk * 2048), id_dq, kk > 0 ? 1u : 0u);
          tc_commit(&dq_full[bj]);
          trace_ev(g.trace, 3, j);
        }
        __syncwarp();
      }
      if (!ok) *abort_flag = 1;
      if (leader) tc_commit(mma_done);
      __syncwarp();
      if (!warp_wait(mma_done, 0, nullptr) && leader) record_status(a.status, kTimeoutDrain);
    }
  } else if (warp >= 8) {
    setmaxnreg_dec<kB3RegsDrain>();
    // -------------------------------------------------------------- dQ drain
    const int quad = warp & 3;          // TMEM lanes = head-dim rows 32*quad.. of dQ^T
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    float* stg = reinterpret_cast<float*>(smem + C::kDQ) + quad * kBQ3 * 32;
    for (int j = 0; j < n; ++j) {
      const int bj = j & 1;
      if (!warp_wait(&dq_full[bj], (j >> 1) & 1, abort_flag)) {
        record_status(a.status, 35);
        *abort_flag = 1;
        break;
      }
      if (lane == 0 && quad == 0) trace_ev(g.trace, 6, j);
      tc_fence_after();
      const bool live = quad * 32 < D;  // TMEM lanes that are rows of dQ^T
      uint32_t v[kBQ3];
      if (live) {
        tmem_ld_32x32b_x32(trow + C::kTdP0 + 128 * bj, *reinterpret_cast<uint32_t(*)[32]>(v));
        tmem_ld_32x32b_x32(trow + C::kTdP0 + 128 * bj + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
        tmem_ld_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_free[bj]);
      if (lane == 0 && quad == 0) trace_ev(g.trace, 7, j);
      if (!live) continue;
      // stage this warp's [64 q x 32 d] slice and reduce-add it into the fp32
      // workspace with one bulk tensor operation (rows past S are clipped)
      if (lane == 0) bulk_wait_group_read<0>();  // previous slice has left smem
      __syncwarp();
#pragma unroll
      for (int c = 0; c < kBQ3; ++c) stg[c * 32 + lane] = __uint_as_float(v[c]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int h = hk * G + j % G, q0 = (qb_lo + j / G) * kBQ3;
        tma_reduce_add_4d(&tmDQ, stg, quad * 32, h, q0, b);
        bulk_commit_group();
      }
      if (lane == 0 && quad == 0) trace_ev(g.trace, 8, j);
    }
    if (lane == 0) bulk_wait_group<0>();  // reductions done before the CTA exits
    __syncwarp();
  } else {
    setmaxnreg_inc<kB3RegsComp>();
    // ----------------------------------------------------------- P / dS warps
    constexpr int kHalf = kBQ3 / 2;  // queries per warp per step
    const int quad = warp & 3, half = warp >> 2;
    const int r = quad * 32 + lane;  // TMEM lane = key row
    const int ki = kv0 + r;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float scale2 = a.scale * kLog2e, scale = a.scale;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int s = j % C::kStages, bj = j & 1;
      if (!warp_wait(&s_full[bj], (j >> 1) & 1, abort_flag) ||
          !warp_wait(&qd_full[s], (j / C::kStages) & 1, abort_flag)) {
        record_status(a.status, 36);
        *abort_flag = 1;
        ok = false;
        break;
      }
      if (lane == 0 && warp == 0) trace_ev(g.trace, 4, j);
      tc_fence_after();
      const int q0 = (qb_lo + j / G) * kBQ3 + half * kHalf;  // first query of this warp
      uint32_t sv[kHalf], dv[kHalf];
      tmem_ld_32x32b_x32(trow + C::kTS0 + 128 * bj + half * kHalf, sv);
      tmem_ld_32x32b_x32(trow + C::kTdP0 + 128 * bj + half * kHalf, dv);
      // [0, 64): -lse * log2(e), [64, 128): -delta * scale of the step's 64 queries
      const float4* st4 = reinterpret_cast<const float4*>(sStats(s)) + half * (kHalf / 4);
      const bool edge = (a.causal && kv0 + BKV - 1 > q0) ||
                        (a.window > 0 && q0 + kHalf - 1 - kv0 >= a.window);
      const int c_lo = a.causal ? ki - q0 : -(1 << 30);
      const int c_hi = a.window > 0 ? ki + a.window - 1 - q0 : (1 << 30);
      tmem_ld_wait();
      if (lane == 0 && warp == 0) trace_ev(g.trace, 9, j);
      uint32_t pk[kHalf / 2], dk[kHalf / 2];
#pragma unroll
      for (int c = 0; c < kHalf; c += 4) {
        const float4 nl = st4[c / 4];                // -lse * log2(e)
        const float4 nd = st4[kBQ3 / 4 + c / 4];     // -delta * scale
        float p0 = fast_exp2(fmaf(__uint_as_float(sv[c]), scale2, nl.x));
        float p1 = fast_exp2(fmaf(__uint_as_float(sv[c + 1]), scale2, nl.y));
        float p2 = fast_exp2(fmaf(__uint_as_float(sv[c + 2]), scale2, nl.z));
        float p3 = fast_exp2(fmaf(__uint_as_float(sv[c + 3]), scale2, nl.w));
        if (edge) {
          p0 = (c >= c_lo && c <= c_hi) ? p0 : 0.f;
          p1 = (c + 1 >= c_lo && c + 1 <= c_hi) ? p1 : 0.f;
          p2 = (c + 2 >= c_lo && c + 2 <= c_hi) ? p2 : 0.f;
          p3 = (c + 3 >= c_lo && c + 3 <= c_hi) ? p3 : 0.f;
        }
        const float t0 = fmaf(__uint_as_float(dv[c]), scale, nd.x) * p0;
        const float t1 = fmaf(__uint_as_float(dv[c + 1]), scale, nd.y) * p1;
        const float t2 = fmaf(__uint_as_float(dv[c + 2]), scale, nd.z) * p2;
        const float t3 = fmaf(__uint_as_float(dv[c + 3]), scale, nd.w) * p3;
        pk[c / 2] = pack_bf16x2(p0, p1);
        pk[c / 2 + 1] = pack_bf16x2(p2, p3);
        dk[c / 2] = pack_bf16x2(t0, t1);
        dk[c / 2 + 1] = pack_bf16x2(t2, t3);
      }
      if (lane == 0 && warp == 0) trace_ev(g.trace, 10, j);
      // P^T and dS^T (two bf16 per column) into the 32 S columns this warp has read
      // itself (the other half's columns may still be unread), dS^T also into this
      // half's 64 bytes of the key row in smem (SW128 rows of 128 bytes) for dQ
      tmem_st_32x32b_x16(trow + C::kTS0 + 128 * bj + half * kHalf, pk);
      tmem_st_32x32b_x16(trow + C::kTS0 + 128 * bj + half * kHalf + kHalf / 2, dk);
      uint8_t* ds_row = sDS(bj) + r * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c16 = half * 4 + i;
        *reinterpret_cast<uint4*>(ds_row + ((c16 ^ (r & 7)) << 4)) =
            make_uint4(dk[i * 4], dk[i * 4 + 1], dk[i * 4 + 2], dk[i * 4 + 3]);
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      if (lane == 0 && warp == 0) trace_ev(g.trace, 11, j);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[bj]);
      if (lane == 0 && warp == 0) trace_ev(g.trace, 5, j);
    }
    // dK, dV of this key tile: each half writes half of the head_dim columns
    constexpr int kCols = D / 2;
    __nv_bfloat16* dkr = reinterpret_cast<__nv_bfloat16*>(g.dk) +
                         (static_cast<long long>(b) * a.S + ki) * g.dk_row + hk * D + half * kCols;
    __nv_bfloat16* dvr = reinterpret_cast<__nv_bfloat16*>(g.dv) +
                         (static_cast<long long>(b) * a.S + ki) * g.dv_row + hk * D + half * kCols;
    if (n == 0) {
      if (ki < a.S)
        for (int c = 0; c < kCols; c += 8) {
          *reinterpret_cast<uint4*>(dkr + c) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(dvr + c) = make_uint4(0, 0, 0, 0);
        }
    } else if (ok) {
      if (warp_wait(mma_done, 0, abort_flag)) {
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < kCols / 32; ++c) {
          uint32_t u[32], w32[32];
          tmem_ld_32x32b_x32(trow + C::kTdV + half * kCols + c * 32, u);
          tmem_ld_32x32b_x32(trow + C::kTdK + half * kCols + c * 32, w32);
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
      } else {
        record_status(a.status, 37);
        *abort_flag = 1;
      }
    }
  }
  __syncthreads();
  if (warp == kB3MmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Backward pre-pass of the pipelined kernel: per (b, h) row of the stats workspace
// [B*Hq][2][S64], -lse*log2(e) and -scale * rowsum(dO * O); queries beyond S get -inf
// and 0. Half a warp per four consecutive positions of one (b, h) (S64 is a multiple of
// 64): D / 16 channels per lane and row, the eight row loads of a lane issued before
// any math, lanes 0..3 writing the four results.
template <int D>
__global__ void attn_bwd_stats_kernel(const __nv_bfloat16* __restrict__ o, long long o_row,
                                      const __nv_bfloat16* __restrict__ dout, long long do_row,
                                      const float* __restrict__ lse, float* __restrict__ stats,
                                      int B, int S, int S64, int H, float scale) {
  static_assert(D == 64 || D == 128, "stats head_dim");
  constexpr int R = 4;
  using V = std::conditional_t<D == 128, uint4, uint2>;  // D / 16 bf16 per lane
  constexpr int NW = sizeof(V) / 4;
  const long long r0 = ((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 4) * R;
  const int l16 = threadIdx.x & 15;
  const long long total = static_cast<long long>(B) * S64 * H;
  const bool valid = r0 < total;
  const long long rid = valid ? r0 : 0;  // every lane takes part in the shuffles
  const int s0 = static_cast<int>(rid % S64);
  const long long bh = rid / S64;
  const int h = static_cast<int>(bh % H), bb = static_cast<int>(bh / H);
  V ov[R], dv[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int s = s0 + r;
    if (valid && s < S) {
      const long long tok = static_cast<long long>(bb) * S + s;
      ov[r] = *reinterpret_cast<const V*>(o + tok * o_row + h * D + l16 * (D / 16));
      dv[r] = *reinterpret_cast<const V*>(dout + tok * do_row + h * D + l16 * (D / 16));
    }
  }
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    acc[r] = 0.f;
    if (valid && s0 + r < S) {
      const uint32_t* ow = reinterpret_cast<const uint32_t*>(&ov[r]);
      const uint32_t* dw = reinterpret_cast<const uint32_t*>(&dv[r]);
#pragma unroll
      for (int e = 0; e < NW; ++e) {
        const float2 x = unpack_bf16x2(ow[e]), y = unpack_bf16x2(dw[e]);
        acc[r] = fmaf(x.x, y.x, fmaf(x.y, y.y, acc[r]));
      }
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
  }
  if (valid && l16 < R) {
    float a = acc[0];
#pragma unroll
    for (int r = 1; r < R; ++r)
      if (l16 == r) a = acc[r];
    const int s = s0 + l16;
    float* row = stats + (static_cast<long long>(bb) * H + h) * 2 * S64;
    if (s >= S) {
      row[s] = -INFINITY;
      row[S64 + s] = 0.f;
    } else {
      row[s] = -lse[(static_cast<long long>(bb) * H + h) * S + s] * kLog2e;
      row[S64 + s] = -a * scale;
    }
  }
}

// dQ workspace (fp32 [B*S, H*D]) -> bf16 rows with stride dq_row; 8 values per access
__global__ void attn_dq_cast8_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                                     long long dq_row, long long tokens, int HD) {
  // flat index over 8-value groups; four groups per thread in flight per iteration
  const int c8 = HD / 8;
  const long long n8 = tokens * c8;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  constexpr int U = 4;
  for (long long i0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < n8;
       i0 += U * stride) {
    float4 x[U], y[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + u * stride;
      if (i < n8) {
        const float4* src = reinterpret_cast<const float4*>(acc) + 2 * i;
        x[u] = src[0];
        y[u] = src[1];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = i0 + u * stride;
      if (i < n8) {
        const long long t = i / c8;
        const int c = static_cast<int>(i - t * c8);
        uint4 v;
        v.x = pack_bf16x2(x[u].x, x[u].y);
        v.y = pack_bf16x2(x[u].z, x[u].w);
        v.z = pack_bf16x2(y[u].x, y[u].y);
        v.w = pack_bf16x2(y[u].z, y[u].w);
        *reinterpret_cast<uint4*>(dq + t * dq_row + c * 8) = v;
      }
    }
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
// [B, S, H, d] bf16 with token stride `row` (elements); box = 64 x 1 x box_rows x 1
static CUtensorMap map_bshd(const void* base, int B, int S, int H, int d, long long row,
                            int box_rows = 128) {
  if (reinterpret_cast<uintptr_t>(base) & 15) throw std::invalid_argument("attention: base not 16B aligned");
  if ((row * 2) % 16) throw std::invalid_argument("attention: token stride must be a multiple of 8");
  CUtensorMap m;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(d) * 2, static_cast<cuuint64_t>(row) * 2,
                           static_cast<cuuint64_t>(row) * 2 * S};
  cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = encode_tensor_map(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base),
                                 dims, strides, box, es, CU_TENSOR_MAP_SWIZZLE_128B);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("attention: cuTensorMapEncodeTiled failed (" + std::to_string(r) +
                             ") dims {" + std::to_string(d) + "," + std::to_string(H) + "," +
                             std::to_string(S) + "," + std::to_string(B) + "} row " +
                             std::to_string(row) + " base " +
                             std::to_string(reinterpret_cast<uintptr_t>(base)));
  return m;
}

// fp32 dQ workspace [B, S, Hq, d] for bulk reduce-add; box = 32 d x 1 x 64 q x 1
static CUtensorMap map_dq_acc(float* base, int B, int S, int H, int d) {
  CUtensorMap m;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(d) * 4, static_cast<cuuint64_t>(H) * d * 4,
                           static_cast<cuuint64_t>(H) * d * 4 * S};
  cuuint32_t box[4] = {32, 1, static_cast<cuuint32_t>(kBQ3), 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = encode_tensor_map(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, box, es,
                                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("attention: dQ workspace tensor map failed (" + std::to_string(r) + ")");
  return m;
}

template <int D, int kPolyMask>
static void fwd_launch_t(const AttnArgs& a, cudaStream_t st);

template <int D>
static void fwd_launch(const AttnArgs& a, cudaStream_t st) {
  // share of the exponentials computed on the FMA pipe, in pairs per eight pairs
  // (PLG_ATTN_POLY = 2, 3 or 4). Measured at B=8, S=4096, 16q/8kv x 128: 2 -> 0.552 ms,
  // 3 -> 0.547 ms, 4 -> 0.575 ms (the FMA pipe becomes the limiter); 3 by default.
  static const int poly = [] {
    const char* e = std::getenv("PLG_ATTN_POLY");
    const int v = e ? std::atoi(e) : 3;
    return (v == 2 || v == 4) ? v : 3;
  }();
  if (poly == 3) return fwd_launch_t<D, 0xA4>(a, st);  // pairs 2, 5, 7
  if (poly == 4) return fwd_launch_t<D, 0xAA>(a, st);  // odd pairs
  return fwd_launch_t<D, 0x88>(a, st);                 // pairs 3, 7
}

template <int D, int kPolyMask>
static void fwd_launch_t(const AttnArgs& a, cudaStream_t st) {
  using C = Fwd<D>;
  CUtensorMap tq = map_bshd(a.q, a.B, a.S, a.Hq, D, a.q_row);
  CUtensorMap tk = map_bshd(a.k, a.B, a.S, a.Hk, D, a.k_row);
  CUtensorMap tv = map_bshd(a.v, a.B, a.S, a.Hk, D, a.v_row);
  set_max_smem_once(reinterpret_cast<const void*>(attn_fwd_kernel<D, kPolyMask>), C::kSmem);
  static const int regs = [] {
    cudaFuncAttributes fa;
    PLG_CUDA_CHECK(cudaFuncGetAttributes(&fa, attn_fwd_kernel<D, kPolyMask>));
    return fa.numRegs;
  }();
  // the setmaxnreg split assumes this launch allocation; with fewer registers
  // the softmax warpgroups' increase could never be granted
  if (regs != kFwdRegsLaunch)
    throw std::runtime_error("attention forward: kernel built with " + std::to_string(regs) +
                             " registers per thread, the register split needs " +
                             std::to_string(kFwdRegsLaunch));
  const int G = a.Hq / a.Hk;
  const int n_q = (a.S + BQ - 1) / BQ;
  const int pair_heads = (G % 2 == 0) ? 1 : 0;
  const long long units = pair_heads ? n_q : (n_q + 1) / 2;
  const long long ctas = units * (pair_heads ? a.Hq / 2 : a.Hq) * a.B;
  if (ctas > 0x7fffffffLL) throw std::invalid_argument("attention: problem too large for one launch");
  attn_fwd_kernel<D, kPolyMask><<<static_cast<unsigned>(ctas), kFwdThreads, C::kSmem, st>>>(tq, tk, tv, a,
                                                                                       pair_heads);
  PLG_CUDA_CHECK(cudaGetLastError());
}

template <int D>
static void bwd3_launch(const AttnBwdArgs& g, cudaStream_t st) {
  using C = Bwd3<D>;
  const AttnArgs& a = g.f;
  CUtensorMap tq = map_bshd(a.q, a.B, a.S, a.Hq, C::D, a.q_row, kBQ3);
  CUtensorMap tk = map_bshd(a.k, a.B, a.S, a.Hk, C::D, a.k_row);
  CUtensorMap tv = map_bshd(a.v, a.B, a.S, a.Hk, C::D, a.v_row);
  CUtensorMap td = map_bshd(g.dout, a.B, a.S, a.Hq, C::D, g.do_row, kBQ3);
  CUtensorMap tdq = map_dq_acc(g.dq_acc, a.B, a.S, a.Hq, C::D);
  set_max_smem_once(reinterpret_cast<const void*>(attn_bwd3_kernel<D>), C::kSmem);
  static const int regs = [] {
    cudaFuncAttributes fa;
    PLG_CUDA_CHECK(cudaFuncGetAttributes(&fa, attn_bwd3_kernel<D>));
    return fa.numRegs;
  }();
  if (regs != kB3RegsLaunch)
    throw std::runtime_error("attention backward: kernel built with " + std::to_string(regs) +
                             " registers per thread, the register split needs " +
                             std::to_string(kB3RegsLaunch));
  const int S64 = (a.S + kBQ3 - 1) / kBQ3 * kBQ3;
  const long long srows = static_cast<long long>(a.B) * S64 * a.Hq;
  if ((a.o_row % 8) || (g.do_row % 8) || (g.dq_row % 8) ||
      (reinterpret_cast<uintptr_t>(a.o) & 15) || (reinterpret_cast<uintptr_t>(g.dout) & 15) ||
      (reinterpret_cast<uintptr_t>(g.dq) & 15))
    throw std::invalid_argument("attention backward: o, dout and dq rows must be 16-byte aligned");
  PLG_CUDA_CHECK(cudaMemsetAsync(g.dq_acc, 0,
                                  sizeof(float) * static_cast<size_t>(a.B) * a.S * a.Hq * D, st));
  attn_bwd_stats_kernel<D><<<(srows * 4 + 255) / 256, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.o), a.o_row,
      reinterpret_cast<const __nv_bfloat16*>(g.dout), g.do_row, a.lse, g.delta, a.B, a.S, S64, a.Hq,
      a.scale);
  PLG_CUDA_CHECK(cudaGetLastError());
  const long long ctas = static_cast<long long>((a.S + BKV - 1) / BKV) * a.Hk * a.B;
  if (ctas > 0x7fffffffLL) throw std::invalid_argument("attention: problem too large for one launch");
  attn_bwd3_kernel<D><<<static_cast<unsigned>(ctas), kB3Threads, C::kSmem, st>>>(tq, tk, tv, td,
                                                                                       tdq, g);
  PLG_CUDA_CHECK(cudaGetLastError());
  const long long tokens = static_cast<long long>(a.B) * a.S;
  const long long groups = tokens * (a.Hq * C::D / 8);
  const long long cblocks = std::max(1LL, std::min<long long>((groups + 255) / 256, 148 * 8));
  attn_dq_cast8_kernel<<<static_cast<unsigned>(cblocks), 256, 0, st>>>(
      g.dq_acc, reinterpret_cast<__nv_bfloat16*>(g.dq), g.dq_row, tokens, a.Hq * C::D);
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
  set_max_smem_once(reinterpret_cast<const void*>(attn_bwd_kernel<D>), C::kSmem);
  const long long rows = static_cast<long long>(a.B) * a.S * a.Hq;
  attn_delta_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.o), a.o_row,
      reinterpret_cast<const __nv_bfloat16*>(g.dout), g.do_row, g.delta, a.B, a.S, a.Hq, D);
  PLG_CUDA_CHECK(cudaMemsetAsync(g.dq_acc, 0, sizeof(float) * rows * D, st));
  dim3 grid((a.S + BKV - 1) / BKV, a.Hk, a.B);
  attn_bwd_kernel<D><<<grid, kBwdThreads, C::kSmem, st>>>(tq, tk, tv, td, g);
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
  if (a.d == 128) return attn::bwd3_launch<128>(g, st);
  if (a.d == 64) {
    // PLG_ATTN_BWD64=group selects the single-group head_dim-64 kernel
    static const bool group = [] {
      const char* e = std::getenv("PLG_ATTN_BWD64");
      return e != nullptr && std::string(e) == "group";
    }();
    return group ? attn::bwd_launch<64>(g, st) : attn::bwd3_launch<64>(g, st);
  }
  throw std::invalid_argument("attention: head_dim must be 64 or 128");
}

}  // namespace plg
