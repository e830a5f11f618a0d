// Persistent bf16 GEMM on the sm_100a 5th-generation tensor cores.
//
//   C[M,N] = alpha * sum_k A(m,k) * B(n,k)  (+ beta * D[M,N])
//
// A is K-major ([M,K] row-major) or M-major ([K,M] row-major); B likewise
// ([N,K] or [K,N]). These three combinations cover a linear layer:
//   forward  y  = x  W^T : A K-major (x [T,K]),  B K-major (W [N,K])
//   dgrad    dx = dy W   : A K-major (dy [T,N]), B N-major (W [N,K] read as [K=N,N=K])
//   wgrad    dW = dy^T x : A M-major (dy [T,N]), B N-major (x [T,K])
// Replaces the reference's cuBLAS calls behind nn.Linear under autocast
// (pluggy/models/qwen3/qwen3.py:94-97,207-215; pluggy/loss/fused_linear_ce.py:31-58).
//
// Structure (one CTA per SM, grid-stride over output tiles):
//   warp 0      TMA producer: per k-block, one elected thread waits for a free
//               smem stage and issues the A and B tile loads (128-byte swizzle,
//               no multicast) onto the stage's mbarrier.
//   warp 1      allocates TMEM (2 accumulators x BN fp32 columns), then one
//               thread issues tcgen05.mma 128xBNx16 per 16-wide k step and
//               commits each stage back to the producer and each finished tile
//               to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows), optional alpha/beta*D, convert,
//               store; split-K partial sums are added with vector fp32 atomics.
// The epilogue of tile i overlaps the main loop of tile i+1 (double-buffered
// accumulator). Every wait is bounded (common.cuh).
#include <cudaTypedefs.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "ops.h"

namespace plg {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;

struct Args {
  int M, N, K;
  void* C;
  long long ldc;
  const void* D;
  long long ldd;
  float alpha, beta;
  int c_fp32, d_fp32;
  int splits;        // >1: fp32 atomic accumulation into C
  int m_tiles, n_tiles, k_blocks;
  int raster_m;      // 1: m-tiles vary fastest
  int* status;
  // reduce-scatter epilogue (see GemmProblem)
  int rs_n, rs_rank;
  int rs_mshift;     // m-tile rotation: each rank starts on a different owner's rows
  long long rs_S, rs_seg, rs_rows;
  long long rs_cap_rows;  // rows of N that fit in every staging buffer
  void* rs_dst[8];
  // grouped GEMM (MoE experts; see GemmProblem): 0 none, 1 a group per m tile,
  // 2 a k range per group
  int grp_mode;
  const int* grp_tile;   // mode 1: [m_tiles] group of each m tile (-1: no work)
  long long grp_b_rows;  // mode 1: rows of B per group (B is [groups * rows, cols])
  const int* grp_koff;   // mode 2: [groups + 1] row offsets of the k ranges (multiples of BK)
  long long grp_c_rows;  // mode 2: rows of C per group (C is [groups * M, N])
  int grp_count;         // mode 2: number of groups
};

// destination of row `row` under the reduce-scatter epilogue; static indices only
// (a dynamically indexed kernel parameter would be copied to local memory)
__device__ __forceinline__ __nv_bfloat16* rs_row_ptr(const Args& args, long long row) {
  const long long b = row / args.rs_S, s = row - b * args.rs_S;
  const int owner = static_cast<int>(s / args.rs_seg);
  const long long lrow = b * args.rs_seg + (s - owner * args.rs_seg);
  void* base = args.rs_dst[0];
#pragma unroll
  for (int j = 1; j < 8; ++j)
    if (owner == j) base = args.rs_dst[j];
  return reinterpret_cast<__nv_bfloat16*>(base) + (args.rs_rank * args.rs_rows + lrow) * args.ldc;
}

// per epilogue warp: a 32 x 64 bf16 chunk for the reduce-scatter epilogue
constexpr int kEpiStageBytes = 4 * 32 * 128;

template <int BN>
struct Cfg {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // 256 or 512: a power of two
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/ +
                                    kEpiStageBytes;
};

// Epilogue of one accumulator row (this thread's TMEM lane): BN fp32 columns at
// t_row -> alpha * acc (+ beta * D) -> C (bf16 / fp32 / split-K fp32 atomics).
// Reduce-scatter epilogue of one warp's 32 accumulator rows: the rows go to a
// peer's staging buffer over NVLink, where 16-byte stores scattered over 32 rows
// would waste most of each link transaction. So the warp writes each 32 x 64
// chunk (bf16) into its shared-memory slot (16-byte groups XOR-swizzled against
// bank conflicts) and stores it back out row-contiguously: 8 lanes cover one
// row's 128 bytes, 4 rows per instruction. A warp's 32 rows lie in one sequence
// segment (segment length % 32 == 0), so they are consecutive rows of one owner.
template <int BN>
__device__ __forceinline__ void store_acc_rows_rs(const Args& args, uint32_t t_row, long long row,
                                                  int col_base, uint8_t* stage) {
  const int lane = threadIdx.x & 31;
  const long long row_base = row - lane;
  if (row_base >= args.M) return;  // warp-uniform
  __nv_bfloat16* wbase = rs_row_ptr(args, row_base);
  {
    // the warp's 32 rows must lie inside the owner's staging buffer
    const long long b = row_base / args.rs_S, s = row_base - b * args.rs_S;
    const long long lrow = b * args.rs_seg + s % args.rs_seg;
    if (args.rs_rank * args.rs_rows + lrow + 32 > args.rs_cap_rows) {
      if ((threadIdx.x & 31) == 0) record_status(args.status, kOutOfBounds);
      return;
    }
  }
#pragma unroll 1
  for (int cp = 0; cp < BN / 64; ++cp) {
    uint32_t u[32];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t r[32];
      __syncwarp();
      tmem_ld_32x32b_x32(t_row + (cp * 2 + h) * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i)
        u[h * 16 + i] = pack_bf16x2(__uint_as_float(r[2 * i]) * args.alpha,
                                    __uint_as_float(r[2 * i + 1]) * args.alpha);
    }
    uint4* srow = reinterpret_cast<uint4*>(stage + lane * 128);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      srow[k ^ (lane & 7)] = make_uint4(u[4 * k], u[4 * k + 1], u[4 * k + 2], u[4 * k + 3]);
    __syncwarp();
    const int col0 = col_base + cp * 64;
    const int k = lane & 7;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int rl = it * 4 + (lane >> 3);
      const int col = col0 + k * 8;
      if (row_base + rl < args.M && col < args.N) {
        const uint4 v = reinterpret_cast<const uint4*>(stage + rl * 128)[k ^ (rl & 7)];
        *reinterpret_cast<uint4*>(wbase + rl * args.ldc + col) = v;
      }
    }
  }
  __syncwarp();
}

template <int BN>
__device__ __forceinline__ void store_acc_row(const Args& args, uint32_t t_row, long long row,
                                              bool row_ok, int col_base, int kb0, uint8_t* stage,
                                              bool zero = false) {
  if (args.rs_n) {
    store_acc_rows_rs<BN>(args, t_row, row, col_base, stage);
    return;
  }
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    __syncwarp();
    tmem_ld_32x32b_x32(t_row + c * 32, r);
    tmem_ld_wait();
    const int col0 = col_base + c * 32;
    if (!row_ok || col0 >= args.N) continue;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = zero ? 0.f : __uint_as_float(r[i]) * args.alpha;
    const bool full = col0 + 32 <= args.N;
    if (args.D != nullptr && args.beta != 0.f && kb0 == 0) {
      if (args.d_fp32) {
        const float* dp = reinterpret_cast<const float*>(args.D) + row * args.ldd + col0;
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float4 d4 = *reinterpret_cast<const float4*>(dp + i);
            v[i] += args.beta * d4.x; v[i + 1] += args.beta * d4.y;
            v[i + 2] += args.beta * d4.z; v[i + 3] += args.beta * d4.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (col0 + i < args.N) v[i] += args.beta * dp[i];
        }
      } else {
        const __nv_bfloat16* dp =
            reinterpret_cast<const __nv_bfloat16*>(args.D) + row * args.ldd + col0;
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 u = *reinterpret_cast<const uint4*>(dp + i);
            float2 f0 = unpack_bf16x2(u.x), f1 = unpack_bf16x2(u.y);
            float2 f2 = unpack_bf16x2(u.z), f3 = unpack_bf16x2(u.w);
            v[i] += args.beta * f0.x; v[i + 1] += args.beta * f0.y;
            v[i + 2] += args.beta * f1.x; v[i + 3] += args.beta * f1.y;
            v[i + 4] += args.beta * f2.x; v[i + 5] += args.beta * f2.y;
            v[i + 6] += args.beta * f3.x; v[i + 7] += args.beta * f3.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (col0 + i < args.N) v[i] += args.beta * __bfloat162float(dp[i]);
        }
      }
    }
    if (args.c_fp32) {
      float* cp = reinterpret_cast<float*>(args.C) + row * args.ldc + col0;
      if (args.splits > 1) {
        if (full) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            atomicAdd(reinterpret_cast<float4*>(cp + i),
                      make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (col0 + i < args.N) atomicAdd(cp + i, v[i]);
        }
      } else if (full) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(cp + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col0 + i < args.N) cp[i] = v[i];
      }
    } else {
      __nv_bfloat16* cp = (args.rs_n ? rs_row_ptr(args, row)
                                     : reinterpret_cast<__nv_bfloat16*>(args.C) + row * args.ldc) + col0;
      if (full) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 u;
          u.x = pack_bf16x2(v[i], v[i + 1]);
          u.y = pack_bf16x2(v[i + 2], v[i + 3]);
          u.z = pack_bf16x2(v[i + 4], v[i + 5]);
          u.w = pack_bf16x2(v[i + 6], v[i + 7]);
          *reinterpret_cast<uint4*>(cp + i) = u;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col0 + i < args.N) cp[i] = __float2bfloat16(v[i]);
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                Args args) {
  using C_ = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C_::kStages * C_::kStageBytes);
  uint64_t* full_bar = bar;                       // [kStages]
  uint64_t* empty_bar = bar + C_::kStages;        // [kStages]
  uint64_t* accf_bar = bar + 2 * C_::kStages;     // [2]
  uint64_t* acce_bar = bar + 2 * C_::kStages + 2; // [2]
  uint64_t* done_bar = bar + 2 * C_::kStages + 4;  // [1]
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(bar + 2 * C_::kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_smem + 1);
  uint8_t* epi_stage = smem + C_::kStages * C_::kStageBytes + 256;  // [4 warps][32][128 B]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C_::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_smem, C_::kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  const int total_tiles = args.m_tiles * args.n_tiles;
  const int total_work = total_tiles * (args.grp_mode == 2 ? args.grp_count : args.splits);
  const int kb_per_split = (args.k_blocks + args.splits - 1) / args.splits;

  // work unit -> tile (mt, nt), k-block range and group g; false: no work (mode 1
  // m tile beyond the last group). Every role decodes the same units.
  auto decode = [&](int w, int& mt, int& nt, int& kb0, int& kb1, int& g) -> bool {
    g = 0;
    int tile, sp = 0;
    if (args.grp_mode == 2) {
      g = w / total_tiles;
      tile = w - g * total_tiles;
    } else {
      tile = w / args.splits;
      sp = w - tile * args.splits;
    }
    if (args.raster_m) {
      mt = tile % args.m_tiles;
      nt = tile / args.m_tiles;
    } else {
      nt = tile % args.n_tiles;
      mt = tile / args.n_tiles;
    }
    if (args.rs_mshift) mt = (mt + args.rs_mshift) % args.m_tiles;
    if (args.grp_mode == 2) {
      kb0 = args.grp_koff[g] / BK;
      kb1 = args.grp_koff[g + 1] / BK;
      return true;
    }
    kb0 = sp * kb_per_split;
    kb1 = min(args.k_blocks, kb0 + kb_per_split);
    if (args.grp_mode == 1) {
      g = args.grp_tile[mt];
      return g >= 0;
    }
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, parity_mask = 0;  // per stage: issued, and the phase parity
      for (int w = blockIdx.x; w < total_work && ok; w += gridDim.x) {
        int mt, nt, kb0, kb1, g;
        if (!decode(w, mt, nt, kb0, kb1, g)) continue;
        // mode 1: B rows of group g start at g * grp_b_rows
        const int b_row0 = args.grp_mode == 1 ? static_cast<int>(g * args.grp_b_rows) : 0;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            record_status(args.status, kTimeoutSmemEmpty);
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* sA = tiles + stage * C_::kStageBytes;
          uint8_t* sB = sA + C_::kABytes;
          mbar_arrive_expect_tx(&full_bar[stage], C_::kStageBytes);
          const int k0 = kb * BK;
          if (A_MN) {
            // [K, M] row-major: boxes of 64 m x 64 k, one per 64-wide m chunk
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(sA + j * (BK * 128), &tmA, &full_bar[stage], mt * BM + j * 64, k0);
          } else {
            tma_load_2d(sA, &tmA, &full_bar[stage], k0, mt * BM);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + j * (BK * 128), &tmB, &full_bar[stage], nt * BN + j * 64, b_row0 + k0);
          } else {
            tma_load_2d(sB, &tmB, &full_bar[stage], k0, b_row0 + nt * BN);
          }
          issued_mask |= 1u << stage;
          parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // unwind: wait (bounded) until every load this thread issued has landed
        // so no bulk copy is still writing into smem when the CTA exits.
        for (int s = 0; s < C_::kStages; ++s) {
          if ((issued_mask >> s) & 1u) {
            if (!mbar_wait_bounded(&full_bar[s], (parity_mask >> s) & 1u, nullptr))
              record_status(args.status, kTimeoutDrain);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = -1;
      bool ok = true;
      for (int w = blockIdx.x; w < total_work && ok; w += gridDim.x) {
        int mt, nt, kb0, kb1, g;
        if (!decode(w, mt, nt, kb0, kb1, g)) continue;
        ++local;
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&acce_bar[buf], acc_phase ^ 1u, abort_flag)) {
          record_status(args.status, kTimeoutAccEmpty);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag)) {
            record_status(args.status, kTimeoutTmaFull);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sA = smem_u32(tiles + stage * C_::kStageBytes);
          const uint32_t sB = sA + C_::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t da, db;
            if (A_MN) da = make_smem_desc(sA + kk * 2048, BK * 128, 1024, kLayoutSW128);
            else da = make_smem_desc(sA + kk * 32, 16, 1024, kLayoutSW128);
            if (B_MN) db = make_smem_desc(sB + kk * 2048, BK * 128, 1024, kLayoutSW128);
            else db = make_smem_desc(sB + kk * 32, 16, 1024, kLayoutSW128);
            tc_mma_ss(d_tmem, da, db, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty_bar[stage]);  // frees the smem stage when these MMAs finish
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&accf_bar[buf]);  // accumulator ready for the epilogue
      }
      // every issued MMA must finish before TMEM is released
      tc_commit(done_bar);
      if (!mbar_wait_bounded(done_bar, 0, nullptr)) record_status(args.status, kTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    int local = -1;
    for (int w = blockIdx.x; w < total_work; w += gridDim.x) {
      int mt, nt, kb0, kb1, g;
      if (!decode(w, mt, nt, kb0, kb1, g)) continue;
      ++local;
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&accf_bar[buf], acc_phase, abort_flag)) {
        record_status(args.status, kTimeoutAccFull);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const long long row = (long long)mt * BM + row_in_tile;
      const bool row_ok = row < args.M;
      // mode 2: group g's rows of C; an empty k range stores zeros
      const long long crow = args.grp_mode == 2 ? g * args.grp_c_rows + row : row;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      // the addend D is applied by the first k split (mode 2 has one split per group)
      store_acc_row<BN>(args, t_row, crow, row_ok, nt * BN, args.grp_mode == 2 ? 0 : kb0,
                        epi_stage + q * 32 * 128, kb1 <= kb0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[buf]);
    }
    // reduce-scatter epilogue: this thread's peer stores are visible system-wide
    // before the kernel ends (the finishing kernel's flags then publish them)
    if (args.rs_n) __threadfence_system();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C_::kTmemCols);
  }
}

// --------------------------------------------------------------------------
// Two-SM variant: a cluster of 2 CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256). CTA rank r loads rows [128r, 128r+128) of
// the A tile and columns [128r, 128r+128) of the B tile (its own halves, no
// multicast), so per SM a k-block costs 32 KB of smem fill instead of 48 KB for
// the same 128 x 256 of output: the L2-to-SM traffic per flop drops by a third.
// Rank 0 issues the MMAs; stage, accumulator and teardown barriers in both CTAs
// are signalled by multicast commits; the epilogues of both CTAs report an
// accumulator drained to rank 0 (8 arrivals). Work units are (256 x 256 tile,
// k-split) pairs walked by the clusters.
// --------------------------------------------------------------------------
struct PairCfg {
  static constexpr int BN = 256;                 // pair tile N (each CTA loads 128)
  static constexpr int kStages = 6;
  static constexpr int kABytes = BM * BK * 2;    // 16 KB: this CTA's 128 rows
  static constexpr int kBBytes = 128 * BK * 2;   // 16 KB: this CTA's 128 of 256 columns
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;       // two 128 x 256 fp32 accumulators per CTA
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256 + kEpiStageBytes;
};

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     Args args) {
  using C_ = PairCfg;
  constexpr int BN = C_::BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C_::kStages * C_::kStageBytes);
  uint64_t* full_bar = bar;                         // [kStages] (rank 0's are used)
  uint64_t* empty_bar = bar + C_::kStages;          // [kStages]
  uint64_t* accf_bar = bar + 2 * C_::kStages;       // [2]
  uint64_t* acce_bar = bar + 2 * C_::kStages + 2;   // [2] (rank 0's are used)
  uint64_t* done_bar = bar + 2 * C_::kStages + 4;
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(bar + 2 * C_::kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_smem + 1);
  uint8_t* epi_stage = smem + C_::kStages * C_::kStageBytes + 256;  // [4 warps][32][128 B]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C_::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 8);  // 4 epilogue warps in each CTA of the pair
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_base_smem, C_::kTmemCols);
    tmem_relinquish_pair();
  }
  // barriers of both CTAs initialised and TMEM allocated before any remote use
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_smem;

  const int total_tiles = args.m_tiles * args.n_tiles;  // 256 x 256 tiles
  const int total_work = total_tiles * args.splits;
  const int kb_per_split = (args.k_blocks + args.splits - 1) / args.splits;
  auto decode = [&](int w, int& mt, int& nt, int& kb0, int& kb1) {
    const int tile = w / args.splits;
    const int sp = w - tile * args.splits;
    if (args.raster_m) {
      mt = tile % args.m_tiles;
      nt = tile / args.m_tiles;
    } else {
      nt = tile % args.n_tiles;
      mt = tile / args.n_tiles;
    }
    if (args.rs_mshift) mt = (mt + args.rs_mshift) % args.m_tiles;
    kb0 = sp * kb_per_split;
    kb1 = min(args.k_blocks, kb0 + kb_per_split);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t armed_mask = 0, parity_mask = 0;
      for (int w = pair; w < total_work && ok; w += npairs) {
        int mt, nt, kb0, kb1;
        decode(w, mt, nt, kb0, kb1);
        const int m0 = mt * 2 * BM + static_cast<int>(rank) * BM;
        const int n0 = nt * BN + static_cast<int>(rank) * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            record_status(args.status, kTimeoutSmemEmpty);
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* sA = tiles + stage * C_::kStageBytes;
          uint8_t* sB = sA + C_::kABytes;
          // rank 0's barrier counts the bytes of both CTAs
          if (leader) {
            mbar_arrive_expect_tx(&full_bar[stage], 2 * C_::kStageBytes);
            armed_mask |= 1u << stage;
            parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
          }
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d_pair(sA + j * (BK * 128), &tmA, &full_bar[stage], m0 + j * 64, k0);
          } else {
            tma_load_2d_pair(sA, &tmA, &full_bar[stage], k0, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
              tma_load_2d_pair(sB + j * (BK * 128), &tmB, &full_bar[stage], n0 + j * 64, k0);
          } else {
            tma_load_2d_pair(sB, &tmB, &full_bar[stage], k0, n0);
          }
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // unwind: let the copies in flight land before the CTA can exit
        if (leader) {
          for (int s = 0; s < C_::kStages; ++s)
            if (((armed_mask >> s) & 1u) &&
                !mbar_wait_bounded(&full_bar[s], (parity_mask >> s) & 1u, nullptr))
              record_status(args.status, kTimeoutDrain);
        } else {
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 2000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(2 * BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int w = pair; w < total_work && ok; w += npairs, ++local) {
        int mt, nt, kb0, kb1;
        decode(w, mt, nt, kb0, kb1);
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&acce_bar[buf], acc_phase ^ 1u, abort_flag)) {
          record_status(args.status, kTimeoutAccEmpty);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, abort_flag)) {
            record_status(args.status, kTimeoutTmaFull);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sA = smem_u32(tiles + stage * C_::kStageBytes);
          const uint32_t sB = sA + C_::kABytes;
          const uint64_t da0 = A_MN ? make_smem_desc(sA, BK * 128, 1024, kLayoutSW128)
                                    : make_smem_desc(sA, 16, 1024, kLayoutSW128);
          const uint64_t db0 = B_MN ? make_smem_desc(sB, BK * 128, 1024, kLayoutSW128)
                                    : make_smem_desc(sB, 16, 1024, kLayoutSW128);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc_mma_ss_pair(d_tmem, desc_advance(da0, A_MN ? kk * 2048 : kk * 32),
                           desc_advance(db0, B_MN ? kk * 2048 : kk * 32), idesc,
                           (kb > kb0 || kk > 0) ? 1u : 0u);
          tc_commit_pair(&empty_bar[stage], 0x3);  // frees the stage in both CTAs
          if (++stage == C_::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(&accf_bar[buf], 0x3);
      }
      if (!ok) *abort_flag = 1;
      tc_commit_pair(done_bar, 0x3);
    }
    // every MMA reading this CTA's smem or writing its TMEM has finished
    if (lane == 0 && !mbar_wait_bounded(done_bar, 0, nullptr)) record_status(args.status, kTimeoutDrain);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    for (int w = pair; w < total_work; w += npairs, ++local) {
      int mt, nt, kb0, kb1;
      decode(w, mt, nt, kb0, kb1);
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&accf_bar[buf], acc_phase, abort_flag)) {
        record_status(args.status, kTimeoutAccFull);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const long long row = (long long)mt * 2 * BM + rank * BM + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      store_acc_row<BN>(args, t_row, row, row < args.M, nt * BN, kb0, epi_stage + q * 32 * 128);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&acce_bar[buf], 0);
    }
    if (args.rs_n) __threadfence_system();
  }

  __syncthreads();
  // the peer must not exit (or free TMEM) while rank 0 may still signal it
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C_::kTmemCols);
  }
}

// --------------------------------------------------------------------------
// host side
// --------------------------------------------------------------------------
// 2-D bf16 tensor map over a row-major [rows, cols] matrix with leading dim `ld`
// (elements); box = box_cols x box_rows; 128-byte swizzle.
static CUtensorMap make_map_2d(const void* base, long long rows, long long cols, long long ld,
                               int box_cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tensor_map(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                                 dims, strides, box, estr, CU_TENSOR_MAP_SWIZZLE_128B);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string(r));
  return m;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    PLG_CUDA_CHECK(cudaGetDevice(&dev));
    PLG_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

// Split-K factor for fp32 outputs: the smallest modelled time over s = 1..8 with
// at least 8 k-blocks per split, where time ~ waves(tiles * s, slots) / s (the
// last wave is paid in full) times the cost of the extra fp32 reductions of C,
// relative to the math about 15/k_blocks per split (>= 2%): the reduction moves
// 4*M*N bytes per split against 2*M*N*K flops.
static int choose_splits(int tiles, int slots, int k_blocks) {
  int best = 1;
  double best_cost = 1e30;
  const double ovh = k_blocks > 0 ? (15.0 / k_blocks > 0.02 ? 15.0 / k_blocks : 0.02) : 0.02;
  for (int s = 1; s <= 8; ++s) {
    if (s > 1 && k_blocks / s < 8) break;
    const long long units = static_cast<long long>(tiles) * s;
    const long long waves = (units + slots - 1) / slots;
    const double cost = static_cast<double>(waves) / s * (1.0 + ovh * (s - 1));
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

static void set_rs_fields(const GemmProblem& p, Args& a, int tile_m) {
  a.rs_n = p.rs_n;
  a.rs_rank = p.rs_rank;
  a.rs_mshift = 0;
  a.rs_S = p.rs_S;
  for (int j = 0; j < 8; ++j) a.rs_dst[j] = p.rs_dst[j];
  if (!p.rs_n) return;
  if (p.rs_n < 1 || p.rs_n > 8 || p.rs_rank < 0 || p.rs_rank >= p.rs_n)
    throw std::invalid_argument("gemm reduce-scatter: 1..8 ranks");
  if (p.c_fp32 || p.D != nullptr || p.splits > 1)
    throw std::invalid_argument("gemm reduce-scatter: bf16 output without addend or split-K only");
  if (p.rs_S <= 0 || p.M % p.rs_S || p.rs_S % p.rs_n || p.ldc != p.N)
    throw std::invalid_argument("gemm reduce-scatter: M = B*S, S divisible by ranks, ldc == N");
  for (int j = 0; j < p.rs_n; ++j)
    if (p.rs_dst[j] == nullptr || (reinterpret_cast<uintptr_t>(p.rs_dst[j]) & 15))
      throw std::invalid_argument("gemm reduce-scatter: staging buffers must be 16-byte aligned");
  a.rs_seg = p.rs_S / p.rs_n;
  a.rs_rows = p.M / p.rs_n;
  a.rs_cap_rows = p.rs_cap / (2LL * p.N);
  if (a.rs_cap_rows < static_cast<long long>(p.M))
    throw std::invalid_argument("gemm reduce-scatter: the staging buffers are smaller than the output");
  if (a.rs_seg % 32 || p.N % 8)
    throw std::invalid_argument("gemm reduce-scatter: S / ranks a multiple of 32, N a multiple of 8");
  // all ranks writing the same owner's rows at once would funnel into one link:
  // rank r starts at owner r's rows
  if (a.m_tiles > 0) a.rs_mshift = static_cast<int>((p.rs_rank * a.rs_seg / tile_m) % a.m_tiles);
}

template <int BN, bool A_MN, bool B_MN>
static void launch(const GemmProblem& p, cudaStream_t stream) {
  using C_ = Cfg<BN>;
  // A map
  CUtensorMap ta = A_MN ? make_map_2d(p.A, p.K, p.M, p.lda, 64, BK)
                        : make_map_2d(p.A, p.M, p.K, p.lda, BK, BM);
  // grouped mode 1: B stacks every group's matrix
  const long long b_rows = (p.grp_mode == 1) ? p.grp_count * p.grp_b_rows : (B_MN ? p.K : p.N);
  CUtensorMap tb = B_MN ? make_map_2d(p.B, b_rows, p.N, p.ldb, 64, BK)
                        : make_map_2d(p.B, b_rows, p.K, p.ldb, BK, BN);
  Args a{};
  a.M = p.M; a.N = p.N; a.K = p.K;
  a.C = p.C; a.ldc = p.ldc; a.D = p.D; a.ldd = p.ldd;
  a.alpha = p.alpha; a.beta = p.beta;
  a.c_fp32 = p.c_fp32; a.d_fp32 = p.d_fp32;
  a.m_tiles = (p.M + BM - 1) / BM;
  a.n_tiles = (p.N + BN - 1) / BN;
  a.k_blocks = (p.K + BK - 1) / BK;
  a.status = p.status;
  set_rs_fields(p, a, BM);
  a.grp_mode = p.grp_mode;
  a.grp_tile = p.grp_tile;
  a.grp_b_rows = p.grp_b_rows;
  a.grp_koff = p.grp_koff;
  a.grp_c_rows = p.M;
  a.grp_count = p.grp_count;
  const int sms = num_sms();
  const int tiles = a.m_tiles * a.n_tiles;
  int splits = p.splits;
  if (splits <= 0) splits = (p.c_fp32 && p.allow_split) ? choose_splits(tiles, sms, a.k_blocks) : 1;
  if (p.rs_n || p.grp_mode) splits = 1;
  if (splits > a.k_blocks) splits = a.k_blocks;
  if (splits < 1) splits = 1;
  // every split must own at least one k-block
  while (splits > 1 && (splits - 1) * ((a.k_blocks + splits - 1) / splits) >= a.k_blocks) --splits;
  a.splits = splits;
  if (splits > 1) {
    // partial sums are atomically added into C: C must start from its base value
    const bool accumulate_into_c = (p.D == p.C && p.beta == 1.f);
    if (accumulate_into_c) {
      a.D = nullptr;
    } else {
      if (p.D == p.C) throw std::invalid_argument("gemm: split-K with D == C needs beta == 1");
      PLG_CUDA_CHECK(cudaMemsetAsync(p.C, 0, sizeof(float) * (size_t)p.ldc * (size_t)(p.M - 1) +
                                                 sizeof(float) * (size_t)p.N, stream));
    }
  }
  // raster: walk along the operand that is re-read from L2 less
  a.raster_m = (static_cast<long long>(p.N) > static_cast<long long>(p.M)) ? 1 : 0;
  // grouped mode 1: consecutive units walk one m tile's n tiles (one expert's rows
  // stay in L2 while its weights stream)
  if (p.grp_mode == 1) a.raster_m = 0;
  const int work = tiles * (p.grp_mode == 2 ? p.grp_count : splits);
  const int grid = work < sms ? work : sms;
  auto kern = gemm_kernel<BN, A_MN, B_MN>;
  set_max_smem_once(reinterpret_cast<const void*>(kern), C_::kSmemBytes);
  kern<<<grid, kThreads, C_::kSmemBytes, stream>>>(ta, tb, a);
  PLG_CUDA_CHECK(cudaGetLastError());
}

template <bool A_MN, bool B_MN>
static void launch_pair(const GemmProblem& p, cudaStream_t stream) {
  using C_ = PairCfg;
  constexpr int BN = C_::BN;
  // per CTA: A box of 128 rows (or two 64-wide M-major boxes), B box of 128 rows
  CUtensorMap ta = A_MN ? make_map_2d(p.A, p.K, p.M, p.lda, 64, BK)
                        : make_map_2d(p.A, p.M, p.K, p.lda, BK, BM);
  CUtensorMap tb = B_MN ? make_map_2d(p.B, p.K, p.N, p.ldb, 64, BK)
                        : make_map_2d(p.B, p.N, p.K, p.ldb, BK, 128);
  Args a{};
  a.M = p.M; a.N = p.N; a.K = p.K;
  a.C = p.C; a.ldc = p.ldc; a.D = p.D; a.ldd = p.ldd;
  a.alpha = p.alpha; a.beta = p.beta;
  a.c_fp32 = p.c_fp32; a.d_fp32 = p.d_fp32;
  a.m_tiles = (p.M + 2 * BM - 1) / (2 * BM);
  a.n_tiles = (p.N + BN - 1) / BN;
  a.k_blocks = (p.K + BK - 1) / BK;
  a.status = p.status;
  set_rs_fields(p, a, 2 * BM);
  auto kern = gemm_pair_kernel<A_MN, B_MN>;
  set_max_smem_once(reinterpret_cast<const void*>(kern), C_::kSmemBytes);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C_::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent grid: as many SM pairs as can hold a cluster at once
  static int max_pairs = 0;
  if (max_pairs == 0) {
    cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
    int n = 0;
    PLG_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    max_pairs = n > 0 ? n : 1;
  }
  const int pairs = max_pairs;
  const int tiles = a.m_tiles * a.n_tiles;
  int splits = p.splits;
  if (splits <= 0) splits = (p.c_fp32 && p.allow_split) ? choose_splits(tiles, pairs, a.k_blocks) : 1;
  if (p.rs_n) splits = 1;
  if (splits > a.k_blocks) splits = a.k_blocks;
  if (splits < 1) splits = 1;
  while (splits > 1 && (splits - 1) * ((a.k_blocks + splits - 1) / splits) >= a.k_blocks) --splits;
  a.splits = splits;
  if (splits > 1) {
    const bool accumulate_into_c = (p.D == p.C && p.beta == 1.f);
    if (accumulate_into_c) {
      a.D = nullptr;
    } else {
      if (p.D == p.C) throw std::invalid_argument("gemm: split-K with D == C needs beta == 1");
      PLG_CUDA_CHECK(cudaMemsetAsync(p.C, 0, sizeof(float) * (size_t)p.ldc * (size_t)(p.M - 1) +
                                                 sizeof(float) * (size_t)p.N, stream));
    }
  }
  a.raster_m = (static_cast<long long>(p.N) > static_cast<long long>(p.M)) ? 1 : 0;
  const int work = tiles * splits;
  const int nclusters = work < pairs ? work : pairs;
  cfg.gridDim = dim3(2 * nclusters, 1, 1);
  PLG_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, a));
}

}  // namespace gemm

void gemm_bf16(const GemmProblem& p, cudaStream_t stream) {
  using namespace gemm;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return;
  if ((p.lda % 8) || (p.ldb % 8)) throw std::invalid_argument("gemm: lda/ldb must be multiples of 8");
  if ((reinterpret_cast<uintptr_t>(p.A) | reinterpret_cast<uintptr_t>(p.B)) & 15)
    throw std::invalid_argument("gemm: A/B must be 16-byte aligned");
  if (p.ldc % (p.c_fp32 ? 4 : 8)) throw std::invalid_argument("gemm: ldc must keep rows 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(p.C) & 15) throw std::invalid_argument("gemm: C must be 16-byte aligned");
  if (p.splits > 1 && !p.c_fp32) throw std::invalid_argument("gemm: split-K needs an fp32 output");
  if (p.grp_mode) {
    if (p.grp_mode < 0 || p.grp_mode > 2 || p.grp_count < 1 || p.rs_n)
      throw std::invalid_argument("gemm grouped: mode 1 or 2, at least one group, no reduce-scatter");
    if (p.grp_mode == 1 && (p.grp_tile == nullptr || p.grp_b_rows <= 0 ||
                            (p.b_mn_major ? (p.K != p.grp_b_rows || p.K % BK)
                                          : p.N > p.grp_b_rows)))
      throw std::invalid_argument("gemm grouped mode 1: a tile table and B blocks of N rows "
                                  "(K-major) or K rows, a multiple of 64 (MN-major)");
    if (p.grp_mode == 2 && (p.grp_koff == nullptr || !p.a_mn_major || !p.b_mn_major))
      throw std::invalid_argument("gemm grouped mode 2: k offsets, A and B both MN-major");
    if (p.grp_mode == 2 && p.D != nullptr && p.D != p.C)
      throw std::invalid_argument("gemm grouped mode 2: the addend can only be C itself");
  }
  const bool wide = p.N >= 256 && p.bn != 128;
  // large problems: 256 x 256 tiles on SM pairs (bn == 256 keeps the one-SM kernel)
  const bool pair = wide && p.bn == 0 && p.M >= 256 && num_sms() >= 2 && !p.grp_mode;
#define PLG_GEMM_CASE(BN_, AM, BMJ) \
  if (p.a_mn_major == AM && p.b_mn_major == BMJ) return launch<BN_, AM, BMJ>(p, stream);
#define PLG_GEMM_PAIR(AM, BMJ) \
  if (p.a_mn_major == AM && p.b_mn_major == BMJ) return launch_pair<AM, BMJ>(p, stream);
  if (pair) {
    PLG_GEMM_PAIR(false, false)
    PLG_GEMM_PAIR(false, true)
    PLG_GEMM_PAIR(true, true)
    PLG_GEMM_PAIR(true, false)
  }
#undef PLG_GEMM_PAIR
  if (wide) {
    PLG_GEMM_CASE(256, false, false)
    PLG_GEMM_CASE(256, false, true)
    PLG_GEMM_CASE(256, true, true)
    PLG_GEMM_CASE(256, true, false)
  } else {
    PLG_GEMM_CASE(128, false, false)
    PLG_GEMM_CASE(128, false, true)
    PLG_GEMM_CASE(128, true, true)
    PLG_GEMM_CASE(128, true, false)
  }
#undef PLG_GEMM_CASE
}

}  // namespace plg
