// Host-side launcher API of the pluggy_b200 sm_100a kernels.
//
// The .cu files implement these with raw pointers and a cudaStream_t so they
// compile without the torch headers; bindings.cpp adapts torch tensors to them.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace plg {

// ---------------------------------------------------------------- GEMM (tcgen05)
struct GemmProblem {
  int M = 0, N = 0, K = 0;
  const void* A = nullptr;  // bf16
  long long lda = 0;
  bool a_mn_major = false;  // false: A is [M,K] row-major; true: A is [K,M] row-major
  const void* B = nullptr;  // bf16
  long long ldb = 0;
  bool b_mn_major = false;  // false: B is [N,K] row-major; true: B is [K,N] row-major
  void* C = nullptr;        // [M, N] row-major, bf16 or fp32
  long long ldc = 0;
  bool c_fp32 = false;
  const void* D = nullptr;  // optional addend [M, N] (may alias C)
  long long ldd = 0;
  bool d_fp32 = false;
  float alpha = 1.f, beta = 0.f;
  int splits = 0;           // 0: automatic split-K for fp32 outputs (when allow_split)
  bool allow_split = true;
  int bn = 0;               // 0 automatic, else 128 or 256
  int* status = nullptr;    // device status word (bounded waits)
  // Reduce-scatter epilogue (tensor parallel, sequence-sharded output): rows are
  // [B, S] flattened; row (b, s) belongs to rank s / (S / rs_n) and is stored as
  // bf16 into that rank's staging buffer rs_dst[owner] at slot rs_rank:
  // staging[rs_rank][b * S/rs_n + s % (S/rs_n)][N]. C is not written.
  int rs_n = 0, rs_rank = 0;
  long long rs_S = 0;
  void* rs_dst[8] = {};
  long long rs_cap = 0;     // bytes of every staging buffer (stores beyond are skipped)
  // Grouped GEMM over grp_count groups (MoE experts), one-SM 128-row tiles, no split-K:
  //  grp_mode 1: the group of each 128-row m tile is grp_tile[m_tile] (device int32,
  //    -1 = no work: the tile is skipped); B stacks the groups' matrices as
  //    [grp_count * grp_b_rows, cols] and a tile reads its group's block (K-major B:
  //    grp_b_rows >= N; MN-major B: grp_b_rows == K, a multiple of 64).
  //  grp_mode 2: M and N are per group; A and B are MN-major over the same rows, and
  //    group g sums over rows [grp_koff[g], grp_koff[g + 1]) (device int32 [grp_count + 1],
  //    multiples of 64), writing rows [g * M, (g + 1) * M) of C; an empty range writes 0.
  int grp_mode = 0;
  const int* grp_tile = nullptr;
  long long grp_b_rows = 0;
  const int* grp_koff = nullptr;
  int grp_count = 0;
};
void gemm_bf16(const GemmProblem& p, cudaStream_t stream);

// ---------------------------------------------------------------- normalisation
// y = x * rsqrt(mean(x^2) + eps) * w  (rows x D), x fp32 or bf16, w fp32 or null,
// y bf16 (and/or fp32), rstd fp32 [rows]
void rmsnorm_fwd(const void* x, bool x_fp32, const float* w, void* y, bool y_fp32, float* rstd,
                 long long rows, int D, float eps, cudaStream_t stream);
// dx = (w*dy - y_hat * mean(w*dy*y_hat)) * rstd (+ dres); dw partial sums into dw_partial
// [blocks, D] (reduced by the caller); dx written as fp32 (dx_f32) and/or bf16 (dx_bf16)
void rmsnorm_bwd(const void* dy, bool dy_fp32, const void* x, bool x_fp32, const float* w,
                 const float* rstd, const float* dres, float* dx_f32, void* dx_bf16,
                 float* dw_partial, int dw_blocks, long long rows, int D, cudaStream_t stream);

// QK-norm + RoPE on a packed projection [T, (Hq + 2*Hk) * d] (q | k | v):
// per head RMSNorm with weights wq/wk (d), then rotate-half RoPE with the
// angle pos * inv_freq[i]; writes q [T, Hq, d], k [T, Hk, d] (bf16) and rstd
// [T, Hq + Hk]. pos = t % S (packed rows) or positions[t] when given.
// rot_dim <= d: only the first rot_dim channels rotate (partial RoPE).
struct QkRopeArgs {
  const void* qkv; long long ld_qkv;
  void* q; void* k; float* rstd;
  const float* wq; const float* wk;
  const float* inv_freq; const int32_t* positions;
  long long T; int S; int Hq; int Hk; int d; int rot_dim; float eps;
  int norm_q; int norm_k;  // 0 skips the norm (Llama)
  int k_offset; int v_offset;  // column offsets (in heads*d units) of k and v within a row
  int full_width_norm;     // OLMo: q/k normalised over all heads' channels jointly
  const float* rope_table; // optional [S][2][rot_dim/2] cos then sin per position (else sincosf)
  int* status = nullptr;   // device status word (bounded waits of the TMA-fed kernels)
};
void qk_norm_rope_fwd(const QkRopeArgs& a, cudaStream_t stream);
// y [B, H, S, d] = RoPE(x) (backward: its transpose); x and y with strides (b, h, s, 1),
// cos/sin fp32 [Bc, S, d] with strides (b, s, 1) (b stride 0 broadcasts)
void rope_apply(const void* x, long long xs_b, long long xs_h, long long xs_s, const float* cos,
                const float* sin, long long cs_b, long long cs_s, void* y, long long ys_b,
                long long ys_h, long long ys_s, int B, int H, int S, int d, bool backward,
                cudaStream_t stream);
// backward: dq [T,Hq,d], dk [T,Hk,d] -> dqkv (q and k parts) ; dwq/dwk partials
void qk_norm_rope_bwd(const QkRopeArgs& a, const void* dq, const void* dk, void* dqkv,
                      long long ld_dqkv, float* dwq_partial, float* dwk_partial, int dw_blocks,
                      cudaStream_t stream);

// ---------------------------------------------------------------- elementwise
// act = silu(g) * u  (kind 0) or gelu_tanh(g) * u (kind 1); gu is [T, 2F] with
// g = gu[:, :F], u = gu[:, F:] (ld_gu >= 2F)
void glu_fwd(const void* gu, long long ld_gu, void* out, long long rows, int F, int kind,
             cudaStream_t stream);
void glu_bwd(const void* gu, long long ld_gu, const void* dout, void* dgu, long long rows, int F,
             int kind, cudaStream_t stream);
void cast_f32_bf16(const float* x, void* y, long long n, cudaStream_t stream);
// out[D] = column sums of part[R, D] (fixed summation order)
void colsum(const float* part, int R, int D, float* out, cudaStream_t stream);
void cast_bf16_f32(const void* x, float* y, long long n, cudaStream_t stream);
void embedding_fwd(const int64_t* ids, const float* w, float* out_f32, long long T, int D,
                   float scale, cudaStream_t stream);
// dw[ids[t]] += scale * dout[t]  (fp32 atomics)
void embedding_bwd(const int64_t* ids, const float* dout, float* dw, long long T, int D,
                   float scale, cudaStream_t stream);
// deterministic form: ids sorted ascending (stable) with their token positions;
// dw[id] += scale * sum of dout rows of that id, summed in token order, no atomics;
// scratch: fp32 [T, D] (rows written only for ids with more than 64 tokens)
void embedding_bwd_sorted(const int64_t* ids_sorted, const int64_t* pos_sorted, const float* dout,
                          float* dw, float* scratch, long long T, int D, float scale,
                          cudaStream_t stream);
// poly[i] = 2^x[i] by the attention kernels' FMA-pipe cubic, ref[i] = exp2f(x[i])
void exp2_poly_eval(const float* x, float* poly, float* ref, long long n, cudaStream_t stream);
// MoE router over logits [T, E]: probs [T, E] fp32 (optional), top-k weights [T, k] fp32
// (renormalised over the k when asked), expert ids [T, k] int64, histogram counts [E] int32
// (optional, accumulated)
void router_topk(const void* logits, bool bf16, long long T, int E, int k, bool renorm, float* probs,
                 float* w, int64_t* idx, int* counts, cudaStream_t stream);
// y = cap * tanh(x / cap)
void softcap_fwd(const void* x, void* y, long long n, float cap, bool bf16, cudaStream_t stream);

// ---------------------------------------------------------------- cross entropy
// Per row of bf16 logits [rows, V]: lse, loss = lse - logit[label] (0 for
// ignored rows), and in place: logits <- (softmax - onehot) * grad_scale.
// row_loss (when given) receives every row's loss, for a deterministic sum by the
// caller; otherwise loss_sum accumulates them (fp32 atomic). softcap > 0 applies
// cap*tanh(x/cap) first (its derivative folded into the gradient).
void ce_rows(void* logits, long long ld, const int64_t* labels, long long rows, int V,
             int ignore_index, float grad_scale, float softcap, float* lse_out, float* loss_sum,
             int* n_valid, cudaStream_t stream, float* row_loss = nullptr,
             float* stats_out = nullptr, const float* lse_in = nullptr, long long label_offset = 0);
// Vocabulary-parallel rows (columns [label_offset, label_offset + V) of the full
// vocabulary): with stats_out [rows][3], only (max, sum of exp, owned target
// logit or 0) are written and the logits are left alone; with lse_in [rows] (the
// full-vocabulary lse), only the in-place gradient pass runs.

// ---------------------------------------------------------------- optimizer
struct TensorRef { void* p; long long n; };
// one launch over every tensor: sum of squares (fp32) into out[0]
void multi_sumsq(const int64_t* table, int ntensors, long long total_chunks, float* out,
                 cudaStream_t stream);
void multi_scale(const int64_t* table, int ntensors, long long total_chunks, const float* coef,
                 cudaStream_t stream);
// table rows: [param f32*, grad f32*, m f32*, v f32*, shadow bf16* (or 0), numel, chunk_start]
void adamw_multi(const int64_t* table, int ntensors, long long total_chunks, float lr, float beta1,
                 float beta2, float eps, float weight_decay, float bc1, float bc2,
                 const float* grad_scale, const float* hyper, cudaStream_t stream);
constexpr int kOptChunk = 65536;

// ---------------------------------------------------------------- attention
struct AttnArgs {
  const void* q; const void* k; const void* v;  // bf16 [B, S, H, d] with row strides
  long long q_row, k_row, v_row;                 // elements between consecutive tokens
  void* o; long long o_row;                      // bf16 [B, S, Hq, d]
  float* lse;                                    // fp32 [B, Hq, S] (natural log)
  int B, S, Hq, Hk, d;
  float scale;
  int causal;
  int window;                                    // > 0: keys k with q - k < window only
  int* status;
};
void attn_fwd(const AttnArgs& a, cudaStream_t stream);
struct AttnBwdArgs {
  AttnArgs f;
  const void* dout; long long do_row;
  void* dq; void* dk; void* dv;                  // bf16, same layouts as q, k, v
  long long dq_row, dk_row, dv_row;
  float* dq_acc;                                 // fp32 workspace [B, S, Hq, d]
  float* delta;                                  // fp32 workspace, attn_bwd_stats_floats()
  long long* trace;                              // optional [kAttnTraceEvents][kAttnTraceSteps]
                                                 // SM clock stamps of CTA 0 (null: off)
};
constexpr int kAttnTraceEvents = 12, kAttnTraceSteps = 256;
// floats the backward's stats workspace needs: [B * Hq][2][S rounded up to 64]
inline long long attn_bwd_stats_floats(int B, int Hq, int S) {
  return static_cast<long long>(B) * Hq * 2 * ((S + 63) / 64 * 64);
}
void attn_bwd(const AttnBwdArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- collectives
// Symmetric (peer-mapped) device memory through CUDA IPC, and the fused
// data-parallel gradient reduction over it (comm.cu).
constexpr int kSymmMaxRanks = 8;
constexpr int kSymmMaxChunks = 128;
void* symm_malloc(size_t bytes, void* ipc_handle_out);  // zeroed; handle is 64 bytes
void* symm_open(const void* ipc_handle);
void symm_close(void* peer_ptr);
void symm_free(void* p);
struct SymmAllReduceArgs {
  float* data[kSymmMaxRanks];      // every rank's data buffer (this rank's own included)
  uint32_t* flags[kSymmMaxRanks];  // every rank's flag table [2][kSymmMaxRanks][kSymmMaxChunks]
  float* sumsq[kSymmMaxRanks];     // every rank's slot table [kSymmMaxRanks][kSymmMaxChunks]
  long long offset;                // first element of the range (multiple of 4)
  long long numel;
  int rank, nranks, chunks;
  uint32_t epoch;                  // grows by one per call on every rank
  int* status;
};
// average data[offset, offset+numel) over the ranks in place on every rank; with
// norm_sq, also (accumulate_norm ? += : =) the sum of squares of the averaged range
// ZeRO-1 inside data parallelism. A bucket [offset, offset + numel) of the grad
// and fp32 param arenas (same layout on every rank) is owned in slices: with
// seg = ceil(numel / n) rounded up to a multiple of 4, rank r owns
// [min(numel, r * seg), min(numel, (r + 1) * seg)).
constexpr int kZero1Kinds = 3;  // flag kinds: 0 RS ready, 1 RS done, 2 AG done
struct Zero1Args {
  float* grads[kSymmMaxRanks];     // every rank's grad arena
  float* params[kSymmMaxRanks];    // every rank's fp32 param arena
  uint32_t* flags[kSymmMaxRanks];  // every rank's flag table [kZero1Kinds][kSymmMaxRanks][kSymmMaxChunks]
  float* sumsq[kSymmMaxRanks];     // every rank's slot table [kSymmMaxRanks][kSymmMaxChunks]
  long long offset, numel;         // bucket range in elements (offset a multiple of 4)
  int rank, nranks, chunks;
  uint32_t epoch;                  // grows by one per call of the same kernel on every rank
  int* status;
};
// Reduce-scatter: the own slice of the own grad arena becomes the average over the
// ranks (peer loads); the sum of squares of the averaged slice goes into every
// rank's slot table, and (accumulate ? += : =) into norm_sq.
void zero1_reduce_scatter(const Zero1Args& a, float* norm_sq, bool accumulate, cudaStream_t st);
struct Zero1Adam {
  float lr[4] = {}, wd[4] = {};    // per param group
  float beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, bc1 = 1.f, bc2 = 1.f;
  const float* grad_scale = nullptr;  // device scalar (clip coefficient) or null
  const int64_t* rows = nullptr;   // device [nrows][3]: start, end (bucket elements), group
  int nrows = 0;                   //   sorted and covering [0, numel)
  float* exp_avg = nullptr;        // own-slice optimizer state (slice length)
  float* exp_avg_sq = nullptr;
};
// AdamW on the own slice (grads already averaged), the updated fp32 params stored
// into every rank's param arena (peer stores); returns once every peer's slice of
// the bucket has landed in this rank's arena.
void zero1_adamw_allgather(const Zero1Args& a, const Zero1Adam& h, cudaStream_t st);

// Tensor-parallel collectives over peer memory (sequence dimension of [B, S, W]
// rows). Flags: each rank's flag words [kTpKinds][kSymmMaxRanks] in symmetric
// memory; `epoch` grows by one per call of a kind; staging/send buffers are
// double-buffered by the caller (epoch parity).
constexpr int kTpKinds = 4;  // 0: reduce-scatter, 1: all-gather
struct TpArgs {
  int n = 1, rank = 0;
  uint32_t epoch = 0;
  int* status = nullptr;
  uint32_t* flags[kSymmMaxRanks] = {};
  void* bufs[kSymmMaxRanks] = {};  // every rank's staging (RS) or send (AG) buffer
  long long B = 0, S = 0, W = 0;   // rows are [B, S] flattened, W bf16 columns
  long long cap16 = 0;             // bytes / 16 of every bufs[p] (stores beyond are skipped)
};
// RS: push this rank's partial [B*S, W] rows into every owner's staging slot
void tp_rs_push(const TpArgs& a, const void* partial, long long ld, cudaStream_t stream);
// RS: signal, wait for every peer, out[B*S/n, W] = sum over slots of own staging
void tp_rs_finish(const TpArgs& a, void* out, long long ld_out, cudaStream_t stream);
// AG: push this rank's shard [B*S/n, W] into slot `rank` of every rank's receive buffer
void tp_ag_push(const TpArgs& a, const void* shard, long long ld, cudaStream_t stream);
// AG: signal, wait for every peer, copy the slots of the own receive buffer into out [B*S, W]
void tp_ag_finish(const TpArgs& a, void* out, long long ld_out, cudaStream_t stream);
// RMSNorm fused with the AG push: y = x * rsqrt(mean(x^2) + eps) * w of this rank's
// shard rows [B*S/n, W] (x fp32 or bf16), stored as bf16 straight into slot `rank` of
// every rank's receive buffer; rstd [B*S/n] kept locally. Finish with tp_ag_finish.
void tp_norm_ag_push(const TpArgs& a, const void* x, bool x_fp32, long long ld, const float* w,
                     float eps, float* rstd, cudaStream_t stream);
// Expert-parallel row exchange (MoE dispatch / combine) over peer memory: segment p
// of the source rows, [src_start[p], src_start[p] + count[p]), goes to rank p's
// buffer (bufs[p]) at row dst_off[p]. Rows are W bf16 (W % 8 == 0; any 2-byte data).
struct EpSegs {
  long long src_start[kSymmMaxRanks] = {};
  long long count[kSymmMaxRanks] = {};
  long long dst_off[kSymmMaxRanks] = {};
};
void ep_push(const TpArgs& a, const EpSegs& sg, const void* src, long long ld, cudaStream_t stream);
// Deadline (ns) of every peer-flag wait in the collective kernels on the
// current device (default 2 s); ordered on `st` and synchronised.
void set_peer_wait_deadline_ns(unsigned long long ns, cudaStream_t st);
// signal (flag kind `kind`), wait for every peer, copy own buffer rows [0, rows) to out
void ep_finish(const TpArgs& a, int kind, void* out, long long rows, long long ld_out,
               cudaStream_t stream);
// FSDP unit all-gather over peer memory: table [k][3] int64 (units of 16 bytes):
// shard offset in this rank's flat shard, offset of the parameter in the unit's full
// layout, shard length. This rank's shard of parameter i goes to every rank's buffer
// at full_off_i + rank * shard_len_i. Finish with ep_finish (rows of 8 2-byte units).
// FSDP gradient reduce-scatter over peer memory: every rank holds its full unit
// gradient (fp32, the unit's full layout) in a staging slot; rank r sums its shard
// of every parameter over the ranks' slots (fixed rank order), scales by `scale` and
// writes (accumulate ? += : =) into its flat fp32 grad-shard accumulator.
// table [k][3] int64 (elements): offset in the flat shard, offset of the parameter in
// the full layout, shard length. Offsets and lengths must be multiples of 4.
struct FsdpRsArgs {
  float* stage[kSymmMaxRanks] = {};
  uint32_t* flags[kSymmMaxRanks] = {};  // [2 kinds][kSymmMaxRanks][kSymmMaxChunks]
  const int64_t* table = nullptr;
  int k = 0;
  long long shard_numel = 0;
  float* out = nullptr;
  int accumulate = 0;
  float scale = 1.f;
  int rank = 0, nranks = 1, chunks = 1;
  uint32_t epoch = 0;
  int* status = nullptr;
};
void fsdp_reduce_scatter(const FsdpRsArgs& a, cudaStream_t stream);
// Low-precision form: fp32 shard in, matrices stored as bf16 (vectors as fp32) straight
// into every rank's slot; table [k][5] (see comm.cu). Finish with ep_finish (0 rows).
void fsdp_push_lowp(const TpArgs& a, const int64_t* table, int k, long long total16, const float* shard,
                    cudaStream_t stream);
void fsdp_push(const TpArgs& a, const int64_t* table, int k, long long total16, const void* shard,
               cudaStream_t stream);
void symm_allreduce_avg(const SymmAllReduceArgs& a, float* norm_sq, bool accumulate_norm,
                        cudaStream_t stream);

}  // namespace plg
