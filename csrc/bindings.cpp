// torch bindings for the pluggy_b200 sm_100a kernels (module pluggy_b200._C).
//
// Thin adapters: validate dtypes/devices/contiguity, pass raw pointers and the
// current CUDA stream to the launchers in ops.h. No computation happens here.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "ops.h"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

bool is_f32(const at::Tensor& t) { return t.scalar_type() == at::kFloat; }
bool is_bf16(const at::Tensor& t) { return t.scalar_type() == at::kBFloat16; }

int* status_ptr(const c10::optional<at::Tensor>& s) {
  if (!s.has_value()) return nullptr;
  TORCH_CHECK(s->scalar_type() == at::kInt, "status must be int32");
  return s->data_ptr<int>();
}

// C = alpha * op(A) op(B)^T (+ beta * D).
// a: [M,K] (a_mn_major=false) or [K,M] (true); b: [N,K] or [K,N]; c: [M,N]
void gemm(const at::Tensor& a, bool a_mn_major, const at::Tensor& b, bool b_mn_major, at::Tensor& c,
          const c10::optional<at::Tensor>& d, double alpha, double beta, int64_t splits, int64_t bn,
          const c10::optional<at::Tensor>& status) {
  check_cuda(a, "a");
  check_cuda(b, "b");
  check_cuda(c, "c");
  TORCH_CHECK(is_bf16(a) && is_bf16(b), "gemm operands must be bf16");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "gemm takes 2-D tensors");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "gemm needs unit inner stride");
  TORCH_CHECK(is_bf16(c) || is_f32(c), "gemm output must be bf16 or fp32");
  const c10::cuda::CUDAGuard guard(a.device());
  plg::GemmProblem p;
  p.M = static_cast<int>(a_mn_major ? a.size(1) : a.size(0));
  p.K = static_cast<int>(a_mn_major ? a.size(0) : a.size(1));
  p.N = static_cast<int>(b_mn_major ? b.size(1) : b.size(0));
  const int kb = static_cast<int>(b_mn_major ? b.size(0) : b.size(1));
  TORCH_CHECK(kb == p.K, "gemm: K mismatch (", p.K, " vs ", kb, ")");
  TORCH_CHECK(c.size(0) == p.M && c.size(1) == p.N, "gemm: C must be [M, N]");
  p.A = a.data_ptr();
  p.lda = a.stride(0);
  p.a_mn_major = a_mn_major;
  p.B = b.data_ptr();
  p.ldb = b.stride(0);
  p.b_mn_major = b_mn_major;
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.c_fp32 = is_f32(c);
  if (d.has_value() && beta != 0.0) {
    check_cuda(*d, "d");
    TORCH_CHECK(d->dim() == 2 && d->size(0) == p.M && d->size(1) == p.N && d->stride(1) == 1,
                "gemm: D must be [M, N] with unit inner stride");
    TORCH_CHECK(is_bf16(*d) || is_f32(*d), "gemm: D must be bf16 or fp32");
    p.D = d->data_ptr();
    p.ldd = d->stride(0);
    p.d_fp32 = is_f32(*d);
  }
  p.alpha = static_cast<float>(alpha);
  p.beta = static_cast<float>(beta);
  p.splits = static_cast<int>(splits);
  p.allow_split = splits != 1;
  p.bn = static_cast<int>(bn);
  p.status = status_ptr(status);
  plg::gemm_bf16(p, cur_stream());
}

// Grouped GEMM (MoE experts). mode 1: a [rows, K] (K-major), b = every group's
// matrix stacked [G * b_rows, ...] (K-major [G*N, K] or MN-major [G*K, N]),
// table = int32 [rows / 128] group of each 128-row tile (-1: skipped);
// c [rows, N]. mode 2: a [rows, M] and b [rows, N] both MN-major over the same
// rows, table = int32 [G + 1] row offsets (multiples of 64); c [G * M, N].
void gemm_grouped(const at::Tensor& a, const at::Tensor& b, bool b_mn_major, at::Tensor& c,
                  int64_t mode, const at::Tensor& table, int64_t groups, int64_t b_rows,
                  double alpha, double beta, const c10::optional<at::Tensor>& status) {
  check_cuda(a, "a");
  check_cuda(b, "b");
  check_cuda(c, "c");
  check_cuda(table, "table");
  TORCH_CHECK(is_bf16(a) && is_bf16(b), "gemm_grouped operands must be bf16");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 &&
                  c.stride(1) == 1, "gemm_grouped takes 2-D tensors with unit inner stride");
  TORCH_CHECK(is_bf16(c) || is_f32(c), "gemm_grouped output must be bf16 or fp32");
  TORCH_CHECK(table.scalar_type() == at::kInt && table.is_contiguous(), "gemm_grouped: int32 table");
  TORCH_CHECK(groups >= 1, "gemm_grouped: at least one group");
  const c10::cuda::CUDAGuard guard(a.device());
  plg::GemmProblem p;
  p.grp_mode = static_cast<int>(mode);
  p.grp_count = static_cast<int>(groups);
  p.A = a.data_ptr();
  p.lda = a.stride(0);
  p.B = b.data_ptr();
  p.ldb = b.stride(0);
  p.b_mn_major = b_mn_major;
  p.C = c.data_ptr();
  p.ldc = c.stride(0);
  p.c_fp32 = is_f32(c);
  if (mode == 1) {
    p.M = static_cast<int>(a.size(0));
    p.K = static_cast<int>(a.size(1));
    p.N = static_cast<int>(b_mn_major ? b.size(1) : b_rows);
    TORCH_CHECK(b.size(0) == groups * b_rows, "gemm_grouped mode 1: b must stack groups * b_rows rows");
    TORCH_CHECK(b_mn_major ? b_rows == p.K : b.size(1) == p.K, "gemm_grouped mode 1: K mismatch");
    TORCH_CHECK(table.numel() >= (p.M + 127) / 128, "gemm_grouped mode 1: one table entry per 128 rows");
    TORCH_CHECK(c.size(0) == p.M && c.size(1) == p.N, "gemm_grouped mode 1: c must be [rows, N]");
    p.grp_tile = table.data_ptr<int>();
    p.grp_b_rows = b_rows;
  } else if (mode == 2) {
    TORCH_CHECK(b_mn_major, "gemm_grouped mode 2: b is MN-major");
    p.a_mn_major = true;
    p.K = static_cast<int>(a.size(0));
    p.M = static_cast<int>(a.size(1));
    p.N = static_cast<int>(b.size(1));
    TORCH_CHECK(b.size(0) == p.K, "gemm_grouped mode 2: a and b must span the same rows");
    TORCH_CHECK(table.numel() == groups + 1, "gemm_grouped mode 2: groups + 1 offsets");
    TORCH_CHECK(c.size(0) == groups * p.M && c.size(1) == p.N, "gemm_grouped mode 2: c must be [G*M, N]");
    p.grp_koff = table.data_ptr<int>();
  } else {
    TORCH_CHECK(false, "gemm_grouped: mode 1 or 2");
  }
  if (beta != 0.0) {
    p.D = c.data_ptr();
    p.ldd = c.stride(0);
    p.d_fp32 = is_f32(c);
  }
  p.alpha = static_cast<float>(alpha);
  p.beta = static_cast<float>(beta);
  p.splits = 1;
  p.allow_split = false;
  p.status = status_ptr(status);
  plg::gemm_bf16(p, cur_stream());
}

void rmsnorm_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& w, at::Tensor& y,
                 const c10::optional<at::Tensor>& rstd, double eps) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous(), "rmsnorm tensors must be contiguous");
  const int D = static_cast<int>(x.size(-1));
  const long long rows = x.numel() / D;
  const float* wp = nullptr;
  if (w.has_value()) {
    TORCH_CHECK(is_f32(*w) && w->numel() == D, "rmsnorm weight must be fp32 [D]");
    wp = w->data_ptr<float>();
  }
  float* rp = rstd.has_value() ? rstd->data_ptr<float>() : nullptr;
  const c10::cuda::CUDAGuard guard(x.device());
  plg::rmsnorm_fwd(x.data_ptr(), is_f32(x), wp, y.data_ptr(), is_f32(y), rp, rows, D,
                   static_cast<float>(eps), cur_stream());
}

void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const c10::optional<at::Tensor>& w,
                 const at::Tensor& rstd, const c10::optional<at::Tensor>& dres,
                 const c10::optional<at::Tensor>& dx_f32, const c10::optional<at::Tensor>& dx_bf16,
                 const c10::optional<at::Tensor>& dw_partial) {
  check_cuda(dy, "dy");
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous(), "rmsnorm_bwd tensors must be contiguous");
  const int D = static_cast<int>(x.size(-1));
  const long long rows = x.numel() / D;
  const float* wp = w.has_value() ? w->data_ptr<float>() : nullptr;
  const float* rp = dres.has_value() ? dres->data_ptr<float>() : nullptr;
  float* dxf = dx_f32.has_value() ? dx_f32->data_ptr<float>() : nullptr;
  void* dxb = dx_bf16.has_value() ? dx_bf16->data_ptr() : nullptr;
  float* dwp = dw_partial.has_value() ? dw_partial->data_ptr<float>() : nullptr;
  const int blocks = dw_partial.has_value() ? static_cast<int>(dw_partial->size(0)) : 592;
  const c10::cuda::CUDAGuard guard(x.device());
  plg::rmsnorm_bwd(dy.data_ptr(), is_f32(dy), x.data_ptr(), is_f32(x), wp,
                   rstd.data_ptr<float>(), rp, dxf, dxb, dwp, blocks, rows, D, cur_stream());
}

plg::QkRopeArgs qk_args(const at::Tensor& qkv, at::Tensor& q, at::Tensor& k, at::Tensor& rstd,
                        const c10::optional<at::Tensor>& wq, const c10::optional<at::Tensor>& wk,
                        const at::Tensor& inv_freq, const c10::optional<at::Tensor>& positions,
                        int64_t S, int64_t Hq, int64_t Hk, int64_t d, int64_t rot_dim, double eps,
                        int64_t k_offset, const c10::optional<at::Tensor>& rope_table) {
  plg::QkRopeArgs a{};
  a.rope_table = nullptr;
  if (rope_table.has_value()) {
    TORCH_CHECK(is_f32(*rope_table) && rope_table->is_contiguous() && rope_table->is_cuda() &&
                    rope_table->numel() >= S * rot_dim,
                "qk_norm_rope: rope_table must be fp32 [S, 2, rot_dim/2] on the device");
    a.rope_table = rope_table->data_ptr<float>();
  }
  a.qkv = qkv.data_ptr();
  a.ld_qkv = qkv.stride(0);
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.rstd = rstd.data_ptr<float>();
  a.wq = wq.has_value() ? wq->data_ptr<float>() : nullptr;
  a.wk = wk.has_value() ? wk->data_ptr<float>() : nullptr;
  a.norm_q = wq.has_value();
  a.norm_k = wk.has_value();
  a.inv_freq = inv_freq.data_ptr<float>();
  a.positions = positions.has_value() ? positions->data_ptr<int32_t>() : nullptr;
  a.T = qkv.size(0);
  a.S = static_cast<int>(S);
  a.Hq = static_cast<int>(Hq);
  a.Hk = static_cast<int>(Hk);
  a.d = static_cast<int>(d);
  a.rot_dim = static_cast<int>(rot_dim);
  a.eps = static_cast<float>(eps);
  a.k_offset = static_cast<int>(k_offset);
  return a;
}

void rope_apply(const at::Tensor& x, const at::Tensor& cos, const at::Tensor& sin, at::Tensor& y,
                bool backward) {
  // x [B, H, S, d] bf16 (last dim contiguous), cos/sin [Bc, 1, S, d] fp32, y contiguous
  TORCH_CHECK(x.is_cuda() && x.dim() == 4 && x.scalar_type() == at::kBFloat16 && x.stride(3) == 1,
              "rope_apply: x must be a [B, H, S, d] bf16 CUDA tensor with a contiguous last dim");
  TORCH_CHECK(cos.scalar_type() == at::kFloat && sin.scalar_type() == at::kFloat && cos.dim() == 4 &&
                  cos.sizes() == sin.sizes() && cos.strides() == sin.strides() && cos.stride(3) == 1,
              "rope_apply: cos/sin must be fp32 [Bc, 1, S, d] tables with equal strides");
  const int B = x.size(0), H = x.size(1), S = x.size(2), d = x.size(3);
  TORCH_CHECK(cos.size(1) == 1 && cos.size(2) == S && cos.size(3) == d &&
                  (cos.size(0) == 1 || cos.size(0) == B),
              "rope_apply: cos/sin shape does not match x");
  TORCH_CHECK(y.sizes() == x.sizes() && y.scalar_type() == at::kBFloat16 && y.stride(3) == 1,
              "rope_apply: y must be a bf16 tensor of x's shape with a contiguous last dim");
  const c10::cuda::CUDAGuard guard(x.device());
  const long long cs_b = cos.size(0) == 1 ? 0 : cos.stride(0);
  plg::rope_apply(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), cos.data_ptr<float>(),
                  sin.data_ptr<float>(), cs_b, cos.stride(2), y.data_ptr(), y.stride(0), y.stride(1),
                  y.stride(2), B, H, S, d, backward, cur_stream());
}

void qk_norm_rope_fwd(const at::Tensor& qkv, at::Tensor& q, at::Tensor& k, at::Tensor& rstd,
                      const c10::optional<at::Tensor>& wq, const c10::optional<at::Tensor>& wk,
                      const at::Tensor& inv_freq, const c10::optional<at::Tensor>& positions,
                      int64_t S, int64_t Hq, int64_t Hk, int64_t d, int64_t rot_dim, double eps,
                      int64_t k_offset, const c10::optional<at::Tensor>& rope_table,
                      const c10::optional<at::Tensor>& status) {
  check_cuda(qkv, "qkv");
  TORCH_CHECK(is_bf16(qkv) && qkv.dim() == 2 && qkv.stride(1) == 1, "qkv must be bf16 [T, W]");
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto a = qk_args(qkv, q, k, rstd, wq, wk, inv_freq, positions, S, Hq, Hk, d, rot_dim, eps, k_offset,
                   rope_table);
  a.status = status.has_value() ? status->data_ptr<int>() : nullptr;
  plg::qk_norm_rope_fwd(a, cur_stream());
}

void qk_norm_rope_bwd(const at::Tensor& qkv, at::Tensor& rstd, const c10::optional<at::Tensor>& wq,
                      const c10::optional<at::Tensor>& wk, const at::Tensor& inv_freq,
                      const c10::optional<at::Tensor>& positions, int64_t S, int64_t Hq, int64_t Hk,
                      int64_t d, int64_t rot_dim, double eps, int64_t k_offset,
                      const at::Tensor& dq, const at::Tensor& dk, at::Tensor& dqkv,
                      const c10::optional<at::Tensor>& dwq_partial,
                      const c10::optional<at::Tensor>& dwk_partial, int64_t blocks,
                      const c10::optional<at::Tensor>& rope_table,
                      const c10::optional<at::Tensor>& status) {
  check_cuda(qkv, "qkv");
  const c10::cuda::CUDAGuard guard(qkv.device());
  at::Tensor q_dummy = dq, k_dummy = dk;
  auto a = qk_args(qkv, q_dummy, k_dummy, rstd, wq, wk, inv_freq, positions, S, Hq, Hk, d, rot_dim,
                   eps, k_offset, rope_table);
  a.status = status.has_value() ? status->data_ptr<int>() : nullptr;
  plg::qk_norm_rope_bwd(a, dq.data_ptr(), dk.data_ptr(), dqkv.data_ptr(), dqkv.stride(0),
                        dwq_partial.has_value() ? dwq_partial->data_ptr<float>() : nullptr,
                        dwk_partial.has_value() ? dwk_partial->data_ptr<float>() : nullptr,
                        static_cast<int>(blocks), cur_stream());
}

void glu_fwd(const at::Tensor& gu, at::Tensor& out, int64_t kind) {
  check_cuda(gu, "gu");
  TORCH_CHECK(is_bf16(gu) && gu.stride(-1) == 1, "glu input must be bf16");
  const int F = static_cast<int>(out.size(-1));
  const long long rows = out.numel() / F;
  const c10::cuda::CUDAGuard guard(gu.device());
  plg::glu_fwd(gu.data_ptr(), gu.stride(-2), out.data_ptr(), rows, F, static_cast<int>(kind),
               cur_stream());
}

void glu_bwd(const at::Tensor& gu, const at::Tensor& dout, at::Tensor& dgu, int64_t kind) {
  check_cuda(gu, "gu");
  TORCH_CHECK(dout.is_contiguous() && dgu.stride(-2) == gu.stride(-2), "glu_bwd layout");
  const int F = static_cast<int>(dout.size(-1));
  const long long rows = dout.numel() / F;
  const c10::cuda::CUDAGuard guard(gu.device());
  plg::glu_bwd(gu.data_ptr(), gu.stride(-2), dout.data_ptr(), dgu.data_ptr(), rows, F,
               static_cast<int>(kind), cur_stream());
}

void cast_f32_bf16(const at::Tensor& x, at::Tensor& y) {
  check_cuda(x, "x");
  TORCH_CHECK(is_f32(x) && is_bf16(y) && x.is_contiguous() && y.is_contiguous() &&
                  x.numel() == y.numel(),
              "cast_f32_bf16 layout");
  const c10::cuda::CUDAGuard guard(x.device());
  plg::cast_f32_bf16(x.data_ptr<float>(), y.data_ptr(), x.numel(), cur_stream());
}

void embedding_fwd(const at::Tensor& ids, const at::Tensor& w, at::Tensor& out, double scale) {
  check_cuda(ids, "ids");
  TORCH_CHECK(ids.scalar_type() == at::kLong && is_f32(w) && is_f32(out), "embedding dtypes");
  TORCH_CHECK(ids.is_contiguous() && w.is_contiguous() && out.is_contiguous(), "embedding layout");
  const c10::cuda::CUDAGuard guard(ids.device());
  plg::embedding_fwd(ids.data_ptr<int64_t>(), w.data_ptr<float>(), out.data_ptr<float>(),
                     ids.numel(), static_cast<int>(w.size(1)), static_cast<float>(scale),
                     cur_stream());
}

void embedding_bwd(const at::Tensor& ids, const at::Tensor& dout, at::Tensor& dw, double scale) {
  check_cuda(ids, "ids");
  TORCH_CHECK(dout.is_contiguous() && dw.is_contiguous() && is_f32(dout) && is_f32(dw),
              "embedding_bwd layout");
  const c10::cuda::CUDAGuard guard(ids.device());
  plg::embedding_bwd(ids.data_ptr<int64_t>(), dout.data_ptr<float>(), dw.data_ptr<float>(),
                     ids.numel(), static_cast<int>(dw.size(1)), static_cast<float>(scale),
                     cur_stream());
}

void softcap(const at::Tensor& x, at::Tensor& y, double cap) {
  check_cuda(x, "x");
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && x.scalar_type() == y.scalar_type(),
              "softcap layout");
  TORCH_CHECK(is_bf16(x) || is_f32(x), "softcap dtype");
  const c10::cuda::CUDAGuard guard(x.device());
  plg::softcap_fwd(x.data_ptr(), y.data_ptr(), x.numel(), static_cast<float>(cap), is_bf16(x),
                   cur_stream());
}

void ce_rows(at::Tensor& logits, const at::Tensor& labels, int64_t ignore_index, double grad_scale,
             double softcap, const c10::optional<at::Tensor>& lse,
             const c10::optional<at::Tensor>& loss_sum, const c10::optional<at::Tensor>& n_valid,
             const c10::optional<at::Tensor>& row_loss, const c10::optional<at::Tensor>& stats,
             const c10::optional<at::Tensor>& lse_in, int64_t label_offset) {
  check_cuda(logits, "logits");
  TORCH_CHECK(is_bf16(logits) && logits.dim() == 2 && logits.stride(1) == 1, "ce logits layout");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "ce labels");
  if (row_loss.has_value())
    TORCH_CHECK(is_f32(*row_loss) && row_loss->is_contiguous() && row_loss->numel() == logits.size(0),
                "ce row_loss: fp32 [rows]");
  if (stats.has_value())
    TORCH_CHECK(is_f32(*stats) && stats->is_contiguous() && stats->numel() == 3 * logits.size(0),
                "ce stats: fp32 [rows, 3]");
  if (lse_in.has_value())
    TORCH_CHECK(is_f32(*lse_in) && lse_in->is_contiguous() && lse_in->numel() == logits.size(0),
                "ce lse_in: fp32 [rows]");
  TORCH_CHECK(!(stats.has_value() && lse_in.has_value()), "ce_rows: stats or lse_in, not both");
  TORCH_CHECK(loss_sum.has_value() || row_loss.has_value() || stats.has_value() || lse_in.has_value(),
              "ce_rows: loss_sum, row_loss, stats or lse_in");
  const c10::cuda::CUDAGuard guard(logits.device());
  plg::ce_rows(logits.data_ptr(), logits.stride(0), labels.data_ptr<int64_t>(), logits.size(0),
               static_cast<int>(logits.size(1)), static_cast<int>(ignore_index),
               static_cast<float>(grad_scale), static_cast<float>(softcap),
               lse.has_value() ? lse->data_ptr<float>() : nullptr,
               loss_sum.has_value() ? loss_sum->data_ptr<float>() : nullptr,
               n_valid.has_value() ? n_valid->data_ptr<int>() : nullptr, cur_stream(),
               row_loss.has_value() ? row_loss->data_ptr<float>() : nullptr,
               stats.has_value() ? stats->data_ptr<float>() : nullptr,
               lse_in.has_value() ? lse_in->data_ptr<float>() : nullptr, label_offset);
}

void router_topk_b(const at::Tensor& logits, int64_t k, bool renorm, const c10::optional<at::Tensor>& probs,
                   at::Tensor& w, at::Tensor& idx, const c10::optional<at::Tensor>& counts) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.is_contiguous() && (is_bf16(logits) || is_f32(logits)),
              "router_topk: logits must be a contiguous [T, E] bf16 or fp32 tensor");
  const long long T = logits.size(0);
  const int E = static_cast<int>(logits.size(1));
  TORCH_CHECK(is_f32(w) && w.is_contiguous() && w.numel() == T * k, "router_topk: w is fp32 [T, k]");
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous() && idx.numel() == T * k,
              "router_topk: idx is int64 [T, k]");
  if (probs.has_value())
    TORCH_CHECK(is_f32(*probs) && probs->is_contiguous() && probs->numel() == T * E,
                "router_topk: probs is fp32 [T, E]");
  if (counts.has_value())
    TORCH_CHECK(counts->scalar_type() == at::kInt && counts->is_contiguous() && counts->numel() == E,
                "router_topk: counts is int32 [E]");
  const c10::cuda::CUDAGuard guard(logits.device());
  plg::router_topk(logits.data_ptr(), is_bf16(logits), T, E, static_cast<int>(k), renorm,
                   probs.has_value() ? probs->data_ptr<float>() : nullptr, w.data_ptr<float>(),
                   idx.data_ptr<int64_t>(), counts.has_value() ? counts->data_ptr<int>() : nullptr,
                   cur_stream());
}

void exp2_poly_eval_b(const at::Tensor& x, at::Tensor& poly, at::Tensor& ref) {
  check_cuda(x, "x");
  TORCH_CHECK(is_f32(x) && is_f32(poly) && is_f32(ref) && x.is_contiguous() && poly.is_contiguous() &&
                  ref.is_contiguous() && poly.numel() == x.numel() && ref.numel() == x.numel(),
              "exp2_poly_eval: fp32 contiguous tensors of one size");
  const c10::cuda::CUDAGuard guard(x.device());
  plg::exp2_poly_eval(x.data_ptr<float>(), poly.data_ptr<float>(), ref.data_ptr<float>(), x.numel(),
                      cur_stream());
}

void embedding_bwd_sorted(const at::Tensor& ids_sorted, const at::Tensor& pos_sorted,
                          const at::Tensor& dout, at::Tensor& dw, double scale) {
  check_cuda(dout, "dout");
  TORCH_CHECK(ids_sorted.scalar_type() == at::kLong && pos_sorted.scalar_type() == at::kLong &&
                  ids_sorted.is_contiguous() && pos_sorted.is_contiguous() &&
                  ids_sorted.numel() == pos_sorted.numel() && ids_sorted.numel() == dout.size(0),
              "embedding_bwd_sorted: int64 sorted ids and positions, one per dout row");
  TORCH_CHECK(is_f32(dout) && is_f32(dw) && dout.is_contiguous() && dw.is_contiguous() &&
                  dout.dim() == 2 && dw.dim() == 2 && dout.size(1) == dw.size(1),
              "embedding_bwd_sorted: fp32 dout [T, D] and dw [V, D]");
  const c10::cuda::CUDAGuard guard(dout.device());
  // partial sums of long runs (rows touched only for ids with more than 64 tokens)
  at::Tensor scratch = at::empty_like(dout);
  plg::embedding_bwd_sorted(ids_sorted.data_ptr<int64_t>(), pos_sorted.data_ptr<int64_t>(),
                            dout.data_ptr<float>(), dw.data_ptr<float>(), scratch.data_ptr<float>(),
                            dout.size(0), static_cast<int>(dout.size(1)), static_cast<float>(scale),
                            cur_stream());
}

void multi_sumsq(const at::Tensor& table, int64_t ntensors, int64_t total_chunks, at::Tensor& out) {
  const c10::cuda::CUDAGuard guard(out.device());
  plg::multi_sumsq(table.data_ptr<int64_t>(), static_cast<int>(ntensors), total_chunks,
                   out.data_ptr<float>(), cur_stream());
}

void multi_scale(const at::Tensor& table, int64_t ntensors, int64_t total_chunks,
                 const at::Tensor& coef) {
  const c10::cuda::CUDAGuard guard(coef.device());
  plg::multi_scale(table.data_ptr<int64_t>(), static_cast<int>(ntensors), total_chunks,
                   coef.data_ptr<float>(), cur_stream());
}

void adamw_multi(const at::Tensor& table, int64_t ntensors, int64_t total_chunks, double lr,
                 double beta1, double beta2, double eps, double wd, double bc1, double bc2,
                 const c10::optional<at::Tensor>& grad_scale,
                 const c10::optional<at::Tensor>& hyper) {
  const c10::cuda::CUDAGuard guard(table.device());
  if (hyper.has_value())
    TORCH_CHECK(hyper->is_cuda() && hyper->scalar_type() == at::kFloat && hyper->numel() >= 3 &&
                    hyper->is_contiguous(),
                "adamw_multi: hyper must be a contiguous fp32 device tensor of (lr, bc1, bc2)");
  plg::adamw_multi(table.data_ptr<int64_t>(), static_cast<int>(ntensors), total_chunks,
                   static_cast<float>(lr), static_cast<float>(beta1), static_cast<float>(beta2),
                   static_cast<float>(eps), static_cast<float>(wd), static_cast<float>(bc1),
                   static_cast<float>(bc2),
                   grad_scale.has_value() ? grad_scale->data_ptr<float>() : nullptr,
                   hyper.has_value() ? hyper->data_ptr<float>() : nullptr, cur_stream());
}

plg::AttnArgs attn_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                        at::Tensor& o, at::Tensor& lse, double scale, bool causal, int64_t window,
                        const c10::optional<at::Tensor>& status) {
  // q: [B, S, Hq, d], k/v: [B, S, Hk, d] with unit inner stride and head stride d
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "attention takes [B, S, H, d]");
  TORCH_CHECK(is_bf16(q) && is_bf16(k) && is_bf16(v) && is_bf16(o), "attention is bf16");
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&q, &k, &v, &o}) {
    TORCH_CHECK(t->stride(3) == 1 && (t->size(2) == 1 || t->stride(2) == t->size(3)),
                "attention: heads must be packed");
    TORCH_CHECK(t->size(0) == 1 || t->stride(0) == t->stride(1) * t->size(1),
                "attention: batch stride = S * row");
  }
  plg::AttnArgs a{};
  a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr(); a.o = o.data_ptr();
  a.q_row = q.stride(1); a.k_row = k.stride(1); a.v_row = v.stride(1); a.o_row = o.stride(1);
  a.lse = lse.data_ptr<float>();
  a.B = static_cast<int>(q.size(0)); a.S = static_cast<int>(q.size(1));
  a.Hq = static_cast<int>(q.size(2)); a.Hk = static_cast<int>(k.size(2));
  a.d = static_cast<int>(q.size(3));
  a.scale = static_cast<float>(scale);
  a.causal = causal ? 1 : 0;
  a.window = static_cast<int>(window);
  a.status = status_ptr(status);
  return a;
}

void attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
              at::Tensor& lse, double scale, bool causal, int64_t window,
              const c10::optional<at::Tensor>& status) {
  check_cuda(q, "q");
  const c10::cuda::CUDAGuard guard(q.device());
  auto a = attn_args(q, k, v, o, lse, scale, causal, window, status);
  plg::attn_fwd(a, cur_stream());
}

void attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
              at::Tensor& lse, const at::Tensor& dout, at::Tensor& dq, at::Tensor& dk,
              at::Tensor& dv, at::Tensor& dq_acc, at::Tensor& delta, double scale, bool causal,
              int64_t window, const c10::optional<at::Tensor>& status,
              const c10::optional<at::Tensor>& trace) {
  check_cuda(q, "q");
  const c10::cuda::CUDAGuard guard(q.device());
  plg::AttnBwdArgs b{};
  b.f = attn_args(q, k, v, o, lse, scale, causal, window, status);
  TORCH_CHECK(dout.stride(3) == 1 && dq.stride(3) == 1 && dk.stride(3) == 1 && dv.stride(3) == 1,
              "attention grads need unit inner stride");
  TORCH_CHECK(dout.dim() == 4 && (dout.size(2) == 1 || dout.stride(2) == dout.size(3)) &&
                  (dout.size(0) == 1 || dout.stride(0) == dout.stride(1) * dout.size(1)),
              "attention backward: dout must be [B, S, Hq, d] with packed heads");
  b.dout = dout.data_ptr(); b.do_row = dout.stride(1);
  b.dq = dq.data_ptr(); b.dk = dk.data_ptr(); b.dv = dv.data_ptr();
  b.dq_row = dq.stride(1); b.dk_row = dk.stride(1); b.dv_row = dv.stride(1);
  TORCH_CHECK(is_f32(dq_acc) && dq_acc.is_contiguous() && is_f32(delta) && delta.is_contiguous(),
              "attention workspaces");
  TORCH_CHECK(dq_acc.numel() >= static_cast<int64_t>(b.f.B) * b.f.S * b.f.Hq * b.f.d &&
                  delta.numel() >= plg::attn_bwd_stats_floats(b.f.B, b.f.Hq, b.f.S),
              "attention backward workspaces too small");
  b.dq_acc = dq_acc.data_ptr<float>();
  b.delta = delta.data_ptr<float>();
  b.trace = nullptr;
  if (trace.has_value()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                    trace->numel() >= plg::kAttnTraceEvents * plg::kAttnTraceSteps,
                "attention trace buffer: int64 cuda tensor of at least 12 x 256");
    b.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  plg::attn_bwd(b, cur_stream());
}

void colsum(const at::Tensor& part, at::Tensor& out) {
  check_cuda(part, "part");
  TORCH_CHECK(is_f32(part) && part.dim() == 2 && part.is_contiguous(), "colsum: fp32 [R, D] input");
  TORCH_CHECK(is_f32(out) && out.is_contiguous() && out.numel() == part.size(1), "colsum: out [D]");
  const c10::cuda::CUDAGuard guard(part.device());
  plg::colsum(part.data_ptr<float>(), static_cast<int>(part.size(0)), static_cast<int>(part.size(1)),
              out.data_ptr<float>(), cur_stream());
}

// ------------------------------------------------------------ symmetric memory
std::tuple<int64_t, at::Tensor> symm_malloc_b(int64_t bytes) {
  at::Tensor h = at::empty({64}, at::TensorOptions().dtype(at::kByte));
  void* p = plg::symm_malloc(static_cast<size_t>(bytes), h.data_ptr());
  return {reinterpret_cast<int64_t>(p), h};
}

int64_t symm_open_b(const at::Tensor& handle) {
  TORCH_CHECK(handle.numel() == 64 && handle.dtype() == at::kByte && !handle.is_cuda(),
              "symm_open: 64-byte CPU handle");
  return reinterpret_cast<int64_t>(plg::symm_open(handle.contiguous().data_ptr()));
}

void symm_close_b(int64_t p) { plg::symm_close(reinterpret_cast<void*>(p)); }
void symm_free_b(int64_t p) { plg::symm_free(reinterpret_cast<void*>(p)); }

// a tensor over device memory this module owns (no deleter: the owner frees it)
at::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype,
                           int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, static_cast<int>(device));
  return at::from_blob(reinterpret_cast<void*>(ptr), shape, [](void*) {}, opts);
}

void symm_allreduce_avg_b(std::vector<int64_t> data, std::vector<int64_t> flags,
                          std::vector<int64_t> sumsq, int64_t offset, int64_t numel, int64_t rank,
                          int64_t epoch, int64_t chunks, const c10::optional<at::Tensor>& norm_sq,
                          bool accumulate, const c10::optional<at::Tensor>& status) {
  const int n = static_cast<int>(data.size());
  TORCH_CHECK(n >= 1 && n <= plg::kSymmMaxRanks && flags.size() == data.size() &&
                  sumsq.size() == data.size(), "symm_allreduce_avg: one pointer per rank");
  plg::SymmAllReduceArgs a{};
  for (int i = 0; i < n; ++i) {
    a.data[i] = reinterpret_cast<float*>(data[i]);
    a.flags[i] = reinterpret_cast<uint32_t*>(flags[i]);
    a.sumsq[i] = reinterpret_cast<float*>(sumsq[i]);
  }
  a.offset = offset;
  a.numel = numel;
  a.rank = static_cast<int>(rank);
  a.nranks = n;
  a.chunks = static_cast<int>(chunks);
  a.epoch = static_cast<uint32_t>(epoch);
  a.status = status.has_value() ? status->data_ptr<int>() : nullptr;
  float* ns = nullptr;
  if (norm_sq.has_value()) {
    TORCH_CHECK(is_f32(*norm_sq) && norm_sq->is_cuda(), "norm_sq: fp32 device tensor");
    ns = norm_sq->data_ptr<float>();
  }
  plg::symm_allreduce_avg(a, ns, accumulate, cur_stream());
}

plg::Zero1Args zero1_args(const std::vector<int64_t>& grads, const std::vector<int64_t>& params,
                          const std::vector<int64_t>& flags, const std::vector<int64_t>& slots,
                          int64_t offset, int64_t numel, int64_t rank, int64_t epoch, int64_t chunks,
                          const c10::optional<at::Tensor>& status) {
  const int n = static_cast<int>(grads.size());
  TORCH_CHECK(n >= 1 && n <= plg::kSymmMaxRanks && params.size() == grads.size() &&
                  flags.size() == grads.size() && slots.size() == grads.size(),
              "zero1: one pointer per rank");
  plg::Zero1Args a{};
  for (int i = 0; i < n; ++i) {
    a.grads[i] = reinterpret_cast<float*>(grads[i]);
    a.params[i] = reinterpret_cast<float*>(params[i]);
    a.flags[i] = reinterpret_cast<uint32_t*>(flags[i]);
    a.sumsq[i] = reinterpret_cast<float*>(slots[i]);
  }
  a.offset = offset;
  a.numel = numel;
  a.rank = static_cast<int>(rank);
  a.nranks = n;
  a.chunks = static_cast<int>(chunks);
  a.epoch = static_cast<uint32_t>(epoch);
  a.status = status.has_value() ? status->data_ptr<int>() : nullptr;
  return a;
}

void zero1_rs_b(std::vector<int64_t> grads, std::vector<int64_t> params, std::vector<int64_t> flags,
                std::vector<int64_t> slots, int64_t offset, int64_t numel, int64_t rank, int64_t epoch,
                int64_t chunks, const c10::optional<at::Tensor>& norm_sq, bool accumulate,
                const c10::optional<at::Tensor>& status) {
  auto a = zero1_args(grads, params, flags, slots, offset, numel, rank, epoch, chunks, status);
  float* ns = nullptr;
  if (norm_sq.has_value()) {
    TORCH_CHECK(is_f32(*norm_sq) && norm_sq->is_cuda(), "norm_sq: fp32 device tensor");
    ns = norm_sq->data_ptr<float>();
  }
  plg::zero1_reduce_scatter(a, ns, accumulate, cur_stream());
}

void zero1_adamw_ag_b(std::vector<int64_t> grads, std::vector<int64_t> params, std::vector<int64_t> flags,
                      std::vector<int64_t> slots, int64_t offset, int64_t numel, int64_t rank,
                      int64_t epoch, int64_t chunks, std::vector<double> lr, std::vector<double> wd,
                      double beta1, double beta2, double eps, double bc1, double bc2,
                      const c10::optional<at::Tensor>& grad_scale, const at::Tensor& rows,
                      at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
                      const c10::optional<at::Tensor>& status) {
  auto a = zero1_args(grads, params, flags, slots, offset, numel, rank, epoch, chunks, status);
  TORCH_CHECK(lr.size() == wd.size() && lr.size() >= 1 && lr.size() <= 4, "zero1 adamw: 1..4 param groups");
  TORCH_CHECK(rows.is_cuda() && rows.scalar_type() == at::kLong && rows.dim() == 2 && rows.size(1) == 3 &&
                  rows.is_contiguous() && rows.size(0) >= 1, "zero1 adamw: int64 rows [k, 3] on the device");
  TORCH_CHECK(is_f32(exp_avg) && is_f32(exp_avg_sq) && exp_avg.is_contiguous() && exp_avg_sq.is_contiguous() &&
                  exp_avg.numel() == exp_avg_sq.numel(), "zero1 adamw: fp32 slice state");
  const int64_t n = static_cast<int64_t>(grads.size());
  const int64_t seg = ((numel + n - 1) / n + 3) / 4 * 4;
  const int64_t s0 = std::min<int64_t>(numel, rank * seg), s1 = std::min<int64_t>(numel, s0 + seg);
  TORCH_CHECK(exp_avg.numel() >= s1 - s0, "zero1 adamw: the slice state is shorter than the owned slice");
  plg::Zero1Adam h;
  for (size_t g = 0; g < lr.size(); ++g) {
    h.lr[g] = static_cast<float>(lr[g]);
    h.wd[g] = static_cast<float>(wd[g]);
  }
  h.beta1 = static_cast<float>(beta1);
  h.beta2 = static_cast<float>(beta2);
  h.eps = static_cast<float>(eps);
  h.bc1 = static_cast<float>(bc1);
  h.bc2 = static_cast<float>(bc2);
  if (grad_scale.has_value()) {
    TORCH_CHECK(is_f32(*grad_scale) && grad_scale->is_cuda(), "grad_scale: fp32 device scalar");
    h.grad_scale = grad_scale->data_ptr<float>();
  }
  h.rows = rows.data_ptr<int64_t>();
  h.nrows = static_cast<int>(rows.size(0));
  h.exp_avg = exp_avg.data_ptr<float>();
  h.exp_avg_sq = exp_avg_sq.data_ptr<float>();
  plg::zero1_adamw_allgather(a, h, cur_stream());
}

// GEMM whose epilogue stores each row into its owner's staging slot (tensor-parallel
// reduce-scatter along the sequence); rs_dst: every rank's staging base address
void gemm_rs(const at::Tensor& a, const at::Tensor& b, bool b_mn_major, std::vector<int64_t> rs_dst,
             int64_t rank, int64_t S, int64_t cap_bytes, const c10::optional<at::Tensor>& status) {
  check_cuda(a, "a");
  check_cuda(b, "b");
  TORCH_CHECK(is_bf16(a) && is_bf16(b) && a.dim() == 2 && b.dim() == 2, "gemm_rs: bf16 2-D operands");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm_rs needs unit inner stride");
  const int n = static_cast<int>(rs_dst.size());
  TORCH_CHECK(n >= 1 && n <= 8, "gemm_rs: 1..8 ranks");
  const c10::cuda::CUDAGuard guard(a.device());
  plg::GemmProblem p;
  p.M = static_cast<int>(a.size(0));
  p.K = static_cast<int>(a.size(1));
  p.N = static_cast<int>(b_mn_major ? b.size(1) : b.size(0));
  TORCH_CHECK((b_mn_major ? b.size(0) : b.size(1)) == p.K, "gemm_rs: K mismatch");
  p.A = a.data_ptr();
  p.lda = a.stride(0);
  p.B = b.data_ptr();
  p.ldb = b.stride(0);
  p.b_mn_major = b_mn_major;
  p.ldc = p.N;
  p.splits = 1;
  p.allow_split = false;
  p.rs_n = n;
  p.rs_rank = static_cast<int>(rank);
  p.rs_S = S;
  for (int j = 0; j < n; ++j) p.rs_dst[j] = reinterpret_cast<void*>(rs_dst[j]);
  p.rs_cap = cap_bytes;
  p.status = status.has_value() ? status->data_ptr<int>() : nullptr;
  plg::gemm_bf16(p, cur_stream());
}

plg::TpArgs tp_args(std::vector<int64_t> flags, std::vector<int64_t> bufs, int64_t rank, int64_t epoch,
                    int64_t B, int64_t S, int64_t W, int64_t cap_bytes,
                    const c10::optional<at::Tensor>& status) {
  const int n = static_cast<int>(flags.size());
  TORCH_CHECK(n >= 1 && n <= plg::kSymmMaxRanks && bufs.size() == flags.size(),
              "tp collective: one flag table and one buffer per rank (1..8)");
  plg::TpArgs a;
  a.n = n;
  a.rank = static_cast<int>(rank);
  a.epoch = static_cast<uint32_t>(epoch);
  a.status = status.has_value() ? status->data_ptr<int>() : nullptr;
  for (int j = 0; j < n; ++j) {
    a.flags[j] = reinterpret_cast<uint32_t*>(flags[j]);
    a.bufs[j] = reinterpret_cast<void*>(bufs[j]);
  }
  a.B = B;
  a.S = S;
  a.W = W;
  a.cap16 = cap_bytes / 16;
  return a;
}

void tp_collective(const std::string& op, const at::Tensor& t, std::vector<int64_t> flags,
                   std::vector<int64_t> bufs, int64_t rank, int64_t epoch, int64_t B, int64_t S,
                   int64_t cap_bytes, const c10::optional<at::Tensor>& status) {
  check_cuda(t, "t");
  TORCH_CHECK(is_bf16(t) && t.dim() == 2 && t.stride(1) == 1, "tp collective: bf16 [rows, W] rows");
  const c10::cuda::CUDAGuard guard(t.device());
  auto a = tp_args(flags, bufs, rank, epoch, B, S, t.size(1), cap_bytes, status);
  const long long full = B * S, part = B * (S / static_cast<long long>(flags.size()));
  if (op == "rs_push") {
    TORCH_CHECK(t.size(0) == full, "rs_push: partial must be [B*S, W]");
    plg::tp_rs_push(a, t.data_ptr(), t.stride(0), cur_stream());
  } else if (op == "rs_finish") {
    TORCH_CHECK(t.size(0) == part, "rs_finish: out must be [B*S/n, W]");
    plg::tp_rs_finish(a, t.data_ptr(), t.stride(0), cur_stream());
  } else if (op == "ag_push") {
    TORCH_CHECK(t.size(0) == part, "ag_push: shard must be [B*S/n, W]");
    plg::tp_ag_push(a, t.data_ptr(), t.stride(0), cur_stream());
  } else if (op == "ag_finish") {
    TORCH_CHECK(t.size(0) == full, "ag_finish: out must be [B*S, W]");
    plg::tp_ag_finish(a, t.data_ptr(), t.stride(0), cur_stream());
  } else {
    TORCH_CHECK(false, "tp collective: unknown op ", op);
  }
}

void ep_exchange(const std::string& op, const at::Tensor& t, std::vector<int64_t> flags,
                 std::vector<int64_t> bufs, int64_t rank, int64_t epoch, int64_t kind,
                 std::vector<int64_t> src_start, std::vector<int64_t> count,
                 std::vector<int64_t> dst_off, int64_t rows, int64_t cap_bytes,
                 const c10::optional<at::Tensor>& status) {
  check_cuda(t, "t");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1 && t.element_size() == 2,
              "ep exchange: 2-D rows of a 2-byte dtype");
  const c10::cuda::CUDAGuard guard(t.device());
  auto a = tp_args(flags, bufs, rank, epoch, 1, static_cast<int64_t>(flags.size()), t.size(1), cap_bytes,
                   status);
  if (op == "push") {
    const size_t n = flags.size();
    TORCH_CHECK(src_start.size() == n && count.size() == n && dst_off.size() == n,
                "ep push: one segment per rank");
    plg::EpSegs sg;
    for (size_t p = 0; p < n; ++p) {
      sg.src_start[p] = src_start[p];
      sg.count[p] = count[p];
      sg.dst_off[p] = dst_off[p];
      TORCH_CHECK(src_start[p] + count[p] <= t.size(0), "ep push: segment past the source rows");
    }
    plg::ep_push(a, sg, t.data_ptr(), t.stride(0), cur_stream());
  } else if (op == "finish") {
    TORCH_CHECK(rows <= t.size(0), "ep finish: out has fewer rows than requested");
    plg::ep_finish(a, static_cast<int>(kind), t.data_ptr(), rows, t.stride(0), cur_stream());
  } else {
    TORCH_CHECK(false, "ep exchange: unknown op ", op);
  }
}

void fsdp_push_b(const at::Tensor& shard, const at::Tensor& table, std::vector<int64_t> flags,
                 std::vector<int64_t> bufs, int64_t rank, int64_t epoch, int64_t cap_bytes,
                 const c10::optional<at::Tensor>& status) {
  check_cuda(shard, "shard");
  check_cuda(table, "table");
  TORCH_CHECK(shard.is_contiguous() && (shard.numel() * shard.element_size()) % 16 == 0,
              "fsdp_push: contiguous shard of whole 16-byte groups");
  TORCH_CHECK(table.scalar_type() == at::kLong && table.dim() == 2 && table.size(1) == 3 &&
                  table.is_contiguous(), "fsdp_push: int64 table [k, 3]");
  const c10::cuda::CUDAGuard guard(shard.device());
  auto a = tp_args(flags, bufs, rank, epoch, 1, static_cast<int64_t>(flags.size()), 8, cap_bytes, status);
  plg::fsdp_push(a, table.data_ptr<int64_t>(), static_cast<int>(table.size(0)),
                 shard.numel() * shard.element_size() / 16, shard.data_ptr(), cur_stream());
}

void fsdp_push_lowp_b(const at::Tensor& shard, const at::Tensor& table, int64_t total16,
                      std::vector<int64_t> flags, std::vector<int64_t> bufs, int64_t rank, int64_t epoch,
                      int64_t cap_bytes, const c10::optional<at::Tensor>& status) {
  check_cuda(shard, "shard");
  check_cuda(table, "table");
  TORCH_CHECK(is_f32(shard) && shard.is_contiguous(), "fsdp_push_lowp: contiguous fp32 shard");
  TORCH_CHECK(table.scalar_type() == at::kLong && table.dim() == 2 && table.size(1) == 5 &&
                  table.is_contiguous(), "fsdp_push_lowp: int64 table [k, 5]");
  const c10::cuda::CUDAGuard guard(shard.device());
  auto a = tp_args(flags, bufs, rank, epoch, 1, static_cast<int64_t>(flags.size()), 8, cap_bytes, status);
  plg::fsdp_push_lowp(a, table.data_ptr<int64_t>(), static_cast<int>(table.size(0)), total16,
                      shard.data_ptr<float>(), cur_stream());
}

void fsdp_rs_b(std::vector<int64_t> stage, std::vector<int64_t> flags, const at::Tensor& table,
               at::Tensor& out, bool accumulate, double scale, int64_t rank, int64_t epoch, int64_t chunks,
               const c10::optional<at::Tensor>& status) {
  check_cuda(out, "out");
  check_cuda(table, "table");
  TORCH_CHECK(is_f32(out) && out.is_contiguous(), "fsdp_rs: contiguous fp32 shard accumulator");
  TORCH_CHECK(table.scalar_type() == at::kLong && table.dim() == 2 && table.size(1) == 3 &&
                  table.is_contiguous(), "fsdp_rs: int64 table [k, 3]");
  const int n = static_cast<int>(stage.size());
  TORCH_CHECK(n >= 1 && n <= plg::kSymmMaxRanks && flags.size() == stage.size(), "fsdp_rs: one slot per rank");
  const c10::cuda::CUDAGuard guard(out.device());
  plg::FsdpRsArgs a;
  for (int i = 0; i < n; ++i) {
    a.stage[i] = reinterpret_cast<float*>(stage[i]);
    a.flags[i] = reinterpret_cast<uint32_t*>(flags[i]);
  }
  a.table = table.data_ptr<int64_t>();
  a.k = static_cast<int>(table.size(0));
  a.shard_numel = out.numel();
  a.out = out.data_ptr<float>();
  a.accumulate = accumulate ? 1 : 0;
  a.scale = static_cast<float>(scale);
  a.rank = static_cast<int>(rank);
  a.nranks = n;
  a.chunks = static_cast<int>(chunks);
  a.epoch = static_cast<uint32_t>(epoch);
  a.status = status.has_value() ? status->data_ptr<int>() : nullptr;
  plg::fsdp_reduce_scatter(a, cur_stream());
}

void tp_norm_ag(const at::Tensor& x, const c10::optional<at::Tensor>& w, at::Tensor& rstd,
                at::Tensor& out, std::vector<int64_t> flags, std::vector<int64_t> bufs, int64_t rank,
                int64_t epoch, int64_t B, int64_t S, double eps, int64_t cap_bytes,
                const c10::optional<at::Tensor>& status) {
  check_cuda(x, "x");
  TORCH_CHECK((is_f32(x) || is_bf16(x)) && x.dim() == 2 && x.stride(1) == 1, "tp_norm_ag: x [rows, W]");
  TORCH_CHECK(is_f32(rstd) && rstd.is_contiguous() && rstd.numel() == x.size(0), "tp_norm_ag: rstd [rows]");
  TORCH_CHECK(is_bf16(out) && out.dim() == 2 && out.size(1) == x.size(1) && out.stride(1) == 1,
              "tp_norm_ag: out bf16 [B*S, W]");
  if (w.has_value()) TORCH_CHECK(is_f32(*w) && w->numel() == x.size(1), "tp_norm_ag: fp32 weight [W]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto a = tp_args(flags, bufs, rank, epoch, B, S, x.size(1), cap_bytes, status);
  TORCH_CHECK(x.size(0) == B * (S / static_cast<int64_t>(flags.size())), "tp_norm_ag: x must be [B*S/n, W]");
  TORCH_CHECK(out.size(0) == B * S, "tp_norm_ag: out must be [B*S, W]");
  plg::tp_norm_ag_push(a, x.data_ptr(), is_f32(x), x.stride(0), w.has_value() ? w->data_ptr<float>() : nullptr,
                       static_cast<float>(eps), rstd.data_ptr<float>(), cur_stream());
  plg::tp_ag_finish(a, out.data_ptr(), out.stride(0), cur_stream());
}

void set_peer_wait_deadline(int64_t ns) {
  TORCH_CHECK(ns > 0, "set_peer_wait_deadline: the deadline must be positive");
  plg::set_peer_wait_deadline_ns(static_cast<unsigned long long>(ns), cur_stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "pluggy_b200 sm_100a kernels";
  m.def("gemm", &gemm);
  m.def("gemm_grouped", &gemm_grouped, py::arg("a"), py::arg("b"), py::arg("b_mn_major"), py::arg("c"),
        py::arg("mode"), py::arg("table"), py::arg("groups"), py::arg("b_rows"), py::arg("alpha"),
        py::arg("beta"), py::arg("status") = py::none());
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rope_apply", &rope_apply);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd, py::arg("qkv"), py::arg("q"), py::arg("k"),
        py::arg("rstd"), py::arg("wq"), py::arg("wk"), py::arg("inv_freq"), py::arg("positions"),
        py::arg("S"), py::arg("Hq"), py::arg("Hk"), py::arg("d"), py::arg("rot_dim"), py::arg("eps"),
        py::arg("k_offset"), py::arg("rope_table"), py::arg("status") = py::none());
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd, py::arg("qkv"), py::arg("rstd"), py::arg("wq"),
        py::arg("wk"), py::arg("inv_freq"), py::arg("positions"), py::arg("S"), py::arg("Hq"),
        py::arg("Hk"), py::arg("d"), py::arg("rot_dim"), py::arg("eps"), py::arg("k_offset"),
        py::arg("dq"), py::arg("dk"), py::arg("dqkv"), py::arg("dwq_partial"), py::arg("dwk_partial"),
        py::arg("blocks"), py::arg("rope_table"), py::arg("status") = py::none());
  m.def("glu_fwd", &glu_fwd);
  m.def("glu_bwd", &glu_bwd);
  m.def("cast_f32_bf16", &cast_f32_bf16);
  m.def("colsum", &colsum);
  m.def("symm_malloc", &symm_malloc_b);
  m.def("symm_open", &symm_open_b);
  m.def("symm_close", &symm_close_b);
  m.def("symm_free", &symm_free_b);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("symm_allreduce_avg", &symm_allreduce_avg_b);
  m.def("gemm_rs", &gemm_rs, py::arg("a"), py::arg("b"), py::arg("b_mn_major"), py::arg("rs_dst"),
        py::arg("rank"), py::arg("S"), py::arg("cap_bytes"), py::arg("status") = py::none());
  m.def("fsdp_push", &fsdp_push_b, py::arg("shard"), py::arg("table"), py::arg("flags"),
        py::arg("bufs"), py::arg("rank"), py::arg("epoch"), py::arg("cap_bytes"),
        py::arg("status") = py::none());
  m.def("fsdp_rs", &fsdp_rs_b, py::arg("stage"), py::arg("flags"), py::arg("table"), py::arg("out"),
        py::arg("accumulate"), py::arg("scale"), py::arg("rank"), py::arg("epoch"), py::arg("chunks"),
        py::arg("status") = py::none());
  m.def("fsdp_push_lowp", &fsdp_push_lowp_b, py::arg("shard"), py::arg("table"), py::arg("total16"),
        py::arg("flags"), py::arg("bufs"), py::arg("rank"), py::arg("epoch"), py::arg("cap_bytes"),
        py::arg("status") = py::none());
  m.def("ep_exchange", &ep_exchange, py::arg("op"), py::arg("t"), py::arg("flags"), py::arg("bufs"),
        py::arg("rank"), py::arg("epoch"), py::arg("kind"), py::arg("src_start"), py::arg("count"),
        py::arg("dst_off"), py::arg("rows"), py::arg("cap_bytes"), py::arg("status") = py::none());
  m.def("tp_norm_ag", &tp_norm_ag, py::arg("x"), py::arg("w"), py::arg("rstd"), py::arg("out"),
        py::arg("flags"), py::arg("bufs"), py::arg("rank"), py::arg("epoch"), py::arg("B"), py::arg("S"),
        py::arg("eps"), py::arg("cap_bytes"), py::arg("status") = py::none());
  m.def("tp_collective", &tp_collective, py::arg("op"), py::arg("t"), py::arg("flags"), py::arg("bufs"),
        py::arg("rank"), py::arg("epoch"), py::arg("B"), py::arg("S"), py::arg("cap_bytes"),
        py::arg("status") = py::none());
  m.def("set_peer_wait_deadline", &set_peer_wait_deadline, py::arg("ns"));
  m.def("zero1_rs", &zero1_rs_b, py::arg("grads"), py::arg("params"), py::arg("flags"),
        py::arg("slots"), py::arg("offset"), py::arg("numel"), py::arg("rank"), py::arg("epoch"),
        py::arg("chunks"), py::arg("norm_sq"), py::arg("accumulate"), py::arg("status") = py::none());
  m.def("zero1_adamw_ag", &zero1_adamw_ag_b, py::arg("grads"), py::arg("params"), py::arg("flags"),
        py::arg("slots"), py::arg("offset"), py::arg("numel"), py::arg("rank"), py::arg("epoch"),
        py::arg("chunks"), py::arg("lr"), py::arg("wd"), py::arg("beta1"), py::arg("beta2"),
        py::arg("eps"), py::arg("bc1"), py::arg("bc2"), py::arg("grad_scale"), py::arg("rows"),
        py::arg("exp_avg"), py::arg("exp_avg_sq"), py::arg("status") = py::none());
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("softcap", &softcap);
  m.def("ce_rows", &ce_rows, py::arg("logits"), py::arg("labels"), py::arg("ignore_index"),
        py::arg("grad_scale"), py::arg("softcap"), py::arg("lse"), py::arg("loss_sum"),
        py::arg("n_valid"), py::arg("row_loss") = py::none(), py::arg("stats") = py::none(),
        py::arg("lse_in") = py::none(), py::arg("label_offset") = 0);
  m.def("embedding_bwd_sorted", &embedding_bwd_sorted);
  m.def("exp2_poly_eval", &exp2_poly_eval_b);
  m.def("router_topk", &router_topk_b, py::arg("logits"), py::arg("k"), py::arg("renorm"),
        py::arg("probs"), py::arg("w"), py::arg("idx"), py::arg("counts") = py::none());
  m.def("multi_sumsq", &multi_sumsq);
  m.def("multi_scale", &multi_scale);
  m.def("adamw_multi", &adamw_multi, py::arg("table"), py::arg("ntensors"), py::arg("total_chunks"),
        py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("wd"),
        py::arg("bc1"), py::arg("bc2"), py::arg("grad_scale") = py::none(),
        py::arg("hyper") = py::none());
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_bwd", &attn_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"),
        py::arg("lse"), py::arg("dout"), py::arg("dq"), py::arg("dk"), py::arg("dv"),
        py::arg("dq_acc"), py::arg("delta"), py::arg("scale"), py::arg("causal"),
        py::arg("window"), py::arg("status") = py::none(), py::arg("trace") = py::none());
}
