// Python bindings of the sm_100a kernels (module centrifuge_b200._kernels).
//
// Each binding checks devices, dtypes, shapes and strides of its tensors, then launches the
// kernel on the current CUDA stream.  A non-zero launcher status raises a RuntimeError: there is
// no fallback path on the GPU.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <tuple>

#include "kernels/launch_api.h"

namespace {

using at::Tensor;

#define CFB_CHECK_RC(rc, what) TORCH_CHECK((rc) == 0, what, " failed with status ", (rc))

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

inline void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
inline void check_bf16_2d(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with unit inner stride");
}
template <typename T>
inline const T* opt_ptr(const c10::optional<Tensor>& t) {
  return (t.has_value() && t->defined()) ? static_cast<const T*>(t->data_ptr()) : nullptr;
}

// Per-device status block handed to every kernel as `err` (layout in sm100_common.cuh):
// [0] first error code, [1] local wait limit (us, 0 = default), [2] peer wait limit (us),
// [3] reserved.
constexpr int64_t kStatusWordsHost = 4;
Tensor& err_word(int device) {
  static std::vector<Tensor> words(64);
  Tensor& w = words.at(device);
  if (!w.defined())
    w = at::zeros({kStatusWordsHost},
                  at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device));
  return w;
}

inline void check_status(const Tensor& err, const char* what) {
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt && err.is_contiguous() &&
                  err.numel() >= kStatusWordsHost,
              what, ": err must be a device status block (int32, >= 4 words; see status_block)");
}

// Work counter of the persistent attention kernels (two int32 words per device, zero at rest;
// forward and backward launches on one device are stream-ordered, so they share it).
Tensor& attn_work_counter(int device) {
  static std::vector<Tensor> words(64);
  Tensor& w = words.at(device);
  if (!w.defined())
    w = at::zeros({2}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device));
  return w;
}

// out[M, N] = epi(alpha * op(a) @ op(b))
//   a: [M, K] (a_mn = false) or [K, M] (a_mn = true)
//   b: [N, K] (b_mn = false) or [K, N] (b_mn = true)
void gemm(const Tensor& a, const Tensor& b, Tensor& out, bool a_mn, bool b_mn, int64_t epi,
          const c10::optional<Tensor>& resid, double alpha, int64_t bn, int64_t max_ctas) {
  check_bf16_2d(a, "a");
  check_bf16_2d(b, "b");
  check_cuda(out, "out");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1, "out must be 2-D row-major");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm: inner dimensions differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm: out has shape ", out.sizes(),
              ", expected [", M, ", ", N, "]");
  if (epi == kEpiBF16 || epi == kEpiBF16Resid) {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "gemm: bf16 epilogue needs a bf16 out");
  } else {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "gemm: fp32 epilogue needs an fp32 out");
  }
  const void* r = nullptr;
  int64_t ldr = 0;
  if (epi == kEpiBF16Resid) {
    TORCH_CHECK(resid.has_value() && resid->defined(), "gemm: residual epilogue needs resid");
    check_bf16_2d(*resid, "resid");
    TORCH_CHECK(resid->size(0) == M && resid->size(1) == N, "gemm: resid shape mismatch");
    r = resid->data_ptr();
    ldr = resid->stride(0);
  }
  if (M == 0 || N == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  if (K == 0) {
    if (epi != kEpiF32Acc && epi != kEpiBF16Resid) out.zero_();
    if (epi == kEpiBF16Resid) out.copy_(*resid);
    return;
  }
  int rc = cfb_gemm_bf16(a.data_ptr(), a.stride(0), a_mn, b.data_ptr(), b.stride(0), b_mn,
                         out.data_ptr(), out.stride(0), static_cast<int>(epi), r, ldr,
                         static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                         static_cast<float>(alpha),
                         err_word(a.get_device()).data_ptr<int>(), static_cast<int>(bn),
                         static_cast<int>(max_ctas), cur_stream());
  CFB_CHECK_RC(rc, "gemm");
}

// out[M, N] = a @ b^T (both K-major) with rotate-half RoPE applied in the epilogue to columns
// [0, rope_cols) (heads of hd columns) at positions pos[M] (int32), table [max_pos, hd/2, 2] fp32.
void gemm_rope(const Tensor& a, const Tensor& b, Tensor& out, const Tensor& pos,
               const Tensor& table, int64_t rope_cols, int64_t hd, int64_t bn) {
  check_bf16_2d(a, "a");
  check_bf16_2d(b, "b");
  check_bf16_2d(out, "out");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(b.size(1) == K, "gemm_rope: inner dimensions differ");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm_rope: out shape");
  TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == at::kInt && pos.numel() == M &&
                  pos.is_contiguous(), "gemm_rope: pos must be int32 [M] on the device");
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kFloat && table.is_contiguous() &&
                  table.dim() == 3 && table.size(1) == hd / 2 && table.size(2) == 2,
              "gemm_rope: table must be fp32 [max_pos, hd/2, 2]");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  CFB_CHECK_RC(cfb_gemm_bf16_rope(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                                  out.data_ptr(), out.stride(0), static_cast<int>(M),
                                  static_cast<int>(N), static_cast<int>(K), pos.data_ptr<int>(),
                                  table.data_ptr<float>(), static_cast<int>(rope_cols),
                                  static_cast<int>(hd), err_word(a.get_device()).data_ptr<int>(),
                                  static_cast<int>(bn), 0, cur_stream()),
               "gemm_rope");
}

// gu [M, 2F] = x @ w^T (w = [gate; up] [2F, K]) and h [M, F] = silu(gate) * up in the epilogue
void gemm_swiglu(const Tensor& x, const Tensor& w, Tensor& gu, Tensor& h) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  check_bf16_2d(gu, "gu");
  check_bf16_2d(h, "h");
  const int64_t M = x.size(0), K = x.size(1), F2 = w.size(0);
  TORCH_CHECK(w.size(1) == K && F2 % 2 == 0, "gemm_swiglu: w must be [2F, K]");
  TORCH_CHECK(gu.size(0) == M && gu.size(1) == F2 && h.size(0) == M && h.size(1) == F2 / 2,
              "gemm_swiglu: outputs");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  CFB_CHECK_RC(cfb_gemm_swiglu(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0),
                               gu.data_ptr(), gu.stride(0), h.data_ptr(), h.stride(0),
                               static_cast<int>(M), static_cast<int>(F2 / 2),
                               static_cast<int>(K), err_word(x.get_device()).data_ptr<int>(),
                               cur_stream()),
               "gemm_swiglu");
}

// lm_head forward fused with cross-entropy statistics: per row and 256-column tile of
// x @ w^T the max and sum of exp (pmax, psum [M, ceil(N / 256)]) and the label logit (ptgt [M]);
// the logits are never stored
void gemm_ce_part(const Tensor& x, const Tensor& w, const Tensor& labels, Tensor& pmax,
                  Tensor& psum, Tensor& ptgt) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0), nt = (N + 255) / 256;
  TORCH_CHECK(w.size(1) == K, "gemm_ce_part: w must be [N, K]");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == M,
              "gemm_ce_part: labels int64 [M]");
  for (const Tensor* t : {&pmax, &psum})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == M * nt,
                "gemm_ce_part: pmax / psum fp32 [M, ceil(N / 256)]");
  TORCH_CHECK(ptgt.scalar_type() == at::kFloat && ptgt.numel() == M, "gemm_ce_part: ptgt");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  CFB_CHECK_RC(cfb_gemm_ce_part(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0),
                                static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                                reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()),
                                pmax.data_ptr<float>(), psum.data_ptr<float>(),
                                ptgt.data_ptr<float>(), err_word(x.get_device()).data_ptr<int>(),
                                cur_stream()),
               "gemm_ce_part");
}

// dlogits [M, N] = (softmax(x @ w^T) - onehot(labels)) * dloss with the logits recomputed
void gemm_ce_grad(const Tensor& x, const Tensor& w, const Tensor& labels, const Tensor& lse,
                  const Tensor& dloss, Tensor& out) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  check_bf16_2d(out, "out");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K && out.size(0) == M && out.size(1) == N, "gemm_ce_grad: shapes");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == M,
              "gemm_ce_grad: labels int64 [M]");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == M &&
                  dloss.scalar_type() == at::kFloat && dloss.is_contiguous() &&
                  dloss.numel() == M,
              "gemm_ce_grad: lse / dloss fp32 [M]");
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  CFB_CHECK_RC(cfb_gemm_ce_grad(x.data_ptr(), x.stride(0), w.data_ptr(), w.stride(0),
                                out.data_ptr(), out.stride(0), static_cast<int>(M),
                                static_cast<int>(N), static_cast<int>(K),
                                reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()),
                                lse.data_ptr<float>(), dloss.data_ptr<float>(),
                                err_word(x.get_device()).data_ptr<int>(), cur_stream()),
               "gemm_ce_grad");
}

void ce_combine(const Tensor& pmax, const Tensor& psum, const Tensor& ptgt, const Tensor& labels,
                int64_t vocab, Tensor& loss, Tensor& lse) {
  const int64_t M = labels.numel();
  TORCH_CHECK(M > 0 && pmax.numel() % M == 0 && psum.numel() == pmax.numel(),
              "ce_combine: statistics");
  const c10::cuda::CUDAGuard guard(pmax.device());
  CFB_CHECK_RC(cfb_ce_combine(pmax.data_ptr<float>(), psum.data_ptr<float>(),
                              ptgt.data_ptr<float>(), static_cast<int>(M),
                              static_cast<int>(pmax.numel() / M),
                              reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()),
                              vocab, loss.data_ptr<float>(), lse.data_ptr<float>(),
                              err_word(pmax.get_device()).data_ptr<int>(), cur_stream()),
               "ce_combine");
}

// (bn, ksplit, pair) the GEMM planner picks for an M x N x K problem on `sms` SMs (host only)
std::tuple<int64_t, int64_t, bool> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t epi,
                                             int64_t bn, int64_t sms) {
  int obn = 0, oks = 0, opair = 0;
  CFB_CHECK_RC(cfb_gemm_plan(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                             static_cast<int>(epi), static_cast<int>(bn), static_cast<int>(sms),
                             &obn, &oks, &opair),
               "gemm_plan");
  return {obn, oks, opair != 0};
}

// dgu [M, 2F] = SwiGLU backward of dh = dy @ wd (wd [H, F], read MN-major) with the gate/up
// activations of row gu_rows[m] (or m) of gu [*, 2F]; dh stays in TMEM.
void gemm_swiglu_bwd(const Tensor& dy, const Tensor& wd, const Tensor& gu,
                     const c10::optional<Tensor>& gu_rows, Tensor& dgu) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(wd, "wd");
  check_bf16_2d(gu, "gu");
  check_bf16_2d(dgu, "dgu");
  const int64_t M = dy.size(0), K = dy.size(1), F = wd.size(1);
  TORCH_CHECK(wd.size(0) == K, "gemm_swiglu_bwd: wd must be [H, F] with H = dy.size(1)");
  TORCH_CHECK(gu.size(1) == 2 * F && dgu.size(0) == M && dgu.size(1) == 2 * F,
              "gemm_swiglu_bwd: gu / dgu must have 2F columns");
  const int* rows = nullptr;
  if (gu_rows.has_value() && gu_rows->defined()) {
    TORCH_CHECK(gu_rows->is_cuda() && gu_rows->scalar_type() == at::kInt &&
                    gu_rows->numel() == M && gu_rows->is_contiguous(),
                "gemm_swiglu_bwd: gu_rows must be int32 [M] on the device");
    rows = gu_rows->data_ptr<int>();
  } else {
    TORCH_CHECK(gu.size(0) == M, "gemm_swiglu_bwd: gu must have M rows without gu_rows");
  }
  if (M == 0) return;
  const c10::cuda::CUDAGuard guard(dy.device());
  CFB_CHECK_RC(cfb_gemm_swiglu_bwd(dy.data_ptr(), dy.stride(0), wd.data_ptr(), wd.stride(0),
                                   gu.data_ptr(), gu.stride(0), rows, dgu.data_ptr(),
                                   dgu.stride(0), static_cast<int>(M), static_cast<int>(F),
                                   static_cast<int>(K), err_word(dy.get_device()).data_ptr<int>(),
                                   cur_stream()),
               "gemm_swiglu_bwd");
}

// ---- tensor-parallel fusion (pointers into symmetric memory are raw device addresses)
// out = a @ b^T (a @ b with b_mn) fused with a sequence-parallel collective over NVLink:
// mode 1 all-gathers this rank's rows of `a` to every rank while computing, mode 2 writes the
// partials into `out` (this rank's symmetric partial buffer) and this rank's reduced rows
// (+resid) into `rs_out`.
void gemm_tp(const Tensor& a, const Tensor& b, Tensor& out, bool b_mn,
             const c10::optional<Tensor>& pos, const c10::optional<Tensor>& table,
             int64_t rope_cols, int64_t hd, int64_t mode, int64_t rank, int64_t P,
             const Tensor& seg, int64_t epoch, int64_t peer_flags_dev, int64_t flag_ready,
             int64_t flag_done, Tensor& tile_cnt, int64_t rot_rows, int64_t ag_mc,
             int64_t ag_peers_dev, int64_t mc_part, int64_t peer_part_dev, int64_t flag_blk,
             int64_t interleave_spb, const c10::optional<Tensor>& resid,
             const c10::optional<Tensor>& rs_out, int64_t bn) {
  check_bf16_2d(a, "a");
  check_bf16_2d(b, "b");
  check_bf16_2d(out, "out");
  const int64_t M = a.size(0), K = a.size(1), N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K && out.size(0) == M && out.size(1) == N,
              "gemm_tp: shapes");
  TORCH_CHECK(seg.is_cuda() && seg.scalar_type() == at::kInt && seg.numel() == P + 1,
              "gemm_tp: seg must be int32 [P + 1] on the device");
  TORCH_CHECK(tile_cnt.scalar_type() == at::kInt &&
                  tile_cnt.numel() >= std::max<int64_t>(P, (M + 127) / 128) + 2,
              "tile_cnt");
  CfbTpGemm t = {};
  t.mode = static_cast<int>(mode);
  t.rank = static_cast<int>(rank);
  t.P = static_cast<int>(P);
  t.seg = seg.data_ptr<int>();
  t.epoch = static_cast<uint32_t>(epoch);
  t.peer_flags = reinterpret_cast<uint32_t* const*>(peer_flags_dev);
  t.flag_ready = static_cast<int>(flag_ready);
  t.flag_done = static_cast<int>(flag_done);
  t.tile_cnt = reinterpret_cast<uint32_t*>(tile_cnt.data_ptr<int>());
  t.rot_rows = static_cast<int>(rot_rows);
  t.ag_mc = reinterpret_cast<void*>(ag_mc);
  t.ag_peers = reinterpret_cast<void* const*>(ag_peers_dev);
  t.mc_part = reinterpret_cast<const void*>(mc_part);
  t.peer_part = reinterpret_cast<const void* const*>(peer_part_dev);
  t.flag_blk = static_cast<int>(flag_blk);
  t.interleave_spb = static_cast<int>(interleave_spb);
  if (resid.has_value() && resid->defined()) {
    check_bf16_2d(*resid, "resid");
    t.resid = resid->data_ptr();
    t.ld_resid = resid->stride(0);
  }
  if (rs_out.has_value() && rs_out->defined()) {
    check_bf16_2d(*rs_out, "rs_out");
    TORCH_CHECK(rs_out->size(1) == N, "rs_out columns");
    t.out = rs_out->data_ptr();
    t.ld_out = rs_out->stride(0);
    t.out_rows = static_cast<int>(rs_out->size(0));
  }
  const int* pp = nullptr;
  const float* cs = nullptr;
  if (table.has_value() && table->defined()) {
    TORCH_CHECK(pos.has_value() && pos->scalar_type() == at::kInt && pos->numel() == M, "pos");
    TORCH_CHECK(table->scalar_type() == at::kFloat && table->is_contiguous(), "table");
    pp = pos->data_ptr<int>();
    cs = table->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(a.device());
  CFB_CHECK_RC(cfb_gemm_tp(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), b_mn ? 1 : 0,
                           out.data_ptr(), out.stride(0), static_cast<int>(M),
                           static_cast<int>(N), static_cast<int>(K), pp, cs,
                           static_cast<int>(rope_cols), static_cast<int>(hd), &t,
                           err_word(a.get_device()).data_ptr<int>(), static_cast<int>(bn),
                           cur_stream()),
               "gemm_tp");
}

int64_t gemm_error_word(int64_t device, bool reset) {
  Tensor& w = err_word(static_cast<int>(device));
  const int64_t v = w[0].item<int>();
  if (reset) w[0].zero_();
  return v;
}

// The device status block itself (shared by every kernel launched on `device`).
Tensor status_block(int64_t device) { return err_word(static_cast<int>(device)); }

// Limits of the bounded device waits on `device`, in microseconds (0 restores the default:
// 4 s for waits on the GPU's own work, 20 s for waits on another GPU).  Stream-ordered.
void set_wait_limits(int64_t device, int64_t local_us, int64_t peer_us) {
  TORCH_CHECK(local_us >= 0 && local_us <= INT32_MAX && peer_us >= 0 && peer_us <= INT32_MAX,
              "set_wait_limits: limits must be in [0, 2^31) microseconds");
  Tensor& w = err_word(static_cast<int>(device));
  w[1].fill_(local_us);
  w[2].fill_(peer_us);
}

void rmsnorm_fwd(const Tensor& x, const Tensor& w, Tensor& y, const c10::optional<Tensor>& rstd,
                 double eps) {
  check_bf16_2d(x, "x");
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && w.is_contiguous(), "rmsnorm: contiguous");
  const int rows = x.size(0), H = x.size(1);
  float* rp = nullptr;
  if (rstd.has_value() && rstd->defined()) {
    TORCH_CHECK(rstd->scalar_type() == at::kFloat && rstd->numel() >= rows, "rstd");
    rp = rstd->data_ptr<float>();
  }
  if (rows == 0) return;
  const c10::cuda::CUDAGuard guard(x.device());
  CFB_CHECK_RC(cfb_rmsnorm_fwd(x.data_ptr(), w.data_ptr(), y.data_ptr(), rp, rows, H,
                               static_cast<float>(eps), cur_stream()),
               "rmsnorm_fwd");
}

void rmsnorm_bwd(const Tensor& dy, const Tensor& x, const c10::optional<Tensor>& x_rows,
                 const Tensor& rstd, const Tensor& w, const c10::optional<Tensor>& dres,
                 Tensor& dx, Tensor& dw_acc, int64_t partial_rows) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dx.is_contiguous(), "contiguous");
  TORCH_CHECK(dw_acc.scalar_type() == at::kFloat && dw_acc.is_contiguous(), "dw_acc fp32");
  const int rows = dy.size(0), H = dy.size(1);
  if (rows == 0) return;
  if (x_rows.has_value() && x_rows->defined())
    TORCH_CHECK(x_rows->scalar_type() == at::kInt && x_rows->numel() == rows, "x_rows int32");
  int P = static_cast<int>(std::min<int64_t>(partial_rows, rows));
  if (P < 1) P = 1;
  const c10::cuda::CUDAGuard guard(dy.device());
  Tensor partial = at::empty({P, H}, dy.options().dtype(at::kFloat));
  CFB_CHECK_RC(cfb_rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), opt_ptr<int>(x_rows),
                               rstd.data_ptr<float>(), w.data_ptr(), opt_ptr<void>(dres),
                               dx.data_ptr(), partial.data_ptr<float>(), dw_acc.data_ptr<float>(),
                               rows, H, P, cur_stream()),
               "rmsnorm_bwd");
}

void rope(Tensor& qkv, const Tensor& pos, int64_t n_heads, int64_t head_dim,
          const Tensor& cos_sin, bool inverse) {
  check_bf16_2d(qkv, "qkv");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.numel() == qkv.size(0), "pos int32 [rows]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos_sin fp32");
  TORCH_CHECK(n_heads * head_dim <= qkv.size(1), "rope: heads exceed the row");
  if (qkv.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(qkv.device());
  CFB_CHECK_RC(cfb_rope(qkv.data_ptr(), qkv.stride(0), pos.data_ptr<int>(), nullptr, qkv.size(0),
                        n_heads, head_dim, cos_sin.data_ptr<float>(), inverse ? 1 : 0,
                        cur_stream()),
               "rope");
}

void swiglu_fwd(const Tensor& gu, Tensor& h) {
  TORCH_CHECK(gu.is_contiguous() && h.is_contiguous(), "swiglu: contiguous");
  const int rows = gu.size(0), F = h.size(1);
  TORCH_CHECK(gu.size(1) == 2 * F, "swiglu: gu must be [rows, 2F]");
  if (rows == 0) return;
  const c10::cuda::CUDAGuard guard(gu.device());
  CFB_CHECK_RC(cfb_swiglu_fwd(gu.data_ptr(), h.data_ptr(), rows, F, cur_stream()), "swiglu_fwd");
}

void swiglu_bwd(const Tensor& dh, const Tensor& gu, const c10::optional<Tensor>& gu_rows,
                Tensor& dgu, const c10::optional<Tensor>& h_out) {
  TORCH_CHECK(dh.is_contiguous() && gu.is_contiguous() && dgu.is_contiguous(), "contiguous");
  const int rows = dh.size(0), F = dh.size(1);
  TORCH_CHECK(dgu.size(0) == rows && dgu.size(1) == 2 * F, "dgu shape");
  void* hp = nullptr;
  if (h_out.has_value() && h_out->defined()) {
    TORCH_CHECK(h_out->is_contiguous() && h_out->size(0) == rows && h_out->size(1) == F &&
                    h_out->scalar_type() == dh.scalar_type(),
                "swiglu_bwd: h_out must be [rows, F] like dh");
    hp = h_out->data_ptr();
  }
  if (rows == 0) return;
  const c10::cuda::CUDAGuard guard(dh.device());
  CFB_CHECK_RC(cfb_swiglu_bwd(dh.data_ptr(), gu.data_ptr(), opt_ptr<int>(gu_rows), dgu.data_ptr(),
                              hp, rows, F, cur_stream()),
               "swiglu_bwd");
}

void gather_rows(const Tensor& src, const Tensor& idx, Tensor& dst) {
  check_cuda(src, "src");
  TORCH_CHECK(src.dim() == 2 && src.stride(1) == 1 && dst.dim() == 2 && dst.stride(1) == 1,
              "gather_rows: 2-D row-major");
  TORCH_CHECK(idx.scalar_type() == at::kInt && idx.numel() == dst.size(0), "idx int32 [rows]");
  TORCH_CHECK(src.size(1) == dst.size(1) && src.scalar_type() == dst.scalar_type(), "gather dims");
  const int64_t es = src.element_size();
  if (dst.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(src.device());
  CFB_CHECK_RC(cfb_gather_rows(src.data_ptr(), src.stride(0) * es, src.size(0),
                               idx.data_ptr<int>(), dst.data_ptr(), dst.stride(0) * es,
                               dst.size(0), static_cast<int>(dst.size(1) * es),
                               err_word(src.get_device()).data_ptr<int>(), cur_stream()),
               "gather_rows");
}

void embedding_fwd(const Tensor& table, const Tensor& ids, Tensor& out) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids int64");
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous(), "contiguous");
  if (ids.numel() == 0) return;
  const c10::cuda::CUDAGuard guard(table.device());
  CFB_CHECK_RC(cfb_embedding_fwd(table.data_ptr(), table.size(0),
                                 reinterpret_cast<const long long*>(ids.data_ptr<int64_t>()),
                                 out.data_ptr(), ids.numel(), table.size(1),
                                 err_word(table.get_device()).data_ptr<int>(), cur_stream()),
               "embedding_fwd");
}

void embedding_bwd(const Tensor& dy, const Tensor& ids, const c10::optional<Tensor>& id_rows,
                   Tensor& dtable, bool deterministic) {
  TORCH_CHECK(dtable.scalar_type() == at::kFloat && dtable.is_contiguous(), "dtable fp32");
  TORCH_CHECK(dy.is_contiguous() && ids.scalar_type() == at::kLong, "dy/ids");
  if (dy.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(dy.device());
  if (deterministic) {
    // each row's token, a stable sort by token, then one warp per run of equal tokens
    int* err = err_word(dy.get_device()).data_ptr<int>();
    Tensor tok = at::empty({dy.size(0)}, ids.options());
    CFB_CHECK_RC(cfb_row_tokens(reinterpret_cast<const long long*>(ids.data_ptr<int64_t>()),
                                ids.numel(), reinterpret_cast<const int*>(opt_ptr<int>(id_rows)),
                                reinterpret_cast<long long*>(tok.data_ptr<int64_t>()),
                                dy.size(0), err, cur_stream()),
                 "row_tokens");
    auto sorted = at::sort(tok, /*stable=*/true, /*dim=*/0, /*descending=*/false);
    const Tensor& stok = std::get<0>(sorted);
    const Tensor& order = std::get<1>(sorted);
    CFB_CHECK_RC(cfb_embedding_bwd_sorted(
                     dy.data_ptr(), reinterpret_cast<const long long*>(stok.data_ptr<int64_t>()),
                     reinterpret_cast<const long long*>(order.data_ptr<int64_t>()),
                     dtable.data_ptr<float>(), dtable.size(0), dy.size(0), dy.size(1), err,
                     cur_stream()),
                 "embedding_bwd_sorted");
    return;
  }
  CFB_CHECK_RC(cfb_embedding_bwd(dy.data_ptr(), reinterpret_cast<const long long*>(ids.data_ptr<int64_t>()),
                                 reinterpret_cast<const int*>(opt_ptr<int>(id_rows)),
                                 dtable.data_ptr<float>(), dtable.size(0), dy.size(0), dy.size(1),
                                 err_word(dy.get_device()).data_ptr<int>(), cur_stream()),
               "embedding_bwd");
}

void ce_fwd(const Tensor& logits, const Tensor& labels, Tensor& loss, Tensor& lse) {
  check_bf16_2d(logits, "logits");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.numel() == logits.size(0), "labels");
  TORCH_CHECK(loss.scalar_type() == at::kFloat && lse.scalar_type() == at::kFloat, "fp32 outs");
  if (logits.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  CFB_CHECK_RC(cfb_ce_fwd(logits.data_ptr(), logits.stride(0), reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()),
                          loss.data_ptr<float>(), lse.data_ptr<float>(), logits.size(0),
                          logits.size(1), err_word(logits.get_device()).data_ptr<int>(),
                          cur_stream()),
               "ce_fwd");
}

void ce_bwd(const Tensor& logits, const c10::optional<Tensor>& rows, const Tensor& labels,
            const Tensor& lse, const Tensor& dloss, Tensor& dlogits, int64_t vocab_start) {
  check_bf16_2d(logits, "logits");
  check_bf16_2d(dlogits, "dlogits");
  TORCH_CHECK(dloss.scalar_type() == at::kFloat && dloss.numel() == dlogits.size(0), "dloss");
  if (dlogits.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  CFB_CHECK_RC(cfb_ce_bwd(logits.data_ptr(), logits.stride(0), opt_ptr<int>(rows),
                          reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()), lse.data_ptr<float>(),
                          dloss.data_ptr<float>(), dlogits.data_ptr(), dlogits.stride(0),
                          dlogits.size(0), logits.size(1), vocab_start, cur_stream()),
               "ce_bwd");
}

void ce_partial(const Tensor& logits, const Tensor& labels, Tensor& pmax, Tensor& psum,
                Tensor& ptgt, int64_t vocab_start) {
  check_bf16_2d(logits, "logits");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.numel() == logits.size(0), "labels");
  if (logits.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  CFB_CHECK_RC(cfb_ce_partial(logits.data_ptr(), logits.stride(0),
                              reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()),
                              pmax.data_ptr<float>(), psum.data_ptr<float>(),
                              ptgt.data_ptr<float>(), logits.size(0), logits.size(1),
                              vocab_start, cur_stream()),
               "ce_partial");
}

void adamw(Tensor& master, const Tensor& grad, Tensor& m, Tensor& v, Tensor& param, double lr,
           double b1, double b2, double eps, double wd, double bc1, double bc2,
           const c10::optional<Tensor>& grad_scale) {
  TORCH_CHECK(master.scalar_type() == at::kFloat && grad.scalar_type() == at::kFloat, "fp32");
  TORCH_CHECK(param.scalar_type() == at::kBFloat16, "param bf16");
  const int64_t n = master.numel();
  TORCH_CHECK(grad.numel() == n && m.numel() == n && v.numel() == n && param.numel() == n, "n");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(master.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(grad.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(m.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(v.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(param.data_ptr()) & 7) == 0,
              "adamw: buffers must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(master.device());
  CFB_CHECK_RC(cfb_adamw(master.data_ptr<float>(), grad.data_ptr<float>(), m.data_ptr<float>(),
                         v.data_ptr<float>(), param.data_ptr(), n, lr, b1, b2, eps, wd, bc1, bc2,
                         opt_ptr<float>(grad_scale), cur_stream()),
               "adamw");
}

// AdamW on a shard with the bf16 result written through the multicast address `param_mc` (raw
// device address into symmetric memory): the ZeRO parameter all-gather fused into the step.
void adamw_multicast(Tensor& master, const Tensor& grad, Tensor& m, Tensor& v, int64_t param_mc,
                     double lr, double b1, double b2, double eps, double wd, double bc1,
                     double bc2, const c10::optional<Tensor>& grad_scale) {
  TORCH_CHECK(master.scalar_type() == at::kFloat && grad.scalar_type() == at::kFloat, "fp32");
  const int64_t n = master.numel();
  TORCH_CHECK(grad.numel() == n && m.numel() == n && v.numel() == n, "n");
  const c10::cuda::CUDAGuard guard(master.device());
  CFB_CHECK_RC(cfb_adamw_multicast(master.data_ptr<float>(), grad.data_ptr<float>(),
                                   m.data_ptr<float>(), v.data_ptr<float>(),
                                   reinterpret_cast<void*>(param_mc), n, lr, b1, b2, eps, wd,
                                   bc1, bc2, opt_ptr<float>(grad_scale), cur_stream()),
               "adamw_multicast");
}

void sumsq(const Tensor& x, Tensor& partial) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && partial.scalar_type() == at::kFloat, "fp32");
  const c10::cuda::CUDAGuard guard(x.device());
  CFB_CHECK_RC(cfb_sumsq(x.data_ptr<float>(), x.numel(), partial.data_ptr<float>(),
                         static_cast<int>(partial.numel()), cur_stream()),
               "sumsq");
}

void clip_coef(const Tensor& partials, double max_norm, double extra_scale, Tensor& coef,
               Tensor& norm) {
  const c10::cuda::CUDAGuard guard(partials.device());
  CFB_CHECK_RC(cfb_clip_coef(partials.data_ptr<float>(), partials.numel(), max_norm, extra_scale,
                             coef.data_ptr<float>(), norm.data_ptr<float>(),
                             err_word(partials.get_device()).data_ptr<int>(), cur_stream()),
               "clip_coef");
}

void drop_smallest(const Tensor& score, Tensor& mask, int64_t start, int64_t end, int64_t k) {
  TORCH_CHECK(score.scalar_type() == at::kFloat && score.dim() == 2 && score.stride(1) == 1,
              "score fp32 2-D");
  TORCH_CHECK(mask.dim() == 2 && mask.stride(1) == 1 && mask.size(0) == score.size(0), "mask");
  TORCH_CHECK(end <= score.size(1) && end <= mask.size(1), "drop_smallest: range");
  int* m32 = nullptr;
  long long* m64 = nullptr;
  if (mask.scalar_type() == at::kLong)
    m64 = reinterpret_cast<long long*>(mask.data_ptr<int64_t>());
  else if (mask.scalar_type() == at::kInt)
    m32 = mask.data_ptr<int>();
  else
    TORCH_CHECK(false, "mask must be int32 or int64");
  if (score.size(0) == 0) return;
  const c10::cuda::CUDAGuard guard(score.device());
  CFB_CHECK_RC(cfb_drop_smallest(score.data_ptr<float>(), score.stride(0), m32, m64,
                                 mask.stride(0), score.size(0), start, end, k, cur_stream()),
               "drop_smallest");
}

void keep_index(const Tensor& mask, int64_t S_keep, Tensor& pos, Tensor& flat_rows, Tensor& err) {
  TORCH_CHECK(mask.scalar_type() == at::kLong && mask.is_contiguous() && mask.dim() == 2,
              "mask int64 [B, S]");
  TORCH_CHECK(pos.scalar_type() == at::kInt && flat_rows.scalar_type() == at::kInt, "int32");
  check_status(err, "keep_index");
  const c10::cuda::CUDAGuard guard(mask.device());
  CFB_CHECK_RC(cfb_keep_index(reinterpret_cast<const long long*>(mask.data_ptr<int64_t>()),
                              mask.size(0), mask.size(1), S_keep, pos.data_ptr<int>(),
                              flat_rows.data_ptr<int>(), err.data_ptr<int>(), cur_stream()),
               "keep_index");
}

void cast_f32_bf16(const Tensor& x, Tensor& y) {
  const c10::cuda::CUDAGuard guard(x.device());
  CFB_CHECK_RC(cfb_cast_f32_bf16(x.data_ptr<float>(), y.data_ptr(), x.numel(), cur_stream()),
               "cast");
}

void scale_f32(Tensor& x, double s) {
  const c10::cuda::CUDAGuard guard(x.device());
  CFB_CHECK_RC(cfb_scale_f32(x.data_ptr<float>(), x.numel(), s, cur_stream()), "scale");
}

void attn_fwd_mma(const Tensor& qkv, Tensor& out, Tensor& lse, int64_t B, int64_t S, int64_t nh,
                  int64_t nkv, int64_t hd, double scale) {
  check_bf16_2d(qkv, "qkv");
  check_bf16_2d(out, "out");
  TORCH_CHECK(qkv.size(0) == B * S && out.size(0) == B * S, "attn_fwd: rows");
  TORCH_CHECK(qkv.size(1) >= (nh + 2 * nkv) * hd && out.size(1) >= nh * hd, "attn_fwd: cols");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * S * nh, "lse [T, nh] fp32");
  const c10::cuda::CUDAGuard guard(qkv.device());
  CFB_CHECK_RC(cfb_attn_fwd(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0),
                            lse.data_ptr<float>(), B, S, nh, nkv, hd, scale, cur_stream()),
               "attn_fwd");
}

// Causal GQA attention forward on tcgen05/TMEM (the production path).
void attn_fwd(const Tensor& qkv, Tensor& out, Tensor& lse, int64_t B, int64_t S, int64_t nh,
              int64_t nkv, int64_t hd, double scale) {
  check_bf16_2d(qkv, "qkv");
  check_bf16_2d(out, "out");
  TORCH_CHECK(qkv.size(0) == B * S && out.size(0) == B * S, "attn_fwd: rows");
  TORCH_CHECK(qkv.size(1) >= (nh + 2 * nkv) * hd && out.size(1) >= nh * hd, "attn_fwd: cols");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * S * nh, "lse [T, nh] fp32");
  const c10::cuda::CUDAGuard guard(qkv.device());
  CFB_CHECK_RC(cfb_attn_fwd_tc(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0),
                               lse.data_ptr<float>(), B, S, nh, nkv, hd, scale,
                               attn_work_counter(qkv.get_device()).data_ptr<int>(),
                               err_word(qkv.get_device()).data_ptr<int>(), cur_stream()),
               "attn_fwd");
}

void check_attn_bwd_args(const Tensor& qkv_k, const Tensor& qkv_full, const Tensor& o_k,
                         const Tensor& do_k, const Tensor& lse_k, const Tensor& pos_k,
                         const Tensor& dqkv_k, const Tensor& delta, int64_t B, int64_t S,
                         int64_t Sk, int64_t nh) {
  check_bf16_2d(qkv_k, "qkv_k");
  check_bf16_2d(qkv_full, "qkv_full");
  check_bf16_2d(o_k, "o_k");
  check_bf16_2d(do_k, "do_k");
  check_bf16_2d(dqkv_k, "dqkv_k");
  TORCH_CHECK(qkv_k.stride(0) == qkv_full.stride(0) && dqkv_k.stride(0) == qkv_k.stride(0),
              "attn_bwd: qkv buffers share the row stride");
  TORCH_CHECK(o_k.stride(0) == do_k.stride(0), "attn_bwd: o and do share the row stride");
  TORCH_CHECK(qkv_k.size(0) == B * Sk && qkv_full.size(0) == B * S, "attn_bwd: rows");
  TORCH_CHECK(pos_k.scalar_type() == at::kInt && pos_k.numel() == B * Sk, "pos_k int32");
  TORCH_CHECK(delta.scalar_type() == at::kFloat && delta.numel() >= B * Sk * nh, "delta");
  TORCH_CHECK(lse_k.scalar_type() == at::kFloat && lse_k.numel() == B * Sk * nh, "lse_k");
}

// Filtered causal GQA attention backward on tcgen05/TMEM (the production path).
void attn_bwd(const Tensor& qkv_k, const Tensor& qkv_full, const Tensor& o_k, const Tensor& do_k,
              const Tensor& lse_k, const Tensor& pos_k, Tensor& dqkv_k, Tensor& delta, int64_t B,
              int64_t S, int64_t Sk, int64_t nh, int64_t nkv, int64_t hd, double scale,
              const c10::optional<Tensor>& rope_table) {
  check_attn_bwd_args(qkv_k, qkv_full, o_k, do_k, lse_k, pos_k, dqkv_k, delta, B, S, Sk, nh);
  const float* cs = nullptr;
  if (rope_table.has_value() && rope_table->defined()) {
    const Tensor& t = *rope_table;
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() &&
                    t.dim() == 3 && t.size(1) == hd / 2 && t.size(2) == 2 && t.size(0) >= S,
                "attn_bwd: rope_table must be fp32 [max_pos >= S, hd/2, 2]");
    cs = t.data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(qkv_k.device());
  CFB_CHECK_RC(cfb_attn_delta(o_k.data_ptr(), do_k.data_ptr(), o_k.stride(0),
                              delta.data_ptr<float>(), B * Sk, nh, hd, cur_stream()),
               "attn_delta");
  CFB_CHECK_RC(cfb_attn_bwd_tc(qkv_k.data_ptr(), qkv_k.stride(0), qkv_full.data_ptr(),
                               do_k.data_ptr(), do_k.stride(0), lse_k.data_ptr<float>(),
                               delta.data_ptr<float>(), pos_k.data_ptr<int>(), dqkv_k.data_ptr(),
                               B, S, Sk, nh, nkv, hd, scale, cs,
                               attn_work_counter(qkv_k.get_device()).data_ptr<int>(),
                               err_word(qkv_k.get_device()).data_ptr<int>(), cur_stream()),
               "attn_bwd");
}

// mma.sync (legacy tensor path) backward, kept as a comparison point.
void attn_bwd_mma(const Tensor& qkv_k, const Tensor& qkv_full, const Tensor& o_k,
                  const Tensor& do_k, const Tensor& lse_k, const Tensor& pos_k, Tensor& dqkv_k,
                  Tensor& delta, int64_t B, int64_t S, int64_t Sk, int64_t nh, int64_t nkv,
                  int64_t hd, double scale) {
  check_attn_bwd_args(qkv_k, qkv_full, o_k, do_k, lse_k, pos_k, dqkv_k, delta, B, S, Sk, nh);
  const c10::cuda::CUDAGuard guard(qkv_k.device());
  CFB_CHECK_RC(cfb_attn_bwd(qkv_k.data_ptr(), qkv_k.stride(0), qkv_full.data_ptr(),
                            o_k.data_ptr(), o_k.stride(0), do_k.data_ptr(),
                            lse_k.data_ptr<float>(), pos_k.data_ptr<int>(), dqkv_k.data_ptr(),
                            nullptr, delta.data_ptr<float>(), B, S, Sk, nh, nkv, hd, scale,
                            cur_stream()),
               "attn_bwd_mma");
}

// ---- NVLink peer-memory gradient reduction (pointers are raw device addresses from the
// symmetric-memory handle; `err` is a device int32 word)
void symm_signal(int64_t peer_flags_dev, int64_t W, int64_t off, int64_t epoch) {
  CFB_CHECK_RC(cfb_symm_signal(reinterpret_cast<uint32_t* const*>(peer_flags_dev), W, off,
                               static_cast<uint32_t>(epoch), cur_stream()),
               "symm_signal");
}

void symm_wait(int64_t flags, int64_t base, int64_t stride, int64_t n, int64_t epoch,
               Tensor& err) {
  check_status(err, "symm_wait");
  CFB_CHECK_RC(cfb_symm_wait(reinterpret_cast<const uint32_t*>(flags), base, stride, n,
                             static_cast<uint32_t>(epoch), err.data_ptr<int>(), cur_stream()),
               "symm_wait");
}

void symm_pull_reduce(int64_t mc_base, int64_t peer_base_dev, int64_t W, int64_t off, int64_t n,
                      Tensor& dst, double scale, Tensor& err) {
  TORCH_CHECK(dst.scalar_type() == at::kFloat && dst.is_contiguous() && dst.numel() == n,
              "symm_pull_reduce: dst must be a contiguous fp32 [n] tensor");
  check_status(err, "symm_pull_reduce");
  CFB_CHECK_RC(cfb_symm_pull_reduce(reinterpret_cast<const float*>(mc_base),
                                    reinterpret_cast<const float* const*>(peer_base_dev), W, off,
                                    n, dst.data_ptr<float>(), static_cast<float>(scale), nullptr,
                                    0, 0, err.data_ptr<int>(), cur_stream()),
               "symm_pull_reduce");
}

void ex2_poly(const Tensor& x, Tensor& y) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && y.scalar_type() == at::kFloat &&
                  x.is_contiguous() && y.is_contiguous() && x.numel() == y.numel(),
              "ex2_poly: contiguous fp32 tensors of equal size");
  const c10::cuda::CUDAGuard guard(x.device());
  CFB_CHECK_RC(cfb_ex2_poly(x.data_ptr<float>(), y.data_ptr<float>(), x.numel(), cur_stream()),
               "ex2_poly");
}

// vocabulary-parallel cross entropy over symmetric per-row statistics (see cfb_ce_exchange)
void ce_exchange(int64_t peer_stats_dev, int64_t P, const Tensor& labels, Tensor& loss,
                 Tensor& lse, int64_t flags, int64_t ready_base, int64_t epoch,
                 int64_t peer_flags_dev, int64_t done_off, int64_t me, Tensor& counter,
                 Tensor& err) {
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "labels int64");
  const int64_t T = labels.numel();
  TORCH_CHECK(loss.scalar_type() == at::kFloat && lse.scalar_type() == at::kFloat &&
                  loss.numel() == T && lse.numel() == T,
              "loss / lse fp32 [T]");
  TORCH_CHECK(counter.scalar_type() == at::kInt && counter.numel() >= 1, "counter");
  check_status(err, "ce_exchange");
  const c10::cuda::CUDAGuard guard(labels.device());
  CFB_CHECK_RC(cfb_ce_exchange(reinterpret_cast<const float* const*>(peer_stats_dev), P, T,
                               reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()),
                               loss.data_ptr<float>(), lse.data_ptr<float>(),
                               reinterpret_cast<const uint32_t*>(flags), ready_base,
                               static_cast<uint32_t>(epoch),
                               reinterpret_cast<uint32_t* const*>(peer_flags_dev), done_off, me,
                               reinterpret_cast<uint32_t*>(counter.data_ptr<int>()),
                               err.data_ptr<int>(), cur_stream()),
               "ce_exchange");
}

// buf = 0 unless err[0] != 0 (a failed peer wait: a peer may still be reading buf)
void zero_unless_error(Tensor& buf, const Tensor& err) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kFloat && buf.is_contiguous(),
              "zero_unless_error: contiguous fp32 CUDA buffer");
  check_status(err, "zero_unless_error");
  const c10::cuda::CUDAGuard guard(buf.device());
  CFB_CHECK_RC(cfb_zero_unless_error(buf.data_ptr<float>(), buf.numel(), err.data_ptr<int>(),
                                     cur_stream()),
               "zero_unless_error");
}

// Dispatcher-visible attention ops on token-major rows, used by the graph rewriter's filtered
// attention node (centrifuge_b200._filter_C) for SDPA graphs of arbitrary models.
std::tuple<Tensor, Tensor> attn_fwd_rows(const Tensor& qkv, int64_t B, int64_t S, int64_t nh,
                                         int64_t nkv, int64_t hd, double scale) {
  Tensor out = at::empty({B * S, nh * hd}, qkv.options());
  Tensor lse = at::empty({B * S, nh}, qkv.options().dtype(at::kFloat));
  attn_fwd(qkv, out, lse, B, S, nh, nkv, hd, scale);
  return {out, lse};
}

Tensor attn_bwd_rows(const Tensor& qkv_k, const Tensor& qkv_full, const Tensor& o_k,
                     const Tensor& do_k, const Tensor& lse_k, const Tensor& pos_k, int64_t B,
                     int64_t S, int64_t Sk, int64_t nh, int64_t nkv, int64_t hd, double scale) {
  Tensor dqkv = at::empty_like(qkv_k);
  Tensor delta = at::empty({B * Sk * nh}, qkv_k.options().dtype(at::kFloat));
  Tensor o = o_k.contiguous(), d = do_k.contiguous();
  attn_bwd(qkv_k, qkv_full, o, d, lse_k, pos_k, dqkv, delta, B, S, Sk, nh, nkv, hd, scale,
           c10::nullopt);
  return dqkv;
}

}  // namespace

TORCH_LIBRARY(cfb, m) {
  m.def("attn_fwd_rows(Tensor qkv, int B, int S, int nh, int nkv, int hd, float scale) -> "
        "(Tensor, Tensor)");
  m.def("attn_bwd_rows(Tensor qkv_k, Tensor qkv_full, Tensor o_k, Tensor do_k, Tensor lse_k, "
        "Tensor pos_k, int B, int S, int Sk, int nh, int nkv, int hd, float scale) -> Tensor");
}

TORCH_LIBRARY_IMPL(cfb, CUDA, m) {
  m.impl("attn_fwd_rows", &attn_fwd_rows);
  m.impl("attn_bwd_rows", &attn_bwd_rows);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of centrifuge_b200";
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM", py::arg("a"), py::arg("b"), py::arg("out"),
        py::arg("a_mn"), py::arg("b_mn"), py::arg("epi"), py::arg("resid") = py::none(),
        py::arg("alpha") = 1.0, py::arg("bn") = 0, py::arg("max_ctas") = 0);
  m.def("gemm_error_word", &gemm_error_word, py::arg("device") = 0, py::arg("reset") = true);
  m.def("status_block", &status_block, "per-device status block of the kernels",
        py::arg("device") = 0);
  m.def("set_wait_limits", &set_wait_limits, py::arg("device"), py::arg("local_us"),
        py::arg("peer_us"));
  m.def("zero_unless_error", &zero_unless_error);
  m.def("gemm_swiglu", &gemm_swiglu, "gate/up projection with the SwiGLU epilogue");
  m.def("gemm_ce_part", &gemm_ce_part, "lm_head GEMM with cross-entropy statistics epilogue");
  m.def("gemm_ce_grad", &gemm_ce_grad, "lm_head recompute GEMM with the cross-entropy gradient");
  m.def("ce_combine", &ce_combine);
  m.def("gemm_plan", &gemm_plan, "tile / split-K choice of the GEMM planner (host only)");
  m.def("gemm_swiglu_bwd", &gemm_swiglu_bwd,
        "down-projection dgrad with the SwiGLU backward in the epilogue");
  m.def("gemm_tp", &gemm_tp, py::arg("a"), py::arg("b"), py::arg("out"), py::arg("b_mn"),
        py::arg("pos"), py::arg("table"), py::arg("rope_cols"), py::arg("hd"), py::arg("mode"),
        py::arg("rank"), py::arg("P"), py::arg("seg"), py::arg("epoch"),
        py::arg("peer_flags_dev"), py::arg("flag_ready"), py::arg("flag_done"),
        py::arg("tile_cnt"), py::arg("rot_rows"), py::arg("ag_mc"), py::arg("ag_peers_dev"),
        py::arg("mc_part"), py::arg("peer_part_dev"), py::arg("flag_blk"),
        py::arg("interleave_spb"), py::arg("resid"), py::arg("rs_out"),
        py::arg("bn") = 0);
  m.def("gemm_rope", &gemm_rope, "tcgen05 bf16 GEMM with RoPE fused into the epilogue",
        py::arg("a"), py::arg("b"), py::arg("out"), py::arg("pos"), py::arg("table"),
        py::arg("rope_cols"), py::arg("hd"), py::arg("bn") = 0);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("rope", &rope);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("gather_rows", &gather_rows);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("ce_exchange", &ce_exchange);
  m.def("ex2_poly", &ex2_poly);
  m.def("embedding_bwd", &embedding_bwd, py::arg("dy"), py::arg("ids"), py::arg("id_rows"),
        py::arg("dtable"), py::arg("deterministic") = true);
  m.def("ce_fwd", &ce_fwd);
  m.def("ce_bwd", &ce_bwd, py::arg("logits"), py::arg("rows"), py::arg("labels"),
        py::arg("lse"), py::arg("dloss"), py::arg("dlogits"), py::arg("vocab_start") = 0);
  m.def("ce_partial", &ce_partial);
  m.def("adamw", &adamw);
  m.def("adamw_multicast", &adamw_multicast);
  m.def("sumsq", &sumsq);
  m.def("clip_coef", &clip_coef);
  m.def("drop_smallest", &drop_smallest);
  m.def("keep_index", &keep_index);
  m.def("cast_f32_bf16", &cast_f32_bf16);
  m.def("scale_f32", &scale_f32);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_fwd_mma", &attn_fwd_mma);
  m.def("attn_bwd", &attn_bwd, py::arg("qkv_k"), py::arg("qkv_full"), py::arg("o_k"),
        py::arg("do_k"), py::arg("lse_k"), py::arg("pos_k"), py::arg("dqkv_k"), py::arg("delta"),
        py::arg("B"), py::arg("S"), py::arg("Sk"), py::arg("nh"), py::arg("nkv"), py::arg("hd"),
        py::arg("scale"), py::arg("rope_table") = py::none());
  m.def("attn_bwd_mma", &attn_bwd_mma);
  m.def("symm_signal", &symm_signal);
  m.def("symm_wait", &symm_wait);
  m.def("symm_pull_reduce", &symm_pull_reduce);
  m.attr("EPI_BF16") = static_cast<int>(kEpiBF16);
  m.attr("EPI_BF16_RESID") = static_cast<int>(kEpiBF16Resid);
  m.attr("EPI_F32") = static_cast<int>(kEpiF32);
  m.attr("EPI_F32_ACC") = static_cast<int>(kEpiF32Acc);
  m.attr("GEMM_TILE_PAIR") = static_cast<int>(kGemmTilePair);
}
