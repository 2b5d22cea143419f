// Host-side launchers of the sm_100a kernels.  Plain C++ entry points over raw device
// pointers; the torch bindings (bindings.cpp) validate tensors and call these on the current
// stream.  Every launcher returns 0 on success and a negative code on a bad argument or a
// launch failure.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

enum {
  kEpiBF16 = 0,
  kEpiBF16Resid = 1,
  kEpiF32 = 2,
  kEpiF32Acc = 3,
  kEpiBF16Rope = 4,
  kEpiSwiGLU = 5,
  kEpiSwiGLUBwd = 6,  // dgrad of the down projection -> d[gate; up] (see cfb_gemm_swiglu_bwd)
  kEpiCEPart = 7,     // lm_head forward fused with cross-entropy statistics (cfb_gemm_ce_part)
  kEpiCEGrad = 8      // lm_head recompute fused with the cross-entropy gradient (cfb_gemm_ce_grad)
};
// `bn` value of cfb_gemm_bf16 that selects the 256 x 256 tile on a CTA pair (cta_group::2);
// 128 / 256 select a single-CTA tile of that width, 0 lets the planner choose
enum { kGemmTilePair = 512 };

// GEMM (gemm_sm100.cu): D = alpha * op(A) op(B) with the epilogue `epi`.
int cfb_gemm_bf16(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn,
                  void* D, long long ldd, int epi, const void* R, long long ldr, int M, int N,
                  int K, float alpha, int* err, int bn, int max_ctas, cudaStream_t st);
// Gate/up projection with SwiGLU in the epilogue: B = [gate; up] [2F, K] (K-major), both halves
// computed per tile (two TMEM accumulators); GU [M, 2F] receives [g | u] (kept for the
// backward), Hout [M, F] silu(g) * u.  F must be a multiple of 128.
int cfb_gemm_swiglu(const void* A, long long lda, const void* B, long long ldb, void* GU,
                    long long ld_gu, void* Hout, long long ld_h, int M, int F, int K, int* err,
                    cudaStream_t st);
// dgu[M, 2F] = SwiGLU backward of dh = dY[M, K] @ Wd[K, F] (Wd read MN-major: the down
// projection's weight [H, F] with K = H), computed in the GEMM epilogue: with g, u the saved
// gate / up of row gu_rows[m] (or m) of gu [*, 2F] (ld_gu), dgu[m, f] = dh * u * s * (1 + g (1 - s))
// and dgu[m, F + f] = dh * g * s, s = sigmoid(g).  dh itself is never stored.
int cfb_gemm_swiglu_bwd(const void* dY, long long ld_dy, const void* Wd, long long ld_w,
                        const void* gu, long long ld_gu, const int* gu_rows, void* dgu,
                        long long ld_dgu, int M, int F, int K, int* err, cudaStream_t st);

// Tensor-parallel fusion of a GEMM (A [M, K] K-major; B [N, K] K-major or, with b_mn, [K, N])
// with a collective over NVLink (gemm_sm100.cu), in one cooperative launch.  The M rows are
// split into per-rank segments seg[q]..seg[q+1] (device array [P + 1]; uniform
// sequence-parallel shards in the forward, each rank's kept rows in the filtered backward).
// Flags are symmetric buffers peer_flags[q] with ready[P] at flag_ready, done[P] at flag_done.
//   mode 1 (all-gather into A): this rank's segment of A is already in place; two extra warps
//     per CTA copy it to every other rank's A (multicast store through the NVSwitch, or peer
//     stores) and raise ready[rank] there, while the TMA producer reads other segments only
//     after their ready flag (own segment first).
//   mode 2 (reduce-scatter of D): D is this rank's partial buffer in symmetric memory; when an
//     m-block is stored, its owners get blk_ready[m][rank] = epoch (at flag_blk); two extra
//     warps per CTA of an owner reduce its segment block by block as soon as all ranks stored
//     the block (multimem.ld_reduce on mc_part, or loads from peer_part), add `resid` and write
//     `out` rows [0, count), zeros up to out_rows.  With interleave_spb > 0 (uniform segments of
//     that many 128-row blocks) the m-blocks run interleaved across owners.
struct CfbTpGemm {
  int mode;
  int rank, P;
  const int* seg;                 // device [P + 1]
  uint32_t epoch;
  uint32_t* const* peer_flags;    // device array [P] of flag buffers (symmetric memory)
  int flag_ready, flag_done;
  uint32_t* tile_cnt;             // local scratch [max(P, m-blocks) + 2], zero at rest
  int rot_rows;                   // mode 1: first row computed (multiple of 128)
  void* ag_mc;                    // mode 1: multicast address of A (or nullptr)
  void* const* ag_peers;          // mode 1: device array [P] of A on every rank
  const void* mc_part;            // mode 2: multicast address of D (or nullptr)
  const void* const* peer_part;   // mode 2: device array [P] of D on every rank
  int flag_blk;                   // mode 2: offset of blk_ready[num m-blocks][P]
  int interleave_spb;             // mode 2: > 0 for uniform segments (m-blocks per segment)
  const void* resid;              // mode 2: [count, N] bf16 (optional)
  long long ld_resid;
  void* out;                      // mode 2: [out_rows, N] bf16
  long long ld_out;
  int out_rows;
};
// The tile shape / split-K choice the GEMM entry points make for an M x N x K problem with
// epilogue `epi` and requested tile `bn` (0, 128, 256, kGemmTilePair) on `sms` SMs (host only;
// the planner that gemm_entry uses with the device's SM count, ignoring the ldd / environment
// conditions).
int cfb_gemm_plan(int M, int N, int K, int epi, int bn, int sms, int* out_bn, int* out_ksplit,
                  int* out_pair);

int cfb_gemm_tp(const void* A, long long lda, const void* B, long long ldb, int b_mn, void* D,
                long long ldd, int M, int N, int K, const int* pos, const float* cos_sin,
                int rope_cols, int head_dim, const CfbTpGemm* tp, int* err, int bn,
                cudaStream_t st);

// Forward projection with rotate-half RoPE fused into the epilogue: D = A B^T (both K-major) and
// columns [0, rope_cols) rotated per head of head_dim (64 or 128) at position pos[row], using the
// [max_pos, head_dim/2, 2] fp32 (cos, sin) table.
int cfb_gemm_bf16_rope(const void* A, long long lda, const void* B, long long ldb, void* D,
                       long long ldd, int M, int N, int K, const int* pos, const float* cos_sin,
                       int rope_cols, int head_dim, int* err, int bn, int max_ctas,
                       cudaStream_t st);

// Row ops (fused_ops.cu).
int cfb_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int rows, int H,
                    float eps, cudaStream_t st);
int cfb_rmsnorm_bwd(const void* dy, const void* x, const int* x_rows, const float* rstd,
                    const void* w, const void* dres, void* dx, float* dw_partial, float* dw_acc,
                    int rows, int H, int partial_rows, cudaStream_t st);
int cfb_rope(void* qkv, long long ld, const int* pos, const int* row_of, int rows, int n_heads,
             int head_dim, const float* cos_sin, int inverse, cudaStream_t st);
int cfb_swiglu_fwd(const void* gu, void* h, int rows, int F, cudaStream_t st);
int cfb_swiglu_bwd(const void* dh, const void* gu, const int* gu_rows, void* dgu, void* h_out,
                   int rows, int F, cudaStream_t st);
// Index checks: a row id outside [0, src_rows), a token id outside [0, V) or a label >= V
// records kErrBounds in `err` (the status block) and the access is skipped (gathered rows and
// embeddings are zero, the loss is 0).
int cfb_gather_rows(const void* src, long long ld_src, long long src_rows, const int* idx,
                    void* dst, long long ld_dst, int rows, int row_bytes, int* err,
                    cudaStream_t st);
int cfb_embedding_fwd(const void* table, long long V, const long long* ids, void* out, int rows,
                      int H, int* err, cudaStream_t st);
int cfb_embedding_bwd(const void* dy, const long long* ids, const int* id_rows, float* dtable,
                      long long V, int rows, int H, int* err, cudaStream_t st);
// Deterministic embedding gradient: cfb_row_tokens gathers each dy row's token (-1 for a row
// id outside ids), the caller sorts them stably, cfb_embedding_bwd_sorted sums every run of
// equal tokens in row order into its table row (no atomics).
int cfb_row_tokens(const long long* ids, long long n_ids, const int* id_rows, long long* tok,
                   int rows, int* err, cudaStream_t st);
int cfb_embedding_bwd_sorted(const void* dy, const long long* sorted_tok,
                             const long long* order, float* dtable, long long V, int rows, int H,
                             int* err, cudaStream_t st);
int cfb_ce_fwd(const void* logits, long long ld, const long long* labels, float* loss,
               float* lse, int rows, int V, int* err, cudaStream_t st);
int cfb_ce_bwd(const void* logits, long long ld, const int* logit_rows, const long long* labels,
               const float* lse, const float* dloss, void* dlogits, long long ld_out, int rows,
               int V, long long vocab_start, cudaStream_t st);
int cfb_ce_partial(const void* logits, long long ld, const long long* labels, float* pmax,
                   float* psum, float* ptgt, int rows, int V, long long vocab_start,
                   cudaStream_t st);
int cfb_adamw(float* master, const float* grad, float* m, float* v, void* param_bf16, long long n,
              float lr, float beta1, float beta2, float eps, float wd, float bc1, float bc2,
              const float* grad_scale, cudaStream_t st);
// AdamW whose bf16 output goes to the NVSwitch multicast address `param_mc` of the parameter
// buffer shared by the data-parallel group (every rank receives the updated shard).
int cfb_adamw_multicast(float* master, const float* grad, float* m, float* v, void* param_mc,
                        long long n, float lr, float beta1, float beta2, float eps, float wd,
                        float bc1, float bc2, const float* grad_scale, cudaStream_t st);
int cfb_sumsq(const float* x, long long n, float* out_partial, int nblocks, cudaStream_t st);
// coef = min(1, max_norm / norm) * extra_scale; when status[0] != 0 (a wait of this step gave
// up) coef = -1, which makes the AdamW kernels skip the update.
int cfb_clip_coef(const float* partials, int n, float max_norm, float extra_scale, float* coef,
                  float* norm_out, const int* status, cudaStream_t st);
int cfb_drop_smallest(const float* score, long long ld, int* mask_i32, long long* mask_i64,
                      long long ld_mask, int rows, int start, int end, int k, cudaStream_t st);
int cfb_keep_index(const long long* mask, int B, int S, int S_keep, int* pos, int* flat_rows,
                   int* err, cudaStream_t st);
int cfb_cast_f32_bf16(const float* x, void* y, long long n, cudaStream_t st);
int cfb_scale_f32(float* x, long long n, float s, cudaStream_t st);

// Attention (attention_fwd.cu / attention_bwd.cu).  Token-major layouts:
//   q/k/v rows of the fused [T, ld] qkv buffer, heads at column offsets.
int cfb_attn_fwd(const void* qkv, long long ld_qkv, void* out, long long ld_out, float* lse,
                 int B, int S, int nh, int nkv, int hd, float scale, cudaStream_t st);
// tcgen05/TMEM forward (attention_sm100.cu); `err` receives a code if a bounded wait gives up.
// Persistent kernel scheduled through `work` (two device int32 words, zero before the first
// launch; the kernel leaves them zero).  Launches sharing one `work` pair must be ordered.
int cfb_attn_fwd_tc(const void* qkv, long long ld_qkv, void* out, long long ld_out, float* lse,
                    int B, int S, int nh, int nkv, int hd, float scale, int* work, int* err,
                    cudaStream_t st);
int cfb_attn_bwd(const void* qkv_k, long long ld_qkv, const void* qkv_full, const void* o_k,
                 long long ld_o, const void* do_k, const float* lse_k, const int* pos_k,
                 void* dqkv_k, float* unused, float* delta, int B, int S, int Sk, int nh,
                 int nkv, int hd, float scale, cudaStream_t st);

// delta[r, h] = <O[r, h, :], dO[r, h, :]> over the kept rows (attention backward prologue).
int cfb_attn_delta(const void* o_k, const void* do_k, long long ld_o, float* delta, long long rows,
                   int nh, int hd, cudaStream_t st);
// tcgen05/TMEM filtered backward (attention_bwd_sm100.cu): dK/dV of the kept keys and dQ of the
// kept queries over all keys by position; `delta` must be computed first.  `rope_cs` (optional,
// [max_pos, hd/2, 2] fp32 cos/sin) folds the RoPE backward of dQ and dK into the epilogue.  Persistent kernel
// scheduled through `work` (two device int32 words, zero before the first launch; the kernel
// leaves them zero).  Launches sharing one `work` pair must be ordered (one stream).
int cfb_attn_bwd_tc(const void* qkv_k, long long ld_qkv, const void* qkv_full, const void* do_k,
                    long long ld_o, const float* lse_k, const float* delta, const int* pos_k,
                    void* dqkv_k, int B, int S, int Sk, int nh, int nkv, int hd, float scale,
                    const float* rope_cs, int* work, int* err, cudaStream_t st);

// lm_head GEMM fused with cross entropy (gemm_sm100.cu, CTA-pair tiles of 256 x 256).
// Forward: logits = X W^T (X [M, K], W [N, K], both K-major) are never stored; for every row r
// and 256-column tile t the epilogue writes pmax[r * nt + t] = max of the tile's fp32 logits,
// psum[r * nt + t] = sum of exp(logit - pmax) over them, and ptgt[r] = the logit of column
// labels[r] (written by the tile that holds it; rows with labels[r] < 0 get nothing).
// nt = ceil(N / 256).  cfb_ce_combine then gives lse and the per-token loss.
int cfb_gemm_ce_part(const void* X, long long ldx, const void* W, long long ldw, int M, int N,
                     int K, const long long* labels, float* pmax, float* psum, float* ptgt,
                     int* err, cudaStream_t st);
// Backward: logits of the M rows of X recomputed in the GEMM, the epilogue stores
// dlogits[r, c] = (exp(logit - lse[r]) - [c == labels[r]]) * dloss[r] (bf16, ld ldd; zero rows
// for labels[r] < 0).
int cfb_gemm_ce_grad(const void* X, long long ldx, const void* W, long long ldw, void* dlogits,
                     long long ldd, int M, int N, int K, const long long* labels,
                     const float* lse, const float* dloss, int* err, cudaStream_t st);
// lse[r] = M + log(sum_t psum[r, t] exp(pmax[r, t] - M)), M = max_t pmax[r, t];
// loss[r] = lse[r] - ptgt[r] for labels[r] >= 0, else 0.
int cfb_ce_combine(const float* pmax, const float* psum, const float* ptgt, int rows, int nt,
                   const long long* labels, long long V, float* loss, float* lse, int* err,
                   cudaStream_t st);

// NVLink peer-memory gradient reduction (comm_sm100.cu).
int cfb_symm_signal(uint32_t* const* peer_flags_dev, int W, int off, uint32_t epoch,
                    cudaStream_t st);
// Vocabulary-parallel cross entropy: combine the P ranks' per-row (max, sum exp, label logit)
// statistics (symmetric buffers [3][T], peer_stats device array [P]) into loss / lse after a
// bounded wait on ready[ready_base + q] >= epoch; then raise done[done_off + me] = epoch at every
// rank.  `counter` is a device word, zero at rest.
int cfb_ce_exchange(const float* const* peer_stats, int P, int T, const long long* labels,
                    float* loss, float* lse, const uint32_t* flags, int ready_base,
                    uint32_t epoch, uint32_t* const* peer_flags, int done_off, int me,
                    uint32_t* counter, int* err, cudaStream_t st);
// The attention forward's software base-2 exponential, element-wise (accuracy tests).
int cfb_ex2_poly(const float* x, float* y, int n, cudaStream_t st);
int cfb_symm_wait(const uint32_t* flags, int base, int stride, int n, uint32_t epoch, int* err,
                  cudaStream_t st);
int cfb_symm_pull_reduce(const float* mc_base, const float* const* peer_base_dev, int W,
                         long long off, long long n, float* dst, float scale,
                         const uint32_t* flags, int bucket, uint32_t epoch, int* err,
                         cudaStream_t st);
// buf[0, n) = 0 unless err[0] != 0 (buf 16-byte aligned)
int cfb_zero_unless_error(float* buf, long long n, const int* err, cudaStream_t st);
