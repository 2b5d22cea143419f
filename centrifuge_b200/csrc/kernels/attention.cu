// Causal GQA attention forward and the filtered ("restore-Q") attention backward.
//
// Forward: O = softmax(scale * Q K^T + causal) V over the full sequence, with the per-row
// log-sum-exp saved for the backward.  GQA is native: query head h reads KV head
// h / (nh / nkv) directly from the fused qkv rows (no repeat_kv copy).
//
// Filtered backward (reference behaviour: grad_filter/token_filter/csrc/backward_filters.cpp:
// 420-505, ScaledDotProductFlashAttentionFilterRestoreQ, default RESTORE_Q build).  Given the
// kept query rows (compact, sorted by position) it computes the exact gradient of the kept
// queries' outputs with K/V of dropped positions treated as constants:
//   dK_j, dV_j  for kept keys j, summed over kept queries i with pos_j <= pos_i
//   dQ_i        for kept queries i, summed over ALL keys j <= pos_i (kept and dropped)
// The reference computes the second part with a second library backward over the dropped keys
// and a materialised -inf bias [B, h, S_keep, S_drop]; here it is one pass over the keys in
// original order with a position predicate, and no bias tensor.  Two kernels:
//   attn_bwd_dkdv  CTA = 64 kept keys of one KV head; loops over the head group's query heads
//                  and the kept query blocks (causal in compact index == causal in position)
//   attn_bwd_dq    CTA = 64 kept queries of one head; loops over key blocks of the full
//                  sequence up to the block's last position
// With every token kept (Sk == S) this is the ordinary dense attention backward.
//
// Tile math uses warp-level mma.sync m16n8k16 (bf16 in, fp32 accumulate) with ldmatrix
// from XOR-swizzled shared memory and cp.async double buffering.
#include "sm100_common.cuh"
#include "launch_api.h"

#include <math_constants.h>

namespace cfb {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of element (row, col) in a [rows][HD] bf16 tile with 16-byte chunks XOR-swizzled
// by (row & 7).  `col` must be a multiple of 8.
template <int HD>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return static_cast<uint32_t>(row * HD * 2 + ((((col >> 3) ^ (row & 7))) << 4));
}

// Copy `rows` rows x HD columns (starting at global row r0, column c0 of a row-major matrix
// with leading dimension ld) into a swizzled tile; rows >= row_end are zero-filled.
template <int HD, int ROWS, int THREADS>
__device__ __forceinline__ void load_tile(uint32_t tile, const __nv_bfloat16* g, long long ld,
                                          long long r0, int row_end_local, int c0) {
  constexpr int CHUNKS = ROWS * HD / 8;
#pragma unroll
  for (int i = threadIdx.x; i < CHUNKS; i += THREADS) {
    const int r = i / (HD / 8);
    const int c = (i % (HD / 8)) * 8;
    const bool valid = r < row_end_local;
    const __nv_bfloat16* src = g + (r0 + (valid ? r : 0)) * ld + c0 + c;
    cp_async16(tile + swz<HD>(r, c), src, valid);
  }
}

// ------------------------------------------------------------------------------ forward
template <int HD>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                       long long ld,
                                                       __nv_bfloat16* __restrict__ out,
                                                       long long ld_out, float* __restrict__ lse,
                                                       int S, int nh, int nkv, float scale) {
  constexpr int BM = 64, BN = 64;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + BM * HD * 2;
  const uint32_t sV0 = sK0 + 2 * BN * HD * 2;
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int g = h / (nh / nkv);
  const int q0 = qb * BM;
  const long long row0 = static_cast<long long>(b) * S;
  const int warp = warp_id(), lane = lane_id();
  const int gid = lane >> 2, tig = lane & 3;
  const int qcol = h * HD, kcol = nh * HD + g * HD, vcol = (nh + nkv) * HD + g * HD;
  const float sl2 = scale * kLog2e;

  load_tile<HD, BM, 128>(sQ, qkv, ld, row0 + q0, S - q0, qcol);
  const int last_q = min(S, q0 + BM) - 1;
  const int n_kb = last_q / BN + 1;
  load_tile<HD, BN, 128>(sK0, qkv, ld, row0, S, kcol);
  load_tile<HD, BN, 128>(sV0, qkv, ld, row0, S, vcol);
  cp_commit();

  uint32_t qf[HD / 16][4];
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-CUDART_INF_F, -CUDART_INF_F};
  float l_r[2] = {0.f, 0.f};
  const int qrow[2] = {q0 + warp * 16 + gid, q0 + warp * 16 + gid + 8};

  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) {
      const int nb = (kb + 1) & 1;
      const int k0n = (kb + 1) * BN;
      load_tile<HD, BN, 128>(sK0 + nb * BN * HD * 2, qkv, ld, row0 + k0n, S - k0n, kcol);
      load_tile<HD, BN, 128>(sV0 + nb * BN * HD * 2, qkv, ld, row0 + k0n, S - k0n, vcol);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kc = 0; kc < HD / 16; ++kc)
        ldsm4(sQ + swz<HD>(warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, kc * 16 + (lane >> 4) * 8),
              qf[kc]);
    }
    const uint32_t sK = sK0 + buf * BN * HD * 2;
    const uint32_t sV = sV0 + buf * BN * HD * 2;
    float s[BN / 8][4];
#pragma unroll
    for (int i = 0; i < BN / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kc = 0; kc < HD / 16; ++kc) {
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        uint32_t r[4];
        ldsm4(sK + swz<HD>(np * 16 + (lane & 7) + (lane >> 4) * 8, kc * 16 + ((lane >> 3) & 1) * 8), r);
        mma16816(s[2 * np], qf[kc], r[0], r[1]);
        mma16816(s[2 * np + 1], qf[kc], r[2], r[3]);
      }
    }
    const int k0 = kb * BN;
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int t = 0; t < BN / 8; ++t) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int key = k0 + t * 8 + 2 * tig + (c & 1);
        const int rr = c >> 1;
        float v = s[t][c] * sl2;
        if (key > qrow[rr] || key >= S) v = -CUDART_INF_F;
        s[t][c] = v;
        mx[rr] = fmaxf(mx[rr], v);
      }
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
    }
    float alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const float ref = (mx[rr] == -CUDART_INF_F) ? 0.f : mx[rr];
      alpha[rr] = exp2f(m_r[rr] - ref);
      m_r[rr] = mx[rr];
      mx[rr] = ref;
    }
#pragma unroll
    for (int t = 0; t < BN / 8; ++t) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float p = exp2f(s[t][c] - mx[c >> 1]);
        s[t][c] = p;
        rs[c >> 1] += p;
      }
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 1);
      rs[rr] += __shfl_xor_sync(0xffffffffu, rs[rr], 2);
      l_r[rr] = l_r[rr] * alpha[rr] + rs[rr];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
#pragma unroll
    for (int kc = 0; kc < BN / 16; ++kc) {
      uint32_t a[4];
      a[0] = pack_bf16x2(s[2 * kc][0], s[2 * kc][1]);
      a[1] = pack_bf16x2(s[2 * kc][2], s[2 * kc][3]);
      a[2] = pack_bf16x2(s[2 * kc + 1][0], s[2 * kc + 1][1]);
      a[3] = pack_bf16x2(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t r[4];
        ldsm4t(sV + swz<HD>(kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8), r);
        mma16816(o[2 * dp], a, r[0], r[1]);
        mma16816(o[2 * dp + 1], a, r[2], r[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int row = qrow[rr];
    if (row >= S) continue;
    const float inv = l_r[rr] > 0.f ? 1.f / l_r[rr] : 0.f;
    __nv_bfloat16* dst = out + (row0 + row) * ld_out + h * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      const int d = i * 8 + 2 * tig;
      *reinterpret_cast<uint32_t*>(dst + d) = pack_bf16x2(o[i][2 * rr] * inv, o[i][2 * rr + 1] * inv);
    }
    if (tig == 0) lse[(row0 + row) * nh + h] = (m_r[rr] + log2f(l_r[rr])) * kLn2;
  }
}

// ------------------------------------------------------------------------------ delta
// delta[r, h] = sum_d dO[r, h*hd + d] * O[r, h*hd + d]
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                  long long ld, float* __restrict__ delta, int rows, int nh, int hd) {
  const long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (t >= static_cast<long long>(rows) * nh) return;
  const long long r = t / nh;
  const int h = static_cast<int>(t % nh);
  const __nv_bfloat16* a = o + r * ld + h * hd;
  const __nv_bfloat16* bb = dout + r * ld + h * hd;
  float s = 0.f;
  for (int d = 0; d < hd; d += 8) {
    uint4 ua = *reinterpret_cast<const uint4*>(a + d);
    uint4 ub = *reinterpret_cast<const uint4*>(bb + d);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&ua);
    const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&ub);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = __bfloat1622float2(ha[i]);
      const float2 fb = __bfloat1622float2(hb[i]);
      s += fa.x * fb.x + fa.y * fb.y;
    }
  }
  delta[t] = s;
}

// ------------------------------------------------------------------------------ dK / dV
// Grid (ceil(Sk/64), nkv, B).  Compact kept layout: row b*Sk + j of qkv_k / do_k / lse_k.
template <int HD, int BQ>
__global__ void __launch_bounds__(128) attn_bwd_dkdv_kernel(
    const __nv_bfloat16* __restrict__ qkv_k, long long ld, const __nv_bfloat16* __restrict__ do_k,
    long long ld_o, const float* __restrict__ lse_k, const float* __restrict__ delta,
    __nv_bfloat16* __restrict__ dqkv_k, int Sk, int nh, int nkv, float scale) {
  constexpr int BK = 64;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BK * HD * 2;
  const uint32_t sQ0 = sV + BK * HD * 2;
  const uint32_t sO0 = sQ0 + 2 * BQ * HD * 2;
  float* sL = reinterpret_cast<float*>(smem + 2 * BK * HD * 2 + 4 * BQ * HD * 2);  // [2][BQ]
  float* sD = sL + 2 * BQ;                                                        // [2][BQ]

  const int kb = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int group = nh / nkv;
  const int j0 = kb * BK;
  const long long row0 = static_cast<long long>(b) * Sk;
  const int warp = warp_id(), lane = lane_id();
  const int gid = lane >> 2, tig = lane & 3;
  const int kcol = nh * HD + g * HD, vcol = (nh + nkv) * HD + g * HD;
  const float sl2 = scale * kLog2e;

  load_tile<HD, BK, 128>(sK, qkv_k, ld, row0 + j0, Sk - j0, kcol);
  load_tile<HD, BK, 128>(sV, qkv_k, ld, row0 + j0, Sk - j0, vcol);

  const int qb_first = j0 / BQ;
  const int n_qb = (Sk + BQ - 1) / BQ - qb_first;
  const int total = group * n_qb;

  auto issue = [&](int it, int buf) {
    const int hi = it / n_qb;
    const int h = g * group + hi;
    const int i0 = (qb_first + it % n_qb) * BQ;
    load_tile<HD, BQ, 128>(sQ0 + buf * BQ * HD * 2, qkv_k, ld, row0 + i0, Sk - i0, h * HD);
    load_tile<HD, BQ, 128>(sO0 + buf * BQ * HD * 2, do_k, ld_o, row0 + i0, Sk - i0, h * HD);
    for (int i = threadIdx.x; i < BQ; i += 128) {
      const bool v = i0 + i < Sk;
      sL[buf * BQ + i] = v ? lse_k[(row0 + i0 + i) * nh + h] * kLog2e : 0.f;
      sD[buf * BQ + i] = v ? delta[(row0 + i0 + i) * nh + h] : 0.f;
    }
  };

  float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) dk[i][c] = dv[i][c] = 0.f;

  if (total > 0) issue(0, 0);
  cp_commit();
  const int key_r[2] = {j0 + warp * 16 + gid, j0 + warp * 16 + gid + 8};

  for (int it = 0; it < total; ++it) {
    const int buf = it & 1;
    __syncthreads();  // previous iteration done with the buffer about to be refilled
    if (it + 1 < total) {
      issue(it + 1, buf ^ 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int i0 = (qb_first + it % n_qb) * BQ;
    const uint32_t sQ = sQ0 + buf * BQ * HD * 2;
    const uint32_t sO = sO0 + buf * BQ * HD * 2;
    const float* L = sL + buf * BQ;
    const float* Dl = sD + buf * BQ;

    float st[BQ / 8][4], dpt[BQ / 8][4];
#pragma unroll
    for (int i = 0; i < BQ / 8; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) st[i][c] = dpt[i][c] = 0.f;
#pragma unroll
    for (int kc = 0; kc < HD / 16; ++kc) {
      uint32_t ak[4], av[4];
      const int ar = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int ac = kc * 16 + (lane >> 4) * 8;
      ldsm4(sK + swz<HD>(ar, ac), ak);
      ldsm4(sV + swz<HD>(ar, ac), av);
#pragma unroll
      for (int np = 0; np < BQ / 16; ++np) {
        const int br = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int bc = kc * 16 + ((lane >> 3) & 1) * 8;
        uint32_t rq[4], ro[4];
        ldsm4(sQ + swz<HD>(br, bc), rq);
        ldsm4(sO + swz<HD>(br, bc), ro);
        mma16816(st[2 * np], ak, rq[0], rq[1]);
        mma16816(st[2 * np + 1], ak, rq[2], rq[3]);
        mma16816(dpt[2 * np], av, ro[0], ro[1]);
        mma16816(dpt[2 * np + 1], av, ro[2], ro[3]);
      }
    }
#pragma unroll
    for (int t = 0; t < BQ / 8; ++t) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int ql = t * 8 + 2 * tig + (c & 1);
        const int q = i0 + ql;
        const int key = key_r[c >> 1];
        const bool valid = (q < Sk) && (key < Sk) && (key <= q);
        const float p = valid ? exp2f(st[t][c] * sl2 - L[ql]) : 0.f;
        st[t][c] = p;
        dpt[t][c] = p * (dpt[t][c] - Dl[ql]);
      }
    }
#pragma unroll
    for (int kc = 0; kc < BQ / 16; ++kc) {
      uint32_t ap[4], as[4];
      ap[0] = pack_bf16x2(st[2 * kc][0], st[2 * kc][1]);
      ap[1] = pack_bf16x2(st[2 * kc][2], st[2 * kc][3]);
      ap[2] = pack_bf16x2(st[2 * kc + 1][0], st[2 * kc + 1][1]);
      ap[3] = pack_bf16x2(st[2 * kc + 1][2], st[2 * kc + 1][3]);
      as[0] = pack_bf16x2(dpt[2 * kc][0], dpt[2 * kc][1]);
      as[1] = pack_bf16x2(dpt[2 * kc][2], dpt[2 * kc][3]);
      as[2] = pack_bf16x2(dpt[2 * kc + 1][0], dpt[2 * kc + 1][1]);
      as[3] = pack_bf16x2(dpt[2 * kc + 1][2], dpt[2 * kc + 1][3]);
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        const int br = kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int bc = dp * 16 + (lane >> 4) * 8;
        uint32_t ro[4], rq[4];
        ldsm4t(sO + swz<HD>(br, bc), ro);
        ldsm4t(sQ + swz<HD>(br, bc), rq);
        mma16816(dv[2 * dp], ap, ro[0], ro[1]);
        mma16816(dv[2 * dp + 1], ap, ro[2], ro[3]);
        mma16816(dk[2 * dp], as, rq[0], rq[1]);
        mma16816(dk[2 * dp + 1], as, rq[2], rq[3]);
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int key = key_r[rr];
    if (key >= Sk) continue;
    __nv_bfloat16* dst = dqkv_k + (row0 + key) * ld;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      const int d = i * 8 + 2 * tig;
      *reinterpret_cast<uint32_t*>(dst + kcol + d) =
          pack_bf16x2(dk[i][2 * rr] * scale, dk[i][2 * rr + 1] * scale);
      *reinterpret_cast<uint32_t*>(dst + vcol + d) = pack_bf16x2(dv[i][2 * rr], dv[i][2 * rr + 1]);
    }
  }
}

// ------------------------------------------------------------------------------ dQ
// Grid (ceil(Sk/64), nh, B).  Keys come from the full-sequence qkv rows (original positions).
template <int HD>
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(
    const __nv_bfloat16* __restrict__ qkv_k, const __nv_bfloat16* __restrict__ qkv_full,
    long long ld, const __nv_bfloat16* __restrict__ do_k, long long ld_o,
    const float* __restrict__ lse_k, const float* __restrict__ delta,
    const int* __restrict__ pos_k, __nv_bfloat16* __restrict__ dqkv_k, int S, int Sk, int nh,
    int nkv, float scale) {
  constexpr int BM = 64, BN = 64;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sO = sQ + BM * HD * 2;
  const uint32_t sK0 = sO + BM * HD * 2;
  const uint32_t sV0 = sK0 + 2 * BN * HD * 2;
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int g = h / (nh / nkv);
  const int i0 = qb * BM;
  const long long rowk = static_cast<long long>(b) * Sk;
  const long long rowf = static_cast<long long>(b) * S;
  const int warp = warp_id(), lane = lane_id();
  const int gid = lane >> 2, tig = lane & 3;
  const int kcol = nh * HD + g * HD, vcol = (nh + nkv) * HD + g * HD;
  const float sl2 = scale * kLog2e;

  load_tile<HD, BM, 128>(sQ, qkv_k, ld, rowk + i0, Sk - i0, h * HD);
  load_tile<HD, BM, 128>(sO, do_k, ld_o, rowk + i0, Sk - i0, h * HD);
  const int last = min(Sk, i0 + BM) - 1;
  const int max_pos = pos_k[rowk + last];
  const int n_kb = min(max_pos, S - 1) / BN + 1;
  load_tile<HD, BN, 128>(sK0, qkv_full, ld, rowf, S, kcol);
  load_tile<HD, BN, 128>(sV0, qkv_full, ld, rowf, S, vcol);
  cp_commit();

  int qpos[2];
  float lq[2], dq_[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int i = i0 + warp * 16 + gid + rr * 8;
    const bool v = i < Sk;
    qpos[rr] = v ? pos_k[rowk + i] : -1;
    lq[rr] = v ? lse_k[(rowk + i) * nh + h] * kLog2e : 0.f;
    dq_[rr] = v ? delta[(rowk + i) * nh + h] : 0.f;
  }
  float dq[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;

  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) {
      const int nb = buf ^ 1;
      const int k0n = (kb + 1) * BN;
      load_tile<HD, BN, 128>(sK0 + nb * BN * HD * 2, qkv_full, ld, rowf + k0n, S - k0n, kcol);
      load_tile<HD, BN, 128>(sV0 + nb * BN * HD * 2, qkv_full, ld, rowf + k0n, S - k0n, vcol);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = sK0 + buf * BN * HD * 2;
    const uint32_t sV = sV0 + buf * BN * HD * 2;
    float s[BN / 8][4], dp[BN / 8][4];
#pragma unroll
    for (int i = 0; i < BN / 8; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[i][c] = dp[i][c] = 0.f;
#pragma unroll
    for (int kc = 0; kc < HD / 16; ++kc) {
      uint32_t aq[4], ao[4];
      const int ar = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
      const int ac = kc * 16 + (lane >> 4) * 8;
      ldsm4(sQ + swz<HD>(ar, ac), aq);
      ldsm4(sO + swz<HD>(ar, ac), ao);
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        const int br = np * 16 + (lane & 7) + (lane >> 4) * 8;
        const int bc = kc * 16 + ((lane >> 3) & 1) * 8;
        uint32_t rk[4], rv[4];
        ldsm4(sK + swz<HD>(br, bc), rk);
        ldsm4(sV + swz<HD>(br, bc), rv);
        mma16816(s[2 * np], aq, rk[0], rk[1]);
        mma16816(s[2 * np + 1], aq, rk[2], rk[3]);
        mma16816(dp[2 * np], ao, rv[0], rv[1]);
        mma16816(dp[2 * np + 1], ao, rv[2], rv[3]);
      }
    }
    const int k0 = kb * BN;
#pragma unroll
    for (int t = 0; t < BN / 8; ++t) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int key = k0 + t * 8 + 2 * tig + (c & 1);
        const int rr = c >> 1;
        const bool valid = key <= qpos[rr] && key < S;
        const float p = valid ? exp2f(s[t][c] * sl2 - lq[rr]) : 0.f;
        s[t][c] = p * (dp[t][c] - dq_[rr]);
      }
    }
#pragma unroll
    for (int kc = 0; kc < BN / 16; ++kc) {
      uint32_t a[4];
      a[0] = pack_bf16x2(s[2 * kc][0], s[2 * kc][1]);
      a[1] = pack_bf16x2(s[2 * kc][2], s[2 * kc][3]);
      a[2] = pack_bf16x2(s[2 * kc + 1][0], s[2 * kc + 1][1]);
      a[3] = pack_bf16x2(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
      for (int dpi = 0; dpi < HD / 16; ++dpi) {
        uint32_t r[4];
        ldsm4t(sK + swz<HD>(kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dpi * 16 + (lane >> 4) * 8), r);
        mma16816(dq[2 * dpi], a, r[0], r[1]);
        mma16816(dq[2 * dpi + 1], a, r[2], r[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int i = i0 + warp * 16 + gid + rr * 8;
    if (i >= Sk) continue;
    __nv_bfloat16* dst = dqkv_k + (rowk + i) * ld + h * HD;
#pragma unroll
    for (int k = 0; k < HD / 8; ++k) {
      const int d = k * 8 + 2 * tig;
      *reinterpret_cast<uint32_t*>(dst + d) =
          pack_bf16x2(dq[k][2 * rr] * scale, dq[k][2 * rr + 1] * scale);
    }
  }
}

template <int HD>
int fwd_launch(const void* qkv, long long ld, void* out, long long ld_out, float* lse, int B,
               int S, int nh, int nkv, float scale, cudaStream_t st) {
  const int smem = (64 * HD + 4 * 64 * HD) * 2;
  auto k = attn_fwd_kernel<HD>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid((S + 63) / 64, nh, B);
  k<<<grid, 128, smem, st>>>(static_cast<const __nv_bfloat16*>(qkv), ld,
                             static_cast<__nv_bfloat16*>(out), ld_out, lse, S, nh, nkv, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <int HD>
int bwd_launch(const void* qkv_k, long long ld, const void* qkv_full, const void* o_k,
               long long ld_o, const void* do_k, const float* lse_k, const int* pos_k,
               void* dqkv_k, float* delta, int B, int S, int Sk, int nh, int nkv, float scale,
               cudaStream_t st) {
  typedef __nv_bfloat16 bf;
  const long long rows = static_cast<long long>(B) * Sk;
  attn_delta_kernel<<<static_cast<int>((rows * nh + 255) / 256), 256, 0, st>>>(
      static_cast<const bf*>(o_k), static_cast<const bf*>(do_k), ld_o, delta,
      static_cast<int>(rows), nh, HD);
  constexpr int BQ = HD == 64 ? 64 : 32;
  const int smem_kv = 2 * 64 * HD * 2 + 4 * BQ * HD * 2 + 4 * BQ * 4;
  auto k1 = attn_bwd_dkdv_kernel<HD, BQ>;
  cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_kv);
  dim3 g1((Sk + 63) / 64, nkv, B);
  k1<<<g1, 128, smem_kv, st>>>(static_cast<const bf*>(qkv_k), ld, static_cast<const bf*>(do_k),
                               ld_o, lse_k, delta, static_cast<bf*>(dqkv_k), Sk, nh, nkv, scale);
  const int smem_q = (2 * 64 * HD + 4 * 64 * HD) * 2;
  auto k2 = attn_bwd_dq_kernel<HD>;
  cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_q);
  dim3 g2((Sk + 63) / 64, nh, B);
  k2<<<g2, 128, smem_q, st>>>(static_cast<const bf*>(qkv_k), static_cast<const bf*>(qkv_full), ld,
                              static_cast<const bf*>(do_k), ld_o, lse_k, delta, pos_k,
                              static_cast<bf*>(dqkv_k), S, Sk, nh, nkv, scale);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace attn
}  // namespace cfb

int cfb_attn_fwd(const void* qkv, long long ld_qkv, void* out, long long ld_out, float* lse,
                 int B, int S, int nh, int nkv, int hd, float scale, cudaStream_t st) {
  if (ld_qkv % 8 || ld_out % 8 || nh % nkv) return -11;
  if (hd == 64) return cfb::attn::fwd_launch<64>(qkv, ld_qkv, out, ld_out, lse, B, S, nh, nkv, scale, st);
  if (hd == 128) return cfb::attn::fwd_launch<128>(qkv, ld_qkv, out, ld_out, lse, B, S, nh, nkv, scale, st);
  return -12;
}

int cfb_attn_bwd(const void* qkv_k, long long ld_qkv, const void* qkv_full, const void* o_k,
                 long long ld_o, const void* do_k, const float* lse_k, const int* pos_k,
                 void* dqkv_k, float* /*dq_acc*/, float* delta, int B, int S, int Sk, int nh,
                 int nkv, int hd, float scale, cudaStream_t st) {
  if (ld_qkv % 8 || ld_o % 8 || nh % nkv || Sk <= 0) return -11;
  if (hd == 64)
    return cfb::attn::bwd_launch<64>(qkv_k, ld_qkv, qkv_full, o_k, ld_o, do_k, lse_k, pos_k,
                                     dqkv_k, delta, B, S, Sk, nh, nkv, scale, st);
  if (hd == 128)
    return cfb::attn::bwd_launch<128>(qkv_k, ld_qkv, qkv_full, o_k, ld_o, do_k, lse_k, pos_k,
                                      dqkv_k, delta, B, S, Sk, nh, nkv, scale, st);
  return -12;
}

int cfb_attn_delta(const void* o_k, const void* do_k, long long ld_o, float* delta, long long rows,
                   int nh, int hd, cudaStream_t st) {
  if (ld_o % 8 || hd % 8) return -11;
  cfb::attn::attn_delta_kernel<<<static_cast<int>((rows * nh + 255) / 256), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(o_k), static_cast<const __nv_bfloat16*>(do_k), ld_o,
      delta, static_cast<int>(rows), nh, hd);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
