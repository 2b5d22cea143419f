// Filtered ("restore-Q") causal GQA attention backward on the 5th-generation tensor cores.
//
// Inputs are the kept query/key rows in compact order (row b*Sk + j of qkv_k / do_k / lse_k /
// delta, sorted by position) and the full-sequence qkv rows for the dropped keys.  Two kernels:
//
// dK/dV (grid: 128 kept keys x KV head x batch).  The CTA keeps K_kv, V_kv (128 keys) in shared
// memory and loops over (query head of the group) x (64-query blocks from the first one that can
// see its keys).  Per block:  S^T = K Q^T and dP^T = V dO^T (M = 128 keys, N = 64 queries) into
// double-buffered TMEM tiles;  softmax warps form P^T = 2^(S^T c - lse) and
// dS^T = P^T (dP^T - delta) (bf16, 128B-swizzled in shared memory);  dV += P^T dO and
// dK += dS^T Q accumulate in TMEM over all blocks and heads of the group (native GQA: no
// per-head dK/dV and no reduction pass).  Causality in compact index == causality in position.
//
// dQ (grid: 128 kept queries x query head x batch).  The CTA keeps Q, dO in shared memory and
// walks 64-key blocks of the FULL sequence up to its last query's position: S = Q K^T,
// dP = dO V^T, dS = P (dP - delta) with the position predicate key_pos <= query_pos, and
// dQ += dS K in TMEM.  Dropped keys therefore contribute to dQ exactly as in the reference's
// second (restore-Q) backward, in one pass and without a bias tensor.
//
// Roles: warp 0 TMA, warp 1 MMA issue (single thread), warps 2-9 softmax (two warps per TMEM
// lane quadrant, each taking half of the 64 columns; no cross-warp exchange is needed since P
// uses the saved log-sum-exp).  All waits are bounded (sm100_common.cuh).
#include "sm100_common.cuh"
#include "launch_api.h"

#include <math_constants.h>

namespace cfb {
namespace attn_bwd_tc {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int BR = 128;  // rows owned by the CTA (keys for dK/dV, queries for dQ)
constexpr int BC = 64;   // columns per step (queries for dK/dV, keys for dQ)
constexpr int STAGES = 2;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

template <int HD>
struct Smem {
  static constexpr int CH_R = BR * 128;  // chunk of a 128-row tile (64 bf16 per row)
  static constexpr int CH_C = BC * 128;  // chunk of a 64-row tile
  static constexpr int ROW_TILE = (HD / 64) * CH_R;  // [128 x HD]
  static constexpr int COL_TILE = (HD / 64) * CH_C;  // [64 x HD]
  static constexpr int OFF_A = 0;                       // K (dK/dV) or Q (dQ)
  static constexpr int OFF_B = OFF_A + ROW_TILE;        // V (dK/dV) or dO (dQ)
  static constexpr int OFF_ST = OFF_B + ROW_TILE;       // stages of [Q_i, dO_i] / [K_j, V_j]
  static constexpr int STAGE = 2 * COL_TILE;
  static constexpr int OFF_P = OFF_ST + STAGES * STAGE; // P^T (dK/dV only), [128 x 64] bf16
  static constexpr int OFF_DS = OFF_P + CH_R;           // dS^T / dS, [128 x 64] bf16
  static constexpr int OFF_BAR = OFF_DS + CH_R;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
  // requested dynamic shared memory: at least 120 KB so that one CTA runs per SM (each CTA
  // allocates all 512 TMEM columns)
  static constexpr int LAUNCH_BYTES = BYTES < 120 * 1024 ? 120 * 1024 : BYTES;
};

struct Params {
  int S, Sk, nh, nkv;
  float scale_log2;  // softmax scale * log2(e)
  float scale;       // softmax scale (dS -> dQ / dK)
  const float* lse_k;  // [B*Sk, nh] natural-log LSE of kept queries
  const float* delta;  // [B*Sk, nh]
  const int* pos_k;    // [B*Sk] positions of kept rows
  __nv_bfloat16* dqkv; // [B*Sk, ld] output rows (compact)
  long long ld;
  int* err;
};

struct Bars {
  uint64_t a_full, st_full[STAGES], st_empty[STAGES], s_full[2], s_free[2], p_ready, mm_done,
      drain;
  uint32_t tmem_slot;
  int abort;
};

__device__ __forceinline__ void init_bars(Bars* b) {
  mbar_init(smem_u32(&b->a_full), 1);
  for (int s = 0; s < STAGES; ++s) {
    mbar_init(smem_u32(&b->st_full[s]), 1);
    mbar_init(smem_u32(&b->st_empty[s]), 1);
  }
  for (int s = 0; s < 2; ++s) {
    mbar_init(smem_u32(&b->s_full[s]), 1);
    mbar_init(smem_u32(&b->s_free[s]), 8);
  }
  mbar_init(smem_u32(&b->p_ready), 8);
  mbar_init(smem_u32(&b->mm_done), 1);
  mbar_init(smem_u32(&b->drain), 1);
  b->abort = 0;
  fence_mbar_init();
}

// Two 64-column score tiles (S, dP) per buffer: S at sb*64, dP at 128 + sb*64; accumulators
// from column 256.
constexpr uint32_t kColS = 0, kColDP = 128, kColAcc = 256;

// Thread's 32 columns of a 64-column bf16 row tile in 128B-swizzled K-major layout.
__device__ __forceinline__ void write_row_half(uint32_t tile, int r, int half, const uint32_t* pk) {
  const uint32_t rowbase = tile + r * 128;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int piece = half * 4 + i;
    st_shared_v4(rowbase + ((piece ^ (r & 7)) << 4), pk[4 * i], pk[4 * i + 1], pk[4 * i + 2],
                 pk[4 * i + 3]);
  }
}

// ======================================================================== dK / dV
template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dkdv_tc(const __grid_constant__ CUtensorMap tmR,  // qkv_k, box 64 x 128 rows
                     const __grid_constant__ CUtensorMap tmQ,  // qkv_k, box 64 x 64 rows
                     const __grid_constant__ CUtensorMap tmO,  // do_k,  box 64 x 64 rows
                     Params p) {
  using L = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  Bars* bar = reinterpret_cast<Bars*>(smem + L::OFF_BAR);
  volatile int* abort_flag = &bar->abort;
  const int warp = warp_id(), lane = lane_id();
  const int kb = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int group = p.nh / p.nkv;
  const int j0 = kb * BR;          // first compact key of the CTA
  const int row0 = b * p.Sk;       // compact row base of this sequence
  const int qb_first = j0 / BC;
  const int nqb = (p.Sk + BC - 1) / BC - qb_first;
  const int n_it = group * nqb;
  const int kcol = (p.nh + g) * HD, vcol = (p.nh + p.nkv + g) * HD;

  if (threadIdx.x == 0) init_bars(bar);
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmR);
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bar->tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_slot;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(smem_u32(&bar->a_full), 2 * L::ROW_TILE);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        tma_load_2d(sbase + L::OFF_A + c * L::CH_R, &tmR, smem_u32(&bar->a_full), kcol + c * 64, row0 + j0);
        tma_load_2d(sbase + L::OFF_B + c * L::CH_R, &tmR, smem_u32(&bar->a_full), vcol + c * 64, row0 + j0);
      }
      int issued = 0;
      for (int it = 0; it < n_it; ++it, ++issued) {
        const int st = it % STAGES;
        if (!mbar_wait(smem_u32(&bar->st_empty[st]), ((it / STAGES) & 1) ^ 1, abort_flag, p.err,
                       kErrWaitProducer))
          break;
        const int h = g * group + it / nqb;
        const int i0 = (qb_first + it % nqb) * BC;
        const uint32_t fb = smem_u32(&bar->st_full[st]);
        mbar_arrive_expect_tx(fb, L::STAGE);
        const uint32_t sq = sbase + L::OFF_ST + st * L::STAGE;
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d(sq + c * L::CH_C, &tmQ, fb, h * HD + c * 64, row0 + i0);
          tma_load_2d(sq + L::COL_TILE + c * L::CH_C, &tmO, fb, h * HD + c * 64, row0 + i0);
        }
      }
      tma_drain_ring(bar->st_full, STAGES, issued);
      tma_drain_ring(&bar->a_full, 1, 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16_f32(BR, BC, false, false);
      constexpr uint32_t ID_ACC = idesc_bf16_f32(BR, HD, false, true);
      bool ok = mbar_wait(smem_u32(&bar->a_full), 0, abort_flag, p.err, kErrWaitMma);
      auto scores = [&](int it) -> bool {
        const int st = it % STAGES, sb = it & 1;
        if (!mbar_wait(smem_u32(&bar->st_full[st]), (it / STAGES) & 1, abort_flag, p.err, kErrWaitMma))
          return false;
        const int use = it >> 1;
        if (use > 0 &&
            !mbar_wait(smem_u32(&bar->s_free[sb]), (use - 1) & 1, abort_flag, p.err, kErrWaitMma))
          return false;
        tc_fence_after();
        const uint32_t sq = sbase + L::OFF_ST + st * L::STAGE;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t oa = (kk >> 2) * L::CH_R + (kk & 3) * 32;
          const uint32_t ob = (kk >> 2) * L::CH_C + (kk & 3) * 32;
          // S^T = K Q^T ; dP^T = V dO^T
          umma_bf16_ss(tmem + kColS + sb * BC, sdesc_sw128(sbase + L::OFF_A + oa, 16, 1024),
                       sdesc_sw128(sq + ob, 16, 1024), ID_S, kk > 0);
          umma_bf16_ss(tmem + kColDP + sb * BC, sdesc_sw128(sbase + L::OFF_B + oa, 16, 1024),
                       sdesc_sw128(sq + L::COL_TILE + ob, 16, 1024), ID_S, kk > 0);
        }
        umma_commit(smem_u32(&bar->s_full[sb]));
        return true;
      };
      auto accumulate = [&](int it) -> bool {
        if (!mbar_wait(smem_u32(&bar->p_ready), it & 1, abort_flag, p.err, kErrWaitMma)) return false;
        tc_fence_after();
        const int st = it % STAGES;
        const uint32_t sq = sbase + L::OFF_ST + st * L::STAGE;
#pragma unroll
        for (int kk = 0; kk < BC / 16; ++kk) {
          // dV += P^T dO ; dK += dS^T Q   (B operands read MN-major: rows = queries)
          umma_bf16_ss(tmem + kColAcc + HD, sdesc_sw128(sbase + L::OFF_P + kk * 32, 16, 1024),
                       sdesc_sw128(sq + L::COL_TILE + kk * 2048, L::CH_C, 1024), ID_ACC,
                       (it > 0 || kk > 0) ? 1u : 0u);
          umma_bf16_ss(tmem + kColAcc, sdesc_sw128(sbase + L::OFF_DS + kk * 32, 16, 1024),
                       sdesc_sw128(sq + kk * 2048, L::CH_C, 1024), ID_ACC,
                       (it > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(smem_u32(&bar->mm_done));
        umma_commit(smem_u32(&bar->st_empty[st]));
        return true;
      };
      if (ok && n_it > 0) ok = scores(0);
      for (int it = 0; it < n_it && ok; ++it) {
        if (it + 1 < n_it && !scores(it + 1)) break;
        if (!accumulate(it)) break;
      }
      umma_commit(smem_u32(&bar->drain));
      volatile int dummy = 0;
      mbar_wait(smem_u32(&bar->drain), 0, &dummy, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax warps 2..9
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;  // key row of the tile
    const int kc = j0 + r;           // compact key index
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      const int sb = it & 1;
      const int h = g * group + it / nqb;
      const int i0 = (qb_first + it % nqb) * BC + half * 32;  // this thread's first query
      if (!mbar_wait(smem_u32(&bar->s_full[sb]), (it >> 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[32], dp[32];
      CFB_TMEM_LD32(lane_addr + kColS + sb * BC + half * 32, s);
      CFB_TMEM_LD32(lane_addr + kColDP + sb * BC + half * 32, dp);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar->s_free[sb]));
      // column k of this thread's 32 is query i0 + k; lane k of the warp holds its statistics
      const int q_lane = min(i0 + lane, p.Sk - 1);
      const long long qr = static_cast<long long>(row0 + q_lane) * p.nh + h;
      const float l2_lane = __ldg(p.lse_k + qr) * kLog2e;
      const float dl_lane = __ldg(p.delta + qr);
      const int lo = kc - i0, hi = p.Sk - i0;  // query column k is visible iff lo <= k < hi
      uint32_t pp[16], pd[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float pv[2], dv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int k = 2 * i + e;
          const float l2 = __shfl_sync(0xffffffffu, l2_lane, k);
          const float dl = __shfl_sync(0xffffffffu, dl_lane, k);
          const float pe = (k >= lo && k < hi)
                               ? ex2_approx(fmaf(__uint_as_float(s[k]), p.scale_log2, -l2))
                               : 0.f;
          pv[e] = pe;
          dv[e] = pe * (__uint_as_float(dp[k]) - dl);
        }
        pp[i] = pack_bf16x2(pv[0], pv[1]);
        pd[i] = pack_bf16x2(dv[0], dv[1]);
      }
      // the previous block's dV/dK MMAs read P^T / dS^T: wait before overwriting
      if (it > 0 &&
          !mbar_wait(smem_u32(&bar->mm_done), (it - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      write_row_half(sbase + L::OFF_P, r, half, pp);
      write_row_half(sbase + L::OFF_DS, r, half, pd);
      fence_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar->p_ready));
    }
    if (ok && n_it > 0 &&
        mbar_wait(smem_u32(&bar->mm_done), (n_it - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
      tc_fence_after();
      constexpr int OH = HD / 2;
      __nv_bfloat16* drow = p.dqkv + static_cast<long long>(row0 + kc) * p.ld;
#pragma unroll
      for (int cc = 0; cc < OH / 32; ++cc) {
        uint32_t dk[32], dv[32];
        CFB_TMEM_LD32(lane_addr + kColAcc + half * OH + cc * 32, dk);
        CFB_TMEM_LD32(lane_addr + kColAcc + HD + half * OH + cc * 32, dv);
        tmem_ld_wait();
        if (kc < p.Sk) {
          uint4* k4 = reinterpret_cast<uint4*>(drow + kcol + half * OH + cc * 32);
          uint4* v4 = reinterpret_cast<uint4*>(drow + vcol + half * OH + cc * 32);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint4 a, c;
            a.x = pack_bf16x2(__uint_as_float(dk[8 * k + 0]) * p.scale, __uint_as_float(dk[8 * k + 1]) * p.scale);
            a.y = pack_bf16x2(__uint_as_float(dk[8 * k + 2]) * p.scale, __uint_as_float(dk[8 * k + 3]) * p.scale);
            a.z = pack_bf16x2(__uint_as_float(dk[8 * k + 4]) * p.scale, __uint_as_float(dk[8 * k + 5]) * p.scale);
            a.w = pack_bf16x2(__uint_as_float(dk[8 * k + 6]) * p.scale, __uint_as_float(dk[8 * k + 7]) * p.scale);
            c.x = pack_bf16x2(__uint_as_float(dv[8 * k + 0]), __uint_as_float(dv[8 * k + 1]));
            c.y = pack_bf16x2(__uint_as_float(dv[8 * k + 2]), __uint_as_float(dv[8 * k + 3]));
            c.z = pack_bf16x2(__uint_as_float(dv[8 * k + 4]), __uint_as_float(dv[8 * k + 5]));
            c.w = pack_bf16x2(__uint_as_float(dv[8 * k + 6]), __uint_as_float(dv[8 * k + 7]));
            k4[k] = a;
            v4[k] = c;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ======================================================================== dQ
template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dq_tc(const __grid_constant__ CUtensorMap tmQk,  // qkv_k, box 64 x 128 rows
                   const __grid_constant__ CUtensorMap tmOk,  // do_k,  box 64 x 128 rows
                   const __grid_constant__ CUtensorMap tmF,   // qkv full, box 64 x 64 rows
                   Params p) {
  using L = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  Bars* bar = reinterpret_cast<Bars*>(smem + L::OFF_BAR);
  volatile int* abort_flag = &bar->abort;
  const int warp = warp_id(), lane = lane_id();
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.nh / p.nkv);
  const int i0 = qb * BR;
  const int rowk = b * p.Sk, rowf = b * p.S;
  const int last = min(p.Sk, i0 + BR) - 1;
  const int max_pos = min(p.pos_k[rowk + last], p.S - 1);
  const int nkb = max_pos / BC + 1;
  const int kcol = (p.nh + g) * HD, vcol = (p.nh + p.nkv + g) * HD;

  if (threadIdx.x == 0) init_bars(bar);
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQk);
    tma_prefetch_desc(&tmOk);
    tma_prefetch_desc(&tmF);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bar->tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_slot;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(smem_u32(&bar->a_full), 2 * L::ROW_TILE);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        tma_load_2d(sbase + L::OFF_A + c * L::CH_R, &tmQk, smem_u32(&bar->a_full), h * HD + c * 64, rowk + i0);
        tma_load_2d(sbase + L::OFF_B + c * L::CH_R, &tmOk, smem_u32(&bar->a_full), h * HD + c * 64, rowk + i0);
      }
      int issued = 0;
      for (int j = 0; j < nkb; ++j, ++issued) {
        const int st = j % STAGES;
        if (!mbar_wait(smem_u32(&bar->st_empty[st]), ((j / STAGES) & 1) ^ 1, abort_flag, p.err,
                       kErrWaitProducer))
          break;
        const uint32_t fb = smem_u32(&bar->st_full[st]);
        mbar_arrive_expect_tx(fb, L::STAGE);
        const uint32_t sk = sbase + L::OFF_ST + st * L::STAGE;
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d(sk + c * L::CH_C, &tmF, fb, kcol + c * 64, rowf + j * BC);
          tma_load_2d(sk + L::COL_TILE + c * L::CH_C, &tmF, fb, vcol + c * 64, rowf + j * BC);
        }
      }
      tma_drain_ring(bar->st_full, STAGES, issued);
      tma_drain_ring(&bar->a_full, 1, 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16_f32(BR, BC, false, false);
      constexpr uint32_t ID_ACC = idesc_bf16_f32(BR, HD, false, true);
      bool ok = mbar_wait(smem_u32(&bar->a_full), 0, abort_flag, p.err, kErrWaitMma);
      auto scores = [&](int j) -> bool {
        const int st = j % STAGES, sb = j & 1;
        if (!mbar_wait(smem_u32(&bar->st_full[st]), (j / STAGES) & 1, abort_flag, p.err, kErrWaitMma))
          return false;
        const int use = j >> 1;
        if (use > 0 &&
            !mbar_wait(smem_u32(&bar->s_free[sb]), (use - 1) & 1, abort_flag, p.err, kErrWaitMma))
          return false;
        tc_fence_after();
        const uint32_t sk = sbase + L::OFF_ST + st * L::STAGE;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t oa = (kk >> 2) * L::CH_R + (kk & 3) * 32;
          const uint32_t ob = (kk >> 2) * L::CH_C + (kk & 3) * 32;
          // S = Q K^T ; dP = dO V^T
          umma_bf16_ss(tmem + kColS + sb * BC, sdesc_sw128(sbase + L::OFF_A + oa, 16, 1024),
                       sdesc_sw128(sk + ob, 16, 1024), ID_S, kk > 0);
          umma_bf16_ss(tmem + kColDP + sb * BC, sdesc_sw128(sbase + L::OFF_B + oa, 16, 1024),
                       sdesc_sw128(sk + L::COL_TILE + ob, 16, 1024), ID_S, kk > 0);
        }
        umma_commit(smem_u32(&bar->s_full[sb]));
        return true;
      };
      auto accumulate = [&](int j) -> bool {
        if (!mbar_wait(smem_u32(&bar->p_ready), j & 1, abort_flag, p.err, kErrWaitMma)) return false;
        tc_fence_after();
        const int st = j % STAGES;
        const uint32_t sk = sbase + L::OFF_ST + st * L::STAGE;
#pragma unroll
        for (int kk = 0; kk < BC / 16; ++kk)  // dQ += dS K   (K read MN-major: rows = keys)
          umma_bf16_ss(tmem + kColAcc, sdesc_sw128(sbase + L::OFF_DS + kk * 32, 16, 1024),
                       sdesc_sw128(sk + kk * 2048, L::CH_C, 1024), ID_ACC,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(smem_u32(&bar->mm_done));
        umma_commit(smem_u32(&bar->st_empty[st]));
        return true;
      };
      if (ok) ok = scores(0);
      for (int j = 0; j < nkb && ok; ++j) {
        if (j + 1 < nkb && !scores(j + 1)) break;
        if (!accumulate(j)) break;
      }
      umma_commit(smem_u32(&bar->drain));
      volatile int dummy = 0;
      mbar_wait(smem_u32(&bar->drain), 0, &dummy, nullptr, 0);
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;  // query row of the tile
    const int qc = i0 + r;
    const bool qvalid = qc < p.Sk;
    const long long qr = static_cast<long long>(rowk + (qvalid ? qc : p.Sk - 1));
    const int qpos = qvalid ? p.pos_k[qr] : -1;
    const float l2 = p.lse_k[qr * p.nh + h] * kLog2e;
    const float dl = p.delta[qr * p.nh + h];
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(smem_u32(&bar->s_full[sb]), (j >> 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[32], dp[32];
      CFB_TMEM_LD32(lane_addr + kColS + sb * BC + half * 32, s);
      CFB_TMEM_LD32(lane_addr + kColDP + sb * BC + half * 32, dp);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar->s_free[sb]));
      const int key0 = j * BC + half * 32;
      const int lim = min(qpos, p.S - 1) - key0;  // keys key0 + i with i <= lim are visible
      uint32_t pd[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float dv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int k = 2 * i + e;
          const float pe = (k <= lim) ? ex2_approx(fmaf(__uint_as_float(s[k]), p.scale_log2, -l2)) : 0.f;
          dv[e] = pe * (__uint_as_float(dp[k]) - dl);
        }
        pd[i] = pack_bf16x2(dv[0], dv[1]);
      }
      if (j > 0 &&
          !mbar_wait(smem_u32(&bar->mm_done), (j - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      write_row_half(sbase + L::OFF_DS, r, half, pd);
      fence_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar->p_ready));
    }
    if (ok && mbar_wait(smem_u32(&bar->mm_done), (nkb - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
      tc_fence_after();
      constexpr int OH = HD / 2;
      __nv_bfloat16* drow = p.dqkv + qr * p.ld + h * HD + half * OH;
#pragma unroll
      for (int cc = 0; cc < OH / 32; ++cc) {
        uint32_t dq[32];
        CFB_TMEM_LD32(lane_addr + kColAcc + half * OH + cc * 32, dq);
        tmem_ld_wait();
        if (qvalid) {
          uint4* d4 = reinterpret_cast<uint4*>(drow + cc * 32);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint4 a;
            a.x = pack_bf16x2(__uint_as_float(dq[8 * k + 0]) * p.scale, __uint_as_float(dq[8 * k + 1]) * p.scale);
            a.y = pack_bf16x2(__uint_as_float(dq[8 * k + 2]) * p.scale, __uint_as_float(dq[8 * k + 3]) * p.scale);
            a.z = pack_bf16x2(__uint_as_float(dq[8 * k + 4]) * p.scale, __uint_as_float(dq[8 * k + 5]) * p.scale);
            a.w = pack_bf16x2(__uint_as_float(dq[8 * k + 6]) * p.scale, __uint_as_float(dq[8 * k + 7]) * p.scale);
            d4[k] = a;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace attn_bwd_tc

int make_tmap_2d_bf16(CUtensorMap* map, const void* ptr, long long rows, long long cols,
                      long long ld, int box_cols, int box_rows);

}  // namespace cfb

int cfb_attn_bwd_tc(const void* qkv_k, long long ld_qkv, const void* qkv_full, const void* do_k,
                    long long ld_o, const float* lse_k, const float* delta, const int* pos_k,
                    void* dqkv_k, int B, int S, int Sk, int nh, int nkv, int hd, float scale,
                    int* err, cudaStream_t st) {
  using namespace cfb;
  using namespace cfb::attn_bwd_tc;
  if (ld_qkv % 8 || ld_o % 8 || nh % nkv || Sk <= 0) return -11;
  if (hd != 64 && hd != 128) return -12;
  if ((reinterpret_cast<uintptr_t>(qkv_k) & 15) || (reinterpret_cast<uintptr_t>(qkv_full) & 15) ||
      (reinterpret_cast<uintptr_t>(do_k) & 15) || (reinterpret_cast<uintptr_t>(dqkv_k) & 15))
    return -12;
  CUtensorMap tR, tQ, tO, tOk, tF;
  int rc = 0;
  const long long rows_k = static_cast<long long>(B) * Sk, rows_f = static_cast<long long>(B) * S;
  rc |= make_tmap_2d_bf16(&tR, qkv_k, rows_k, ld_qkv, ld_qkv, 64, 128);
  rc |= make_tmap_2d_bf16(&tQ, qkv_k, rows_k, ld_qkv, ld_qkv, 64, 64);
  rc |= make_tmap_2d_bf16(&tO, do_k, rows_k, ld_o, ld_o, 64, 64);
  rc |= make_tmap_2d_bf16(&tOk, do_k, rows_k, ld_o, ld_o, 64, 128);
  rc |= make_tmap_2d_bf16(&tF, qkv_full, rows_f, ld_qkv, ld_qkv, 64, 64);
  if (rc) return -13;
  Params p;
  p.S = S;
  p.Sk = Sk;
  p.nh = nh;
  p.nkv = nkv;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.lse_k = lse_k;
  p.delta = delta;
  p.pos_k = pos_k;
  p.dqkv = static_cast<__nv_bfloat16*>(dqkv_k);
  p.ld = ld_qkv;
  p.err = err;
  auto go = [&](auto kdkdv, auto kdq, int bytes, bool& configured) -> int {
    if (!configured) {
      cudaFuncSetAttribute(kdkdv, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      cudaFuncSetAttribute(kdq, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      configured = true;
    }
    dim3 g1((Sk + BR - 1) / BR, nkv, B);
    kdkdv<<<g1, 320, bytes, st>>>(tR, tQ, tO, p);
    dim3 g2((Sk + BR - 1) / BR, nh, B);
    kdq<<<g2, 320, bytes, st>>>(tR, tOk, tF, p);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  };
  static bool configured64 = false, configured128 = false;
  if (hd == 64)
    return go(attn_bwd_dkdv_tc<64>, attn_bwd_dq_tc<64>, Smem<64>::LAUNCH_BYTES, configured64);
  return go(attn_bwd_dkdv_tc<128>, attn_bwd_dq_tc<128>, Smem<128>::LAUNCH_BYTES, configured128);
}
