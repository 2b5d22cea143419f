// Filtered ("restore-Q") causal GQA attention backward on the 5th-generation tensor cores.
//
// Inputs are the kept query/key rows in compact order (row b*Sk + j of qkv_k / do_k / lse_k /
// delta, sorted by position) and the full-sequence qkv rows for the dropped keys.  The work
// splits into two kinds of item:
//
// dK/dV item (128 kept keys x KV head x batch).  K_kv, V_kv of the 128 keys stay in shared
// memory while the item loops over (query head of the group) x (64-query blocks from the first
// one that can see its keys).  Per block:  S^T = K Q^T and dP^T = V dO^T (M = 128 keys,
// N = 64 queries) into double-buffered TMEM tiles;  the softmax warps form
// P^T = 2^(S^T c - lse) and dS^T = P^T (dP^T - delta) (bf16, 128B-swizzled in shared memory);
// dV += P^T dO and dK += dS^T Q accumulate in TMEM over all blocks and heads of the group
// (native GQA: no per-head dK/dV and no reduction pass).  Causality in compact index ==
// causality in position.
//
// dQ item (128 kept queries x query head x batch).  Q, dO stay in shared memory while the item
// walks 64-key blocks of the FULL sequence up to its last query's position: S = Q K^T,
// dP = dO V^T, dS = P (dP - delta) with the position predicate key_pos <= query_pos, and
// dQ += dS K in TMEM.  Dropped keys therefore contribute to dQ exactly as in the reference's
// second (restore-Q) backward, in one pass and without a bias tensor.
//
// With a RoPE table the dQ and dK epilogues also apply the RoPE backward (rotation by the negated
// angle of the row's position), so no separate pass runs over dqkv.
//
// Persistent kernel: one CTA per SM takes items from a global counter (heaviest first: dK/dV
// items by ascending key block, then dQ items by descending query block).  The A/B tiles of an
// item (K,V or Q,dO) are double-buffered so the next item's tiles load while the current one
// finishes, and an item's epilogue (TMEM -> global) overlaps the next item's first score tiles.
// Roles: warp 0 TMA + scheduling, warp 1 MMA issue (one thread), NSW = 8 (or 16) softmax /
// epilogue warps: NSW / 4 warps per TMEM lane quadrant, each taking 64 / (NSW / 4) of the 64
// columns.  Every barrier phase is
// derived from running counters (items taken, score tiles processed) that all roles advance
// identically.  All waits are bounded (sm100_common.cuh).
#include "sm100_common.cuh"
#include "launch_api.h"

#include <math_constants.h>
#include <cstdlib>

namespace cfb {
namespace attn_bwd_tc {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int BR = 128;  // rows owned by an item (keys for dK/dV, queries for dQ)
constexpr int BC = 64;   // columns per step (queries for dK/dV, keys for dQ)
constexpr int MAX_STAGES = 4;

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
struct Cfg {
  static constexpr int STAGES = HD == 64 ? 4 : 2;
  static constexpr int CH_R = BR * 128;              // chunk of a 128-row tile (64 bf16 per row)
  static constexpr int CH_C = BC * 128;              // chunk of a 64-row tile
  static constexpr int ROW_TILE = (HD / 64) * CH_R;  // [128 x HD]
  static constexpr int COL_TILE = (HD / 64) * CH_C;  // [64 x HD]
  static constexpr int AB = 2 * ROW_TILE;            // A (K or Q) and B (V or dO) of an item
  static constexpr int OFF_AB = 0;                   // two buffers
  static constexpr int OFF_ST = OFF_AB + 2 * AB;     // stages of [Q_i, dO_i] / [K_j, V_j]
  static constexpr int STAGE = 2 * COL_TILE;
  static constexpr int OFF_P = OFF_ST + STAGES * STAGE;  // P^T (dK/dV items), [128 x 64] bf16
  static constexpr int OFF_DS = OFF_P + CH_R;            // dS^T / dS, [128 x 64] bf16
  static constexpr int OFF_BAR = OFF_DS + CH_R;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;     // + barriers + alignment slack
  static_assert(STAGES <= MAX_STAGES, "stage ring");
  static_assert(BYTES <= 232448, "shared memory per CTA");
};

struct Params {
  int B, S, Sk, nh, nkv, nblk, n_dkdv, n_items;
  float scale_log2;  // softmax scale * log2(e)
  float scale;       // softmax scale (dS -> dQ / dK)
  const float* lse_k;  // [B*Sk, nh] natural-log LSE of kept queries
  const float* delta;  // [B*Sk, nh]
  const int* pos_k;    // [B*Sk] positions of kept rows
  __nv_bfloat16* dqkv; // [B*Sk, ld] output rows (compact)
  long long ld;
  int* work;           // [2]: next item, finished CTAs (zero between launches)
  int* err;
  const float* cs;     // optional RoPE table [max_pos, HD/2, 2] (cos, sin): dQ and dK leave
                       // rotated back by -angle(position) (the RoPE backward), else nullptr
};

struct Bars {
  uint64_t a_full[2], a_empty[2], st_full[MAX_STAGES], st_empty[MAX_STAGES], s_full[2],
      s_free[2], p_ready, mm_done, acc_free, drain;
  int item[2];
  uint32_t tmem_slot;
  int abort;
};

// Two 64-column score tiles (S, dP) per buffer: S at sb*64, dP at 128 + sb*64; accumulators
// (dK, dV or dQ) from column 256.
constexpr uint32_t kColS = 0, kColDP = 128, kColAcc = 256;

struct Item {
  bool dkdv;
  int blk, head, b;  // key/query block, KV/query head, sequence
  int n_it;          // score tiles of the item
};

__device__ __forceinline__ Item decode(int id, const Params& p) {
  Item t;
  if (id < p.n_dkdv) {
    t.dkdv = true;
    t.blk = id / (p.nkv * p.B);
    const int rem = id % (p.nkv * p.B);
    t.head = rem % p.nkv;
    t.b = rem / p.nkv;
    const int nqb = (p.Sk + BC - 1) / BC - t.blk * (BR / BC);
    t.n_it = (p.nh / p.nkv) * nqb;
  } else {
    id -= p.n_dkdv;
    t.dkdv = false;
    t.blk = p.nblk - 1 - id / (p.nh * p.B);
    const int rem = id % (p.nh * p.B);
    t.head = rem % p.nh;
    t.b = rem / p.nh;
    const int last = min(p.Sk, (t.blk + 1) * BR) - 1;
    const int max_pos = min(__ldg(p.pos_k + t.b * p.Sk + last), p.S - 1);
    t.n_it = max_pos / BC + 1;
  }
  return t;
}

// Thread's CPT columns (part `part` of the row) of a 64-column bf16 row tile in 128B-swizzled
// K-major layout: CPT / 8 pieces of 16 bytes.
template <int CPT>
__device__ __forceinline__ void write_row_part(uint32_t tile, int r, int part, const uint32_t* pk) {
  const uint32_t rowbase = tile + r * 128;
#pragma unroll
  for (int i = 0; i < CPT / 8; ++i) {
    const int piece = part * (CPT / 8) + i;
    st_shared_v4(rowbase + ((piece ^ (r & 7)) << 4), pk[4 * i], pk[4 * i + 1], pk[4 * i + 2],
                 pk[4 * i + 3]);
  }
}

// Load N (8, 16 or 32) consecutive TMEM columns of the thread's lane.
template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, uint32_t* r) {
  if constexpr (N == 32) {
    CFB_TMEM_LD32(taddr, r);
  } else if constexpr (N == 16) {
    CFB_TMEM_LD16(taddr, r);
  } else {
    static_assert(N == 8, "TMEM load width");
    CFB_TMEM_LD8(taddr, r);
  }
}

// Store N (a multiple of 8) fp32 TMEM columns as bf16 (times `mul`) to 2 N contiguous bytes.
template <int N>
__device__ __forceinline__ void store_row_n(__nv_bfloat16* dst, const uint32_t* v, float mul) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int k = 0; k < N / 8; ++k) {
    uint4 a;
    a.x = pack_bf16x2(__uint_as_float(v[8 * k + 0]) * mul, __uint_as_float(v[8 * k + 1]) * mul);
    a.y = pack_bf16x2(__uint_as_float(v[8 * k + 2]) * mul, __uint_as_float(v[8 * k + 3]) * mul);
    a.z = pack_bf16x2(__uint_as_float(v[8 * k + 4]) * mul, __uint_as_float(v[8 * k + 5]) * mul);
    a.w = pack_bf16x2(__uint_as_float(v[8 * k + 6]) * mul, __uint_as_float(v[8 * k + 7]) * mul);
    d4[k] = a;
  }
}

// Epilogue of dQ or dK: the thread (TMEM lane = row, part `part` of the QPR threads of the row)
// owns columns [i0, i0 + Q) and [HD/2 + i0, HD/2 + i0 + Q) with Q = HD / (2 QPR) and
// i0 = part * Q, i.e. both members of every rotate-half pair it stores.  Scaled by `mul`; with a
// table, rotated by -angle(pos).
template <int HD, int QPR>
__device__ __forceinline__ void store_rot_pairs(uint32_t t_acc, __nv_bfloat16* head_dst, int part,
                                                float mul, const float* cs, int pos, bool valid) {
  constexpr int Q4 = HD / (2 * QPR), H2 = HD / 2;
  const int i0 = part * Q4;
  uint32_t a[Q4], b[Q4];
  tmem_ld_n<Q4>(t_acc + i0, a);
  tmem_ld_n<Q4>(t_acc + H2 + i0, b);
  tmem_ld_wait();
  if (!valid) return;
  uint32_t oa[Q4 / 2], ob[Q4 / 2];
  const float2* c2 = cs ? reinterpret_cast<const float2*>(cs) + static_cast<long long>(pos) * H2 + i0
                        : nullptr;
#pragma unroll
  for (int t = 0; t < Q4 / 2; ++t) {
    float x0 = __uint_as_float(a[2 * t]) * mul, x1 = __uint_as_float(a[2 * t + 1]) * mul;
    float y0 = __uint_as_float(b[2 * t]) * mul, y1 = __uint_as_float(b[2 * t + 1]) * mul;
    if (c2) {
      const float2 q0 = __ldg(c2 + 2 * t), q1 = __ldg(c2 + 2 * t + 1);
      const float rx0 = x0 * q0.x + y0 * q0.y, ry0 = y0 * q0.x - x0 * q0.y;
      const float rx1 = x1 * q1.x + y1 * q1.y, ry1 = y1 * q1.x - x1 * q1.y;
      x0 = rx0; y0 = ry0; x1 = rx1; y1 = ry1;
    }
    oa[t] = pack_bf16x2(x0, x1);
    ob[t] = pack_bf16x2(y0, y1);
  }
  uint4* da = reinterpret_cast<uint4*>(head_dst + i0);
  uint4* db = reinterpret_cast<uint4*>(head_dst + H2 + i0);
#pragma unroll
  for (int j = 0; j < Q4 / 8; ++j) {
    da[j] = make_uint4(oa[4 * j], oa[4 * j + 1], oa[4 * j + 2], oa[4 * j + 3]);
    db[j] = make_uint4(ob[4 * j], ob[4 * j + 1], ob[4 * j + 2], ob[4 * j + 3]);
  }
}

// NSW softmax / epilogue warps (8 or 16): QPR = NSW / 4 threads share a row of the 64-column
// score tiles, CPT = 64 / QPR columns each.
template <int HD, int NSW = 8>
__global__ void __launch_bounds__(64 + 32 * NSW, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmR,   // qkv_k, box 64 x 128 rows
                       const __grid_constant__ CUtensorMap tmQ,   // qkv_k, box 64 x 64 rows
                       const __grid_constant__ CUtensorMap tmO,   // do_k,  box 64 x 64 rows
                       const __grid_constant__ CUtensorMap tmOk,  // do_k,  box 64 x 128 rows
                       const __grid_constant__ CUtensorMap tmF,   // qkv full, box 64 x 64 rows
                       const Params p) {
  using L = Cfg<HD>;
  constexpr int STAGES = L::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  Bars* bar = reinterpret_cast<Bars*>(smem + L::OFF_BAR);
  volatile int* abort_flag = &bar->abort;
  volatile int* item_slot = bar->item;
  const int warp = warp_id(), lane = lane_id();
  const int group = p.nh / p.nkv;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bar->a_full[i]), 1);
      mbar_init(smem_u32(&bar->a_empty[i]), 1);
      mbar_init(smem_u32(&bar->s_full[i]), 1);
      mbar_init(smem_u32(&bar->s_free[i]), NSW);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bar->st_full[s]), 1);
      mbar_init(smem_u32(&bar->st_empty[s]), 1);
    }
    mbar_init(smem_u32(&bar->p_ready), NSW);
    mbar_init(smem_u32(&bar->mm_done), 1);
    mbar_init(smem_u32(&bar->acc_free), NSW);
    mbar_init(smem_u32(&bar->drain), 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmR);
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmO);
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
      // ------------------------------------------------------------ scheduler + TMA producer
      int k = 0, g = 0;  // items taken (incl. the final "none left"), score tiles loaded
      bool ok = true;
      for (; ok; ++k) {
        const int ab = k & 1;
        if (!mbar_wait(smem_u32(&bar->a_empty[ab]), ((k >> 1) & 1) ^ 1, abort_flag, p.err,
                       kErrWaitProducer)) {
          ok = false;
          break;
        }
        int id = atomicAdd(p.work, 1);
        if (id >= p.n_items) id = -1;
        item_slot[ab] = id;
        if (id < 0) {
          mbar_arrive(smem_u32(&bar->a_full[ab]));
          ++k;
          break;
        }
        const Item t = decode(id, p);
        const uint32_t afb = smem_u32(&bar->a_full[ab]);
        const uint32_t sa = sbase + L::OFF_AB + ab * L::AB;
        mbar_arrive_expect_tx(afb, L::AB);
        if (t.dkdv) {
          const int row = t.b * p.Sk + t.blk * BR;
          const int kcol = (p.nh + t.head) * HD, vcol = (p.nh + p.nkv + t.head) * HD;
#pragma unroll
          for (int c = 0; c < HD / 64; ++c) {
            tma_load_2d(sa + c * L::CH_R, &tmR, afb, kcol + c * 64, row);
            tma_load_2d(sa + L::ROW_TILE + c * L::CH_R, &tmR, afb, vcol + c * 64, row);
          }
        } else {
          const int row = t.b * p.Sk + t.blk * BR;
#pragma unroll
          for (int c = 0; c < HD / 64; ++c) {
            tma_load_2d(sa + c * L::CH_R, &tmR, afb, t.head * HD + c * 64, row);
            tma_load_2d(sa + L::ROW_TILE + c * L::CH_R, &tmOk, afb, t.head * HD + c * 64, row);
          }
        }
        const int qb_first = t.blk * (BR / BC);
        const int nqb = t.dkdv ? t.n_it / group : 0;
        const int g_kv = t.dkdv ? 0 : t.head / group;
        const int kcol = (p.nh + g_kv) * HD, vcol = (p.nh + p.nkv + g_kv) * HD;
        for (int it = 0; it < t.n_it; ++it, ++g) {
          const int st = g % STAGES;
          if (!mbar_wait(smem_u32(&bar->st_empty[st]), ((g / STAGES) & 1) ^ 1, abort_flag,
                         p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&bar->st_full[st]);
          mbar_arrive_expect_tx(fb, L::STAGE);
          const uint32_t ss = sbase + L::OFF_ST + st * L::STAGE;
          if (t.dkdv) {
            const int h = t.head * group + it / nqb;
            const int row = t.b * p.Sk + (qb_first + it % nqb) * BC;
#pragma unroll
            for (int c = 0; c < HD / 64; ++c) {
              tma_load_2d(ss + c * L::CH_C, &tmQ, fb, h * HD + c * 64, row);
              tma_load_2d(ss + L::COL_TILE + c * L::CH_C, &tmO, fb, h * HD + c * 64, row);
            }
          } else {
            const int row = t.b * p.S + it * BC;
#pragma unroll
            for (int c = 0; c < HD / 64; ++c) {
              tma_load_2d(ss + c * L::CH_C, &tmF, fb, kcol + c * 64, row);
              tma_load_2d(ss + L::COL_TILE + c * L::CH_C, &tmF, fb, vcol + c * 64, row);
            }
          }
        }
      }
      tma_drain_ring(bar->st_full, STAGES, g);
      tma_drain_ring(bar->a_full, 2, k);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t ID_S = idesc_bf16_f32(BR, BC, false, false);
      constexpr uint32_t ID_ACC = idesc_bf16_f32(BR, HD, false, true);
      int k = 0, g = 0;
      for (;; ++k) {
        const int ab = k & 1;
        if (!mbar_wait(smem_u32(&bar->a_full[ab]), (k >> 1) & 1, abort_flag, p.err, kErrWaitMma))
          break;
        const int id = item_slot[ab];
        if (id < 0) break;
        const Item t = decode(id, p);
        tc_fence_after();
        const uint32_t sa = sbase + L::OFF_AB + ab * L::AB;
        // S (or S^T) = A X^T and dP (or dP^T) = B Y^T for the stage's [X, Y] tiles
        auto scores = [&](int it) -> bool {
          const int gg = g + it;
          const int st = gg % STAGES, sb = gg & 1;
          if (!mbar_wait(smem_u32(&bar->st_full[st]), (gg / STAGES) & 1, abort_flag, p.err,
                         kErrWaitMma))
            return false;
          const int use = gg >> 1;
          if (use > 0 &&
              !mbar_wait(smem_u32(&bar->s_free[sb]), (use - 1) & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          tc_fence_after();
          const uint32_t ss = sbase + L::OFF_ST + st * L::STAGE;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t oa = (kk >> 2) * L::CH_R + (kk & 3) * 32;
            const uint32_t ob = (kk >> 2) * L::CH_C + (kk & 3) * 32;
            umma_bf16_ss(tmem + kColS + sb * BC, sdesc_sw128(sa + oa, 16, 1024),
                         sdesc_sw128(ss + ob, 16, 1024), ID_S, kk > 0);
            umma_bf16_ss(tmem + kColDP + sb * BC, sdesc_sw128(sa + L::ROW_TILE + oa, 16, 1024),
                         sdesc_sw128(ss + L::COL_TILE + ob, 16, 1024), ID_S, kk > 0);
          }
          umma_commit(smem_u32(&bar->s_full[sb]));
          return true;
        };
        // dK += dS^T X and dV += P^T Y (dK/dV item), dQ += dS X (dQ item); X, Y read MN-major
        auto accumulate = [&](int it) -> bool {
          const int gg = g + it;
          if (it == 0 && k > 0 &&
              !mbar_wait(smem_u32(&bar->acc_free), (k - 1) & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          if (!mbar_wait(smem_u32(&bar->p_ready), gg & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          tc_fence_after();
          const int st = gg % STAGES;
          const uint32_t ss = sbase + L::OFF_ST + st * L::STAGE;
#pragma unroll
          for (int kk = 0; kk < BC / 16; ++kk) {
            const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
            umma_bf16_ss(tmem + kColAcc, sdesc_sw128(sbase + L::OFF_DS + kk * 32, 16, 1024),
                         sdesc_sw128(ss + kk * 2048, L::CH_C, 1024), ID_ACC, acc);
            if (t.dkdv)
              umma_bf16_ss(tmem + kColAcc + HD, sdesc_sw128(sbase + L::OFF_P + kk * 32, 16, 1024),
                           sdesc_sw128(ss + L::COL_TILE + kk * 2048, L::CH_C, 1024), ID_ACC, acc);
          }
          umma_commit(smem_u32(&bar->mm_done));
          umma_commit(smem_u32(&bar->st_empty[st]));
          return true;
        };
        bool ok = scores(0);
        for (int it = 0; it < t.n_it && ok; ++it) {
          if (it + 1 < t.n_it && !scores(it + 1)) ok = false;
          if (ok && !accumulate(it)) ok = false;
        }
        if (!ok) break;
        umma_commit(smem_u32(&bar->a_empty[ab]));
        g += t.n_it;
      }
      umma_commit(smem_u32(&bar->drain));
      volatile int no_abort = 0;
      mbar_wait(smem_u32(&bar->drain), 0, &no_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue, warps 2-9
    constexpr int QPR = NSW / 4;     // threads per tile row
    constexpr int CPT = BC / QPR;    // score columns per thread
    const int quad = warp & 3;
    const int part = (warp - 2) >> 2;
    const int r = quad * 32 + lane;  // tile row == TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    constexpr int OH = HD / QPR;     // dV output columns per thread in the epilogue
    constexpr int OCH = OH < 32 ? OH : 32;
    int k = 0, g = 0;
    bool ok = true;
    for (; ok; ++k) {
      const int ab = k & 1;
      if (!mbar_wait(smem_u32(&bar->a_full[ab]), (k >> 1) & 1, abort_flag, p.err, kErrWaitSoftmax))
        break;
      const int id = item_slot[ab];
      if (id < 0) break;
      const Item t = decode(id, p);
      const int rowk = t.b * p.Sk;
      if (t.dkdv) {
        const int j0 = t.blk * BR;
        const int kc = j0 + r;  // compact key of this row
        const int qb_first = j0 / BC;
        const int nqb = t.n_it / group;
        // lse / delta of the CPT queries of a step: lane k holds query i0 + k % CPT; loaded one
        // step ahead so that the global-load latency is off the critical path
        auto stat_row = [&](int it) -> long long {
          const int hh = t.head * group + it / nqb;
          const int q = (qb_first + it % nqb) * BC + part * CPT + (lane % CPT);
          return static_cast<long long>(rowk + min(q, p.Sk - 1)) * p.nh + hh;
        };
        float l2_next, dl_next;
        {
          const long long qr = stat_row(0);
          l2_next = __ldg(p.lse_k + qr) * kLog2e;
          dl_next = __ldg(p.delta + qr);
        }
        for (int it = 0; it < t.n_it; ++it) {
          const int gg = g + it, sb = gg & 1;
          const int i0 = (qb_first + it % nqb) * BC + part * CPT;  // this thread's first query
          const float l2_lane = l2_next, dl_lane = dl_next;
          if (it + 1 < t.n_it) {
            const long long qr = stat_row(it + 1);
            l2_next = __ldg(p.lse_k + qr) * kLog2e;
            dl_next = __ldg(p.delta + qr);
          }
          if (!mbar_wait(smem_u32(&bar->s_full[sb]), (gg >> 1) & 1, abort_flag, p.err,
                         kErrWaitSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t s[CPT], dp[CPT];
          tmem_ld_n<CPT>(lane_addr + kColS + sb * BC + part * CPT, s);
          tmem_ld_n<CPT>(lane_addr + kColDP + sb * BC + part * CPT, dp);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&bar->s_free[sb]));
          const int lo = kc - i0, hi = p.Sk - i0;  // query column c is visible iff lo <= c < hi
          uint32_t pp[CPT / 2], pd[CPT / 2];
#pragma unroll
          for (int i = 0; i < CPT / 2; ++i) {
            float pv[2], dv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int c = 2 * i + e;
              const float l2 = __shfl_sync(0xffffffffu, l2_lane, c);
              const float dl = __shfl_sync(0xffffffffu, dl_lane, c);
              const float pe = (c >= lo && c < hi)
                                   ? ex2_approx(fmaf(__uint_as_float(s[c]), p.scale_log2, -l2))
                                   : 0.f;
              pv[e] = pe;
              dv[e] = pe * (__uint_as_float(dp[c]) - dl);
            }
            pp[i] = pack_bf16x2(pv[0], pv[1]);
            pd[i] = pack_bf16x2(dv[0], dv[1]);
          }
          // the previous step's accumulate MMAs read P^T / dS^T: wait before overwriting
          if (gg > 0 &&
              !mbar_wait(smem_u32(&bar->mm_done), (gg - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
            ok = false;
            break;
          }
          write_row_part<CPT>(sbase + L::OFF_P, r, part, pp);
          write_row_part<CPT>(sbase + L::OFF_DS, r, part, pd);
          fence_async_shared();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&bar->p_ready));
        }
        if (!ok) break;
        const int gl = g + t.n_it - 1;
        if (!mbar_wait(smem_u32(&bar->mm_done), gl & 1, abort_flag, p.err, kErrWaitSoftmax)) break;
        tc_fence_after();
        const int kcol = (p.nh + t.head) * HD, vcol = (p.nh + p.nkv + t.head) * HD;
        const bool kvalid = kc < p.Sk;
        const long long krow = static_cast<long long>(rowk + min(kc, p.Sk - 1));
        __nv_bfloat16* drow = p.dqkv + krow * p.ld;
        store_rot_pairs<HD, QPR>(lane_addr + kColAcc, drow + kcol, part, p.scale, p.cs,
                                 kvalid ? __ldg(p.pos_k + krow) : 0, kvalid);
#pragma unroll
        for (int cc = 0; cc < OH / OCH; ++cc) {
          uint32_t dv[OCH];
          tmem_ld_n<OCH>(lane_addr + kColAcc + HD + part * OH + cc * OCH, dv);
          tmem_ld_wait();
          if (kvalid) store_row_n<OCH>(drow + vcol + part * OH + cc * OCH, dv, 1.f);
        }
      } else {
        const int qc = t.blk * BR + r;  // compact query of this row
        const bool qvalid = qc < p.Sk;
        const long long qr = static_cast<long long>(rowk + (qvalid ? qc : p.Sk - 1));
        const int qpos = qvalid ? __ldg(p.pos_k + qr) : -1;
        const float l2 = __ldg(p.lse_k + qr * p.nh + t.head) * kLog2e;
        const float dl = __ldg(p.delta + qr * p.nh + t.head);
        for (int j = 0; j < t.n_it; ++j) {
          const int gg = g + j, sb = gg & 1;
          if (!mbar_wait(smem_u32(&bar->s_full[sb]), (gg >> 1) & 1, abort_flag, p.err,
                         kErrWaitSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t s[CPT], dp[CPT];
          tmem_ld_n<CPT>(lane_addr + kColS + sb * BC + part * CPT, s);
          tmem_ld_n<CPT>(lane_addr + kColDP + sb * BC + part * CPT, dp);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&bar->s_free[sb]));
          const int lim = min(qpos, p.S - 1) - (j * BC + part * CPT);  // key column c visible iff c <= lim
          uint32_t pd[CPT / 2];
#pragma unroll
          for (int i = 0; i < CPT / 2; ++i) {
            float dv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int c = 2 * i + e;
              const float pe =
                  (c <= lim) ? ex2_approx(fmaf(__uint_as_float(s[c]), p.scale_log2, -l2)) : 0.f;
              dv[e] = pe * (__uint_as_float(dp[c]) - dl);
            }
            pd[i] = pack_bf16x2(dv[0], dv[1]);
          }
          if (gg > 0 &&
              !mbar_wait(smem_u32(&bar->mm_done), (gg - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
            ok = false;
            break;
          }
          write_row_part<CPT>(sbase + L::OFF_DS, r, part, pd);
          fence_async_shared();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&bar->p_ready));
        }
        if (!ok) break;
        const int gl = g + t.n_it - 1;
        if (!mbar_wait(smem_u32(&bar->mm_done), gl & 1, abort_flag, p.err, kErrWaitSoftmax)) break;
        tc_fence_after();
        store_rot_pairs<HD, QPR>(lane_addr + kColAcc, p.dqkv + qr * p.ld + t.head * HD, part,
                                 p.scale, p.cs, qpos, qvalid);
      }
      // accumulators read: the next item's first accumulate may overwrite them
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar->acc_free));
      g += t.n_it;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
  if (threadIdx.x == 0) {
    // the last CTA to finish resets the work counter for the next launch
    __threadfence();
    if (atomicAdd(p.work + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      atomicExch(p.work, 0);
      atomicExch(p.work + 1, 0);
    }
  }
}

}  // namespace attn_bwd_tc

int make_tmap_2d_bf16(CUtensorMap* map, const void* ptr, long long rows, long long cols,
                      long long ld, int box_cols, int box_rows);

}  // namespace cfb

int cfb_attn_bwd_tc(const void* qkv_k, long long ld_qkv, const void* qkv_full, const void* do_k,
                    long long ld_o, const float* lse_k, const float* delta, const int* pos_k,
                    void* dqkv_k, int B, int S, int Sk, int nh, int nkv, int hd, float scale,
                    const float* rope_cs, int* work, int* err, cudaStream_t st) {
  using namespace cfb;
  using namespace cfb::attn_bwd_tc;
  if (ld_qkv % 8 || ld_o % 8 || nh % nkv || Sk <= 0 || !work) return -11;
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
  p.B = B;
  p.S = S;
  p.Sk = Sk;
  p.nh = nh;
  p.nkv = nkv;
  p.nblk = (Sk + BR - 1) / BR;
  p.n_dkdv = p.nblk * nkv * B;
  p.n_items = p.n_dkdv + p.nblk * nh * B;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.lse_k = lse_k;
  p.delta = delta;
  p.pos_k = pos_k;
  p.dqkv = static_cast<__nv_bfloat16*>(dqkv_k);
  p.ld = ld_qkv;
  p.work = work;
  p.err = err;
  p.cs = rope_cs;
  static int n_sm = 0;
  if (n_sm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  }
  const int grid = p.n_items < n_sm ? p.n_items : n_sm;
  auto go = [&](auto kern, int bytes, int threads, bool& configured) -> int {
    if (!configured) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
      configured = true;
    }
    kern<<<grid, threads, bytes, st>>>(tR, tQ, tO, tOk, tF, p);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  };
  // CFB_ATTN_BWD_WARPS: softmax / epilogue warps per CTA, 8 (default) or 16.  16 measured
  // slower (TinyLlama layer, keep 0.5: 0.528 vs 0.499 ms; hd 128: 1.564 vs 1.526 ms).
  static const int nsw = [] {
    const char* e = std::getenv("CFB_ATTN_BWD_WARPS");
    return (e && std::atoi(e) == 16) ? 16 : 8;
  }();
  static bool cfg[4] = {false, false, false, false};
  if (nsw == 16) {
    if (hd == 64) return go(attn_bwd_tc_kernel<64, 16>, Cfg<64>::BYTES, 576, cfg[0]);
    return go(attn_bwd_tc_kernel<128, 16>, Cfg<128>::BYTES, 576, cfg[1]);
  }
  if (hd == 64) return go(attn_bwd_tc_kernel<64, 8>, Cfg<64>::BYTES, 320, cfg[2]);
  return go(attn_bwd_tc_kernel<128, 8>, Cfg<128>::BYTES, 320, cfg[3]);
}
