// Causal GQA attention forward on the 5th-generation tensor cores (sm_100a).
//
// Work item: 128 query rows of one head against the causal key range, 128 keys per step.
// Persistent kernel (one CTA per SM) taking items from a global counter, heaviest (latest
// query block) first.  Roles:
//   warp 0      scheduler + TMA producer: item id, Q once per item (double-buffered for
//               hd 64 so the next item's Q loads during the current one), then K_j and V_j
//               tiles through two separate rings: a K slot frees as soon as S_j = Q K_j^T is
//               done, a V slot only after P_j V_j, so K loads run well ahead of the softmax
//   warp 1      MMA issuer:   S_j into one of two TMEM tiles (128 x 128 fp32), then
//                             O += P_j V_j into the TMEM accumulators
//   warps 2..   softmax:      NQ = 2 threads per query row (= TMEM lane): warps w, w+4 share a
//                             lane quadrant and take key groups [0, 64), [64, 128) of every step.
//                             Each group keeps its own running max, row sum and O accumulator
//                             (O_0 .. O_{NQ-1} in TMEM, fed by one PV MMA chain per group), so
//                             the groups never synchronise per step; the epilogue merges them
//                             once (O = sum_q O_q 2^(m_q-m), same for l).  Online softmax in
//                             fp32 with one FMA + ex2 per score; P (bf16) is written back into
//                             TMEM over the thread's own S columns and feeds P V as the TMEM A
//                             operand, so P never touches shared memory; a running max only
//                             moves (and its O is rescaled in TMEM) when it grows by more than 2^8
// S_{j+1} is issued before P_j V_j so that the tensor cores compute the next scores while the
// softmax warps work on the current ones, and the next item's first scores overlap this item's
// epilogue.  Q, K and V are read straight from the fused [T, (nh + 2 nkv) hd] qkv rows with one
// 2-D tensor map (box 64 x 128): K tiles serve as the K-major B operand of Q K^T and V tiles,
// bit-identical in shared memory, as the MN-major B operand of P V.  Barrier phases follow
// running counters (items, K/V tiles, score tiles) that every role advances identically.  All
// waits are bounded (sm100_common.cuh).
#include "sm100_common.cuh"
#include "launch_api.h"

#include <math_constants.h>
#include <cstdlib>

namespace cfb {
namespace attn_tc {

constexpr int BM = 128, BN = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int MAX_RING = 4;

template <int HD>
struct Smem {
  static constexpr int QBUF = HD == 64 ? 2 : 1;           // Q buffers (items in flight)
  static constexpr int KV_STAGES = HD == 64 ? 4 : 2;      // slots of each of the K and V rings
  static constexpr int CHUNK = BM * 128;                  // 128 rows x 128 B (64 bf16)
  static constexpr int Q_BYTES = (HD / 64) * CHUNK;       // Q [128 x HD], K-major chunks
  static constexpr int KV_TILE = (HD / 64) * CHUNK;       // K_j or V_j [128 x HD]
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + QBUF * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KV_STAGES * KV_TILE;
  // key groups (threads) per query row.  Four groups (16 softmax warps) at hd 64 measured
  // slower than two (307 vs 441 TFLOP/s at B8 S2048 32q/4kv): the per-group PV MMAs become
  // K = 32 chains and the epilogue merge costs more than the extra warps hide.
  static constexpr int NQ = 2;
  static constexpr int THREADS = 64 + 128 * NQ;           // TMA + MMA warps, 4 NQ softmax warps
  static constexpr int OFF_RED = OFF_V + KV_STAGES * KV_TILE;  // exchange: [2][NQ][128] fp32
  static constexpr int OFF_FLAG = OFF_RED + 2 * NQ * BM * 4;   // [NQ][128] exchange counters
  static constexpr int OFF_BAR = OFF_FLAG + NQ * BM * 4;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;     // + barriers + alignment slack
  static_assert(KV_STAGES <= MAX_RING && QBUF <= 2, "rings");
  static_assert(BYTES <= 232448, "shared memory per CTA");
};

struct Params {
  const __nv_bfloat16* qkv;
  long long ld;
  __nv_bfloat16* out;
  long long ld_out;
  float* lse;
  int B, S, nh, nkv, nqb, n_items;
  float scale_log2;
  int* work;  // [2]: next item, finished CTAs (zero between launches)
  int* err;
};

struct Bars {
  uint64_t q_full[2], q_empty[2], k_full[MAX_RING], k_empty[MAX_RING], v_full[MAX_RING],
      v_empty[MAX_RING], s_full[2], s_free[2], p_ready, o_done, o_free, drain;
  int item[2];
  uint32_t tmem_slot;
  int abort;
};

struct Item {
  int qb, h, b, nkb;
};

__device__ __forceinline__ Item decode(int id, const Params& p) {
  Item t;
  t.qb = p.nqb - 1 - id / (p.nh * p.B);
  const int rem = id % (p.nh * p.B);
  t.h = rem % p.nh;
  t.b = rem / p.nh;
  const int last_q = min(p.S, (t.qb + 1) * BM) - 1;
  t.nkb = last_q / BN + 1;
  return t;
}

// Hardware base-2 exponential (MUFU); flushes denormal results to zero.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Software base-2 exponential on the FMA pipe, for a share of the scores while the MUFU unit
// is the busiest pipe.  Cody-Waite style range reduction x = j + f with j = round(x) (the
// 1.5 * 2^23 rounding constant) and f in [-1/2, 1/2], a degree-3 polynomial for 2^f fitted
// here by the Remez exchange algorithm on the relative error (max relative error 7.5e-5, far
// below the bf16 rounding of P), and 2^j added into the exponent field.  Inputs below -125
// are clamped (result about 2^-125 instead of 0; masked scores are -inf).
__device__ __forceinline__ float ex2_poly(float x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  x = fmaxf(x, -125.0f);
  const float t = x + kRound;
  const float f = x - (t - kRound);
  float p = fmaf(0.0551716685295105f, f, 0.2426111251115799f);
  p = fmaf(p, f, 0.6932609677314758f);
  p = fmaf(p, f, 0.9999280571937561f);
  const int j = __float_as_int(t) - __float_as_int(kRound);
  return __int_as_float(__float_as_int(p) + (j << 23));
}

// Three-input maximum (sm_100).
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Exchange one float per row among the NQ groups of the same lane quadrant.  Each thread
// publishes its value in slot `slot` and a sequence number in shared memory, then spins
// (bounded) until every other group's sequence number arrives, and returns all NQ values
// (vals_out[q], its own included).  A slot is only rewritten two exchanges later, after every
// other group has provably read it (it published the following exchange's sequence number only
// after reading).  Returns false if the wait gave up.
template <int NQ>
__device__ __forceinline__ bool group_exchange(float* vals, volatile int* flags, int slot,
                                               int grp, int r, int seq, float mine,
                                               float (&vals_out)[NQ], volatile int* abort_flag,
                                               int* err) {
  constexpr int BMr = 128;
  vals[(slot * NQ + grp) * BMr + r] = mine;
  __threadfence_block();
  flags[grp * BMr + r] = seq;
  const uint64_t t0 = globaltimer_ns();
  uint64_t limit = 0;  // read from the status block only once a wait has spun 256 times
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    if (q == grp) continue;
    uint32_t spins = 0;
    while (flags[q * BMr + r] < seq) {
      if ((++spins & 255u) == 0) {
        if (*abort_flag) return false;
        if (limit == 0) limit = local_wait_limit_ns(err);
        if (globaltimer_ns() - t0 > limit) {
          *abort_flag = 1;
          atomicCAS(err, 0, kErrWaitSoftmax);
          return false;
        }
      }
    }
  }
  __threadfence_block();
#pragma unroll
  for (int q = 0; q < NQ; ++q) vals_out[q] = q == grp ? mine : vals[(slot * NQ + q) * BMr + r];
  return true;
}

template <int HD>
__global__ void __launch_bounds__(Smem<HD>::THREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, const Params p) {
  using L = Smem<HD>;
  constexpr int QBUF = L::QBUF, KVS = L::KV_STAGES, NQ = L::NQ;
  constexpr int NSW = 4 * NQ;  // softmax warps
  constexpr int CW = BN / NQ;  // keys per softmax thread per step
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  Bars* bar = reinterpret_cast<Bars*>(smem + L::OFF_BAR);
  volatile int* abort_flag = &bar->abort;
  volatile int* item_slot = bar->item;
  const int warp = warp_id(), lane = lane_id();
  const int group = p.nh / p.nkv;

  if (threadIdx.x == 0) {
    for (int i = 0; i < QBUF; ++i) {
      mbar_init(smem_u32(&bar->q_full[i]), 1);
      mbar_init(smem_u32(&bar->q_empty[i]), 1);
    }
    for (int s = 0; s < KVS; ++s) {
      mbar_init(smem_u32(&bar->k_full[s]), 1);
      mbar_init(smem_u32(&bar->k_empty[s]), 1);
      mbar_init(smem_u32(&bar->v_full[s]), 1);
      mbar_init(smem_u32(&bar->v_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&bar->s_full[s]), 1);
      mbar_init(smem_u32(&bar->s_free[s]), NSW);
    }
    mbar_init(smem_u32(&bar->p_ready), NSW);
    mbar_init(smem_u32(&bar->o_done), 1);
    mbar_init(smem_u32(&bar->o_free), NSW);
    mbar_init(smem_u32(&bar->drain), 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < NQ * BM; i += blockDim.x)
    reinterpret_cast<volatile int*>(smem + L::OFF_FLAG)[i] = 0;
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
  if (warp == 1) {
    tmem_alloc(smem_u32(&bar->tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_slot;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t o_col = 2 * BN;  // O_0 .. O_{NQ-1} (HD columns each) after the S tiles
  static_assert(2 * BN + NQ * HD <= 512, "TMEM columns");

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ scheduler + TMA producer
      int k = 0;       // items taken (incl. the final "none left")
      int gk = 0;      // K tiles issued
      int gv = 0;      // V tiles issued
      bool ok = true;
      for (; ok; ++k) {
        const int qs = k % QBUF;
        if (!mbar_wait(smem_u32(&bar->q_empty[qs]), ((k / QBUF) & 1) ^ 1, abort_flag, p.err,
                       kErrWaitProducer)) {
          ok = false;
          break;
        }
        int id = atomicAdd(p.work, 1);
        if (id >= p.n_items) id = -1;
        item_slot[qs] = id;
        if (id < 0) {
          mbar_arrive(smem_u32(&bar->q_full[qs]));
          ++k;
          break;
        }
        const Item t = decode(id, p);
        const int row0 = t.b * p.S;
        const int kvh = t.h / group;
        const int qcol = t.h * HD, kcol = (p.nh + kvh) * HD, vcol = (p.nh + p.nkv + kvh) * HD;
        const uint32_t qfb = smem_u32(&bar->q_full[qs]);
        mbar_arrive_expect_tx(qfb, L::Q_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(sbase + L::OFF_Q + qs * L::Q_BYTES + c * L::CHUNK, &tm, qfb, qcol + c * 64,
                      row0 + t.qb * BM);
        // issue order K_0, K_1, V_0, K_2, V_1, ...: a K load never queues behind the V load
        // of the previous tile (whose slot frees only after that tile's P V)
        for (int j = 0; j <= t.nkb && ok; ++j) {
          if (j < t.nkb) {
            const int st = gk % KVS;
            if (!mbar_wait(smem_u32(&bar->k_empty[st]), ((gk / KVS) & 1) ^ 1, abort_flag, p.err,
                           kErrWaitProducer)) {
              ok = false;
              break;
            }
            const uint32_t fb = smem_u32(&bar->k_full[st]);
            mbar_arrive_expect_tx(fb, L::KV_TILE);
#pragma unroll
            for (int c = 0; c < HD / 64; ++c)
              tma_load_2d(sbase + L::OFF_K + st * L::KV_TILE + c * L::CHUNK, &tm, fb,
                          kcol + c * 64, row0 + j * BN);
            ++gk;
          }
          if (j >= 1) {
            const int st = gv % KVS;
            if (!mbar_wait(smem_u32(&bar->v_empty[st]), ((gv / KVS) & 1) ^ 1, abort_flag, p.err,
                           kErrWaitProducer)) {
              ok = false;
              break;
            }
            const uint32_t fb = smem_u32(&bar->v_full[st]);
            mbar_arrive_expect_tx(fb, L::KV_TILE);
#pragma unroll
            for (int c = 0; c < HD / 64; ++c)
              tma_load_2d(sbase + L::OFF_V + st * L::KV_TILE + c * L::CHUNK, &tm, fb,
                          vcol + c * 64, row0 + (j - 1) * BN);
            ++gv;
          }
        }
      }
      // wait for copies in flight (bounded) before the CTA may exit
      tma_drain_ring(bar->k_full, KVS, gk);
      tma_drain_ring(bar->v_full, KVS, gv);
      tma_drain_ring(bar->q_full, QBUF, k);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, false, true);
      int k = 0, g = 0;  // items, K/V (== score) tiles
      for (;; ++k) {
        const int qs = k % QBUF;
        if (!mbar_wait(smem_u32(&bar->q_full[qs]), (k / QBUF) & 1, abort_flag, p.err, kErrWaitMma))
          break;
        const int id = item_slot[qs];
        if (id < 0) break;
        const Item t = decode(id, p);
        tc_fence_after();
        const uint32_t sq = sbase + L::OFF_Q + qs * L::Q_BYTES;
        auto issue_s = [&](int j) -> bool {
          const int gg = g + j, st = gg % KVS, sb = gg & 1;
          if (!mbar_wait(smem_u32(&bar->k_full[st]), (gg / KVS) & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          const int use = gg >> 1;  // previous use of this S tile must have been read
          if (use > 0 &&
              !mbar_wait(smem_u32(&bar->s_free[sb]), (use - 1) & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          tc_fence_after();
          // descriptors of consecutive K steps differ only in the start-address field
          const uint64_t qd = sdesc_sw128(sq, 16, 1024);
          const uint64_t kd = sdesc_sw128(sbase + L::OFF_K + st * L::KV_TILE, 16, 1024);
          const uint32_t dst = tmem + sb * BN;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * L::CHUNK + (kk & 3) * 32) >> 4;
            umma_bf16_ss(dst, qd + off, kd + off, IDESC_S, kk > 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&bar->s_full[sb]));
          umma_commit(smem_u32(&bar->k_empty[st]));
          return true;
        };
        auto issue_pv = [&](int j) -> bool {
          const int gg = g + j, st = gg % KVS;
          if (j == 0 && k > 0 &&
              !mbar_wait(smem_u32(&bar->o_free), (k - 1) & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          if (!mbar_wait(smem_u32(&bar->v_full[st]), (gg / KVS) & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          if (!mbar_wait(smem_u32(&bar->p_ready), gg & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          tc_fence_after();
          const uint64_t vd = sdesc_sw128(sbase + L::OFF_V + st * L::KV_TILE, L::CHUNK, 1024);
          const uint32_t pa = tmem + (gg & 1) * BN;
          const uint32_t acc0 = j > 0 ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            // keys of group q = [q CW, (q + 1) CW) accumulate into O_q; P_j (bf16, two per
            // column) sits in the first CW / 2 columns of the group's CW columns of S_j
            constexpr int KPG = CW / 16;  // K steps per group
            const int q = kk / KPG, kq = kk % KPG;
            umma_bf16_ts(tmem + o_col + q * HD, pa + q * CW + kq * 8, vd + ((kk * 2048) >> 4),
                         IDESC_O, kq > 0 ? 1u : acc0);
          }
          umma_commit(smem_u32(&bar->o_done));
          umma_commit(smem_u32(&bar->v_empty[st]));
          return true;
        };
        bool ok = issue_s(0);
        for (int j = 0; j < t.nkb && ok; ++j) {
          if (j + 1 < t.nkb && !issue_s(j + 1)) ok = false;
          if (ok && !issue_pv(j)) ok = false;
        }
        if (!ok) break;
        umma_commit(smem_u32(&bar->q_empty[qs]));
        g += t.nkb;
      }
      umma_commit(smem_u32(&bar->drain));
      volatile int no_abort = 0;
      mbar_wait(smem_u32(&bar->drain), 0, &no_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue, warps 2-9
    constexpr int OH = HD / NQ;        // output columns per thread in the epilogue
    const int quad = warp & 3;
    const int grp = (warp - 2) >> 2;   // key group: warps 2-5 -> 0, 6-9 -> 1, ...
    const int r = quad * 32 + lane;    // query row in the tile == TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t my_o = o_col + grp * HD;
    const float c = p.scale_log2;
    float* red = reinterpret_cast<float*>(smem + L::OFF_RED);
    volatile int* xflag = reinterpret_cast<volatile int*>(smem + L::OFF_FLAG);
    int k = 0, g = 0;
    bool ok = true;
    for (; ok; ++k) {
      const int qs = k % QBUF;
      if (!mbar_wait(smem_u32(&bar->q_full[qs]), (k / QBUF) & 1, abort_flag, p.err, kErrWaitSoftmax))
        break;
      const int id = item_slot[qs];
      if (id < 0) break;
      const Item t = decode(id, p);
      const int q0 = t.qb * BM;
      const int qpos = q0 + r;
      float m_ref = -CUDART_INF_F;  // running reference max of this group, log2 units
      float l = 0.f;                // running row sum of this group
      for (int j = 0; j < t.nkb; ++j) {
        const int gg = g + j, sb = gg & 1;
        if (!mbar_wait(smem_u32(&bar->s_full[sb]), (gg >> 1) & 1, abort_flag, p.err,
                       kErrWaitSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[CW];
        {
          uint32_t* su = reinterpret_cast<uint32_t*>(sv);
#pragma unroll
          for (int cc = 0; cc < CW / 32; ++cc)
            CFB_TMEM_LD32(lane_addr + sb * BN + grp * CW + cc * 32, (su + cc * 32));
        }
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar->s_free[sb]));
        const int k0 = j * BN + grp * CW;
        if ((k0 + CW - 1 > q0) || (k0 + CW > p.S)) {  // diagonal / ragged block: mask
          const int lim = min(qpos, p.S - 1) - k0;  // keys with index <= lim are visible
#pragma unroll
          for (int i = 0; i < CW; ++i)
            if (i > lim) sv[i] = -CUDART_INF_F;
        }
        float m4[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
        for (int i = 0; i < CW; i += 8) {  // four independent max chains
#pragma unroll
          for (int q = 0; q < 4; ++q) m4[q] = fmax3f(m4[q], sv[i + 2 * q], sv[i + 2 * q + 1]);
        }
        float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        mx *= c;  // raw max -> log2 units (c > 0)
        const bool grow = (mx > m_ref + kRescaleThreshold) || (m_ref == -CUDART_INF_F);
        float alpha = 1.f;
        if (grow) {
          const float m_new = fmaxf(m_ref, mx);
          alpha = (m_ref == -CUDART_INF_F) ? 0.f : ex2_approx(m_ref - m_new);
          m_ref = m_new;
        }
        const float nref = (m_ref == -CUDART_INF_F) ? 0.f : -m_ref;
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[CW / 2];
#pragma unroll
        for (int i = 0; i < CW / 2; ++i) {
          const float e0 = ex2_approx(fmaf(sv[2 * i], c, nref));
          const float e1 = ex2_approx(fmaf(sv[2 * i + 1], c, nref));
          rs[(2 * i) & 3] += e0;
          rs[(2 * i + 1) & 3] += e1;
          pk[i] = pack_bf16x2(e0, e1);
        }
        l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
        // P_{j-1} V_{j-1} must be complete before P_j is written to TMEM (and before O is
        // rescaled).  Writing P_j while that MMA was still in flight corrupted rows of O on
        // B200, although P_j and P_{j-1} occupy different TMEM columns.
        if (gg > 0 &&
            !mbar_wait(smem_u32(&bar->o_done), (gg - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // P_j (bf16, CW / 2 columns) overwrites the first half of this thread's CW S columns
        if constexpr (CW == 64) {
          CFB_TMEM_ST32(lane_addr + sb * BN + grp * CW, pk);
        } else {
          CFB_TMEM_ST16(lane_addr + sb * BN + grp * CW, pk);
        }
        if (j > 0 && __any_sync(0xffffffffu, grow)) {  // a grown max rescales this group's O
#pragma unroll
          for (int cc = 0; cc < HD / 32; ++cc) {
            uint32_t o[32];
            CFB_TMEM_LD32(lane_addr + my_o + cc * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            CFB_TMEM_ST32(lane_addr + my_o + cc * 32, o);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar->p_ready));
      }
      if (!ok) break;
      // epilogue: merge the NQ groups' (m, l, O) once, write O / l and the LSE
      const int gl = g + t.nkb - 1;
      if (!mbar_wait(smem_u32(&bar->o_done), gl & 1, abort_flag, p.err, kErrWaitSoftmax)) break;
      tc_fence_after();
      float mq[NQ], lq[NQ];
      if (!group_exchange<NQ>(red, xflag, 0, grp, r, 2 * k + 1, m_ref, mq, abort_flag, p.err) ||
          !group_exchange<NQ>(red, xflag, 1, grp, r, 2 * k + 2, l, lq, abort_flag, p.err))
        break;
      float M = mq[0];
#pragma unroll
      for (int q = 1; q < NQ; ++q) M = fmaxf(M, mq[q]);
      float fq[NQ], Lt = 0.f;
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        fq[q] = (mq[q] == -CUDART_INF_F) ? 0.f : ex2_approx(mq[q] - M);
        Lt += lq[q] * fq[q];
      }
      const float inv = Lt > 0.f ? 1.f / Lt : 0.f;
#pragma unroll
      for (int q = 0; q < NQ; ++q) fq[q] *= inv;
      const int row0 = t.b * p.S;
      // this thread writes output columns [grp OH, (grp + 1) OH) of its row
      __nv_bfloat16* dst = p.out + static_cast<long long>(row0 + min(qpos, p.S - 1)) * p.ld_out +
                           t.h * HD + grp * OH;
      constexpr int CH = OH < 32 ? OH : 32;  // columns per TMEM load
#pragma unroll
      for (int cc = 0; cc < OH / CH; ++cc) {
        float v[CH];
#pragma unroll
        for (int e = 0; e < CH; ++e) v[e] = 0.f;
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
          uint32_t a[CH];
          if constexpr (CH == 32) {
            CFB_TMEM_LD32(lane_addr + o_col + q * HD + grp * OH + cc * CH, a);
          } else {
            CFB_TMEM_LD16(lane_addr + o_col + q * HD + grp * OH + cc * CH, a);
          }
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < CH; ++e) v[e] = fmaf(__uint_as_float(a[e]), fq[q], v[e]);
        }
        if (qpos < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + cc * CH);
#pragma unroll
          for (int kq = 0; kq < CH / 8; ++kq) {
            uint4 u;
            u.x = pack_bf16x2(v[8 * kq + 0], v[8 * kq + 1]);
            u.y = pack_bf16x2(v[8 * kq + 2], v[8 * kq + 3]);
            u.z = pack_bf16x2(v[8 * kq + 4], v[8 * kq + 5]);
            u.w = pack_bf16x2(v[8 * kq + 6], v[8 * kq + 7]);
            d4[kq] = u;
          }
        }
      }
      if (qpos < p.S && grp == 0)
        p.lse[static_cast<long long>(row0 + qpos) * p.nh + t.h] = (M + log2f(Lt)) * kLn2;
      // O read: the next item's first PV may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar->o_free));
      g += t.nkb;
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

// ------------------------------------------------------------------ two-tile ("ping-pong") form
// Work item: one 128-query block of TWO heads of the same GQA group (heads 2 hp, 2 hp + 1 share
// their K/V head, so both query tiles walk the same K_j / V_j tiles and the same causal range).
// Each tile has its own softmax group of four warps (one per TMEM lane quadrant; a thread owns a
// whole query row and all 128 keys of a step) and its own S and O in TMEM:
//   TMEM columns  [0, 128) S_A (P_A packed bf16 into the first 64)   [128, 256) S_B
//                 [256, 256 + HD) O_A                                 [256 + HD, 256 + 2 HD) O_B
// MMA issue order per key step j:  P_A V_j, S_A(j+1) = Q_A K_{j+1}^T, P_B V_j, S_B(j+1).  Tile
// A's softmax of step j+1 thus runs while the tensor cores do tile B's P V and next scores, and
// the other way round, so the exponentials of one tile overlap the other tile's MMAs.  A tile's
// S is rewritten only by the MMA after its own P V (issued in order by one thread), and the
// scores of step j being ready imply that P V of step j-1 is complete, which makes the O
// rescale of step j safe without a further wait.
template <int HD>
struct SmemPP {
  static constexpr int QBUF = HD == 64 ? 2 : 1;       // items whose Q tiles are in flight
  static constexpr int KV_STAGES = HD == 64 ? 4 : 2;  // slots of each of the K and V rings
  static constexpr int CHUNK = BM * 128;              // 128 rows x 128 B (64 bf16)
  static constexpr int Q_TILE = (HD / 64) * CHUNK;    // one head's Q [128 x HD]
  static constexpr int Q_BYTES = 2 * Q_TILE;          // both tiles of an item
  static constexpr int KV_TILE = (HD / 64) * CHUNK;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + QBUF * Q_BYTES;
  static constexpr int OFF_V = OFF_K + KV_STAGES * KV_TILE;
  static constexpr int OFF_BAR = OFF_V + KV_STAGES * KV_TILE;
  static constexpr int THREADS = 64 + 2 * 128;        // TMA + MMA warps, 2 x 4 softmax warps
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
  static_assert(KV_STAGES <= MAX_RING && QBUF <= 2, "rings");
  static_assert(BYTES <= 232448, "shared memory per CTA");
};

struct BarsPP {
  uint64_t q_full[2], q_empty[2], k_full[MAX_RING], k_empty[MAX_RING], v_full[MAX_RING],
      v_empty[MAX_RING], s_full[2], p_ready[2], o_done[2], o_free[2], drain;
  int item[2];
  uint32_t tmem_slot;
  int abort;
};

// item id -> (query block, first head of the pair, batch); heaviest query blocks first
__device__ __forceinline__ Item decode_pp(int id, const Params& p) {
  const int nhp = p.nh >> 1;
  Item t;
  t.qb = p.nqb - 1 - id / (nhp * p.B);
  const int rem = id % (nhp * p.B);
  t.h = 2 * (rem % nhp);
  t.b = rem / nhp;
  const int last_q = min(p.S, (t.qb + 1) * BM) - 1;
  t.nkb = last_q / BN + 1;
  return t;
}

// PE: every PE-th pair of scores takes the software exponential (0: all on MUFU)
template <int HD, int PE = 0>
__global__ void __launch_bounds__(SmemPP<HD>::THREADS, 1)
    attn_fwd_pp_kernel(const __grid_constant__ CUtensorMap tm, const Params p) {
  using L = SmemPP<HD>;
  constexpr int QBUF = L::QBUF, KVS = L::KV_STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  BarsPP* bar = reinterpret_cast<BarsPP*>(smem + L::OFF_BAR);
  volatile int* abort_flag = &bar->abort;
  volatile int* item_slot = bar->item;
  const int warp = warp_id(), lane = lane_id();
  const int group = p.nh / p.nkv;

  if (threadIdx.x == 0) {
    for (int i = 0; i < QBUF; ++i) {
      mbar_init(smem_u32(&bar->q_full[i]), 1);
      mbar_init(smem_u32(&bar->q_empty[i]), 1);
    }
    for (int s = 0; s < KVS; ++s) {
      mbar_init(smem_u32(&bar->k_full[s]), 1);
      mbar_init(smem_u32(&bar->k_empty[s]), 1);
      mbar_init(smem_u32(&bar->v_full[s]), 1);
      mbar_init(smem_u32(&bar->v_empty[s]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(smem_u32(&bar->s_full[t]), 1);
      mbar_init(smem_u32(&bar->p_ready[t]), 4);
      mbar_init(smem_u32(&bar->o_done[t]), 1);
      mbar_init(smem_u32(&bar->o_free[t]), 4);
    }
    mbar_init(smem_u32(&bar->drain), 1);
    bar->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
  if (warp == 1) {
    tmem_alloc(smem_u32(&bar->tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_slot;
  const uint32_t sbase = smem_u32(smem);
  constexpr uint32_t kOCol = 2 * BN;  // O_A, O_B after the two S tiles
  static_assert(2 * BN + 2 * HD <= 512, "TMEM columns");

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ scheduler + TMA producer
      int k = 0, gk = 0, gv = 0;
      bool ok = true;
      for (; ok; ++k) {
        const int qs = k % QBUF;
        if (!mbar_wait(smem_u32(&bar->q_empty[qs]), ((k / QBUF) & 1) ^ 1, abort_flag, p.err,
                       kErrWaitProducer)) {
          ok = false;
          break;
        }
        int id = atomicAdd(p.work, 1);
        if (id >= p.n_items) id = -1;
        item_slot[qs] = id;
        if (id < 0) {
          mbar_arrive(smem_u32(&bar->q_full[qs]));
          ++k;
          break;
        }
        const Item t = decode_pp(id, p);
        const int row0 = t.b * p.S;
        const int kvh = t.h / group;
        const int kcol = (p.nh + kvh) * HD, vcol = (p.nh + p.nkv + kvh) * HD;
        const uint32_t qfb = smem_u32(&bar->q_full[qs]);
        mbar_arrive_expect_tx(qfb, L::Q_BYTES);
#pragma unroll
        for (int tt = 0; tt < 2; ++tt)
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(sbase + L::OFF_Q + qs * L::Q_BYTES + tt * L::Q_TILE + c * L::CHUNK, &tm,
                        qfb, (t.h + tt) * HD + c * 64, row0 + t.qb * BM);
        // K_0, K_1, V_0, K_2, V_1, ...: a K load never queues behind the previous tile's V
        for (int j = 0; j <= t.nkb && ok; ++j) {
          if (j < t.nkb) {
            const int st = gk % KVS;
            if (!mbar_wait(smem_u32(&bar->k_empty[st]), ((gk / KVS) & 1) ^ 1, abort_flag, p.err,
                           kErrWaitProducer)) {
              ok = false;
              break;
            }
            const uint32_t fb = smem_u32(&bar->k_full[st]);
            mbar_arrive_expect_tx(fb, L::KV_TILE);
#pragma unroll
            for (int c = 0; c < HD / 64; ++c)
              tma_load_2d(sbase + L::OFF_K + st * L::KV_TILE + c * L::CHUNK, &tm, fb,
                          kcol + c * 64, row0 + j * BN);
            ++gk;
          }
          if (j >= 1) {
            const int st = gv % KVS;
            if (!mbar_wait(smem_u32(&bar->v_empty[st]), ((gv / KVS) & 1) ^ 1, abort_flag, p.err,
                           kErrWaitProducer)) {
              ok = false;
              break;
            }
            const uint32_t fb = smem_u32(&bar->v_full[st]);
            mbar_arrive_expect_tx(fb, L::KV_TILE);
#pragma unroll
            for (int c = 0; c < HD / 64; ++c)
              tma_load_2d(sbase + L::OFF_V + st * L::KV_TILE + c * L::CHUNK, &tm, fb,
                          vcol + c * 64, row0 + (j - 1) * BN);
            ++gv;
          }
        }
      }
      tma_drain_ring(bar->k_full, KVS, gk);
      tma_drain_ring(bar->v_full, KVS, gv);
      tma_drain_ring(bar->q_full, QBUF, k);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, false, true);
      int k = 0, g = 0;  // items, key steps
      bool ok = true;
      for (; ok; ++k) {
        const int qs = k % QBUF;
        if (!mbar_wait(smem_u32(&bar->q_full[qs]), (k / QBUF) & 1, abort_flag, p.err, kErrWaitMma))
          break;
        const int id = item_slot[qs];
        if (id < 0) break;
        const Item t = decode_pp(id, p);
        tc_fence_after();
        // S_t(j) = Q_t K_j^T into tile t's S columns (K slot of step j already full)
        auto issue_s = [&](int tt, int j) {
          const int st = (g + j) % KVS;
          const uint64_t qd = sdesc_sw128(sbase + L::OFF_Q + qs * L::Q_BYTES + tt * L::Q_TILE,
                                          16, 1024);
          const uint64_t kd = sdesc_sw128(sbase + L::OFF_K + st * L::KV_TILE, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = ((kk >> 2) * L::CHUNK + (kk & 3) * 32) >> 4;
            umma_bf16_ss(tmem + tt * BN, qd + off, kd + off, IDESC_S, kk > 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&bar->s_full[tt]));
        };
        auto wait_k = [&](int j) -> bool {
          const int gg = g + j;
          if (!mbar_wait(smem_u32(&bar->k_full[gg % KVS]), (gg / KVS) & 1, abort_flag, p.err,
                         kErrWaitMma))
            return false;
          tc_fence_after();
          return true;
        };
        // O_t += P_t(j) V_j once tile t's softmax has written P_t(j)
        auto issue_pv = [&](int tt, int j) -> bool {
          const int gg = g + j, st = gg % KVS;
          if (j == 0 && k > 0 &&
              !mbar_wait(smem_u32(&bar->o_free[tt]), (k - 1) & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          if (!mbar_wait(smem_u32(&bar->p_ready[tt]), gg & 1, abort_flag, p.err, kErrWaitMma))
            return false;
          tc_fence_after();
          const uint64_t vd = sdesc_sw128(sbase + L::OFF_V + st * L::KV_TILE, L::CHUNK, 1024);
          const uint32_t pa = tmem + tt * BN;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            umma_bf16_ts(tmem + kOCol + tt * HD, pa + kk * 8, vd + ((kk * 2048) >> 4), IDESC_O,
                         (kk > 0 || j > 0) ? 1u : 0u);
          return true;
        };
        ok = wait_k(0);
        if (ok) {
          issue_s(0, 0);
          issue_s(1, 0);
          umma_commit(smem_u32(&bar->k_empty[g % KVS]));
        }
        for (int j = 0; j < t.nkb && ok; ++j) {
          const int gg = g + j;
          if (!mbar_wait(smem_u32(&bar->v_full[gg % KVS]), (gg / KVS) & 1, abort_flag, p.err,
                         kErrWaitMma)) {
            ok = false;
            break;
          }
          const bool more = j + 1 < t.nkb;
          if (more && !wait_k(j + 1)) {
            ok = false;
            break;
          }
          if (!issue_pv(0, j)) {
            ok = false;
            break;
          }
          if (!more) umma_commit(smem_u32(&bar->o_done[0]));
          if (more) issue_s(0, j + 1);
          if (!issue_pv(1, j)) {
            ok = false;
            break;
          }
          umma_commit(smem_u32(&bar->v_empty[gg % KVS]));
          if (more) {
            issue_s(1, j + 1);
            umma_commit(smem_u32(&bar->k_empty[(gg + 1) % KVS]));
          } else {
            umma_commit(smem_u32(&bar->o_done[1]));
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&bar->q_empty[qs]));
        g += t.nkb;
      }
      umma_commit(smem_u32(&bar->drain));
      volatile int no_abort = 0;
      mbar_wait(smem_u32(&bar->drain), 0, &no_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue, warps 2-9
    const int quad = warp & 3;
    const int tt = (warp - 2) >> 2;  // tile: warps 2-5 -> A (head 2 hp), 6-9 -> B (2 hp + 1)
    const int r = quad * 32 + lane;  // query row in the tile == TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t s_col = tt * BN, o_col = kOCol + tt * HD;
    const float c = p.scale_log2;
    int k = 0, g = 0;
    bool ok = true;
    for (; ok; ++k) {
      const int qs = k % QBUF;
      if (!mbar_wait(smem_u32(&bar->q_full[qs]), (k / QBUF) & 1, abort_flag, p.err, kErrWaitSoftmax))
        break;
      const int id = item_slot[qs];
      if (id < 0) break;
      const Item t = decode_pp(id, p);
      const int q0 = t.qb * BM;
      const int qpos = q0 + r;
      float m_ref = -CUDART_INF_F;  // running reference max, log2 units
      float l = 0.f;                // running row sum
      for (int j = 0; j < t.nkb; ++j) {
        const int gg = g + j;
        if (!mbar_wait(smem_u32(&bar->s_full[tt]), gg & 1, abort_flag, p.err, kErrWaitSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sv[BN];
        {
          uint32_t* su = reinterpret_cast<uint32_t*>(sv);
#pragma unroll
          for (int cc = 0; cc < BN / 32; ++cc) CFB_TMEM_LD32(lane_addr + s_col + cc * 32, (su + cc * 32));
        }
        tmem_ld_wait();
        const int k0 = j * BN;
        if ((k0 + BN - 1 > q0) || (k0 + BN > p.S)) {  // diagonal / ragged block: mask
          const int lim = min(qpos, p.S - 1) - k0;  // keys with index <= lim are visible
#pragma unroll
          for (int i = 0; i < BN; ++i)
            if (i > lim) sv[i] = -CUDART_INF_F;
        }
        float m4[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
        for (int i = 0; i < BN; i += 8) {
#pragma unroll
          for (int q = 0; q < 4; ++q) m4[q] = fmax3f(m4[q], sv[i + 2 * q], sv[i + 2 * q + 1]);
        }
        const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * c;
        const bool grow = (mx > m_ref + kRescaleThreshold) || (m_ref == -CUDART_INF_F);
        float alpha = 1.f;
        if (grow) {
          const float m_new = fmaxf(m_ref, mx);
          alpha = (m_ref == -CUDART_INF_F) ? 0.f : ex2_approx(m_ref - m_new);
          m_ref = m_new;
        }
        const float nref = (m_ref == -CUDART_INF_F) ? 0.f : -m_ref;
        float rs[4] = {0.f, 0.f, 0.f, 0.f};
        // P (bf16, two keys per column) over the first 64 of the tile's 128 S columns; the whole
        // row of S is already in registers
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float x0 = fmaf(sv[cc * 32 + 2 * i], c, nref);
            const float x1 = fmaf(sv[cc * 32 + 2 * i + 1], c, nref);
            const bool soft = PE > 0 && (i % (PE > 0 ? PE : 1)) == (PE > 0 ? PE : 1) - 1;
            const float e0 = soft ? ex2_poly(x0) : ex2_approx(x0);
            const float e1 = soft ? ex2_poly(x1) : ex2_approx(x1);
            rs[(2 * i) & 3] += e0;
            rs[(2 * i + 1) & 3] += e1;
            pk[i] = pack_bf16x2(e0, e1);
          }
          CFB_TMEM_ST16(lane_addr + s_col + cc * 16, pk);
        }
        l = l * alpha + ((rs[0] + rs[1]) + (rs[2] + rs[3]));
        // a grown max rescales O (P V of step j-1 is complete: S of step j was issued after it)
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int cc = 0; cc < HD / 32; ++cc) {
            uint32_t o[32];
            CFB_TMEM_LD32(lane_addr + o_col + cc * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            CFB_TMEM_ST32(lane_addr + o_col + cc * 32, o);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar->p_ready[tt]));
      }
      if (!ok) break;
      // epilogue: O / l and the LSE of this tile's head
      if (!mbar_wait(smem_u32(&bar->o_done[tt]), k & 1, abort_flag, p.err, kErrWaitSoftmax)) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int row0 = t.b * p.S, h = t.h + tt;
      __nv_bfloat16* dst =
          p.out + static_cast<long long>(row0 + min(qpos, p.S - 1)) * p.ld_out + h * HD;
#pragma unroll
      for (int cc = 0; cc < HD / 32; ++cc) {
        uint32_t a[32];
        CFB_TMEM_LD32(lane_addr + o_col + cc * 32, a);
        tmem_ld_wait();
        if (qpos < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + cc * 32);
#pragma unroll
          for (int kq = 0; kq < 4; ++kq) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(a[8 * kq + 0]) * inv, __uint_as_float(a[8 * kq + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(a[8 * kq + 2]) * inv, __uint_as_float(a[8 * kq + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(a[8 * kq + 4]) * inv, __uint_as_float(a[8 * kq + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(a[8 * kq + 6]) * inv, __uint_as_float(a[8 * kq + 7]) * inv);
            d4[kq] = u;
          }
        }
      }
      if (qpos < p.S)
        p.lse[static_cast<long long>(row0 + qpos) * p.nh + h] = (m_ref + log2f(l)) * kLn2;
      // O read: the next item's first P V of this tile may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar->o_free[tt]));
      g += t.nkb;
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

// y[i] = ex2_poly(x[i]): the software exponential on its own, for accuracy tests
__global__ void ex2_poly_kernel(const float* __restrict__ x, float* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = ex2_poly(x[i]);
}

int make_tmap_qkv(CUtensorMap* map, const void* qkv, long long rows, long long ld);

template <int HD>
int launch(const void* qkv, long long ld, void* out, long long ld_out, float* lse, int B, int S,
           int nh, int nkv, float scale, int* work, int* err, cudaStream_t st) {
  CUtensorMap tm;
  const int rc = make_tmap_qkv(&tm, qkv, static_cast<long long>(B) * S, ld);
  if (rc) return rc;
  Params p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.ld = ld;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.lse = lse;
  p.B = B;
  p.S = S;
  p.nh = nh;
  p.nkv = nkv;
  p.nqb = (S + BM - 1) / BM;
  p.n_items = p.nqb * nh * B;
  p.scale_log2 = scale * kLog2e;
  p.work = work;
  p.err = err;
  static int n_sm = 0;
  if (n_sm == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  }
  // Two-tile kernel when head pairs share a K/V head (even GQA group); CFB_ATTN_PP=0 keeps the
  // one-tile kernel.
  static const bool pp_on = [] {
    const char* e = std::getenv("CFB_ATTN_PP");
    return !(e && e[0] == '0');
  }();
  // CFB_ATTN_POLY=n (4 or 8): every n-th pair of scores uses the FMA-pipe exponential
  static const int poly = [] {
    const char* e = std::getenv("CFB_ATTN_POLY");
    return e ? std::atoi(e) : 0;
  }();
  if (pp_on && (nh / nkv) % 2 == 0) {
    p.n_items = p.nqb * (nh / 2) * B;
    auto kpp = poly == 4 ? attn_fwd_pp_kernel<HD, 4>
             : poly == 8 ? attn_fwd_pp_kernel<HD, 8> : attn_fwd_pp_kernel<HD, 0>;
    static bool configured_pp[3] = {false, false, false};
    const int pi = poly == 4 ? 1 : poly == 8 ? 2 : 0;
    if (!configured_pp[pi]) {
      cudaFuncSetAttribute(kpp, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemPP<HD>::BYTES);
      configured_pp[pi] = true;
    }
    const int grid = p.n_items < n_sm ? p.n_items : n_sm;
    kpp<<<grid, SmemPP<HD>::THREADS, SmemPP<HD>::BYTES, st>>>(tm, p);
    return cudaGetLastError() == cudaSuccess ? 0 : -3;
  }
  auto kern = attn_fwd_tc_kernel<HD>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<HD>::BYTES);
    configured = true;
  }
  const int grid = p.n_items < n_sm ? p.n_items : n_sm;
  kern<<<grid, Smem<HD>::THREADS, Smem<HD>::BYTES, st>>>(tm, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace attn_tc

int make_tmap_2d_bf16(CUtensorMap* map, const void* ptr, long long rows, long long cols,
                      long long ld, int box_cols, int box_rows);

int attn_tc::make_tmap_qkv(CUtensorMap* map, const void* qkv, long long rows, long long ld) {
  return make_tmap_2d_bf16(map, qkv, rows, ld, ld, 64, 128);
}

}  // namespace cfb

int cfb_attn_fwd_tc(const void* qkv, long long ld_qkv, void* out, long long ld_out, float* lse,
                    int B, int S, int nh, int nkv, int hd, float scale, int* work, int* err,
                    cudaStream_t st) {
  if (ld_qkv % 8 || ld_out % 8 || nh % nkv || !work) return -11;
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return -12;
  if (hd == 64)
    return cfb::attn_tc::launch<64>(qkv, ld_qkv, out, ld_out, lse, B, S, nh, nkv, scale, work,
                                    err, st);
  if (hd == 128)
    return cfb::attn_tc::launch<128>(qkv, ld_qkv, out, ld_out, lse, B, S, nh, nkv, scale, work,
                                     err, st);
  return -12;
}

int cfb_ex2_poly(const float* x, float* y, int n, cudaStream_t st) {
  if (n <= 0) return n == 0 ? 0 : -11;
  cfb::attn_tc::ex2_poly_kernel<<<(n + 255) / 256, 256, 0, st>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
