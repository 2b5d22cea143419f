// Causal GQA attention forward on the 5th-generation tensor cores (sm_100a).
//
// One CTA computes 128 query rows of one head against the causal key range, 128 keys per step:
//   warp 0      TMA producer: Q once, then K_j / V_j tiles (2-stage ring) from the fused qkv rows
//   warp 1      MMA issuer:   S_j = Q K_j^T into one of two TMEM tiles (128 x 128 fp32), then
//                             O += P_j V_j into the TMEM accumulator (128 x hd fp32)
//   warps 2-9   softmax:      two threads per query row (= TMEM lane): warps w and w+4 share a
//                             lane quadrant and take keys [0, 64) / [64, 128) of every step.
//                             Each half keeps its own running max, row sum and O accumulator
//                             (O0, O1 in TMEM, fed by two K=64 PV MMAs), so the halves never
//                             synchronise per step; the epilogue merges them once
//                             (O = O0 2^(m0-m) + O1 2^(m1-m), same for l).  Online softmax in
//                             fp32 with one FMA + ex2 per score, P written to shared memory as
//                             bf16 (128B-swizzled K-major operand); a running max only moves
//                             (and its O is rescaled in TMEM) when it grows by more than 2^8
// S_{j+1} is issued before P_j V_j so that the tensor cores compute the next scores while the
// softmax warps work on the current ones.  Q, K and V are read straight from the fused
// [T, (nh + 2 nkv) hd] qkv rows with one 2-D tensor map (box 64 x 128): K tiles serve as the
// K-major B operand of Q K^T and V tiles, bit-identical in shared memory, as the MN-major B
// operand of P V.  All waits are bounded (sm100_common.cuh).
#include "sm100_common.cuh"
#include "launch_api.h"

#include <math_constants.h>

namespace cfb {
namespace attn_tc {

constexpr int BM = 128, BN = 128;
constexpr int KV_STAGES = 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int HD>
struct Smem {
  static constexpr int CHUNK = BM * 128;                  // 128 rows x 128 B (64 bf16)
  static constexpr int Q_BYTES = (HD / 64) * CHUNK;       // Q [128 x HD], K-major chunks
  static constexpr int KV_TILE = (HD / 64) * CHUNK;       // K_j or V_j [128 x HD]
  static constexpr int P_BYTES = 2 * CHUNK;               // P [128 x 128 keys], 2 K-chunks
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + KV_STAGES * KV_TILE;
  static constexpr int OFF_P = OFF_V + KV_STAGES * KV_TILE;
  static constexpr int OFF_RED = OFF_P + P_BYTES;  // epilogue exchange: [2][2 half][128] fp32
  static constexpr int OFF_FLAG = OFF_RED + 3 * 2 * BM * 4;  // [2 half][128] exchange counters
  static constexpr int OFF_BAR = OFF_FLAG + 2 * BM * 4;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;     // + barriers + alignment slack
};

struct Params {
  const __nv_bfloat16* qkv;
  long long ld;
  __nv_bfloat16* out;
  long long ld_out;
  float* lse;
  int S, nh, nkv;
  float scale_log2;
  int* err;
};

// Hardware base-2 exponential (MUFU); flushes denormal results to zero.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

// Exchange one float per row with the partner warp of the same lane quadrant.  Each side
// publishes its value and a sequence number in shared memory and spins (bounded) until the
// partner's sequence number arrives; values are double-buffered by sequence parity so a slot is
// only rewritten after the partner has read it.  Returns false if the wait gave up.
__device__ __forceinline__ bool pair_exchange(float* vals, volatile int* flags, int slot_base,
                                              int half, int r, int seq, float mine, float& theirs,
                                              volatile int* abort_flag, int* err) {
  constexpr int BMr = 128;
  vals[(slot_base + half) * BMr + r] = mine;
  __threadfence_block();
  flags[half * BMr + r] = seq;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (flags[(half ^ 1) * BMr + r] < seq) {
    if ((++spins & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        atomicCAS(err, 0, kErrWaitSoftmax);
        return false;
      }
    }
  }
  __threadfence_block();
  theirs = vals[(slot_base + (half ^ 1)) * BMr + r];
  return true;
}

template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm, Params p) {
  using L = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + KV_STAGES;
  uint64_t* s_full = kv_empty + KV_STAGES;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_ready = s_free + 2;
  uint64_t* o_done = p_ready + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.nh / p.nkv);
  const int q0 = qb * BM;
  const int row0 = b * p.S;
  const int last_q = min(p.S, q0 + BM) - 1;
  const int nkb = last_q / BN + 1;
  const int qcol = h * HD, kcol = (p.nh + g) * HD, vcol = (p.nh + p.nkv + g) * HD;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(smem_u32(&kv_full[s]), 1);
      mbar_init(smem_u32(&kv_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&s_full[s]), 1);
      mbar_init(smem_u32(&s_free[s]), 8);
    }
    mbar_init(smem_u32(p_ready), 8);
    mbar_init(smem_u32(o_done), 1);
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 2 * BM; i += blockDim.x)
    reinterpret_cast<volatile int*>(smem + L::OFF_FLAG)[i] = 0;
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tm);
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t o_col = 2 * BN;  // O0, O1 accumulators (HD columns each) after the S tiles

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- producer
      mbar_arrive_expect_tx(smem_u32(q_full), L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        tma_load_2d(sbase + L::OFF_Q + c * L::CHUNK, &tm, smem_u32(q_full), qcol + c * 64,
                    row0 + q0);
      int issued = 0;
      for (int j = 0; j < nkb; ++j, ++issued) {
        const int st = j % KV_STAGES;
        if (!mbar_wait(smem_u32(&kv_empty[st]), ((j / KV_STAGES) & 1) ^ 1, abort_flag, p.err,
                       kErrWaitProducer))
          break;
        const uint32_t fb = smem_u32(&kv_full[st]);
        mbar_arrive_expect_tx(fb, 2 * L::KV_TILE);
        const int k0 = row0 + j * BN;
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d(sbase + L::OFF_K + st * L::KV_TILE + c * L::CHUNK, &tm, fb, kcol + c * 64, k0);
          tma_load_2d(sbase + L::OFF_V + st * L::KV_TILE + c * L::CHUNK, &tm, fb, vcol + c * 64, k0);
        }
      }
      tma_drain_ring(kv_full, KV_STAGES, issued);
      tma_drain_ring(q_full, 1, 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, false, true);
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, p.err, kErrWaitMma);
      auto issue_s = [&](int j) -> bool {
        const int st = j % KV_STAGES, sb = j & 1;
        if (!mbar_wait(smem_u32(&kv_full[st]), (j / KV_STAGES) & 1, abort_flag, p.err, kErrWaitMma))
          return false;
        const int use = j >> 1;  // previous use of this S tile must have been read
        if (use > 0 &&
            !mbar_wait(smem_u32(&s_free[sb]), (use - 1) & 1, abort_flag, p.err, kErrWaitMma))
          return false;
        tc_fence_after();
        const uint32_t kst = sbase + L::OFF_K + st * L::KV_TILE;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::CHUNK + (kk & 3) * 32;
          umma_bf16_ss(tmem + sb * BN, sdesc_sw128(sbase + L::OFF_Q + off, 16, 1024),
                       sdesc_sw128(kst + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(&s_full[sb]));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkb && ok; ++j) {
        if (j + 1 < nkb && !issue_s(j + 1)) break;
        if (!mbar_wait(smem_u32(p_ready), j & 1, abort_flag, p.err, kErrWaitMma)) break;
        tc_fence_after();
        const int st = j % KV_STAGES;
        const uint32_t vst = sbase + L::OFF_V + st * L::KV_TILE;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // keys [0, 64) accumulate into O0, keys [64, 128) into O1
          const int hh = kk >> 2;
          const uint32_t aoff = hh * L::CHUNK + (kk & 3) * 32;
          umma_bf16_ss(tmem + o_col + hh * HD, sdesc_sw128(sbase + L::OFF_P + aoff, 16, 1024),
                       sdesc_sw128(vst + kk * 2048, L::CHUNK, 1024), IDESC_O,
                       (j > 0 || (kk & 3) > 0) ? 1u : 0u);
        }
        umma_commit(smem_u32(o_done));
        umma_commit(smem_u32(&kv_empty[st]));
      }
      umma_commit(smem_u32(drain));
      volatile int dummy = 0;
      mbar_wait(smem_u32(drain), 0, &dummy, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------------ softmax (warps 2..9)
    constexpr int HALF = BN / 2;       // keys per thread per step
    constexpr int OH = HD / 2;         // output columns per thread in the epilogue
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // 0: warps 2-5, 1: warps 6-9
    const int r = quad * 32 + lane;    // query row in the tile == TMEM lane
    const int qpos = q0 + r;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t my_o = o_col + half * HD;
    const float c = p.scale_log2;
    float m_ref = -CUDART_INF_F;  // running reference max of this half, log2 units
    float l = 0.f;                // running row sum of this half
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(smem_u32(&s_full[sb]), (j >> 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[HALF];
      {
        uint32_t* su = reinterpret_cast<uint32_t*>(sv);
#pragma unroll
        for (int cc = 0; cc < HALF / 32; ++cc)
          CFB_TMEM_LD32(lane_addr + sb * BN + half * HALF + cc * 32, (su + cc * 32));
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s_free[sb]));
      const int k0 = j * BN + half * HALF;
      if ((k0 + HALF - 1 > q0) || (k0 + HALF > p.S)) {  // diagonal / ragged block: mask
        const int lim = min(qpos, p.S - 1) - k0;      // keys with index <= lim are visible
#pragma unroll
        for (int i = 0; i < HALF; ++i)
          if (i > lim) sv[i] = -CUDART_INF_F;
      }
      float mx = -CUDART_INF_F;
#pragma unroll
      for (int i = 0; i < HALF; i += 2) mx = fmax3f(mx, sv[i], sv[i + 1]);
      mx *= c;  // raw max -> log2 units (c > 0)
      const bool grow = (mx > m_ref + kRescaleThreshold) || (m_ref == -CUDART_INF_F);
      float alpha = 1.f;
      if (grow) {
        const float m_new = fmaxf(m_ref, mx);
        alpha = (m_ref == -CUDART_INF_F) ? 0.f : ex2_approx(m_ref - m_new);
        m_ref = m_new;
      }
      const float nref = (m_ref == -CUDART_INF_F) ? 0.f : -m_ref;
      float rs0 = 0.f, rs1 = 0.f;
      uint32_t pk[HALF / 2];
#pragma unroll
      for (int i = 0; i < HALF / 2; ++i) {
        const float e0 = ex2_approx(fmaf(sv[2 * i], c, nref));
        const float e1 = ex2_approx(fmaf(sv[2 * i + 1], c, nref));
        rs0 += e0;
        rs1 += e1;
        pk[i] = pack_bf16x2(e0, e1);
      }
      l = l * alpha + (rs0 + rs1);
      // P_{j-1} V_{j-1} must be complete before P is overwritten and O rescaled
      if (j > 0 &&
          !mbar_wait(smem_u32(o_done), (j - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int cc = 0; cc < HD / 32; ++cc) {
          uint32_t o[32];
          CFB_TMEM_LD32(lane_addr + my_o + cc * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          CFB_TMEM_ST32(lane_addr + my_o + cc * 32, o);
        }
        tmem_st_wait();
      }
      // this thread's 64 keys of the P row = K-chunk `half` of the PV operand (128B swizzle)
      const uint32_t rowbase = sbase + L::OFF_P + half * L::CHUNK + r * 128;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        st_shared_v4(rowbase + ((i ^ (r & 7)) << 4), pk[4 * i], pk[4 * i + 1], pk[4 * i + 2],
                     pk[4 * i + 3]);
      fence_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(p_ready));
    }
    // epilogue: merge the two halves' (m, l, O) once, write O / l and the LSE
    if (ok && mbar_wait(smem_u32(o_done), (nkb - 1) & 1, abort_flag, p.err, kErrWaitSoftmax)) {
      tc_fence_after();
      float* red = reinterpret_cast<float*>(smem + L::OFF_RED);
      volatile int* xflag = reinterpret_cast<volatile int*>(smem + L::OFF_FLAG);
      float m_o = 0.f, l_o = 0.f;
      ok = pair_exchange(red, xflag, 0, half, r, 1, m_ref, m_o, abort_flag, p.err) &&
           pair_exchange(red, xflag, 2, half, r, 2, l, l_o, abort_flag, p.err);
      const float m0 = half == 0 ? m_ref : m_o, m1 = half == 0 ? m_o : m_ref;
      const float l0 = half == 0 ? l : l_o, l1 = half == 0 ? l_o : l;
      const float M = fmaxf(m0, m1);
      const float f0 = (m0 == -CUDART_INF_F) ? 0.f : ex2_approx(m0 - M);
      const float f1 = (m1 == -CUDART_INF_F) ? 0.f : ex2_approx(m1 - M);
      const float Lt = l0 * f0 + l1 * f1;
      const float inv = Lt > 0.f ? 1.f / Lt : 0.f;
      const float g0 = f0 * inv, g1 = f1 * inv;
      __nv_bfloat16* dst = p.out + static_cast<long long>(row0 + qpos) * p.ld_out + h * HD + half * OH;
#pragma unroll
      for (int cc = 0; cc < OH / 32; ++cc) {
        uint32_t a0[32], a1[32];
        CFB_TMEM_LD32(lane_addr + o_col + half * OH + cc * 32, a0);
        CFB_TMEM_LD32(lane_addr + o_col + HD + half * OH + cc * 32, a1);
        tmem_ld_wait();
        if (ok && qpos < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + cc * 32);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              v[e] = __uint_as_float(a0[8 * k + e]) * g0 + __uint_as_float(a1[8 * k + e]) * g1;
            uint4 u;
            u.x = pack_bf16x2(v[0], v[1]);
            u.y = pack_bf16x2(v[2], v[3]);
            u.z = pack_bf16x2(v[4], v[5]);
            u.w = pack_bf16x2(v[6], v[7]);
            d4[k] = u;
          }
        }
      }
      if (ok && qpos < p.S && half == 0)
        p.lse[static_cast<long long>(row0 + qpos) * p.nh + h] = (M + log2f(Lt)) * kLn2;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

int make_tmap_qkv(CUtensorMap* map, const void* qkv, long long rows, long long ld);

template <int HD>
int launch(const void* qkv, long long ld, void* out, long long ld_out, float* lse, int B, int S,
           int nh, int nkv, float scale, int* err, cudaStream_t st) {
  CUtensorMap tm;
  const int rc = make_tmap_qkv(&tm, qkv, static_cast<long long>(B) * S, ld);
  if (rc) return rc;
  Params p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.ld = ld;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.lse = lse;
  p.S = S;
  p.nh = nh;
  p.nkv = nkv;
  p.scale_log2 = scale * kLog2e;
  p.err = err;
  auto kern = attn_fwd_tc_kernel<HD>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem<HD>::BYTES);
    configured = true;
  }
  dim3 grid((S + BM - 1) / BM, nh, B);
  kern<<<grid, 320, Smem<HD>::BYTES, st>>>(tm, p);
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
                    int B, int S, int nh, int nkv, int hd, float scale, int* err,
                    cudaStream_t st) {
  if (ld_qkv % 8 || ld_out % 8 || nh % nkv) return -11;
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return -12;
  if (hd == 64)
    return cfb::attn_tc::launch<64>(qkv, ld_qkv, out, ld_out, lse, B, S, nh, nkv, scale, err, st);
  if (hd == 128)
    return cfb::attn_tc::launch<128>(qkv, ld_qkv, out, ld_out, lse, B, S, nh, nkv, scale, err, st);
  return -12;
}
