// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation tensor cores.
//
//   D[M, N] = epilogue( alpha * sum_k A[m, k] * B[k, n] )
//
// A is given either K-major (row-major [M, K]) or MN-major (row-major [K, M]); B either
// K-major (row-major [N, K]) or MN-major (row-major [K, N]).  This covers the three GEMMs of a
// linear layer without any transposes:
//   forward   Y  = X  W^T     A = X  [T, K] K-major,   B = W [N, K]  K-major
//   dgrad     dX = dY W       A = dY [T, N] K-major,   B = W [N, K]  MN-major
//   wgrad     dW = dY^T X     A = dY [T, N] MN-major,  B = X [T, K]  MN-major
//
// Roles (192 threads, one CTA per SM, grid = min(#tiles, #SMs)):
//   warp 0  TMA producer: 128B-swizzled tiles of A and B into a STAGES-deep smem ring
//   warp 1  MMA issuer:   tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM accumulators
//   warps 2-5 epilogue:   tcgen05.ld of the accumulator, fused epilogue, global stores
// The two TMEM accumulators (2 x BN fp32 columns) let the epilogue of tile i overlap the
// MMAs of tile i+1.  Weight-gradient GEMMs (fp32 accumulate into the gradient) may split K so
// that the number of work units fills whole waves of the 148 SMs.  Every mbarrier wait is bounded (see sm100_common.cuh); on timeout the
// kernel records an error code, drains its own in-flight work and frees TMEM.
#include "sm100_common.cuh"
#include "launch_api.h"

#include <cudaTypedefs.h>
#include <cstdlib>
#include <mutex>

namespace cfb {

// Hardware base-2 exponential (MUFU, ftz).
__device__ __forceinline__ float exp2f_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct GemmArgs {
  int M, N, K;
  // split-K (kEpiF32Acc only): every output tile is computed as ksplit work units over
  // consecutive k-block ranges, each adding its partial sum into D with fp32 vector reductions
  int ksplit;
  // kEpiF32Acc: add into D with fp32 vector reductions (no read of D on the SM, so the
  // epilogue never waits on memory; with one unit per tile each element gets exactly one add,
  // the same result as load + add + store) instead of load + add + store
  int acc_red;
  void* D;
  long long ldd;
  const __nv_bfloat16* R;
  long long ldr;
  float alpha;
  int* err;
  // kEpiBF16Rope: rotate-half RoPE of columns [0, rope_cols) in heads of hd columns, at
  // position pos[row], with the table cs [max_pos, hd/2, 2] fp32 (cos, sin)
  const int* pos;
  const float* cs;
  int rope_cols, hd;
  // kEpiSwiGLU: B rows [n, n + N) are the gate, rows dual_off + n the up projection; D [M, 2F]
  // receives gate at column n and up at column dual_off + n, aux [M, F] (ld_aux) silu(g) * u
  int dual_off;
  __nv_bfloat16* aux;
  long long ld_aux;
  // kEpiSwiGLUBwd: aux = gu [*, 2F] (read; gate at column n, up at dual_off + n) of row
  // aux_rows[m] (or m); D [M, 2F] receives d gate at column n and d up at dual_off + n
  const int* aux_rows;
  // kEpiCEPart / kEpiCEGrad (256-column tiles): labels [M] (< 0: ignored row); per row and
  // tile the statistics ce_pmax / ce_psum [M, ce_nt] and the label logit ce_ptgt [M]
  // (forward); lse [M] and dloss [M] (backward, D = dlogits bf16)
  const long long* ce_labels;
  float *ce_pmax, *ce_psum, *ce_ptgt;
  const float *ce_lse, *ce_dloss;
  int ce_nt;
  // ---- tensor-parallel fusion.  Row segments: rank q owns rows [seg[q], seg[q+1]) of A / D
  // (device array [P + 1]; uniform shards in the forward, kept rows in the backward).  Flags
  // live in symmetric buffers peer_flags[q]: ready[P] at flag_ready, done[P] at flag_done.
  int rank, P;
  const int* seg;
  uint32_t epoch;
  uint32_t* const* peer_flags;
  int flag_ready, flag_done;
  uint32_t* tile_cnt;  // local scratch [P + 2], zero at rest
  // all-gather consumer (TPM 1): this rank's rows of A are local; two push warps per CTA copy
  // them to every other rank (multicast store, or peer stores) and raise ready[rank] there;
  // the TMA producer waits on ready[q] before reading rows of segment q != rank.  m-blocks are
  // rotated by rot_mblocks so the local segment is computed first.
  int rot_mblocks;
  long long lda;
  __nv_bfloat16* ag_mc;            // multicast address of A, or nullptr
  __nv_bfloat16* const* ag_peers;  // A of every rank (peer stores without multicast)
  // reduce-scatter producer (TPM 2): D is this rank's partial buffer (symmetric memory).  When
  // all of an m-block's tiles are stored, the rank raises blk_ready[m][rank] (at flag_blk +
  // m * P + rank) at every owner of a row of that block; two pull warps per CTA of the owner
  // reduce its segment block by block as soon as every rank has stored the block (one
  // multimem.ld_reduce per 8 bf16 through the NVSwitch, fp32 accumulation, or peer loads).
  // With uniform segments of interleave_spb m-blocks the m-blocks are computed interleaved
  // across owners, so every owner's blocks complete (and are pulled) during the GEMM.
  const __nv_bfloat16* mc_part;
  const __nv_bfloat16* const* peer_part;
  int flag_blk, interleave_spb;
  const __nv_bfloat16* rs_resid;   // [count, N] added to the reduced rows
  __nv_bfloat16* rs_out;           // [out_rows, N] reduced rows of this rank, then zeros
  long long ld_resid, ld_out;
  int out_rows;
};

namespace tpc {
__device__ __forceinline__ uint4 ld_reduce_bf16x8(const __nv_bfloat16* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* f) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* f, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
// Bounded wait until (int)(flags[i] - epoch) >= 0 for i < n.  On timeout raises *abort and
// records kErrPeerWait; returns false.
__device__ __forceinline__ bool wait_epoch(const uint32_t* flags, int n, uint32_t epoch,
                                           volatile int* abort, int* err) {
  const uint64_t t0 = globaltimer_ns();
  uint64_t limit = 0;  // read from the status block only once a wait has spun 256 times
  for (int i = 0; i < n; ++i) {
    uint32_t spins = 0;
    while (static_cast<int32_t>(ld_acquire_sys(flags + i) - epoch) < 0) {
      if ((++spins & 255u) == 0) {
        if (*abort) return false;
        if (limit == 0) limit = peer_wait_limit_ns(err);
        if (globaltimer_ns() - t0 > limit) {
          *abort = 1;
          atomicCAS(err, 0, kErrPeerWait);
          return false;
        }
      }
    }
  }
  return true;
}
// atomicAdd with acquire-release semantics at GPU scope: publishes this thread's earlier writes
// (and those it observed) to whoever observes the new count
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
}  // namespace tpc

// DUAL (the SwiGLU epilogue): every stage also holds the B tile dual_off rows further down
// (the up projection next to the gate), and each accumulator buffer has two BN-column halves.
template <int BN, bool DUAL = false>
struct GemmShape {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B1_BYTES = BN * BK * 2;
  static constexpr int B_BYTES = (DUAL ? 2 : 1) * B1_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (STAGE_BYTES >= 48 * 1024) ? 4 : 6;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int ACC_COLS = (DUAL ? 2 : 1) * BN;  // one accumulator buffer
  static constexpr int TMEM_COLS = (2 * ACC_COLS <= 32) ? 32 : (2 * ACC_COLS <= 64 ? 64 : (2 * ACC_COLS <= 128 ? 128 : (2 * ACC_COLS <= 256 ? 256 : 512)));
  static_assert(2 * ACC_COLS <= 512, "TMEM");
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& tm, int& tn) {
  constexpr int GROUP = 16;
  const int per_group = GROUP * num_n;
  const int g = tile / per_group;
  const int first_m = g * GROUP;
  const int gsize = min(num_m - first_m, GROUP);
  const int r = tile - g * per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

// Epilogue of one accumulator row (TMEM lane) of a 128 x BN tile: tcgen05.ld of the fp32
// accumulator at `taddr` (this warp's lane quadrant), then the EPI-specific conversion and
// global stores of row `row`, columns [n0, n0 + BN) (clipped to N).
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_row(const GemmArgs& p, uint32_t taddr, int row,
                                             int n0) {
  constexpr bool DUAL = EPI == kEpiSwiGLU;
  const int ksplit = p.ksplit;
  (void)ksplit;
  if (EPI == kEpiCEPart) {
    // online max / sum of exp over the tile's columns, in log2 units; fp32 logits
    constexpr float kL2e = 1.4426950408889634f, kLn2f = 0.6931471805599453f;
    const long long lab = row < p.M ? p.ce_labels[row] : -1;
    float m = -INFINITY, sum = 0.f;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int col = n0 + c * 32;
      if (col >= p.N) break;  // warp-uniform (N % 32 == 0)
      uint32_t r[32];
      CFB_TMEM_LD32(taddr + c * 32, r);
      tmem_ld_wait();
      float cm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) cm = fmaxf(cm, __uint_as_float(r[i]));
      const float mn = fmaxf(m, cm * p.alpha * kL2e);
      float acc = (m == -INFINITY) ? 0.f : sum * exp2f_approx(m - mn);
#pragma unroll
      for (int i = 0; i < 32; ++i) acc += exp2f_approx(fmaf(__uint_as_float(r[i]), p.alpha * kL2e, -mn));
      sum = acc;
      m = mn;
      if (lab >= col && lab < col + 32) {
        float t = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (lab - col == i) t = __uint_as_float(r[i]);
        p.ce_ptgt[row] = t * p.alpha;
      }
    }
    if (row < p.M) {
      const long long o = static_cast<long long>(row) * p.ce_nt + n0 / BN;
      p.ce_pmax[o] = m * kLn2f;
      p.ce_psum[o] = sum;
    }
    return;
  }
  if (EPI == kEpiCEGrad) {
    constexpr float kL2e = 1.4426950408889634f;
    const bool live = row < p.M;
    const long long lab = live ? p.ce_labels[row] : -1;
    const float nl = live ? -p.ce_lse[row] * kL2e : 0.f;
    const float dl = (live && lab >= 0) ? p.ce_dloss[row] : 0.f;
    __nv_bfloat16* grow = reinterpret_cast<__nv_bfloat16*>(p.D) + row * p.ldd;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int col = n0 + c * 32;
      if (col >= p.N) break;  // warp-uniform
      uint32_t r[32];
      CFB_TMEM_LD32(taddr + c * 32, r);
      tmem_ld_wait();
      if (!live) continue;
      uint32_t o[16];
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        float g0 = exp2f_approx(fmaf(__uint_as_float(r[2 * t]), p.alpha * kL2e, nl));
        float g1 = exp2f_approx(fmaf(__uint_as_float(r[2 * t + 1]), p.alpha * kL2e, nl));
        if (lab == col + 2 * t) g0 -= 1.f;
        if (lab == col + 2 * t + 1) g1 -= 1.f;
        o[t] = pack_bf16x2(g0 * dl, g1 * dl);
      }
      uint4* d4 = reinterpret_cast<uint4*>(grow + col);
#pragma unroll
      for (int j = 0; j < 4; ++j) d4[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
    }
    return;
  }
  __nv_bfloat16* drow = reinterpret_cast<__nv_bfloat16*>(p.D) + row * p.ldd;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    const int col = n0 + c * 32;
    if (col >= p.N) break;  // warp-uniform
    if (DUAL) {
      uint32_t rg[32], ru[32];
      CFB_TMEM_LD32(taddr + c * 32, rg);
      CFB_TMEM_LD32(taddr + BN + c * 32, ru);
      tmem_ld_wait();
      if (row < p.M) {
        uint32_t og[16], ou[16], oh[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float g0 = __uint_as_float(rg[2 * t]) * p.alpha;
          const float g1 = __uint_as_float(rg[2 * t + 1]) * p.alpha;
          const float u0 = __uint_as_float(ru[2 * t]) * p.alpha;
          const float u1 = __uint_as_float(ru[2 * t + 1]) * p.alpha;
          og[t] = pack_bf16x2(g0, g1);
          ou[t] = pack_bf16x2(u0, u1);
          // silu of the bf16-rounded gate, as a separate SwiGLU pass over gu would see it
          const float2 gr = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&og[t]));
          const float2 ur = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ou[t]));
          // silu(g) = g sigmoid(g) = g (1 + tanh(g / 2)) / 2: one MUFU tanh per element (the
          // result is rounded to bf16, well above tanh.approx's error)
          oh[t] = pack_bf16x2(silu_tanh(gr.x) * ur.x, silu_tanh(gr.y) * ur.y);
        }
        __nv_bfloat16* gd = drow + col;
        __nv_bfloat16* ud = drow + p.dual_off + col;
        __nv_bfloat16* hd = p.aux + row * p.ld_aux + col;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          reinterpret_cast<uint4*>(gd)[j] = make_uint4(og[4 * j], og[4 * j + 1], og[4 * j + 2], og[4 * j + 3]);
          reinterpret_cast<uint4*>(ud)[j] = make_uint4(ou[4 * j], ou[4 * j + 1], ou[4 * j + 2], ou[4 * j + 3]);
          reinterpret_cast<uint4*>(hd)[j] = make_uint4(oh[4 * j], oh[4 * j + 1], oh[4 * j + 2], oh[4 * j + 3]);
        }
      }
      continue;
    }
    if (EPI == kEpiSwiGLUBwd) {
      uint32_t rd[32];
      CFB_TMEM_LD32(taddr + c * 32, rd);
      tmem_ld_wait();
      if (row < p.M) {
        const long long src = p.aux_rows ? p.aux_rows[row] : row;
        const uint4* g4 = reinterpret_cast<const uint4*>(p.aux + src * p.ld_aux + col);
        const uint4* u4 = reinterpret_cast<const uint4*>(p.aux + src * p.ld_aux + p.dual_off + col);
        uint4* dg4 = reinterpret_cast<uint4*>(drow + col);
        uint4* du4 = reinterpret_cast<uint4*>(drow + p.dual_off + col);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 gq = g4[j], uq = u4[j];
          const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gq);
          const __nv_bfloat162* uh = reinterpret_cast<const __nv_bfloat162*>(&uq);
          uint32_t og[4], ou[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 g = __bfloat1622float2(gh[e]);
            const float2 u = __bfloat1622float2(uh[e]);
            const float d0 = __uint_as_float(rd[8 * j + 2 * e]) * p.alpha;
            const float d1 = __uint_as_float(rd[8 * j + 2 * e + 1]) * p.alpha;
            const float s0 = 1.f / (1.f + __expf(-g.x)), s1 = 1.f / (1.f + __expf(-g.y));
            og[e] = pack_bf16x2(d0 * u.x * s0 * (1.f + g.x * (1.f - s0)),
                                d1 * u.y * s1 * (1.f + g.y * (1.f - s1)));
            ou[e] = pack_bf16x2(d0 * g.x * s0, d1 * g.y * s1);
          }
          dg4[j] = make_uint4(og[0], og[1], og[2], og[3]);
          du4[j] = make_uint4(ou[0], ou[1], ou[2], ou[3]);
        }
      }
      continue;
    }
    if (EPI == kEpiBF16Rope && col < p.rope_cols) {
      // the first-half chunk of a head rotates together with its partner hd/2 columns on
      const int half = p.hd >> 1;
      const int hc = col % p.hd;
      if (hc >= half) continue;  // already written with its partner (warp-uniform)
      uint32_t ra[32], rb[32];
      CFB_TMEM_LD32(taddr + c * 32, ra);
      CFB_TMEM_LD32(taddr + c * 32 + half, rb);
      tmem_ld_wait();
      if (row < p.M) {
        const float4* cs =
            reinterpret_cast<const float4*>(p.cs + (static_cast<long long>(p.pos[row]) * half + hc) * 2);
        uint32_t oa[16], ob[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float4 q = __ldg(cs + t);  // cos, sin of pairs 2t and 2t+1
          const float a0 = __uint_as_float(ra[2 * t]) * p.alpha;
          const float a1 = __uint_as_float(ra[2 * t + 1]) * p.alpha;
          const float b0 = __uint_as_float(rb[2 * t]) * p.alpha;
          const float b1 = __uint_as_float(rb[2 * t + 1]) * p.alpha;
          oa[t] = pack_bf16x2(a0 * q.x - b0 * q.y, a1 * q.z - b1 * q.w);
          ob[t] = pack_bf16x2(b0 * q.x + a0 * q.y, b1 * q.z + a1 * q.w);
        }
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.D) + row * p.ldd + col;
        uint4* da = reinterpret_cast<uint4*>(dst);
        uint4* db = reinterpret_cast<uint4*>(dst + half);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          da[j] = make_uint4(oa[4 * j], oa[4 * j + 1], oa[4 * j + 2], oa[4 * j + 3]);
          db[j] = make_uint4(ob[4 * j], ob[4 * j + 1], ob[4 * j + 2], ob[4 * j + 3]);
        }
      }
      continue;
    }
    uint32_t r[32];
    CFB_TMEM_LD32(taddr + c * 32, r);
    tmem_ld_wait();
    if (row < p.M) {
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
      if (EPI == kEpiBF16 || EPI == kEpiBF16Resid || EPI == kEpiBF16Rope) {
        __nv_bfloat16* dst = drow + col;
        if (EPI == kEpiBF16Resid) {
          const uint4* rs = reinterpret_cast<const uint4*>(p.R + row * p.ldr + col);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 u = rs[j];
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float2 f = __bfloat1622float2(h[e]);
              v[j * 8 + 2 * e] += f.x;
              v[j * 8 + 2 * e + 1] += f.y;
            }
          }
        }
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 u;
          u.x = pack_bf16x2(v[j * 8 + 0], v[j * 8 + 1]);
          u.y = pack_bf16x2(v[j * 8 + 2], v[j * 8 + 3]);
          u.z = pack_bf16x2(v[j * 8 + 4], v[j * 8 + 5]);
          u.w = pack_bf16x2(v[j * 8 + 6], v[j * 8 + 7]);
          d4[j] = u;
        }
      } else {
        float* dst = reinterpret_cast<float*>(p.D) + row * p.ldd + col;
        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          if (EPI == kEpiF32Acc && (ksplit > 1 || p.acc_red)) {
            // with split-K the k-splits of this tile add into D concurrently (fp32, order
            // not fixed)
            asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(
                             d4 + j),
                         "f"(o.x), "f"(o.y), "f"(o.z), "f"(o.w)
                         : "memory");
            continue;
          }
          if (EPI == kEpiF32Acc) {
            const float4 old = d4[j];
            o.x += old.x;
            o.y += old.y;
            o.z += old.z;
            o.w += old.w;
          }
          d4[j] = o;
        }
      }
    }
  }
}

// ------------------------------------------------------------------ TP collective warps
// All-gather push (TPM 1, warps 6 and 7 of every CTA, pw = 0 / 1): copy this rank's rows of A
// to every other rank while the tensor cores start on them; the last push warp of the grid
// raises ready[rank] at every peer.
__device__ __forceinline__ void tp_push_rows(const GemmArgs& p, int pw, int lane,
                                             volatile int* abort) {
  // 32-bit index arithmetic (the host keeps rows x K / 8 below 2^31): the division by the
  // vectors per row is a short multiply sequence, where 64-bit division would dominate the loop
  const int r_lo = p.seg[p.rank];
  const uint32_t rows = static_cast<uint32_t>(p.seg[p.rank + 1] - r_lo);
  const uint32_t vec_per_row = static_cast<uint32_t>(p.K / 8);
  const uint32_t total = rows * vec_per_row;
  const uint32_t stride = gridDim.x * 64u;
  const __nv_bfloat16* A = p.ag_peers[p.rank];
  constexpr int U = 4;
  for (uint32_t v0 = blockIdx.x * 64u + pw * 32 + lane; v0 < total && !*abort;
       v0 += U * stride) {
    uint4 val[U];
    long long off[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t v = v0 + u * stride;
      off[u] = -1;
      if (v < total) {
        const uint32_t rr = v / vec_per_row, cv = v - rr * vec_per_row;
        off[u] = static_cast<long long>(r_lo + static_cast<int>(rr)) * p.lda + cv * 8;
        val[u] = *reinterpret_cast<const uint4*>(A + off[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (off[u] < 0) continue;
      if (p.ag_mc) {
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(
                         p.ag_mc + off[u]),
                     "f"(__uint_as_float(val[u].x)), "f"(__uint_as_float(val[u].y)),
                     "f"(__uint_as_float(val[u].z)), "f"(__uint_as_float(val[u].w))
                     : "memory");
      } else {
        for (int q2 = 0; q2 < p.P; ++q2)
          if (q2 != p.rank) *reinterpret_cast<uint4*>(p.ag_peers[q2] + off[u]) = val[u];
      }
    }
  }
  __syncwarp();
  if (lane == 0) {
    if (tpc::atom_add_acq_rel_gpu(p.tile_cnt, 1u) == 2u * gridDim.x - 1u) {
      __threadfence_system();
      for (int q2 = 0; q2 < p.P; ++q2)
        if (q2 != p.rank) tpc::st_release_sys(p.peer_flags[q2] + p.flag_ready + p.rank, p.epoch);
    }
  }
}

// Reduce-scatter pull (TPM 2, warps 6 and 7): for every 128-row block of this rank's segment,
// wait until every rank has stored its partial rows of the block, then sum them (multimem
// ld_reduce with fp32 accumulation, or peer loads), add the residual and store the result.
template <int BM>
__device__ __forceinline__ void tp_pull_rows(const GemmArgs& p, int pw, int lane, int num_m128,
                                             volatile int* abort) {
  // 32-bit index arithmetic within a 128-row block (see tp_push_rows)
  const int lo = p.seg[p.rank], hi = p.seg[p.rank + 1];
  const uint32_t vec_per_row = static_cast<uint32_t>(p.N / 8);
  const uint32_t stride = gridDim.x * 64u;
  const uint32_t t0 = blockIdx.x * 64u + pw * 32 + lane;
  bool ok = true;
  for (int blk = lo / BM; lo < hi && blk <= (hi - 1) / BM && ok; ++blk) {
    if (lane == 0)
      ok = tpc::wait_epoch(p.peer_flags[p.rank] + p.flag_blk + blk * p.P, p.P, p.epoch,
                           abort, p.err);
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (!ok) break;
    const int r_a = max(lo, blk * BM), r_b = min(hi, blk * BM + BM);
    const uint32_t total = static_cast<uint32_t>(r_b - r_a) * vec_per_row;
    constexpr int U = 8;  // independent 16-byte reductions in flight per thread
    for (uint32_t v0 = t0; v0 < total; v0 += U * stride) {
      uint4 red[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t v = v0 + u * stride;
        if (v >= total) continue;
        const uint32_t rr = v / vec_per_row, cv = v - rr * vec_per_row;
        const long long off = static_cast<long long>(r_a + static_cast<int>(rr)) * p.ldd + cv * 8;
        if (p.mc_part) {
          red[u] = tpc::ld_reduce_bf16x8(p.mc_part + off);
        } else {
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int q2 = 0; q2 < p.P; ++q2) {
            const uint4 w4 = *reinterpret_cast<const uint4*>(p.peer_part[q2] + off);
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w4);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h[e]);
              acc[2 * e] += f.x;
              acc[2 * e + 1] += f.y;
            }
          }
          red[u] = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                              pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t v = v0 + u * stride;
        if (v >= total) continue;
        const uint32_t rr = v / vec_per_row;
        const int r = r_a - lo + static_cast<int>(rr);  // row of out
        const int c = static_cast<int>(v - rr * vec_per_row) * 8;
        float acc[8];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&red[u]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] = f.x;
          acc[2 * e + 1] = f.y;
        }
        if (p.rs_resid) {
          const uint4 u4 = *reinterpret_cast<const uint4*>(
              p.rs_resid + static_cast<long long>(r) * p.ld_resid + c);
          const __nv_bfloat162* hr = reinterpret_cast<const __nv_bfloat162*>(&u4);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(hr[e]);
            acc[2 * e] += f.x;
            acc[2 * e + 1] += f.y;
          }
        }
        *reinterpret_cast<uint4*>(p.rs_out + static_cast<long long>(r) * p.ld_out + c) =
            make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                       pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
      }
    }
  }
  if (ok) {
    // padding rows of out
    const uint32_t zt = static_cast<uint32_t>(max(0, p.out_rows - (hi - lo))) * vec_per_row;
    for (uint32_t v = t0; v < zt; v += stride) {
      const uint32_t rr = v / vec_per_row;
      const int r = (hi - lo) + static_cast<int>(rr);
      const int c = static_cast<int>(v - rr * vec_per_row) * 8;
      *reinterpret_cast<uint4*>(p.rs_out + static_cast<long long>(r) * p.ld_out + c) =
          make_uint4(0u, 0u, 0u, 0u);
    }
    // this rank has read its rows of every partial buffer: the last pull warp of the grid
    // tells all ranks (their buffer of this epoch's parity may be rewritten at epoch + 2)
    __syncwarp();
    if (lane == 0) {
      __threadfence_system();
      if (atomicAdd(p.tile_cnt + num_m128, 1u) == 2u * gridDim.x - 1u) {
        for (int q2 = 0; q2 < p.P; ++q2)
          tpc::st_release_sys(p.peer_flags[q2] + p.flag_done + p.rank, p.epoch);
      }
    }
  }
}

// The last CTA to finish clears the local counters for the next launch.
template <int TPM>
__device__ __forceinline__ void tp_clear_counters(const GemmArgs& p, int num_m128) {
  const int ncnt = TPM == 2 ? num_m128 + 2 : p.P + 2;
  __threadfence();
  if (atomicAdd(p.tile_cnt + ncnt - 1, 1u) == gridDim.x - 1u) {
    for (int i = 0; i < ncnt; ++i) atomicExch(p.tile_cnt + i, 0u);
  }
}

// TPM: 0 plain; 1 all-gather consumer (push warps + per-segment waits); 2 reduce-scatter
// producer (partial rows stored to their owners + sum warps)
template <int BN, bool A_MN, bool B_MN, int EPI, int TPM = 0>
__global__ void __launch_bounds__(TPM != 0 ? 256 : 192, 1)
    gemm_bf16_sm100(const __grid_constant__ CUtensorMap tmA,
                    const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
  constexpr bool DUAL = EPI == kEpiSwiGLU;
  using S = GemmShape<BN, DUAL>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* bar_area = smem + S::STAGES * S::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty = full + S::STAGES;
  uint64_t* tfull = empty + S::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_m = (p.M + S::BM - 1) / S::BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + S::BK - 1) / S::BK;
  const int ksplit = p.ksplit;
  const int num_units = num_tiles * ksplit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 4);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t smem_base = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int last_stage = -1;
      uint32_t last_phase = 0;
      bool ok = true;
      uint64_t ready_mask = 0;  // TPM 1: shards known to be gathered
      for (int unit = blockIdx.x; unit < num_units && ok; unit += gridDim.x) {
        const int tile = unit / ksplit, ks = unit - tile * ksplit;
        int tm, tn;
        tile_coords(tile, num_m, num_n, tm, tn);
        if (TPM == 2 && p.interleave_spb > 0) tm = (tm % p.P) * p.interleave_spb + tm / p.P;
        if (TPM == 1) {
          tm = (tm + p.rot_mblocks) % num_m;
          // wait for every segment that intersects this m-block
          const int r0 = tm * S::BM, r1 = min(p.M, r0 + S::BM);
          bool waited = false;
          for (int q = 0; q < p.P && ok; ++q) {
            if (q == p.rank || ((ready_mask >> q) & 1ull) || p.seg[q] >= r1 ||
                p.seg[q + 1] <= r0)
              continue;
            if (!tpc::wait_epoch(p.peer_flags[p.rank] + p.flag_ready + q, 1, p.epoch, abort_flag,
                                 p.err))
              ok = false;
            ready_mask |= 1ull << q;
            waited = true;
          }
          if (!ok) break;
          // rows written by peers' generic stores are read below by the TMA (async proxy)
          if (waited) asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        const int m0 = tm * S::BM, n0 = tn * BN;
        const int kb_end = (ks + 1) * num_kb / ksplit;
        for (int kb = ks * num_kb / ksplit; kb < kb_end; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.err,
                         kErrWaitProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, S::STAGE_BYTES);
          const uint32_t sa = smem_base + stage * S::STAGE_BYTES;
          const uint32_t sb = sa + S::A_BYTES;
          const int k0 = kb * S::BK;
          if (!A_MN) {
            tma_load_2d(sa, &tmA, fb, k0, m0);
          } else {
            tma_load_2d(sa, &tmA, fb, m0, k0);
            tma_load_2d(sa + 8192, &tmA, fb, m0 + 64, k0);
          }
          if (!B_MN) {
            tma_load_2d(sb, &tmB, fb, k0, n0);
            if (DUAL) tma_load_2d(sb + S::B1_BYTES, &tmB, fb, k0, n0 + p.dual_off);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_2d(sb + c * 8192, &tmB, fb, n0 + c * 64, k0);
          }
          last_stage = stage;
          last_phase = phase;
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && last_stage >= 0) {
        // Let our own last copies land before the CTA exits (bounded).
        volatile int dummy = 0;
        mbar_wait(smem_u32(&full[last_stage]), last_phase, &dummy, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t IDESC = idesc_bf16_f32(128, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < num_units && ok; unit += gridDim.x, ++it) {
        const int ks = unit % ksplit;
        const int kb_beg = ks * num_kb / ksplit, kb_end = (ks + 1) * num_kb / ksplit;
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag, p.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * S::ACC_COLS;
        for (int kb = kb_beg; kb < kb_end; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * S::STAGE_BYTES;
          const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < S::BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(sa + k * 2048, 8192, 1024)
                                     : sdesc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(sb + k * 2048, 8192, 1024)
                                     : sdesc_sw128(sb + k * 32, 16, 1024);
            const uint32_t accum = (kb != kb_beg || k != 0) ? 1u : 0u;
            umma_bf16_ss(d_tmem, ad, bd, IDESC, accum);
            if (DUAL)
              umma_bf16_ss(d_tmem + BN, ad, sdesc_sw128(sb + S::B1_BYTES + k * 32, 16, 1024), IDESC,
                           accum);
          }
          umma_commit(smem_u32(&empty[stage]));
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&tfull[acc]));
      }
      // All issued MMAs complete before TMEM is released.
      umma_commit(smem_u32(drain));
      volatile int dummy = 0;
      mbar_wait(smem_u32(drain), 0, &dummy, nullptr, 0);
    }
  } else if (warp < 6) {
    // -------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    int it = 0;
    if (TPM == 2) {
      // the partial buffer of this epoch's parity was last read by the pulls of epoch - 2
      bool okw = true;
      if (lane == 0)
        okw = tpc::wait_epoch(p.peer_flags[p.rank] + p.flag_done, p.P, p.epoch - 2, abort_flag,
                              p.err);
      (void)__shfl_sync(0xffffffffu, okw ? 1 : 0, 0);  // on timeout abort_flag is raised
    }
    for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x, ++it) {
      if (TPM == 2 && *abort_flag) break;
      const int tile = unit / ksplit;
      int tm, tn;
      tile_coords(tile, num_m, num_n, tm, tn);
      if (TPM == 2 && p.interleave_spb > 0) tm = (tm % p.P) * p.interleave_spb + tm / p.P;
      if (TPM == 1) tm = (tm + p.rot_mblocks) % num_m;
      const int m0 = tm * S::BM, n0 = tn * BN;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, p.err, kErrWaitEpilogue))
        break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * S::ACC_COLS;
      epilogue_row<BN, EPI>(p, taddr, row, n0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
      if (TPM == 2 && lane == 0) {
        // count this warp's quarter of the tile; the last of the m-block's 4 * num_n quarters
        // tells every owner of a row of the block
        if (tpc::atom_add_acq_rel_gpu(p.tile_cnt + tm, 1u) == 4u * num_n - 1u) {
          __threadfence_system();
          const int r1 = min(p.M, m0 + S::BM);
          for (int o = 0; o < p.P; ++o)
            if (p.seg[o] < r1 && p.seg[o + 1] > m0)
              tpc::st_release_sys(p.peer_flags[o] + p.flag_blk + tm * p.P + p.rank, p.epoch);
        }
      }
    }
  } else if (TPM == 1) {
    // -------------------------------------------------------------- push warps (6, 7)
    tp_push_rows(p, warp - 6, lane, abort_flag);
  } else if (TPM == 2) {
    // -------------------------------------------------------------- pull warps (6, 7)
    tp_pull_rows<S::BM>(p, warp - 6, lane, num_m, abort_flag);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, S::TMEM_COLS);
  if (TPM != 0 && threadIdx.x == 0) tp_clear_counters<TPM>(p, num_m);
}

// ------------------------------------------------------------------ CTA-pair GEMM
// Two CTAs of a cluster (one per SM) compute a 256 x 256 tile with tcgen05.mma.cta_group::2.
// Per k-block each CTA stages its 128 rows of A and 128 of the 256 B columns (32 KB, where a
// single CTA computing a 128 x 256 tile stages 48 KB), so the L2 -> shared-memory traffic per
// FLOP drops by a third and the ring is 6 stages deep.  Roles as in the single-CTA kernel.
// The leader (cluster rank 0) issues the MMAs and owns the full and accumulator-empty
// barriers: both CTAs' TMA copies count their bytes on the leader's full barrier and both
// CTAs' epilogue warps arrive on its accumulator-empty barrier; MMA completion is signalled to
// the same barrier offsets of both CTAs.  Each CTA's TMEM holds the fp32 accumulators of its
// 128 rows (2 x 256 columns), which its own epilogue warps drain.  No tensor-parallel modes;
// split-K as in the single-CTA kernel.  SwiGLU (dual-B): the leader stages 128 gate rows of B
// and its peer the 128 matching up rows (dual_off further down), so one N = 256 MMA leaves gate
// in accumulator columns [0, 128) and up in [128, 256) of every row, and a tile covers 128
// output columns of F.
struct PairShape {
  static constexpr int BM = 128;  // rows per CTA; the pair tile is 256 rows
  static constexpr int BN = 256;  // pair tile columns; each CTA stages BN / 2 rows of B
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 6;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int ACC_COLS = BN;
  static constexpr int TMEM_COLS = 512;
};

template <bool A_MN, bool B_MN, int EPI, int TPM = 0>
__global__ void __launch_bounds__(TPM != 0 ? 256 : 192, 1)
    gemm_bf16_sm100_pair(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB, GemmArgs p) {
  using S = PairShape;
  constexpr bool DUAL = EPI == kEpiSwiGLU;
  constexpr int TN = DUAL ? S::BN / 2 : S::BN;  // output columns of a tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* bar_area = smem + S::STAGES * S::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty = full + S::STAGES;
  uint64_t* tfull = empty + S::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_m = (p.M + 2 * S::BM - 1) / (2 * S::BM);
  const int num_m128 = (p.M + S::BM - 1) / S::BM;  // 128-row blocks (flags, counters)
  const int num_n = (p.N + TN - 1) / TN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + S::BK - 1) / S::BK;
  const int ksplit = p.ksplit;
  const int num_units = num_tiles * ksplit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 8);  // 4 epilogue warps of each CTA
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t smem_base = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      uint64_t ready_mask = 0;  // TPM 1: segments known to be gathered
      for (int unit = pair; unit < num_units && ok; unit += num_pairs) {
        const int tile = unit / ksplit, ks = unit - tile * ksplit;
        int tm, tn;
        tile_coords(tile, num_m, num_n, tm, tn);
        if (TPM == 2 && p.interleave_spb > 0) tm = (tm % p.P) * p.interleave_spb + tm / p.P;
        if (TPM == 1) tm = (tm + p.rot_mblocks) % num_m;
        const int m0 = tm * 2 * S::BM + static_cast<int>(crank) * S::BM;
        if (TPM == 1) {
          // this CTA stages rows [m0, m0 + 128) of A: wait for every other rank's segment
          // that intersects them (the peer CTA waits for its own rows)
          const int r1 = min(p.M, m0 + S::BM);
          bool waited = false;
          for (int q = 0; q < p.P && ok; ++q) {
            if (q == p.rank || ((ready_mask >> q) & 1ull) || p.seg[q] >= r1 ||
                p.seg[q + 1] <= m0)
              continue;
            if (!tpc::wait_epoch(p.peer_flags[p.rank] + p.flag_ready + q, 1, p.epoch, abort_flag,
                                 p.err))
              ok = false;
            ready_mask |= 1ull << q;
            waited = true;
          }
          if (!ok) break;
          // rows written by peers' generic stores are read below by the TMA (async proxy)
          if (waited) asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        const int nb0 = DUAL ? tn * TN + (crank ? p.dual_off : 0)
                             : tn * S::BN + static_cast<int>(crank) * (S::BN / 2);
        const int kb_end = (ks + 1) * num_kb / ksplit;
        for (int kb = ks * num_kb / ksplit; kb < kb_end; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.err,
                         kErrWaitProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          if (leader) mbar_arrive_expect_tx(fb, 2 * S::STAGE_BYTES);
          const uint32_t fb_leader = mapa_shared(fb, 0);
          const uint32_t sa = smem_base + stage * S::STAGE_BYTES;
          const uint32_t sb = sa + S::A_BYTES;
          const int k0 = kb * S::BK;
          if (!A_MN) {
            tma_load_2d_pair(sa, &tmA, fb_leader, k0, m0);
          } else {
            tma_load_2d_pair(sa, &tmA, fb_leader, m0, k0);
            tma_load_2d_pair(sa + 8192, &tmA, fb_leader, m0 + 64, k0);
          }
          if (!B_MN) {
            tma_load_2d_pair(sb, &tmB, fb_leader, k0, nb0);
          } else {
            tma_load_2d_pair(sb, &tmB, fb_leader, nb0, k0);
            tma_load_2d_pair(sb + 8192, &tmB, fb_leader, nb0 + 64, k0);
          }
          ++issued;
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // On the error path let the copies land before the CTA exits (bounded); only the leader
      // can wait on the barrier they count on.
      if (!ok && leader) tma_drain_ring(full, S::STAGES, issued);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader)
      constexpr uint32_t IDESC = idesc_bf16_f32(2 * S::BM, S::BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int unit = pair; unit < num_units && ok; unit += num_pairs, ++it) {
        const int ks = unit % ksplit;
        const int kb_beg = ks * num_kb / ksplit, kb_end = (ks + 1) * num_kb / ksplit;
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1u, abort_flag, p.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * S::ACC_COLS;
        for (int kb = kb_beg; kb < kb_end; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * S::STAGE_BYTES;
          const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < S::BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(sa + k * 2048, 8192, 1024)
                                     : sdesc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(sb + k * 2048, 8192, 1024)
                                     : sdesc_sw128(sb + k * 32, 16, 1024);
            umma_bf16_ss_pair(d_tmem, ad, bd, IDESC, (kb != kb_beg || k != 0) ? 1u : 0u);
          }
          umma_commit_pair_mc(smem_u32(&empty[stage]), 0x3);
          if (++stage == S::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(smem_u32(&tfull[acc]), 0x3);
      }
      // All issued MMAs complete (they read both CTAs' shared memory) before either CTA moves on.
      umma_commit_pair(smem_u32(drain));
      volatile int dummy = 0;
      mbar_wait(smem_u32(drain), 0, &dummy, nullptr, 0);
    }
  } else if (warp < 6) {
    // -------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[0]), 0);
    int it = 0;
    if (TPM == 2) {
      // the partial buffer of this epoch's parity was last read by the pulls of epoch - 2
      bool okw = true;
      if (lane == 0)
        okw = tpc::wait_epoch(p.peer_flags[p.rank] + p.flag_done, p.P, p.epoch - 2, abort_flag,
                              p.err);
      (void)__shfl_sync(0xffffffffu, okw ? 1 : 0, 0);  // on timeout abort_flag is raised
    }
    for (int unit = pair; unit < num_units; unit += num_pairs, ++it) {
      if (TPM == 2 && *abort_flag) break;
      const int tile = unit / ksplit;
      int tm, tn;
      tile_coords(tile, num_m, num_n, tm, tn);
      if (TPM == 2 && p.interleave_spb > 0) tm = (tm % p.P) * p.interleave_spb + tm / p.P;
      if (TPM == 1) tm = (tm + p.rot_mblocks) % num_m;
      const int m0 = tm * 2 * S::BM + static_cast<int>(crank) * S::BM, n0 = tn * TN;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, p.err, kErrWaitEpilogue))
        break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * S::ACC_COLS;
      epilogue_row<TN, EPI>(p, taddr, m0 + row_in_tile, n0);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + acc * 8);
      if (TPM == 2 && lane == 0 && m0 < p.M) {
        // count this warp's quarter of the CTA's 128 x 256 share; the last of the 128-row
        // block's 4 * num_n quarters tells every owner of a row of the block
        const int blk = m0 / S::BM;
        if (tpc::atom_add_acq_rel_gpu(p.tile_cnt + blk, 1u) == 4u * num_n - 1u) {
          __threadfence_system();
          const int r1 = min(p.M, m0 + S::BM);
          for (int o = 0; o < p.P; ++o)
            if (p.seg[o] < r1 && p.seg[o + 1] > m0)
              tpc::st_release_sys(p.peer_flags[o] + p.flag_blk + blk * p.P + p.rank, p.epoch);
        }
      }
    }
  } else if (TPM == 1) {
    // -------------------------------------------------------------- push warps (6, 7)
    tp_push_rows(p, warp - 6, lane, abort_flag);
  } else if (TPM == 2) {
    // -------------------------------------------------------------- pull warps (6, 7)
    tp_pull_rows<S::BM>(p, warp - 6, lane, num_m128, abort_flag);
  }

  tc_fence_before();
  cluster_sync();  // the leader's MMAs no longer read this CTA's shared memory
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
  }
  if (TPM != 0 && threadIdx.x == 0) tp_clear_counters<TPM>(p, num_m128);
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult qres;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) ==
            cudaSuccess &&
        qres == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix of `rows` x `cols` with leading dimension `ld`
// (elements); boxes of `box_cols` x `box_rows` with 128-byte swizzle.
int make_tmap_2d_bf16(CUtensorMap* map, const void* ptr, long long rows, long long cols,
                      long long ld, int box_cols, int box_rows) {
  auto fn = get_encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -2;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, bool A_MN, bool B_MN, int EPI, int TPM = 0>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                       cudaStream_t st, int max_ctas) {
  using S = GemmShape<BN, EPI == kEpiSwiGLU>;
  auto kern = gemm_bf16_sm100<BN, A_MN, B_MN, EPI, TPM>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM_BYTES);
    configured = true;
  }
  const int tiles = ((a.M + 127) / 128) * ((a.N + BN - 1) / BN) * a.ksplit;
  int grid = tiles < num_sms() ? tiles : num_sms();
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  if (TPM != 0) {
    // CTAs wait on one another's work (through the flags, also across GPUs): cooperative launch
    // makes the whole grid co-resident
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = S::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, a);
    return e == cudaSuccess ? 0 : -3;
  }
  kern<<<grid, 192, S::SMEM_BYTES, st>>>(ta, tb, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

template <int BN, int EPI>
static int dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const GemmArgs& a, cudaStream_t st, int max_ctas) {
  if (!a_mn && !b_mn) return launch_gemm<BN, false, false, EPI>(ta, tb, a, st, max_ctas);
  if (!a_mn && b_mn) return launch_gemm<BN, false, true, EPI>(ta, tb, a, st, max_ctas);
  if (a_mn && b_mn) return launch_gemm<BN, true, true, EPI>(ta, tb, a, st, max_ctas);
  return launch_gemm<BN, true, false, EPI>(ta, tb, a, st, max_ctas);
}

template <int BN>
static int dispatch_epi(int epi, bool a_mn, bool b_mn, const CUtensorMap& ta,
                        const CUtensorMap& tb, const GemmArgs& a, cudaStream_t st, int max_ctas) {
  switch (epi) {
    case kEpiBF16: return dispatch_major<BN, kEpiBF16>(a_mn, b_mn, ta, tb, a, st, max_ctas);
    case kEpiBF16Resid:
      return dispatch_major<BN, kEpiBF16Resid>(a_mn, b_mn, ta, tb, a, st, max_ctas);
    case kEpiF32: return dispatch_major<BN, kEpiF32>(a_mn, b_mn, ta, tb, a, st, max_ctas);
    case kEpiF32Acc: return dispatch_major<BN, kEpiF32Acc>(a_mn, b_mn, ta, tb, a, st, max_ctas);
    case kEpiBF16Rope:  // forward projections only: both operands K-major
      if (a_mn || b_mn) return -4;
      return launch_gemm<BN, false, false, kEpiBF16Rope>(ta, tb, a, st, max_ctas);
    case kEpiSwiGLUBwd:
      if (a_mn || !b_mn) return -4;
      return launch_gemm<BN, false, true, kEpiSwiGLUBwd>(ta, tb, a, st, max_ctas);
  }
  return -4;
}

// TPM != 0: the CTAs wait on one another's work (through the flags, also across GPUs), so the
// launch is also cooperative, which makes the whole grid co-resident.
template <bool A_MN, bool B_MN, int EPI, int TPM = 0>
static int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                            cudaStream_t st) {
  using S = PairShape;
  auto kern = gemm_bf16_sm100_pair<A_MN, B_MN, EPI, TPM>;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.blockDim = dim3(TPM != 0 ? 256 : 192);
  cfg.dynamicSmemBytes = S::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = TPM != 0 ? 2 : 1;
  static int max_pairs = 0;
  if (max_pairs == 0) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM_BYTES);
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    max_pairs = n < num_sms() / 2 ? n : num_sms() / 2;
  }
  constexpr int TN = EPI == kEpiSwiGLU ? 128 : 256;
  const long long units =
      static_cast<long long>((a.M + 255) / 256) * ((a.N + TN - 1) / TN) * a.ksplit;
  const int pairs = units < max_pairs ? static_cast<int>(units) : max_pairs;
  cfg.gridDim = dim3(2 * pairs);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, a);
  return e == cudaSuccess ? 0 : -3;
}

template <int EPI>
static int dispatch_pair_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                               const GemmArgs& a, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_gemm_pair<false, false, EPI>(ta, tb, a, st);
  if (!a_mn && b_mn) return launch_gemm_pair<false, true, EPI>(ta, tb, a, st);
  if (a_mn && b_mn) return launch_gemm_pair<true, true, EPI>(ta, tb, a, st);
  return launch_gemm_pair<true, false, EPI>(ta, tb, a, st);
}

static int dispatch_pair(int epi, bool a_mn, bool b_mn, const CUtensorMap& ta,
                         const CUtensorMap& tb, const GemmArgs& a, cudaStream_t st) {
  switch (epi) {
    case kEpiBF16: return dispatch_pair_major<kEpiBF16>(a_mn, b_mn, ta, tb, a, st);
    case kEpiBF16Resid: return dispatch_pair_major<kEpiBF16Resid>(a_mn, b_mn, ta, tb, a, st);
    case kEpiF32: return dispatch_pair_major<kEpiF32>(a_mn, b_mn, ta, tb, a, st);
    case kEpiF32Acc: return dispatch_pair_major<kEpiF32Acc>(a_mn, b_mn, ta, tb, a, st);
    case kEpiBF16Rope:
      if (a_mn || b_mn) return -4;
      return launch_gemm_pair<false, false, kEpiBF16Rope>(ta, tb, a, st);
    case kEpiSwiGLUBwd:  // down-projection dgrad only: A K-major, B MN-major
      if (a_mn || !b_mn) return -4;
      return launch_gemm_pair<false, true, kEpiSwiGLUBwd>(ta, tb, a, st);
    case kEpiCEPart:  // lm_head forward / recompute: both operands K-major
      if (a_mn || b_mn) return -4;
      return launch_gemm_pair<false, false, kEpiCEPart>(ta, tb, a, st);
    case kEpiCEGrad:
      if (a_mn || b_mn) return -4;
      return launch_gemm_pair<false, false, kEpiCEGrad>(ta, tb, a, st);
  }
  return -4;
}

}  // namespace cfb

using namespace cfb;

// Tile shape and split-K factor of a GEMM.  Candidates: a 256 x 256 tile on a CTA pair
// (`pair`), or a 128 x bn tile on one CTA (bn = 128 or 256); with `can_split` (fp32 accumulate
// epilogue) each tile may also be split into s <= 4 ranges of at least 16 k-blocks, whose
// partial sums are reduced into D.  The estimated time of a candidate is
//   waves * (k-blocks per unit) * (SM time per k-block)
// with waves = ceil(units / slots) (slots: SMs, or co-resident CTA pairs), and the SM time per
// k-block of a 128 x 256 share measured relative to the single-CTA bn = 256 kernel: the bn = 128
// kernel moves 4/3 as many operand bytes per FLOP and runs about 1/3 slower, the pair kernel
// moves 2/3 as many.  Splits pay 2% each for their fp32 reduction traffic.  A later candidate
// must win by 3% (the pair kernel without split is tried first).
struct GemmPlan {
  int bn;
  int ksplit;
  bool pair;
};

// bn_req: 0 any tile, 128 / 256 that single-CTA tile only, -1 the pair tile only
static GemmPlan plan_gemm(int M, int N, int K, int bn_req, bool can_split, bool can_pair,
                          int sms) {
  const int num_kb = (K + 63) / 64;
  GemmPlan best{256, 1, false};
  double best_t = 1e300;
  auto consider = [&](int bn, bool pair, int s) {
    if (s > 1 && num_kb / s < 16) return;
    const long long tiles = pair ? ((M + 255LL) / 256) * ((N + 255LL) / 256)
                                 : ((M + 127LL) / 128) * ((N + bn - 1LL) / bn);
    const long long units = tiles * s;
    const int slots = pair ? sms / 2 : sms;
    const long long waves = (units + slots - 1) / slots;
    const double kbpu = static_cast<double>((num_kb + s - 1) / s);
    const double per_kb = pair ? 0.9 : (bn == 256 ? 1.0 : 0.5 * 1.33);
    double t = static_cast<double>(waves) * kbpu * per_kb * (1.0 + 0.02 * (s - 1));
    if (t < best_t * 0.97) {
      best_t = t;
      best = GemmPlan{pair ? 256 : bn, s, pair};
    }
  };
  const int max_s = can_split ? 4 : 1;
  const bool single256 = bn_req == 256 || (bn_req == 0 && N > 128);
  const bool single128 = bn_req == 128 || bn_req == 0;
  for (int s = 1; s <= max_s; ++s) {
    if (can_pair) consider(256, true, s);
    if (single256) consider(256, false, s);
    if (single128) consider(128, false, s);
  }
  return best;
}

// operands of the dual-column epilogues (SwiGLU backward) that the other entries leave unset
struct EpiExtra {
  int dual_off;
  const void* aux;
  long long ld_aux;
  const int* aux_rows;
  // cross-entropy epilogues
  const long long* ce_labels = nullptr;
  float *ce_pmax = nullptr, *ce_psum = nullptr, *ce_ptgt = nullptr;
  const float *ce_lse = nullptr, *ce_dloss = nullptr;
  int ce_nt = 0;
};

static int gemm_entry(const void* A, long long lda, int a_mn, const void* B, long long ldb,
                      int b_mn, void* D, long long ldd, int epi, const void* R, long long ldr,
                      int M, int N, int K, float alpha, int* err, int bn, int max_ctas,
                      const int* pos, const float* cs, int rope_cols, int hd,
                      const CfbTpGemm* tp, cudaStream_t st, const EpiExtra* ex = nullptr) {
  if (M <= 0 || N <= 0 || K <= 0) return -10;
  if ((N % 32) != 0 || (lda % 8) != 0 || (ldb % 8) != 0) return -11;
  const int tp_bn_req = tp ? bn : 0;  // a single-CTA tile width asked for by a TP caller
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) ||
      (reinterpret_cast<uintptr_t>(D) & 15))
    return -12;
  // CFB_GEMM_SPLIT_K=0 keeps one unit per tile (fixed fp32 summation order);
  // CFB_GEMM_PAIR=0 keeps every GEMM on single-CTA tiles
  static const bool split_k_on = [] {
    const char* e = std::getenv("CFB_GEMM_SPLIT_K");
    return !(e && e[0] == '0');
  }();
  static const bool pair_on = [] {
    const char* e = std::getenv("CFB_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  // CFB_GEMM_ACC_RED=0: fp32-accumulate epilogues load, add and store instead of reducing
  static const bool acc_red = [] {
    const char* e = std::getenv("CFB_GEMM_ACC_RED");
    return !(e && e[0] == '0');
  }();
  int ksplit = 1;
  bool pair = false;
  if (!tp && max_ctas <= 0 && epi != kEpiSwiGLU) {
    const bool can_split = epi == kEpiF32Acc && (ldd % 4) == 0 && split_k_on;
    const bool force_pair = bn == kGemmTilePair;
    const bool can_pair = force_pair || (pair_on && bn == 0);
    const GemmPlan pl =
        plan_gemm(M, N, K, force_pair ? -1 : bn, can_split, can_pair, num_sms());
    bn = pl.bn;
    ksplit = pl.ksplit;
    pair = pl.pair;
  } else if (bn != 128 && bn != 256) {
    const long long tiles256 = ((M + 127LL) / 128) * ((N + 255LL) / 256);
    bn = (N <= 128 || tiles256 < num_sms()) ? 128 : 256;
  }
  // Tensor-parallel fused modes on the CTA pair (256 x 256 tiles, push / pull warps in both
  // CTAs).  CFB_TP_PAIR: 1 (default) the all-gather consumers only, 2 also the reduce-scatter
  // producers, 0 neither.  Measured at TP = 2, 16384 x 4096 Llama-3-8B layer shapes: the gate /
  // up all-gather GEMM runs 11% faster on the pair (1.24 vs 1.39 ms, NCCL path 1.39 ms), the
  // reduce-scatter GEMMs are within noise or slower (o-proj 0.90-0.95 vs 0.82-0.92 ms).
  static const int tp_pair_mode = [] {
    const char* e = std::getenv("CFB_TP_PAIR");
    return e ? std::atoi(e) : 1;
  }();
  const bool tp_pair = tp && pair_on && max_ctas <= 0 && tp_bn_req == 0 &&
                       (tp->mode == 1 ? tp_pair_mode >= 1 : tp_pair_mode >= 2);
  CUtensorMap ta, tb;
  int rc;
  // A: K-major [M, K] (ld=lda) or MN-major [K, M]
  rc = a_mn ? make_tmap_2d_bf16(&ta, A, K, M, lda, 64, 64)
            : make_tmap_2d_bf16(&ta, A, M, K, lda, 64, 128);
  if (rc) return rc * 100 - 1;
  rc = b_mn ? make_tmap_2d_bf16(&tb, B, K, N, ldb, 64, 64)
            : make_tmap_2d_bf16(&tb, B, N, K, ldb, 64, (pair || tp_pair) ? 128 : bn);
  if (rc) return rc * 100 - 2;
  GemmArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.ksplit = ksplit;
  a.acc_red = (acc_red && (ldd % 4) == 0) ? 1 : 0;
  a.D = D;
  a.ldd = ldd;
  a.R = reinterpret_cast<const __nv_bfloat16*>(R);
  a.ldr = ldr;
  a.alpha = alpha;
  a.err = err;
  a.pos = pos;
  a.cs = cs;
  a.rope_cols = rope_cols;
  a.hd = hd;
  a.dual_off = ex ? ex->dual_off : 0;
  a.aux = ex ? const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(ex->aux)) : nullptr;
  a.ld_aux = ex ? ex->ld_aux : 0;
  a.aux_rows = ex ? ex->aux_rows : nullptr;
  a.ce_labels = ex ? ex->ce_labels : nullptr;
  a.ce_pmax = ex ? ex->ce_pmax : nullptr;
  a.ce_psum = ex ? ex->ce_psum : nullptr;
  a.ce_ptgt = ex ? ex->ce_ptgt : nullptr;
  a.ce_lse = ex ? ex->ce_lse : nullptr;
  a.ce_dloss = ex ? ex->ce_dloss : nullptr;
  a.ce_nt = ex ? ex->ce_nt : 0;
  a.rank = 0;
  a.P = 1;
  a.seg = nullptr;
  a.epoch = 0;
  a.peer_flags = nullptr;
  a.flag_ready = a.flag_done = 0;
  a.tile_cnt = nullptr;
  a.rot_mblocks = 0;
  a.lda = lda;
  a.ag_mc = nullptr;
  a.ag_peers = nullptr;
  a.mc_part = nullptr;
  a.peer_part = nullptr;
  a.flag_blk = 0;
  a.interleave_spb = 0;
  a.rs_resid = nullptr;
  a.rs_out = nullptr;
  a.ld_resid = a.ld_out = 0;
  a.out_rows = 0;
  if (tp) {
    if (tp->mode != 1 && tp->mode != 2) return -13;
    if (a_mn) return -13;  // rows of A are the sequence-parallel rows
    if (tp->P < 1 || tp->P > 64 || !tp->seg || !tp->peer_flags || !tp->tile_cnt) return -13;
    // the collective warps index a rank's rows x (K or N) / 8 vectors with 32-bit integers
    if (static_cast<long long>(M) * ((K > N ? K : N) / 8) >= (1LL << 31)) return -13;
    a.rank = tp->rank;
    a.P = tp->P;
    a.seg = tp->seg;
    a.epoch = tp->epoch;
    a.peer_flags = tp->peer_flags;
    a.flag_ready = tp->flag_ready;
    a.flag_done = tp->flag_done;
    a.tile_cnt = tp->tile_cnt;
    if (tp->mode == 1) {
      if (tp->rot_rows % 128 || !tp->ag_peers || (K % 8) || (lda % 8)) return -13;
      a.rot_mblocks = tp->rot_rows / 128;
      a.ag_mc = static_cast<__nv_bfloat16*>(tp->ag_mc);
      a.ag_peers = reinterpret_cast<__nv_bfloat16* const*>(tp->ag_peers);
      if (tp_pair) {
        GemmArgs ap = a;
        ap.rot_mblocks = tp->rot_rows / 256;  // in 256-row pair blocks
        int rc2 = -4;
        if (epi == kEpiBF16)
          rc2 = b_mn ? launch_gemm_pair<false, true, kEpiBF16, 1>(ta, tb, ap, st)
                     : launch_gemm_pair<false, false, kEpiBF16, 1>(ta, tb, ap, st);
        else if (epi == kEpiBF16Rope && !b_mn)
          rc2 = launch_gemm_pair<false, false, kEpiBF16Rope, 1>(ta, tb, ap, st);
        if (rc2 != -3) return rc2;
        cudaGetLastError();  // launch refused (configuration): single-CTA tiles below
        if (b_mn == 0 && make_tmap_2d_bf16(&tb, B, N, K, ldb, 64, bn)) return -2;
      }
#define CFB_TP1(BNV, BMN, E) launch_gemm<BNV, false, BMN, E, 1>(ta, tb, a, st, max_ctas)
      if (epi == kEpiBF16) {
        if (b_mn) return bn == 256 ? CFB_TP1(256, true, kEpiBF16) : CFB_TP1(128, true, kEpiBF16);
        return bn == 256 ? CFB_TP1(256, false, kEpiBF16) : CFB_TP1(128, false, kEpiBF16);
      }
      if (epi == kEpiBF16Rope && !b_mn)
        return bn == 256 ? CFB_TP1(256, false, kEpiBF16Rope) : CFB_TP1(128, false, kEpiBF16Rope);
#undef CFB_TP1
      return -4;
    }
    if (epi != kEpiBF16 || !tp->out || (N % 8) || tp->out_rows < 0 ||
        (!tp->mc_part && !tp->peer_part))
      return -13;
    a.mc_part = static_cast<const __nv_bfloat16*>(tp->mc_part);
    a.peer_part = reinterpret_cast<const __nv_bfloat16* const*>(tp->peer_part);
    a.flag_blk = tp->flag_blk;
    a.interleave_spb = tp->interleave_spb;
    if (a.interleave_spb > 0 && (M != tp->P * a.interleave_spb * 128)) return -13;
    a.rs_resid = static_cast<const __nv_bfloat16*>(tp->resid);
    a.rs_out = static_cast<__nv_bfloat16*>(tp->out);
    a.ld_resid = tp->ld_resid;
    a.ld_out = tp->ld_out;
    a.out_rows = tp->out_rows;
    if (tp_pair && (a.interleave_spb % 2) == 0) {
      GemmArgs ap = a;
      ap.interleave_spb = a.interleave_spb / 2;  // in 256-row pair blocks
      const int rc2 = b_mn ? launch_gemm_pair<false, true, kEpiBF16, 2>(ta, tb, ap, st)
                           : launch_gemm_pair<false, false, kEpiBF16, 2>(ta, tb, ap, st);
      if (rc2 != -3) return rc2;
      cudaGetLastError();  // launch refused (configuration): single-CTA tiles below
      if (b_mn == 0 && make_tmap_2d_bf16(&tb, B, N, K, ldb, 64, bn)) return -2;
    }
#define CFB_TP2(BNV, BMN) launch_gemm<BNV, false, BMN, kEpiBF16, 2>(ta, tb, a, st, max_ctas)
    if (b_mn) return bn == 256 ? CFB_TP2(256, true) : CFB_TP2(128, true);
    return bn == 256 ? CFB_TP2(256, false) : CFB_TP2(128, false);
#undef CFB_TP2
  }
  if (pair) return dispatch_pair(epi, a_mn, b_mn, ta, tb, a, st);
  if (bn == 256) return dispatch_epi<256>(epi, a_mn, b_mn, ta, tb, a, st, max_ctas);
  return dispatch_epi<128>(epi, a_mn, b_mn, ta, tb, a, st, max_ctas);
}

int cfb_gemm_ce_part(const void* X, long long ldx, const void* W, long long ldw, int M, int N,
                     int K, const long long* labels, float* pmax, float* psum, float* ptgt,
                     int* err, cudaStream_t st) {
  if (!labels || !pmax || !psum || !ptgt) return -13;
  EpiExtra ex{0, nullptr, 0, nullptr};
  ex.ce_labels = labels;
  ex.ce_pmax = pmax;
  ex.ce_psum = psum;
  ex.ce_ptgt = ptgt;
  ex.ce_nt = (N + 255) / 256;
  return gemm_entry(X, ldx, 0, W, ldw, 0, nullptr, 0, kEpiCEPart, nullptr, 0, M, N, K, 1.0f,
                    err, kGemmTilePair, 0, nullptr, nullptr, 0, 0, nullptr, st, &ex);
}

int cfb_gemm_ce_grad(const void* X, long long ldx, const void* W, long long ldw, void* dlogits,
                     long long ldd, int M, int N, int K, const long long* labels,
                     const float* lse, const float* dloss, int* err, cudaStream_t st) {
  if (!labels || !lse || !dloss || !dlogits || (ldd % 8)) return -13;
  EpiExtra ex{0, nullptr, 0, nullptr};
  ex.ce_labels = labels;
  ex.ce_lse = lse;
  ex.ce_dloss = dloss;
  return gemm_entry(X, ldx, 0, W, ldw, 0, dlogits, ldd, kEpiCEGrad, nullptr, 0, M, N, K, 1.0f,
                    err, kGemmTilePair, 0, nullptr, nullptr, 0, 0, nullptr, st, &ex);
}

int cfb_gemm_bf16(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn,
                  void* D, long long ldd, int epi, const void* R, long long ldr, int M, int N,
                  int K, float alpha, int* err, int bn, int max_ctas, cudaStream_t st) {
  if (epi == kEpiBF16Rope || epi == kEpiSwiGLU || epi == kEpiSwiGLUBwd || epi == kEpiCEPart ||
      epi == kEpiCEGrad)
    return -4;
  return gemm_entry(A, lda, a_mn, B, ldb, b_mn, D, ldd, epi, R, ldr, M, N, K, alpha, err, bn,
                    max_ctas, nullptr, nullptr, 0, 0, nullptr, st);
}

int cfb_gemm_bf16_rope(const void* A, long long lda, const void* B, long long ldb, void* D,
                       long long ldd, int M, int N, int K, const int* pos, const float* cos_sin,
                       int rope_cols, int head_dim, int* err, int bn, int max_ctas,
                       cudaStream_t st) {
  if (head_dim != 64 && head_dim != 128) return -13;
  if (rope_cols < 0 || rope_cols % head_dim || rope_cols > N || !pos || !cos_sin) return -13;
  if (reinterpret_cast<uintptr_t>(cos_sin) & 15) return -12;
  return gemm_entry(A, lda, 0, B, ldb, 0, D, ldd, kEpiBF16Rope, nullptr, 0, M, N, K, 1.0f, err,
                    bn, max_ctas, pos, cos_sin, rope_cols, head_dim, nullptr, st);
}

int cfb_gemm_swiglu(const void* A, long long lda, const void* B, long long ldb, void* GU,
                    long long ld_gu, void* Hout, long long ld_h, int M, int F, int K, int* err,
                    cudaStream_t st) {
  if (M <= 0 || F <= 0 || K <= 0) return -10;
  if ((F % 128) || (lda % 8) || (ldb % 8) || (ld_gu % 8) || (ld_h % 8)) return -11;
  if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15) ||
      (reinterpret_cast<uintptr_t>(GU) & 15) || (reinterpret_cast<uintptr_t>(Hout) & 15))
    return -12;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d_bf16(&ta, A, M, K, lda, 64, 128);
  if (rc) return rc * 100 - 1;
  rc = make_tmap_2d_bf16(&tb, B, 2LL * F, K, ldb, 64, 128);
  if (rc) return rc * 100 - 2;
  GemmArgs a = {};
  a.M = M;
  a.N = F;
  a.K = K;
  a.ksplit = 1;
  a.D = GU;
  a.ldd = ld_gu;
  a.alpha = 1.0f;
  a.err = err;
  a.dual_off = F;
  a.aux = static_cast<__nv_bfloat16*>(Hout);
  a.ld_aux = ld_h;
  a.P = 1;
  static const bool pair_on = [] {
    const char* e = std::getenv("CFB_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  if (pair_on) return launch_gemm_pair<false, false, kEpiSwiGLU>(ta, tb, a, st);
  return launch_gemm<128, false, false, kEpiSwiGLU>(ta, tb, a, st, 0);
}

int cfb_gemm_plan(int M, int N, int K, int epi, int bn, int sms, int* out_bn, int* out_ksplit,
                  int* out_pair) {
  if (M <= 0 || N <= 0 || K <= 0 || sms <= 0) return -10;
  const bool force_pair = bn == kGemmTilePair;
  const GemmPlan pl = plan_gemm(M, N, K, force_pair ? -1 : bn, epi == kEpiF32Acc,
                                force_pair || bn == 0, sms);
  *out_bn = pl.bn;
  *out_ksplit = pl.ksplit;
  *out_pair = pl.pair ? 1 : 0;
  return 0;
}

int cfb_gemm_swiglu_bwd(const void* dY, long long ld_dy, const void* Wd, long long ld_w,
                        const void* gu, long long ld_gu, const int* gu_rows, void* dgu,
                        long long ld_dgu, int M, int F, int K, int* err, cudaStream_t st) {
  if ((ld_gu % 8) || (ld_dgu % 8) || (F % 8) || !gu) return -11;
  if (reinterpret_cast<uintptr_t>(gu) & 15) return -12;
  const EpiExtra ex{F, gu, ld_gu, gu_rows};
  return gemm_entry(dY, ld_dy, 0, Wd, ld_w, 1, dgu, ld_dgu, kEpiSwiGLUBwd, nullptr, 0, M, F, K,
                    1.0f, err, 0, 0, nullptr, nullptr, 0, 0, nullptr, st, &ex);
}

int cfb_gemm_tp(const void* A, long long lda, const void* B, long long ldb, int b_mn, void* D,
                long long ldd, int M, int N, int K, const int* pos, const float* cos_sin,
                int rope_cols, int head_dim, const CfbTpGemm* tp, int* err, int bn,
                cudaStream_t st) {
  if (!tp) return -13;
  const int epi = cos_sin ? kEpiBF16Rope : kEpiBF16;
  if (cos_sin && (head_dim != 64 && head_dim != 128)) return -13;
  return gemm_entry(A, lda, 0, B, ldb, b_mn, D, ldd, epi, nullptr, 0, M, N, K, 1.0f, err, bn, 0,
                    pos, cos_sin, rope_cols, head_dim, tp, st);
}
