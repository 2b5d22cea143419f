// Memory-bound fused kernels of the filtered training step (sm_100a).
//
// Each is written for HBM3e streaming: 16-byte vector loads/stores, one warp or one block per
// row, fp32 math, a single bf16 rounding on output.  The backward kernels take a row-index
// array so that they read saved activations of kept tokens in place (no separate gather pass).
//
//   rmsnorm_fwd / rmsnorm_bwd   RMSNorm with saved rstd; bwd fuses the residual-gradient add
//                               and a blocked dgamma reduction
//   rope                        rotate-half RoPE on the q and k heads of the fused qkv rows,
//                               forward or inverse (backward), at original token positions
//   swiglu_fwd / swiglu_bwd     h = silu(g) * u and its gradient
//   gather_rows                 kept-row gather of a [T, C] activation
//   embedding_fwd / _bwd        row gather and fp32 scatter-add of kept rows
//   ce_fwd / ce_bwd             per-token cross entropy (loss, lse) and kept-row dlogits
//   adamw                       fused AdamW on a flat fp32 master shard, bf16 param write
//   sumsq / clip_coef           global grad-norm and clip coefficient, kept on the device
//   drop_smallest               per-row selection of the k smallest scores (bitonic sort)
//   keep_index                  kept positions / flattened kept-row ids from the mask
#include "sm100_common.cuh"
#include "launch_api.h"

#include <math_constants.h>

namespace cfb {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

// ---------------------------------------------------------------- RMSNorm
// One warp per row.  y = x * rstd * w ; rstd = (mean(x^2) + eps)^-1/2.
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                   int rows, int H, float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (row >= rows) return;
  const int lane = lane_id();
  const __nv_bfloat16* xr = x + static_cast<long long>(row) * H;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(H) + eps);
  if (lane == 0 && rstd) rstd[row] = r;
  __nv_bfloat16* yr = y + static_cast<long long>(row) * H;
  for (int c = lane * 8; c < H; c += 256) {
    float f[8], g[8];
    load8(xr + c, f);
    load8(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = f[i] * r * g[i];
    store8(yr + c, f);
  }
}

// Block of 256 threads walks a contiguous range of rows; each thread owns H/2048 groups of 8
// columns and keeps their dgamma partial sums in registers.
template <int GROUPS>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const int* __restrict__ x_rows, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ dres,
    __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_partial, int rows, int H) {
  __shared__ float red[8];
  const int tid = threadIdx.x;
  const int per = (rows + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * per;
  const int r1 = min(rows, r0 + per);
  float dw[GROUPS][8];
  float wv[GROUPS][8];
#pragma unroll
  for (int g = 0; g < GROUPS; ++g) {
    const int c = (tid + g * 256) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) dw[g][i] = 0.f;
    if (c < H) load8(w + c, wv[g]);
  }
  for (int r = r0; r < r1; ++r) {
    const long long xr = x_rows ? x_rows[r] : r;
    const float rs = rstd[xr];
    float dyv[GROUPS][8], xv[GROUPS][8];
    float dot = 0.f;
#pragma unroll
    for (int g = 0; g < GROUPS; ++g) {
      const int c = (tid + g * 256) * 8;
      if (c < H) {
        load8(dy + static_cast<long long>(r) * H + c, dyv[g]);
        load8(x + xr * H + c, xv[g]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          dot += wv[g][i] * dyv[g][i] * xv[g][i];
          dw[g][i] += dyv[g][i] * xv[g][i] * rs;
        }
      }
    }
    dot = warp_sum(dot);
    if ((tid & 31) == 0) red[tid >> 5] = dot;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    __syncthreads();
    const float coef = tot * rs * rs * rs / static_cast<float>(H);
#pragma unroll
    for (int g = 0; g < GROUPS; ++g) {
      const int c = (tid + g * 256) * 8;
      if (c < H) {
        float o[8];
        if (dres) {
          load8(dres + static_cast<long long>(r) * H + c, o);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += rs * wv[g][i] * dyv[g][i] - xv[g][i] * coef;
        store8(dx + static_cast<long long>(r) * H + c, o);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GROUPS; ++g) {
    const int c = (tid + g * 256) * 8;
    if (c < H) {
      float* dst = dw_partial + static_cast<long long>(blockIdx.x) * H + c;
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = dw[g][i];
    }
  }
}

// Warp per row: the lane owns NG groups of 8 columns, c = (lane + 32 g) * 8, and keeps their
// dgamma partial sums in registers across the rows of its warp.  Pass 1 reads dy, x for the row
// dot product; pass 2 re-reads them (L1-resident) to write dx.  No block barrier per row.
template <int NG>
__global__ void __launch_bounds__(256) rmsnorm_bwd_warp_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const int* __restrict__ x_rows, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ dres,
    __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_partial, int rows, int H) {
  const int lane = lane_id(), wp = warp_id();
  float dw[NG][8];
#pragma unroll
  for (int g = 0; g < NG; ++g)
#pragma unroll
    for (int i = 0; i < 8; ++i) dw[g][i] = 0.f;
  const float inv_h = 1.f / static_cast<float>(H);
  for (int r = blockIdx.x * 8 + wp; r < rows; r += gridDim.x * 8) {
    const long long xr = x_rows ? x_rows[r] : r;
    const float rs = rstd[xr];
    const __nv_bfloat16* dyr = dy + static_cast<long long>(r) * H;
    const __nv_bfloat16* xrp = x + xr * H;
    float dot = 0.f;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const int c = (lane + 32 * g) * 8;
      if (c < H) {
        float a[8], b[8], wv[8];
        load8(dyr + c, a);
        load8(xrp + c, b);
        load8(w + c, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float t = a[i] * b[i];
          dot += wv[i] * t;
          dw[g][i] += t * rs;
        }
      }
    }
    dot = warp_sum(dot);
    const float coef = dot * rs * rs * rs * inv_h;
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      const int c = (lane + 32 * g) * 8;
      if (c < H) {
        float a[8], b[8], wv[8], o[8];
        load8(dyr + c, a);
        load8(xrp + c, b);
        load8(w + c, wv);
        if (dres) {
          load8(dres + static_cast<long long>(r) * H + c, o);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += rs * wv[i] * a[i] - b[i] * coef;
        store8(dx + static_cast<long long>(r) * H + c, o);
      }
    }
  }
  // block reduction of the eight warps' partial sums (256 columns at a time), then one partial
  // row per block
  __shared__ float red[8][256];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
#pragma unroll
    for (int i = 0; i < 8; ++i) red[wp][lane * 8 + i] = dw[g][i];
    __syncthreads();
    const int c = g * 256 + threadIdx.x;
    if (c < H) {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) t += red[k][threadIdx.x];
      dw_partial[static_cast<long long>(blockIdx.x) * H + c] = t;
    }
    __syncthreads();
  }
}

// out[c] += sum_p partial[p, c].  Block = 32 columns x 8 row slices; the slices are combined
// in a fixed order (deterministic).
__global__ void __launch_bounds__(256) colsum_acc_kernel(const float* __restrict__ partial,
                                                         float* __restrict__ out, int P, int H) {
  __shared__ float red[8][33];
  const int cx = threadIdx.x & 31, ry = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cx;
  float s = 0.f;
  if (c < H)
    for (int p = ry; p < P; p += 8) s += partial[static_cast<long long>(p) * H + c];
  red[ry][cx] = s;
  __syncthreads();
  if (ry == 0 && c < H) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][cx];
    out[c] += t;
  }
}

// ---------------------------------------------------------------- RoPE
// Rotate-half RoPE on heads [0, n_heads) of each row (q heads then k heads of a qkv row).
// cos_sin: [max_pos, hd/2, 2] fp32.  inverse=1 applies the transpose rotation (backward).
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qkv, long long ld,
                            const int* __restrict__ pos, int rows, int n_heads, int hd,
                            const float2* __restrict__ cs, int inverse) {
  const int half = hd >> 1;
  const long long total = static_cast<long long>(rows) * n_heads * half;
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(t % half);
    const long long rh = t / half;
    const int h = static_cast<int>(rh % n_heads);
    const int r = static_cast<int>(rh / n_heads);
    const float2 c = cs[static_cast<long long>(pos[r]) * half + i];
    const float sn = inverse ? -c.y : c.y;
    __nv_bfloat16* base = qkv + r * ld + h * hd;
    const float x1 = __bfloat162float(base[i]);
    const float x2 = __bfloat162float(base[i + half]);
    base[i] = __float2bfloat16(x1 * c.x - x2 * sn);
    base[i + half] = __float2bfloat16(x2 * c.x + x1 * sn);
  }
}

// ---------------------------------------------------------------- SwiGLU
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ h, int rows, int F) {
  const long long groups = static_cast<long long>(rows) * (F / 8);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < groups;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = t / (F / 8);
    const int c = static_cast<int>(t % (F / 8)) * 8;
    float g[8], u[8], o[8];
    load8(gu + r * 2 * F + c, g);
    load8(gu + r * 2 * F + F + c, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      // the bf16-rounded gate / up as stored, the same formula as the GEMM epilogue
      o[i] = silu_tanh(g[i]) * u[i];
    }
    store8(h + r * F + c, o);
  }
}

// With h_out, also writes h = silu(g) * u of the processed rows (the forward's activation of
// the kept rows, recomputed instead of gathered).
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh,
                                  const __nv_bfloat16* __restrict__ gu,
                                  const int* __restrict__ gu_rows,
                                  __nv_bfloat16* __restrict__ dgu,
                                  __nv_bfloat16* __restrict__ h_out, int rows, int F) {
  const long long groups = static_cast<long long>(rows) * (F / 8);
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < groups;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = t / (F / 8);
    const int c = static_cast<int>(t % (F / 8)) * 8;
    const long long src = gu_rows ? gu_rows[r] : r;
    float g[8], u[8], d[8], dg[8], du[8];
    load8(gu + src * 2 * F + c, g);
    load8(gu + src * 2 * F + F + c, u);
    load8(dh + r * F + c, d);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = sigmoidf_(g[i]);
      const float silu = g[i] * s;
      du[i] = d[i] * silu;
      dg[i] = d[i] * u[i] * s * (1.f + g[i] * (1.f - s));
    }
    store8(dgu + r * 2 * F + c, dg);
    store8(dgu + r * 2 * F + F + c, du);
    if (h_out) {
      float h[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = silu_tanh(g[i]) * u[i];
      store8(h_out + r * F + c, h);
    }
  }
}

// ---------------------------------------------------------------- gathers
// dst[i, :] = src[idx[i], :]; row_bytes is a multiple of 16.  One warp per row.
// An index outside [0, n) records kErrBounds in the status block; the caller skips the access.
__device__ __forceinline__ bool index_ok(long long i, long long n, int* err) {
  if (i >= 0 && i < n) return true;
  if (err) atomicCAS(err, 0, kErrBounds);
  return false;
}

__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, long long ld_src,
                                   long long src_rows, const int* __restrict__ idx,
                                   uint8_t* __restrict__ dst, long long ld_dst, int rows,
                                   int row_bytes, int* err) {
  const int row = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (row >= rows) return;
  const long long i = idx[row];
  uint4* d = reinterpret_cast<uint4*>(dst + static_cast<long long>(row) * ld_dst);
  if (!index_ok(i, src_rows, err)) {  // out-of-range row id: zero row instead of a stray read
    for (int c = lane_id(); c < row_bytes / 16; c += 32) d[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(src + i * ld_src);
  for (int c = lane_id(); c < row_bytes / 16; c += 32) d[c] = s[c];
}

__global__ void embedding_fwd_kernel(const __nv_bfloat16* __restrict__ table, long long V,
                                     const long long* __restrict__ ids,
                                     __nv_bfloat16* __restrict__ out, int rows, int H, int* err) {
  const int row = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (row >= rows) return;
  const long long tok = ids[row];
  uint4* d = reinterpret_cast<uint4*>(out + static_cast<long long>(row) * H);
  if (!index_ok(tok, V, err)) {  // token id outside the vocabulary: zero embedding
    for (int c = lane_id(); c < H / 8; c += 32) d[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* s = reinterpret_cast<const uint4*>(table + tok * H);
  for (int c = lane_id(); c < H / 8; c += 32) d[c] = s[c];
}

__global__ void embedding_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                     const long long* __restrict__ ids,
                                     const int* __restrict__ id_rows, float* __restrict__ dtable,
                                     long long V, int rows, int H, int* err) {
  const int row = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (row >= rows) return;
  const long long tok = ids[id_rows ? id_rows[row] : row];
  if (!index_ok(tok, V, err)) return;
  float* dst = dtable + tok * H;
  const __nv_bfloat16* src = dy + static_cast<long long>(row) * H;
  for (int c = lane_id() * 8; c < H; c += 256) {
    float f[8];
    load8(src + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) atomicAdd(dst + c + i, f[i]);
  }
}

// Deterministic embedding gradient, in two steps around a stable sort of the rows by token:
//   1. row_tokens: tok[r] = ids[id_rows[r]] (or ids[r]), -1 for a row id outside ids;
//   2. (stable sort of tok on the host side, giving sorted tokens and their source rows)
//   3. embedding_bwd_sorted: the first warp of each run of equal tokens sums the run's rows of
//      dy in ascending row order and adds the sum into the table row, which no other warp
//      touches.  The result does not depend on scheduling (no atomics), so two runs give the
//      same bits.  Token ids outside [0, V) record kErrBounds and are skipped.
__global__ void row_tokens_kernel(const long long* __restrict__ ids, long long n_ids,
                                  const int* __restrict__ id_rows, long long* __restrict__ tok,
                                  int rows, int* err) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const long long i = id_rows ? id_rows[r] : r;
  tok[r] = index_ok(i, n_ids, err) ? ids[i] : -1;
}

__global__ void embedding_bwd_sorted_kernel(const __nv_bfloat16* __restrict__ dy,
                                            const long long* __restrict__ stok,
                                            const long long* __restrict__ order,
                                            float* __restrict__ dtable, long long V, int rows,
                                            int H, int* err) {
  const int i = blockIdx.x * (blockDim.x / 32) + warp_id();
  if (i >= rows) return;
  const long long tok = stok[i];
  if (i > 0 && stok[i - 1] == tok) return;  // not the first row of its run
  if (!index_ok(tok, V, tok < 0 ? nullptr : err)) return;  // -1: row id already reported
  float* dst = dtable + tok * H;
  for (int c = lane_id() * 8; c < H; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = i; j < rows && stok[j] == tok; ++j) {
      float f[8];
      load8(dy + order[j] * H + c, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += f[k];
    }
    float4* d = reinterpret_cast<float4*>(dst + c);
    float4 a = d[0], b = d[1];
    a.x += acc[0]; a.y += acc[1]; a.z += acc[2]; a.w += acc[3];
    b.x += acc[4]; b.y += acc[5]; b.z += acc[6]; b.w += acc[7];
    d[0] = a;
    d[1] = b;
  }
}

// ---------------------------------------------------------------- cross entropy
__device__ __forceinline__ void block_max_sum(float& m, float& s, float* sm_m, float* sm_s) {
  // combine (max, sum-of-exp) pairs across the block (blockDim = 256)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -CUDART_INF_F ? 0.f : s * __expf(m - nm)) +
        (om == -CUDART_INF_F ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sm_m[w] = m;
    sm_s[w] = s;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? sm_m[threadIdx.x] : -CUDART_INF_F;
    s = threadIdx.x < (blockDim.x >> 5) ? sm_s[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, m, o);
      const float os = __shfl_xor_sync(0xffffffffu, s, o);
      const float nm = fmaxf(m, om);
      s = (m == -CUDART_INF_F ? 0.f : s * __expf(m - nm)) +
          (om == -CUDART_INF_F ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (threadIdx.x == 0) {
      sm_m[0] = m;
      sm_s[0] = s;
    }
  }
  __syncthreads();
  m = sm_m[0];
  s = sm_s[0];
}

// One block per row; labels < 0 are ignored (loss 0).
__global__ void __launch_bounds__(256) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits,
                                                     long long ld,
                                                     const long long* __restrict__ labels,
                                                     float* __restrict__ loss,
                                                     float* __restrict__ lse, int V, int* err) {
  __shared__ float sm_m[8], sm_s[8];
  const int row = blockIdx.x;
  const __nv_bfloat16* lr = logits + static_cast<long long>(row) * ld;
  float m = -CUDART_INF_F, s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += 256 * 8) {
    float f[8];
    load8(lr + c, f);
    float lm = f[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, f[i]);
    const float nm = fmaxf(m, lm);
    float acc = (m == -CUDART_INF_F) ? 0.f : s * __expf(m - nm);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += __expf(f[i] - nm);
    s = acc;
    m = nm;
  }
  block_max_sum(m, s, sm_m, sm_s);
  if (threadIdx.x == 0) {
    const float l = m + __logf(s);
    lse[row] = l;
    const long long lab = labels[row];
    // negative labels are ignored positions; labels >= V are errors (recorded, loss 0)
    loss[row] = (lab >= 0 && index_ok(lab, V, err)) ? (l - __bfloat162float(lr[lab])) : 0.f;
  }
}

// dlogits[i, v] = (softmax(logits[src_i])[v] - [v == label]) * dloss[i]; with a vocabulary
// shard the columns are global vocabulary ids vocab_start + v.

// Vocabulary-parallel partial statistics of one shard: row max, sum of exp(logit - max) and
// the logit of the label when it falls in [vocab_start, vocab_start + V) (else 0).
__global__ void __launch_bounds__(256) ce_partial_kernel(
    const __nv_bfloat16* __restrict__ logits, long long ld, const long long* __restrict__ labels,
    float* __restrict__ pmax, float* __restrict__ psum, float* __restrict__ ptgt, int V,
    long long vocab_start) {
  __shared__ float sm_m[8], sm_s[8];
  const int row = blockIdx.x;
  const __nv_bfloat16* lr = logits + static_cast<long long>(row) * ld;
  float m = -CUDART_INF_F, s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += 256 * 8) {
    float f[8];
    load8(lr + c, f);
    float lm = f[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, f[i]);
    const float nm = fmaxf(m, lm);
    float acc = (m == -CUDART_INF_F) ? 0.f : s * __expf(m - nm);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += __expf(f[i] - nm);
    s = acc;
    m = nm;
  }
  block_max_sum(m, s, sm_m, sm_s);
  if (threadIdx.x == 0) {
    pmax[row] = m;
    psum[row] = s;
    const long long lab = labels[row] - vocab_start;
    ptgt[row] = (labels[row] >= 0 && lab >= 0 && lab < V) ? __bfloat162float(lr[lab]) : 0.f;
  }
}
__global__ void __launch_bounds__(256) ce_bwd_kernel(
    const __nv_bfloat16* __restrict__ logits, long long ld, const int* __restrict__ logit_rows,
    const long long* __restrict__ labels, const float* __restrict__ lse,
    const float* __restrict__ dloss, __nv_bfloat16* __restrict__ dlogits, long long ld_out,
    int V, long long vocab_start) {
  const int row = blockIdx.x;
  const long long src = logit_rows ? logit_rows[row] : row;
  const __nv_bfloat16* lr = logits + src * ld;
  __nv_bfloat16* out = dlogits + static_cast<long long>(row) * ld_out;
  const float l = lse[src];
  const float g = dloss[row];
  const long long lab = labels[src];
  for (int c = threadIdx.x * 8; c < V; c += 256 * 8) {
    float f[8];
    load8(lr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float p = __expf(f[i] - l);
      if (c + i + vocab_start == lab) p -= 1.f;
      f[i] = (lab >= 0) ? p * g : 0.f;
    }
    store8(out + c, f);
  }
}

// ---------------------------------------------------------------- optimizer
// MC: `param` is the NVSwitch multicast address of the data-parallel group's bf16 parameters,
// so each updated value is written once and lands on every rank (the ZeRO parameter
// all-gather fused into the optimizer step); n must then be a multiple of 4.
template <bool MC = false>
__global__ void adamw_kernel(float* __restrict__ master, const float* __restrict__ grad,
                             float* __restrict__ m, float* __restrict__ v,
                             __nv_bfloat16* __restrict__ param, long long n, float lr,
                             float b1, float b2, float eps, float wd, float bc1, float bc2,
                             const float* __restrict__ grad_scale) {
  const float gs = grad_scale ? *grad_scale : 1.f;
  if (gs < 0.f) return;  // clip_coef marked the step as failed: no update
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 p = reinterpret_cast<float4*>(master)[i];
    const float4 g = reinterpret_cast<const float4*>(grad)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pp = &p.x;
    const float* gg = &g.x;
    float* m_ = &mm.x;
    float* v_ = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gj = gg[j] * gs;
      pp[j] -= lr * wd * pp[j];
      m_[j] = b1 * m_[j] + (1.f - b1) * gj;
      v_[j] = b2 * v_[j] + (1.f - b2) * gj * gj;
      const float denom = sqrtf(v_[j]) * inv_sqrt_bc2 + eps;
      pp[j] -= step_size * m_[j] / denom;
    }
    reinterpret_cast<float4*>(master)[i] = p;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    uint2 o;
    o.x = pack_bf16x2(p.x, p.y);
    o.y = pack_bf16x2(p.z, p.w);
    if (MC) {
      asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(
                       reinterpret_cast<uint2*>(param) + i),
                   "f"(__uint_as_float(o.x)), "f"(__uint_as_float(o.y))
                   : "memory");
    } else {
      reinterpret_cast<uint2*>(param)[i] = o;
    }
  }
  // tail
  if (!MC && blockIdx.x == 0 && threadIdx.x < (n & 3)) {
    const long long j = n4 * 4 + threadIdx.x;
    const float gj = grad[j] * gs;
    float pj = master[j];
    pj -= lr * wd * pj;
    m[j] = b1 * m[j] + (1.f - b1) * gj;
    v[j] = b2 * v[j] + (1.f - b2) * gj * gj;
    pj -= step_size * m[j] / (sqrtf(v[j]) * inv_sqrt_bc2 + eps);
    master[j] = pj;
    param[j] = __float2bfloat16(pj);
  }
}

__global__ void sumsq_kernel(const float* __restrict__ x, long long n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float t = x[i];
    s += t * t;
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) out[blockIdx.x] = s;
  }
}

// coef = min(1, max_norm / (norm + 1e-6)) * extra_scale  (max_norm <= 0: no clipping)
// status[0] != 0 (a bounded wait of this step gave up): coef = -1, the AdamW kernels' signal to
// leave parameters and moments untouched.
__global__ void clip_coef_kernel(const float* __restrict__ partials, int n, float max_norm,
                                 float extra_scale, float* __restrict__ coef,
                                 float* __restrict__ norm_out, const int* status) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += partials[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) {
      // partials hold sum(g^2) of the raw gradients; the true gradient is g * extra_scale
      const float norm = sqrtf(s) * extra_scale;
      float c = 1.f;
      if (max_norm > 0.f && norm > max_norm) c = max_norm / (norm + 1e-6f);
      const bool failed = status != nullptr && *reinterpret_cast<const volatile int*>(status) != 0;
      if (coef) *coef = failed ? -1.f : c * extra_scale;
      if (norm_out) *norm_out = norm;
    }
  }
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                     long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = __float2bfloat16(x[i]);
}
__global__ void scale_f32_kernel(float* __restrict__ x, long long n, float s) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    x[i] *= s;
}

// ---------------------------------------------------------------- token selection
// Per row: sort (score, index) pairs of [start, end) ascending with a bitonic network in
// shared memory (padded with +inf), then zero the mask at the first k indices.
__global__ void __launch_bounds__(1024) drop_smallest_kernel(
    const float* __restrict__ score, long long ld, int* __restrict__ mask_i32,
    long long* __restrict__ mask_i64, long long ld_mask, int start, int end, int k, int P) {
  extern __shared__ uint8_t sm[];
  float* key = reinterpret_cast<float*>(sm);
  int* val = reinterpret_cast<int*>(key + P);
  const int row = blockIdx.x;
  const int n = end - start;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    if (i < n) {
      float s = score[row * ld + start + i];
      if (s != s) s = CUDART_INF_F;  // NaN sorts last
      key[i] = s;
      val[i] = i;
    } else {
      key[i] = CUDART_INF_F;
      val[i] = 0x7fffffff;
    }
  }
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;
          const float ki = key[i], kj = key[j];
          const int vi = val[i], vj = val[j];
          const bool gt = (ki > kj) || (ki == kj && vi > vj);
          if (gt == up) {
            key[i] = kj;
            key[j] = ki;
            val[i] = vj;
            val[j] = vi;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const long long off = row * ld_mask + start + val[i];
    if (mask_i64) mask_i64[off] = 0;
    if (mask_i32) mask_i32[off] = 0;
  }
}

// Kept positions of each row: pos[b, j] ascending, flat_rows[b*S_keep + j] = b*S + pos.
__global__ void __launch_bounds__(1024) keep_index_kernel(const long long* __restrict__ mask,
                                                          int S, int S_keep, int* __restrict__ pos,
                                                          int* __restrict__ flat_rows,
                                                          int* __restrict__ err) {
  __shared__ int counts[1024];
  const int b = blockIdx.x;
  const int per = (S + blockDim.x - 1) / blockDim.x;
  const int s0 = threadIdx.x * per;
  const int s1 = min(S, s0 + per);
  const long long* mr = mask + static_cast<long long>(b) * S;
  int c = 0;
  for (int s = s0; s < s1; ++s) c += (mr[s] != 0);
  counts[threadIdx.x] = c;
  __syncthreads();
  // inclusive scan (Hillis-Steele)
  for (int o = 1; o < blockDim.x; o <<= 1) {
    const int t = threadIdx.x >= o ? counts[threadIdx.x - o] : 0;
    __syncthreads();
    counts[threadIdx.x] += t;
    __syncthreads();
  }
  const int total = counts[blockDim.x - 1];
  if (threadIdx.x == 0 && total != S_keep && err) atomicCAS(err, 0, kErrKeepCount);
  int j = counts[threadIdx.x] - c;
  for (int s = s0; s < s1; ++s) {
    if (mr[s] != 0) {
      if (j < S_keep) {
        pos[static_cast<long long>(b) * S_keep + j] = s;
        flat_rows[static_cast<long long>(b) * S_keep + j] = b * S + s;
      }
      ++j;
    }
  }
}

static inline int grid_for(long long work, int block, int cap = 148 * 16) {
  long long g = (work + block - 1) / block;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

}  // namespace cfb

using namespace cfb;
typedef __nv_bfloat16 bf16;

static inline int last_err() { return cudaGetLastError() == cudaSuccess ? 0 : -3; }

int cfb_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int rows, int H,
                    float eps, cudaStream_t st) {
  if (H % 8) return -11;
  rmsnorm_fwd_kernel<<<(rows + 7) / 8, 256, 0, st>>>(static_cast<const bf16*>(x),
                                                      static_cast<const bf16*>(w),
                                                      static_cast<bf16*>(y), rstd, rows, H, eps);
  return last_err();
}

int cfb_rmsnorm_bwd(const void* dy, const void* x, const int* x_rows, const float* rstd,
                    const void* w, const void* dres, void* dx, float* dw_partial, float* dw_acc,
                    int rows, int H, int partial_rows, cudaStream_t st) {
  if (H % 8 || H > 8192) return -11;
  const int groups = (H / 8 + 255) / 256;
  const bf16* a = static_cast<const bf16*>(dy);
  const bf16* b = static_cast<const bf16*>(x);
  const bf16* c = static_cast<const bf16*>(w);
  const bf16* d = static_cast<const bf16*>(dres);
  bf16* o = static_cast<bf16*>(dx);
  bool done = false;
  if (H % 256 == 0) {  // warp-per-row kernel
    done = true;
    switch (H / 256) {
      case 1: rmsnorm_bwd_warp_kernel<1><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
      case 2: rmsnorm_bwd_warp_kernel<2><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
      case 4: rmsnorm_bwd_warp_kernel<4><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
      case 8: rmsnorm_bwd_warp_kernel<8><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
      case 16: rmsnorm_bwd_warp_kernel<16><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
      default: done = false;
    }
  }
  if (!done) {
    switch (groups) {
      case 1: rmsnorm_bwd_kernel<1><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
      case 2: rmsnorm_bwd_kernel<2><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
      case 3: rmsnorm_bwd_kernel<3><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
      default: rmsnorm_bwd_kernel<4><<<partial_rows, 256, 0, st>>>(a, b, x_rows, rstd, c, d, o, dw_partial, rows, H); break;
    }
  }
  colsum_acc_kernel<<<(H + 31) / 32, 256, 0, st>>>(dw_partial, dw_acc, partial_rows, H);
  return last_err();
}

int cfb_rope(void* qkv, long long ld, const int* pos, const int* /*row_of*/, int rows,
             int n_heads, int head_dim, const float* cos_sin, int inverse, cudaStream_t st) {
  const long long work = static_cast<long long>(rows) * n_heads * (head_dim / 2);
  rope_kernel<<<grid_for(work, 256, 148 * 32), 256, 0, st>>>(
      static_cast<bf16*>(qkv), ld, pos, rows, n_heads, head_dim,
      reinterpret_cast<const float2*>(cos_sin), inverse);
  return last_err();
}

int cfb_swiglu_fwd(const void* gu, void* h, int rows, int F, cudaStream_t st) {
  if (F % 8) return -11;
  const long long work = static_cast<long long>(rows) * (F / 8);
  swiglu_fwd_kernel<<<grid_for(work, 256, 148 * 32), 256, 0, st>>>(
      static_cast<const bf16*>(gu), static_cast<bf16*>(h), rows, F);
  return last_err();
}

int cfb_swiglu_bwd(const void* dh, const void* gu, const int* gu_rows, void* dgu, void* h_out,
                   int rows, int F, cudaStream_t st) {
  if (F % 8) return -11;
  const long long work = static_cast<long long>(rows) * (F / 8);
  swiglu_bwd_kernel<<<grid_for(work, 256, 148 * 32), 256, 0, st>>>(
      static_cast<const bf16*>(dh), static_cast<const bf16*>(gu), gu_rows,
      static_cast<bf16*>(dgu), static_cast<bf16*>(h_out), rows, F);
  return last_err();
}

int cfb_gather_rows(const void* src, long long ld_src, long long src_rows, const int* idx,
                    void* dst, long long ld_dst, int rows, int row_bytes, int* err,
                    cudaStream_t st) {
  if (row_bytes % 16 || ld_src % 16 || ld_dst % 16) return -11;
  if (rows == 0) return 0;
  gather_rows_kernel<<<(rows + 7) / 8, 256, 0, st>>>(static_cast<const uint8_t*>(src), ld_src,
                                                     src_rows, idx, static_cast<uint8_t*>(dst),
                                                     ld_dst, rows, row_bytes, err);
  return last_err();
}

int cfb_embedding_fwd(const void* table, long long V, const long long* ids, void* out, int rows,
                      int H, int* err, cudaStream_t st) {
  if (H % 8) return -11;
  embedding_fwd_kernel<<<(rows + 7) / 8, 256, 0, st>>>(static_cast<const bf16*>(table), V, ids,
                                                       static_cast<bf16*>(out), rows, H, err);
  return last_err();
}

int cfb_embedding_bwd(const void* dy, const long long* ids, const int* id_rows, float* dtable,
                      long long V, int rows, int H, int* err, cudaStream_t st) {
  if (H % 8) return -11;
  if (rows == 0) return 0;
  embedding_bwd_kernel<<<(rows + 7) / 8, 256, 0, st>>>(static_cast<const bf16*>(dy), ids,
                                                       id_rows, dtable, V, rows, H, err);
  return last_err();
}

int cfb_row_tokens(const long long* ids, long long n_ids, const int* id_rows, long long* tok,
                   int rows, int* err, cudaStream_t st) {
  if (rows == 0) return 0;
  row_tokens_kernel<<<(rows + 255) / 256, 256, 0, st>>>(ids, n_ids, id_rows, tok, rows, err);
  return last_err();
}

int cfb_embedding_bwd_sorted(const void* dy, const long long* sorted_tok,
                             const long long* order, float* dtable, long long V, int rows, int H,
                             int* err, cudaStream_t st) {
  if (H % 8 || (reinterpret_cast<uintptr_t>(dtable) & 15)) return -11;
  if (rows == 0) return 0;
  embedding_bwd_sorted_kernel<<<(rows + 7) / 8, 256, 0, st>>>(
      static_cast<const bf16*>(dy), sorted_tok, order, dtable, V, rows, H, err);
  return last_err();
}

int cfb_ce_fwd(const void* logits, long long ld, const long long* labels, float* loss,
               float* lse, int rows, int V, int* err, cudaStream_t st) {
  if (V % 8 || ld % 8) return -11;
  ce_fwd_kernel<<<rows, 256, 0, st>>>(static_cast<const bf16*>(logits), ld, labels, loss, lse, V,
                                      err);
  return last_err();
}

// One warp per row: lse and loss from the per-tile statistics of the fused lm_head GEMM.
__global__ void __launch_bounds__(256) ce_combine_kernel(
    const float* __restrict__ pmax, const float* __restrict__ psum,
    const float* __restrict__ ptgt, int rows, int nt, const long long* __restrict__ labels,
    long long V, float* __restrict__ loss, float* __restrict__ lse, int* err) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* pm = pmax + static_cast<long long>(row) * nt;
  const float* ps = psum + static_cast<long long>(row) * nt;
  float m = -CUDART_INF_F;
  for (int t = lane; t < nt; t += 32) m = fmaxf(m, pm[t]);
  m = warp_max(m);
  float s = 0.f;
  for (int t = lane; t < nt; t += 32) s += ps[t] * __expf(pm[t] - m);
  s = warp_sum(s);
  if (lane == 0) {
    const float l = m + __logf(s);
    lse[row] = l;
    const long long lab = labels[row];
    loss[row] = (lab >= 0 && index_ok(lab, V, err)) ? l - ptgt[row] : 0.f;
  }
}

int cfb_ce_combine(const float* pmax, const float* psum, const float* ptgt, int rows, int nt,
                   const long long* labels, long long V, float* loss, float* lse, int* err,
                   cudaStream_t st) {
  if (rows <= 0) return 0;
  ce_combine_kernel<<<(rows + 7) / 8, 256, 0, st>>>(pmax, psum, ptgt, rows, nt, labels, V, loss,
                                                    lse, err);
  return last_err();
}

int cfb_ce_bwd(const void* logits, long long ld, const int* logit_rows, const long long* labels,
               const float* lse, const float* dloss, void* dlogits, long long ld_out, int rows,
               int V, long long vocab_start, cudaStream_t st) {
  if (V % 8 || ld % 8 || ld_out % 8) return -11;
  if (rows == 0) return 0;
  ce_bwd_kernel<<<rows, 256, 0, st>>>(static_cast<const bf16*>(logits), ld, logit_rows, labels,
                                      lse, dloss, static_cast<bf16*>(dlogits), ld_out, V,
                                      vocab_start);
  return last_err();
}

int cfb_ce_partial(const void* logits, long long ld, const long long* labels, float* pmax,
                   float* psum, float* ptgt, int rows, int V, long long vocab_start,
                   cudaStream_t st) {
  if (V % 8 || ld % 8) return -11;
  if (rows == 0) return 0;
  ce_partial_kernel<<<rows, 256, 0, st>>>(static_cast<const bf16*>(logits), ld, labels, pmax,
                                          psum, ptgt, V, vocab_start);
  return last_err();
}

int cfb_adamw(float* master, const float* grad, float* m, float* v, void* param_bf16, long long n,
              float lr, float beta1, float beta2, float eps, float wd, float bc1, float bc2,
              const float* grad_scale, cudaStream_t st) {
  if (n == 0) return 0;
  adamw_kernel<<<grid_for(n / 4 + 1, 256, 148 * 8), 256, 0, st>>>(
      master, grad, m, v, static_cast<bf16*>(param_bf16), n, lr, beta1, beta2, eps, wd, bc1, bc2,
      grad_scale);
  return last_err();
}

int cfb_adamw_multicast(float* master, const float* grad, float* m, float* v, void* param_mc,
                        long long n, float lr, float beta1, float beta2, float eps, float wd,
                        float bc1, float bc2, const float* grad_scale, cudaStream_t st) {
  if (n == 0) return 0;
  if (n % 4 || (reinterpret_cast<uintptr_t>(param_mc) & 7)) return -11;
  adamw_kernel<true><<<grid_for(n / 4, 256, 148 * 8), 256, 0, st>>>(
      master, grad, m, v, static_cast<bf16*>(param_mc), n, lr, beta1, beta2, eps, wd, bc1, bc2,
      grad_scale);
  return last_err();
}

int cfb_sumsq(const float* x, long long n, float* out_partial, int nblocks, cudaStream_t st) {
  sumsq_kernel<<<nblocks, 256, 0, st>>>(x, n, out_partial);
  return last_err();
}

int cfb_clip_coef(const float* partials, int n, float max_norm, float extra_scale, float* coef,
                  float* norm_out, const int* status, cudaStream_t st) {
  clip_coef_kernel<<<1, 256, 0, st>>>(partials, n, max_norm, extra_scale, coef, norm_out, status);
  return last_err();
}

int cfb_drop_smallest(const float* score, long long ld, int* mask_i32, long long* mask_i64,
                      long long ld_mask, int rows, int start, int end, int k, cudaStream_t st) {
  const int n = end - start;
  if (n <= 0 || k <= 0) return 0;
  int P = 1;
  while (P < n) P <<= 1;
  if (P > 16384) return -11;
  const int smem = P * 8;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(drop_smallest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  drop_smallest_kernel<<<rows, 1024, smem, st>>>(score, ld, mask_i32, mask_i64, ld_mask, start,
                                                 end, k, P);
  return last_err();
}

int cfb_keep_index(const long long* mask, int B, int S, int S_keep, int* pos, int* flat_rows,
                   int* err, cudaStream_t st) {
  keep_index_kernel<<<B, 1024, 0, st>>>(mask, S, S_keep, pos, flat_rows, err);
  return last_err();
}

int cfb_cast_f32_bf16(const float* x, void* y, long long n, cudaStream_t st) {
  cast_f32_bf16_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, static_cast<bf16*>(y), n);
  return last_err();
}

int cfb_scale_f32(float* x, long long n, float s, cudaStream_t st) {
  scale_f32_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n, s);
  return last_err();
}
