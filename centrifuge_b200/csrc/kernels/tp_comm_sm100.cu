// Sequence-parallel all-gather fused into the producing RMSNorm (sm_100a).
//
// The rank normalises its shard of rows and writes each output row once, to the NVSwitch
// multicast address of the gather buffer (every rank's copy receives it: one store per 16 bytes,
// replicated by the switch), or without multicast to every rank's buffer in turn.  When all of
// its CTAs are done the rank raises ready[rank] = epoch in every rank's flag buffer (release,
// system scope).  The consuming GEMM (gemm_sm100.cu, all-gather mode) waits per shard on its
// local copy of those flags and starts with its own shard, so the transfer of the other shards
// overlaps its math.  No NCCL on this path; no TMA here.
#include "sm100_common.cuh"
#include "launch_api.h"

#include <cuda_bf16.h>

namespace cfb {
namespace tpcomm {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* f, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ void multimem_st16(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}

// Warp per row of the local rows.  Row r goes to row (row_base + r) of the gather buffer.
__global__ void __launch_bounds__(256) rmsnorm_push_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w, int rows, int H,
    float eps, __nv_bfloat16* mc_dst, __nv_bfloat16* const* peer_dst, long long ld_dst,
    float* __restrict__ rstd, uint32_t* const* peer_flags, int flag_off, int rank, int P,
    int row_base, uint32_t epoch, uint32_t* cnt) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row < rows) {
    const __nv_bfloat16* xr = x + static_cast<long long>(row) * H;
    float ss = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(H) + eps);
    if (lane == 0) rstd[row] = r;
    const long long drow = static_cast<long long>(row_base) + row;
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      const uint4 g = *reinterpret_cast<const uint4*>(w + c);
      const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&u);
      const __nv_bfloat162* hw = reinterpret_cast<const __nv_bfloat162*>(&g);
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fx = __bfloat1622float2(hx[e]);
        const float2 fw = __bfloat1622float2(hw[e]);
        o[e] = pack_bf16x2(fx.x * r * fw.x, fx.y * r * fw.y);
      }
      const uint4 v = make_uint4(o[0], o[1], o[2], o[3]);
      if (mc_dst) {
        multimem_st16(mc_dst + drow * ld_dst + c, v);
      } else {
        for (int q = 0; q < P; ++q)
          *reinterpret_cast<uint4*>(peer_dst[q] + drow * ld_dst + c) = v;
      }
    }
  }
  // all rows of the grid stored -> ready[rank] = epoch on every rank
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(cnt, 1u) == gridDim.x - 1u) {
      __threadfence_system();
      for (int q = 0; q < P; ++q) st_release_sys(peer_flags[q] + flag_off + rank, epoch);
      atomicExch(cnt, 0u);
    }
  }
}

}  // namespace tpcomm
}  // namespace cfb

int cfb_tp_rmsnorm_push(const void* x, const void* w, int rows, int H, float eps, void* mc_dst,
                        void* const* peer_dst, long long ld_dst, float* rstd,
                        uint32_t* const* peer_flags, int flag_off, int rank, int P,
                        int row_base, uint32_t epoch, uint32_t* cnt, cudaStream_t st) {
  if (H % 8 || ld_dst % 8 || (!mc_dst && !peer_dst) || !peer_flags || !cnt) return -11;
  const int grid = rows > 0 ? (rows + 7) / 8 : 1;
  cfb::tpcomm::rmsnorm_push_kernel<<<grid, 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), rows, H, eps,
      static_cast<__nv_bfloat16*>(mc_dst), reinterpret_cast<__nv_bfloat16* const*>(peer_dst),
      ld_dst, rstd, peer_flags, flag_off, rank, P, row_base, epoch, cnt);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
