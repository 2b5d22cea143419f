// RMSNorm backward without device allocation (see rmsnorm_noalloc.h for the contract).
//
// No counterpart in the reference.  Variant of the rmsnorm backward in fused_ops.cu whose
// per-block dgamma partial sums go to a fixed file-scope device array instead of a buffer
// allocated per call.
#include "rmsnorm_noalloc.h"

#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>

namespace {

// Scratch shared by every call on a device (4 MiB).  In host code this name is only a host-side
// stand-in; kernels receive its device address from cudaGetSymbolAddress.
static __device__ __align__(256) float g_rmsnorm_scratch[CFB_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {};

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  u.x = *reinterpret_cast<uint32_t*>(&h[0]);
  u.y = *reinterpret_cast<uint32_t*>(&h[1]);
  u.z = *reinterpret_cast<uint32_t*>(&h[2]);
  u.w = *reinterpret_cast<uint32_t*>(&h[3]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Block b handles a contiguous row range and writes its dgamma partial sums to
// scratch[b * H, (b + 1) * H) -- every element of that row of the scratch, every call.
template <int GROUPS>
__global__ void __launch_bounds__(256) rms_bwd_partial(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const int* __restrict__ x_rows, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ dres,
    __nv_bfloat16* __restrict__ dx, float* __restrict__ scratch, int rows, int H) {
  __shared__ float red[8];
  const int tid = threadIdx.x;
  const int per = (rows + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * per;
  const int r1 = min(rows, r0 + per);
  float acc[GROUPS][8], wv[GROUPS][8];
#pragma unroll
  for (int g = 0; g < GROUPS; ++g) {
    const int c = (tid + g * 256) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[g][i] = 0.f;
    if (c < H) ld8(w + c, wv[g]);
  }
  for (int r = r0; r < r1; ++r) {
    const long long xr = x_rows ? x_rows[r] : r;
    const float rs = rstd[xr];
    float a[GROUPS][8], b[GROUPS][8];
    float dot = 0.f;
#pragma unroll
    for (int g = 0; g < GROUPS; ++g) {
      const int c = (tid + g * 256) * 8;
      if (c < H) {
        ld8(dy + static_cast<long long>(r) * H + c, a[g]);
        ld8(x + xr * H + c, b[g]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          dot += wv[g][i] * a[g][i] * b[g][i];
          acc[g][i] += a[g][i] * b[g][i] * rs;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
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
          ld8(dres + static_cast<long long>(r) * H + c, o);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] += rs * wv[g][i] * a[g][i] - b[g][i] * coef;
        st8(dx + static_cast<long long>(r) * H + c, o);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GROUPS; ++g) {
    const int c = (tid + g * 256) * 8;
    if (c < H) {
      float* dst = scratch + static_cast<long long>(blockIdx.x) * H + c;
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = acc[g][i];
    }
  }
}

__global__ void rms_bwd_colsum(const float* __restrict__ scratch, float* __restrict__ dw_acc,
                               int P, int H) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int p = 0; p < P; ++p) s += scratch[static_cast<long long>(p) * H + c];
  dw_acc[c] += s;
}

// Device address of the scratch array on the current device (looked up once per device).
float* scratch_for_current_device(int* err) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = CFB_NOALLOC_ERR_SYMBOL;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_rmsnorm_scratch);
    if (rc != cudaSuccess || p == nullptr) {
      *err = CFB_NOALLOC_ERR_SYMBOL;
      return nullptr;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int cfb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const int* x_rows,
                                       const float* rstd, const void* w, const void* dres,
                                       void* dx, float* dw_acc, int rows, int H,
                                       cudaStream_t stream) {
  if (!dy || !x || !rstd || !w || !dx || !dw_acc || rows < 0 || H <= 0 || (H % 8) != 0)
    return CFB_NOALLOC_ERR_BAD_ARGS;
  // the kernels move 8 bf16 values (16 bytes) per access of dy, x, w, dres and dx
  const auto misaligned = [](const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) != 0;
  };
  if (misaligned(dy) || misaligned(x) || misaligned(w) || misaligned(dx) ||
      (dres != nullptr && misaligned(dres)))
    return CFB_NOALLOC_ERR_BAD_ARGS;
  if (H > 8192) return CFB_NOALLOC_ERR_TOO_LARGE;
  if (rows == 0) return CFB_NOALLOC_OK;
  // An error left pending by earlier work on this thread belongs to its owner: report it
  // without launching and without clearing it.
  if (cudaPeekAtLastError() != cudaSuccess) return CFB_NOALLOC_ERR_PENDING;
  int err = CFB_NOALLOC_OK;
  float* scratch = scratch_for_current_device(&err);
  if (scratch == nullptr) return err;
  int P = rows < 296 ? rows : 296;
  const int cap = static_cast<int>(CFB_NOALLOC_SCRATCH_FLOATS / static_cast<unsigned>(H));
  if (P > cap) P = cap;
  if (P < 1) return CFB_NOALLOC_ERR_TOO_LARGE;
  const int groups = (H / 8 + 255) / 256;
  typedef __nv_bfloat16 bf;
  const bf* a = static_cast<const bf*>(dy);
  const bf* b = static_cast<const bf*>(x);
  const bf* c = static_cast<const bf*>(w);
  const bf* d = static_cast<const bf*>(dres);
  bf* o = static_cast<bf*>(dx);
  switch (groups) {
    case 1: rms_bwd_partial<1><<<P, 256, 0, stream>>>(a, b, x_rows, rstd, c, d, o, scratch, rows, H); break;
    case 2: rms_bwd_partial<2><<<P, 256, 0, stream>>>(a, b, x_rows, rstd, c, d, o, scratch, rows, H); break;
    case 3: rms_bwd_partial<3><<<P, 256, 0, stream>>>(a, b, x_rows, rstd, c, d, o, scratch, rows, H); break;
    default: rms_bwd_partial<4><<<P, 256, 0, stream>>>(a, b, x_rows, rstd, c, d, o, scratch, rows, H); break;
  }
  if (cudaGetLastError() != cudaSuccess) return CFB_NOALLOC_ERR_LAUNCH;
  rms_bwd_colsum<<<(H + 255) / 256, 256, 0, stream>>>(scratch, dw_acc, P, H);
  if (cudaGetLastError() != cudaSuccess) return CFB_NOALLOC_ERR_LAUNCH;
  return CFB_NOALLOC_OK;
}

extern "C" const char* cfb_noalloc_strerror(int code) {
  switch (code) {
    case CFB_NOALLOC_OK: return "ok";
    case CFB_NOALLOC_ERR_BAD_ARGS:
      return "bad arguments (null pointer, negative size, H % 8 != 0, or a bf16 buffer not "
             "16-byte aligned)";
    case CFB_NOALLOC_ERR_TOO_LARGE:
      return "hidden size beyond the fixed scratch limit (H must be <= 8192)";
    case CFB_NOALLOC_ERR_SYMBOL: return "could not resolve the device scratch address";
    case CFB_NOALLOC_ERR_LAUNCH: return "kernel launch failed";
    case CFB_NOALLOC_ERR_PENDING:
      return "an earlier CUDA error is pending on this thread (left for its owner; nothing "
             "launched)";
  }
  return "unknown error";
}
