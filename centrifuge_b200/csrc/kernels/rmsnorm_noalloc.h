// RMSNorm backward entry point that allocates no device memory.
//
// This entry point has no counterpart in the reference: it is an addition of this library.
//
// Who needs it: callers that may not allocate device memory themselves -- code running inside a
// host application whose framework owns every device allocation through its own pool and forbids
// plug-ins from calling cudaMalloc/cudaFree, and callers that must not trigger the device-wide
// synchronisation that cudaFree implies or an allocation failure in the middle of a step.  They
// still pass every input and output buffer; the kernel's only scratch (per-block dgamma partial
// sums) lives in a fixed file-scope device array instead of a per-call allocation.
//
//   dx[r, :]  = dres[r, :] + d(rmsnorm)/dx at row x[x_rows[r]]      (bf16, [rows, H])
//   dw_acc   += sum_r dy[r] * x[x_rows[r]] * rstd[x_rows[r]]         (fp32, [H])
//
// Same semantics and argument meaning as cfb_rmsnorm_bwd (launch_api.h); x_rows and dres may be
// null.  dy, x, w, dres and dx are read and written 16 bytes at a time, so each must start on a
// 16-byte boundary (otherwise CFB_NOALLOC_ERR_BAD_ARGS).  If an earlier CUDA error is pending on
// the calling thread, the call launches nothing, leaves that error in place for its owner and
// returns CFB_NOALLOC_ERR_PENDING.
// Limits: H % 8 == 0, H <= 8192, and at most CFB_NOALLOC_SCRATCH_FLOATS fp32 scratch
// elements (4 MiB), which this entry point never exceeds for H <= 8192 by using fewer partial
// rows; larger H is rejected with CFB_NOALLOC_ERR_TOO_LARGE.
//
// Set-up: the first call on a device looks up the device address of the scratch array with
// cudaGetSymbolAddress for the current device and caches it; make that first call before any
// CUDA stream capture.  The scratch array is shared by every call on a device and keeps the
// last call's contents (this entry point fully rewrites the part it reads, so nothing needs
// clearing); calls that overlap on the GPU (different streams, no ordering) race on it.  The
// array stays allocated on every GPU that loads the library until the process exits.
#pragma once
#include <cuda_runtime.h>

#define CFB_NOALLOC_SCRATCH_FLOATS (1u << 20)

enum {
  CFB_NOALLOC_OK = 0,
  CFB_NOALLOC_ERR_BAD_ARGS = -1,
  CFB_NOALLOC_ERR_TOO_LARGE = -2,
  CFB_NOALLOC_ERR_SYMBOL = -3,
  CFB_NOALLOC_ERR_LAUNCH = -4,
  CFB_NOALLOC_ERR_PENDING = -5,
};

#ifdef __cplusplus
extern "C" {
#endif

// Returns CFB_NOALLOC_OK or a negative CFB_NOALLOC_ERR_* code; the launch is asynchronous on
// `stream`.
int cfb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const int* x_rows, const float* rstd,
                            const void* w, const void* dres, void* dx, float* dw_acc, int rows,
                            int H, cudaStream_t stream);

// Human-readable text of a return code.
const char* cfb_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
