// Gradient reduce-scatter over NVLink peer memory, fused with the fp32 accumulation into the
// rank's ZeRO-2 gradient shard (sm_100a).
//
// Every rank's flat fp32 gradient buffer lives in symmetric memory (same offsets on every
// GPU).  For a bucket [lo, hi), rank r owns chunk r.  Protocol per micro-batch `epoch`:
//   1. bucket ready: after the backward has produced bucket b, each rank stores `epoch` into
//      ready[b * W + me] of every peer's flag buffer (release, system scope);
//   2. pull-reduce: each rank waits (bounded, in a one-block kernel so that no SMs spin) until
//      ready[b * W + p] >= epoch for all p, then reads its chunk from every rank and adds the
//      sum into its fp32 shard:
//        * NVLS: one multimem.ld_reduce.add.v4.f32 per 16 bytes on the multicast address --
//          the NVSwitch sums the W copies, each GPU receives one reduced copy;
//        * otherwise plain 16-byte loads from each peer's buffer;
//   3. micro-batch done: after its last bucket each rank stores `epoch` into done[me] of every
//      peer and waits (bounded) for done[p] >= epoch of all peers before its gradient buffer is
//      cleared for the next micro-batch.
// Waits give up after the peer wait limit of the status block (err[2], default 20 s) and record
// kErrPeerWait in err[0], which the host reads one step later; they never trap.  Every kernel
// after a failed wait sees err[0] != 0 and skips its work: the pull does not sum half-written
// peer buffers, and the local gradient buffer is not cleared while a peer may still read it.
// No TMA is used here.
#include "sm100_common.cuh"
#include "launch_api.h"

namespace cfb {
namespace comm {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float4 multimem_ld_reduce_add_v4(const float* mc) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

// Wait until flags[base + i*stride] >= epoch for i < n.  Returns false on timeout.
__device__ bool wait_flags(const uint32_t* flags, int base, int stride, int n, uint32_t epoch,
                           int* err, int code) {
  const uint64_t t0 = globaltimer_ns();
  uint64_t limit = 0;  // read from the status block only once a wait has spun 1024 times
  for (int i = 0; i < n; ++i) {
    const uint32_t* f = flags + base + i * stride;
    uint32_t spins = 0;
    while (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
      if ((++spins & 1023u) == 0) {
        if (limit == 0) limit = peer_wait_limit_ns(err);
        if (globaltimer_ns() - t0 > limit) {
          atomicCAS(err, 0, code);
          return false;
        }
      }
    }
  }
  return true;
}

// One thread per peer stores `epoch` at offset `off` of that peer's flag buffer.
__global__ void signal_peers_kernel(uint32_t* const* peer_flags, int W, int off, uint32_t epoch) {
  const int p = threadIdx.x;
  if (p < W) {
    __threadfence_system();
    st_release_sys(peer_flags[p] + off, epoch);
  }
}

__global__ void wait_kernel(const uint32_t* flags, int base, int stride, int n, uint32_t epoch,
                            int* err) {
  if (threadIdx.x == 0) wait_flags(flags, base, stride, n, epoch, err, kErrPeerWait);
}

// dst[i] += scale * sum_p src_p[off + i]  for i < n  (n % 4 == 0, 16-byte aligned)
__global__ void __launch_bounds__(512) pull_reduce_kernel(
    const float* mc_base, const float* const* peer_base, int W, long long off, long long n,
    float* __restrict__ dst, float scale, const uint32_t* flags, int bucket, uint32_t epoch,
    int* err) {
  if (flags != nullptr) {  // optional in-kernel wait (the host path waits in wait_kernel)
    __shared__ int ok;
    if (threadIdx.x == 0)
      ok = wait_flags(flags, bucket * W, 1, W, epoch, err, kErrPeerWait) ? 1 : 0;
    __syncthreads();
    if (!ok) return;
  } else if (*reinterpret_cast<volatile int*>(err) != 0) {
    return;  // an earlier wait of this step gave up: peer buffers may be half written
  }
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 s;
    if (mc_base != nullptr) {
      s = multimem_ld_reduce_add_v4(mc_base + off + 4 * i);
    } else {
      s = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int p = 0; p < W; ++p) {
        const float4 v = *reinterpret_cast<const float4*>(peer_base[p] + off + 4 * i);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
    }
    float4 d = reinterpret_cast<float4*>(dst)[i];
    d.x += scale * s.x;
    d.y += scale * s.y;
    d.z += scale * s.z;
    d.w += scale * s.w;
    reinterpret_cast<float4*>(dst)[i] = d;
  }
}

// buf[0, n) = 0 unless err[0] != 0 (then a peer may still be reading the buffer: keep it)
__global__ void __launch_bounds__(512) zero_unless_error_kernel(float* __restrict__ buf,
                                                                long long n, const int* err) {
  if (*reinterpret_cast<const volatile int*>(err) != 0) return;
  const long long n4 = n / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += stride)
    reinterpret_cast<float4*>(buf)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (long long i = 4 * n4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
       i < n; i += stride)
    buf[i] = 0.f;
}

// Vocabulary-parallel cross entropy: every rank of the tensor-parallel group holds, per row,
// (max, sum of exp(logit - max), label logit or 0) of its vocabulary shard in a symmetric
// buffer [3][T] (stats_q of rank q through peer_stats[q]).  Each block waits (bounded) until
// every rank has raised ready[q] >= epoch, then one thread per row combines the P triples:
//   M = max_q m_q,  Z = sum_q s_q exp(m_q - M),  lse = M + log Z,  loss = lse - sum_q t_q
// (loss 0 for labels < 0).  The last block to finish tells every rank that this rank has read
// their buffers (done[me] = epoch), after which they may be rewritten.  After a failed wait
// nothing is read and the rows keep loss 0.
__global__ void __launch_bounds__(256) ce_exchange_kernel(
    const float* const* peer_stats, int P, int T, const long long* __restrict__ labels,
    float* __restrict__ loss, float* __restrict__ lse, const uint32_t* flags, int ready_base,
    uint32_t epoch, uint32_t* const* peer_flags, int done_off, int me, uint32_t* counter,
    int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_flags(flags, ready_base, 1, P, epoch, err, kErrPeerWait) ? 1 : 0;
  __syncthreads();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row < T) {
    float l = 0.f, z = 0.f;
    if (ok) {
      float M = -INFINITY;
      for (int q = 0; q < P; ++q) M = fmaxf(M, peer_stats[q][row]);
      float tgt = 0.f;
      for (int q = 0; q < P; ++q) {
        const float* st = peer_stats[q];
        z += st[T + row] * __expf(st[row] - M);
        tgt += st[2 * T + row];
      }
      z = M + __logf(z);
      l = labels[row] >= 0 ? z - tgt : 0.f;
    }
    loss[row] = l;
    lse[row] = z;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(counter, 1u) == gridDim.x - 1u) {
      atomicExch(counter, 0u);
      if (ok)
        for (int q = 0; q < P; ++q) st_release_sys(peer_flags[q] + done_off + me, epoch);
    }
  }
}

}  // namespace comm
}  // namespace cfb

using namespace cfb::comm;

int cfb_symm_signal(uint32_t* const* peer_flags_dev, int W, int off, uint32_t epoch,
                    cudaStream_t st) {
  if (W <= 0 || W > 1024) return -11;
  signal_peers_kernel<<<1, 32 * ((W + 31) / 32), 0, st>>>(peer_flags_dev, W, off, epoch);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int cfb_symm_wait(const uint32_t* flags, int base, int stride, int n, uint32_t epoch, int* err,
                  cudaStream_t st) {
  wait_kernel<<<1, 32, 0, st>>>(flags, base, stride, n, epoch, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int cfb_symm_pull_reduce(const float* mc_base, const float* const* peer_base_dev, int W,
                         long long off, long long n, float* dst, float scale,
                         const uint32_t* flags, int bucket, uint32_t epoch, int* err,
                         cudaStream_t st) {
  if ((n % 4) != 0 || (off % 4) != 0) return -11;
  if (n == 0) return 0;
  long long blocks = (n / 4 + 511) / 512;
  if (blocks > 148 * 4) blocks = 148 * 4;
  pull_reduce_kernel<<<static_cast<int>(blocks), 512, 0, st>>>(
      mc_base, peer_base_dev, W, off, n, dst, scale, flags, bucket, epoch, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int cfb_ce_exchange(const float* const* peer_stats, int P, int T, const long long* labels,
                    float* loss, float* lse, const uint32_t* flags, int ready_base,
                    uint32_t epoch, uint32_t* const* peer_flags, int done_off, int me,
                    uint32_t* counter, int* err, cudaStream_t st) {
  if (P <= 0 || P > 1024 || T < 0) return -11;
  if (T == 0) return 0;
  ce_exchange_kernel<<<(T + 255) / 256, 256, 0, st>>>(peer_stats, P, T, labels, loss, lse, flags,
                                                     ready_base, epoch, peer_flags, done_off, me,
                                                     counter, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

int cfb_zero_unless_error(float* buf, long long n, const int* err, cudaStream_t st) {
  if (n <= 0) return 0;
  if ((reinterpret_cast<uintptr_t>(buf) & 15) != 0) return -11;
  long long blocks = (n / 4 + 511) / 512;
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  zero_unless_error_kernel<<<static_cast<int>(blocks), 512, 0, st>>>(buf, n, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
