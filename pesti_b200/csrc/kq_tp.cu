// kq_tp.cu -- all-gather of row-sharded linear outputs over NVLink peer memory.
//
// A linear's N output rows are split into contiguous per-rank blocks
// [r0, r1); every rank computes its block y_local[m][r1-r0] and the ranks
// then need the whole y[m][N].  Instead of a library all-gather, each rank
// stores its block straight into every rank's exchange buffer (IPC-mapped
// peer memory: plain stores travel over NVLink), at its columns of a y[m][N]
// image, then publishes the call's epoch in every rank's flag array (release
// store, system scope).  Each rank waits until all ranks' flags reach the
// epoch (acquire load) and copies its now complete image out.
//
// Exchange buffer of one rank: two image slots of max_elems floats (epoch
// parity picks the slot) followed by one 32-bit flag per source rank.  Double
// buffering is enough: a rank writes slot e%2 of a peer only after it has seen
// every rank's epoch e-1 flag, and a rank publishes e-1 only after its own
// call e-2 -- including the copy out of slot e%2 -- has finished (stream
// order).  Flags only grow, so waits test flag >= epoch.
//
// All waits are bounded: on timeout the kernel sets *err and returns (the
// host reports it); it never traps or spins forever.
#include "kq_kernels.h"

#include <cuda_runtime.h>

namespace kq {
namespace {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int ERR_TP_WAIT = 31;

__global__ void __launch_bounds__(512) tp_allgather_kernel(const __grid_constant__ TpArgs A) {
  const int64_t nl = A.r1 - A.r0;
  const int64_t total = A.m * nl;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // phase 1: my block into every rank's image (peer stores over NVLink)
  for (int p = 0; p < A.world; ++p) {
    float* dst = A.peer_slot[p];
    for (int64_t e = tid; e < total; e += stride) {
      const int64_t t = e / nl, j = e - t * nl;
      dst[t * A.n + A.r0 + j] = A.y_local[e];
    }
  }
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = atomicAdd(A.ctr, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last) {
    // every CTA's stores are fenced: publish the epoch to every rank
    __threadfence_system();
    if (threadIdx.x < A.world) st_release_sys(A.peer_flags[threadIdx.x] + A.rank, A.epoch);
    if (threadIdx.x == 0) *A.ctr = 0u;  // ready for the next call (stream-ordered)
  }
  // phase 2: wait for every rank's block, then copy the image out
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int r = 0; r < A.world && ok; ++r) {
      uint32_t i = 0;
      while (ld_acquire_sys(A.local_flags + r) < A.epoch) {
        if (++i >= (1u << 24) || *(volatile int*)A.err) {
          atomicCAS(A.err, 0, ERR_TP_WAIT);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  const int64_t all = A.m * A.n;
  for (int64_t e = tid; e < all; e += stride) A.y_out[e] = A.local_slot[e];
}

}  // namespace

cudaError_t launch_tp_allgather(const TpArgs& a, int blocks, cudaStream_t s) {
  if (a.world < 1 || a.world > TP_MAX_WORLD || blocks < 1) return cudaErrorInvalidValue;
  tp_allgather_kernel<<<blocks, 512, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace kq
