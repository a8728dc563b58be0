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
// order).  Flags only grow, so waits test flag >= epoch.  The epoch lives in
// device memory and each call advances it, so a captured CUDA graph can be
// replayed.
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
  // let the next kernel launch (it waits for our completion before reading
  // the gathered output); wait for the kernel that produced y_local
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // This call's epoch: one more than the last completed call's (a device
  // counter, so CUDA-graph replays advance it); its parity picks the slot.
  __shared__ unsigned epoch_sh;
  if (threadIdx.x == 0) epoch_sh = *(volatile unsigned*)A.epoch + 1u;
  __syncthreads();
  const unsigned epoch = epoch_sh;
  const size_t slot = (size_t)(epoch & 1u) * (size_t)A.max_elems;
  const int64_t nl = A.r1 - A.r0;
  const int64_t total = A.m * nl;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // phase 1: my block into every rank's image (peer stores over NVLink)
  for (int p = 0; p < A.world; ++p) {
    float* dst = A.exch[p] + slot;
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
    // every CTA's stores are fenced and every CTA has read the epoch: publish
    // it to every rank and advance the local counter
    __threadfence_system();
    if (threadIdx.x < A.world)
      st_release_sys(reinterpret_cast<unsigned*>(reinterpret_cast<char*>(A.exch[threadIdx.x]) + A.flags_off) + A.rank,
                     epoch);
    if (threadIdx.x == 0) {
      *A.ctr = 0u;  // ready for the next call (stream-ordered)
      *A.epoch = epoch;
    }
  }
  // phase 2: wait for every rank's block, then copy the image out
  const unsigned* flags = reinterpret_cast<const unsigned*>(reinterpret_cast<const char*>(A.exch[A.rank]) + A.flags_off);
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    for (int r = 0; r < A.world && ok; ++r) {
      uint32_t i = 0;
      while (ld_acquire_sys(flags + r) < epoch) {
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
  const float* image = A.exch[A.rank] + slot;
  const int64_t all = A.m * A.n;
  for (int64_t e = tid; e < all; e += stride) {
    const int64_t t = e / A.n, j = e - t * A.n;
    float* dst = A.y_out + t * A.y_ld + j;
    *dst = A.accumulate ? *dst + image[e] : image[e];
  }
}

}  // namespace

cudaError_t launch_tp_allgather(const TpArgs& a, int blocks, cudaStream_t s) {
  if (a.world < 1 || a.world > TP_MAX_WORLD || blocks < 1) return cudaErrorInvalidValue;
  return launch_pdl(tp_allgather_kernel, dim3(blocks), dim3(512), 0, s, a);
}

}  // namespace kq
