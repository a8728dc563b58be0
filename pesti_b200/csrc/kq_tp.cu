// kq_tp.cu -- all-gather of row-sharded linear outputs (and all-reduce of
// column-split partials) over NVLink peer memory.
//
// A linear's N output rows are split into contiguous per-rank blocks
// [r0, r1); every rank computes its block y_local[m][r1-r0] and the ranks
// then need the whole y[m][N].  Each rank stores its block straight into
// every rank's exchange buffer (IPC-mapped peer memory: plain stores travel
// over NVLink) at its columns of a y[m][N] image, and every rank then reads
// its own complete image.
//
// Low-latency words: every element travels as one 8-byte word {f32 bits,
// epoch of the call}, written and read with single 64-bit accesses, so a
// reader knows a value has arrived when its word carries the current epoch --
// no fences, flags or second round trip.  The epoch lives in device memory
// (one more per call; the last CTA to arrive advances it), so a captured CUDA
// graph can be replayed.  Two slots alternate by epoch parity: a rank writes
// slot e%2 of a peer only after its own call e-1 saw every rank's e-1 words,
// which every rank wrote after finishing its call e-2 (stream order) -- the
// last reader of that slot.
//
// All waits are bounded: on timeout the kernel sets *err and stops waiting
// (the host reports it); it never traps or spins forever.
#include "kq_kernels.h"

#include <cuda_runtime.h>

namespace kq {
namespace {

__device__ __forceinline__ void st_word(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

constexpr int ERR_TP_WAIT = 31;

__global__ void __launch_bounds__(512) tp_allgather_kernel(const __grid_constant__ TpArgs A) {
  // let the next kernel launch (it waits for our completion before reading
  // the gathered output); wait for the kernel that produced y_local
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ unsigned epoch_sh;
  if (threadIdx.x == 0) epoch_sh = *(volatile unsigned*)A.epoch + 1u;
  __syncthreads();
  const unsigned epoch = epoch_sh;
  const unsigned long long tag = (unsigned long long)epoch << 32;
  const size_t slot = (size_t)(epoch & 1u) * (size_t)A.max_elems;
  const int64_t nl = A.r1 - A.r0;
  const int64_t total = A.m * nl;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // phase 1: my block into every rank's image
  for (int64_t e = tid; e < total; e += stride) {
    const int64_t t = e / nl, j = e - t * nl;
    const unsigned long long w = tag | __float_as_uint(A.y_local[e]);
    for (int p = 0; p < A.world; ++p) st_word(A.exch[p] + slot + t * A.n + A.r0 + j, w);
  }
  // every CTA has read the epoch once all have arrived: the last one advances it
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(A.ctr, 1u) == gridDim.x - 1) {
    *A.ctr = 0u;
    *A.epoch = epoch;
  }
  // phase 2: each element of my image once its word carries this epoch;
  // a thread reads up to 8 words at once and re-reads only while one is old
  constexpr int U = 8;
  const unsigned long long* image = A.exch[A.rank] + slot;
  const int64_t all = A.m * A.n;
  bool ok = true;
  for (int64_t e0 = tid; e0 < all && ok; e0 += stride * U) {
    unsigned long long w[U];
    for (uint32_t it = 0;; ++it) {
      bool ready = true;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t e = e0 + (int64_t)u * stride;
        w[u] = e < all ? ld_word(image + e) : tag;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) ready = ready && (unsigned)(w[u] >> 32) == epoch;
      if (ready) break;
      if (it >= (1u << 22) || ((it & 255u) == 255u && *(volatile int*)A.err)) {
        atomicCAS(A.err, 0, ERR_TP_WAIT);
        ok = false;
        break;
      }
      __nanosleep(32);
    }
    if (!ok) break;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t e = e0 + (int64_t)u * stride;
      if (e < all) {
        const int64_t t = e / A.n, j = e - t * A.n;
        float* dst = A.y_out + t * A.y_ld + j;
        const float v = __uint_as_float((unsigned)w[u]);
        *dst = A.accumulate ? *dst + v : v;
      }
    }
  }
}

// All-reduce of per-rank partials (the column-split projections at batch >
// 1): each rank's y_local[m][n] goes to section `rank` of every rank's image
// (slot layout [world][m][n]); every rank then sums the world sections of its
// own image in rank order -- the same order everywhere, so every rank holds
// bit-identical sums -- into y_out (or adds them to it).  Same epoch words,
// slots and bounded waits as the all-gather.
__global__ void __launch_bounds__(512) tp_allreduce_kernel(const __grid_constant__ TpArgs A) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ unsigned epoch_sh;
  if (threadIdx.x == 0) epoch_sh = *(volatile unsigned*)A.epoch + 1u;
  __syncthreads();
  const unsigned epoch = epoch_sh;
  const unsigned long long tag = (unsigned long long)epoch << 32;
  const size_t slot = (size_t)(epoch & 1u) * (size_t)A.max_elems;
  const int64_t all = A.m * A.n;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const size_t mine = slot + (size_t)A.rank * (size_t)all;
  for (int64_t e = tid; e < all; e += stride) {
    const unsigned long long w = tag | __float_as_uint(A.y_local[e]);
    for (int p = 0; p < A.world; ++p) st_word(A.exch[p] + mine + e, w);
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(A.ctr, 1u) == gridDim.x - 1) {
    *A.ctr = 0u;
    *A.epoch = epoch;
  }
  constexpr int U = 4;
  const unsigned long long* image = A.exch[A.rank] + slot;
  bool ok = true;
  for (int64_t e0 = tid; e0 < all && ok; e0 += stride * U) {
    unsigned long long w[TP_MAX_WORLD][U];
    for (uint32_t it = 0;; ++it) {
      bool ready = true;
#pragma unroll
      for (int r = 0; r < TP_MAX_WORLD; ++r)
        if (r < A.world)
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int64_t e = e0 + (int64_t)u * stride;
            w[r][u] = e < all ? ld_word(image + (size_t)r * (size_t)all + e) : tag;
            ready = ready && (unsigned)(w[r][u] >> 32) == epoch;
          }
      if (ready) break;
      if (it >= (1u << 22) || ((it & 255u) == 255u && *(volatile int*)A.err)) {
        atomicCAS(A.err, 0, ERR_TP_WAIT);
        ok = false;
        break;
      }
      __nanosleep(32);
    }
    if (!ok) break;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t e = e0 + (int64_t)u * stride;
      if (e < all) {
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < TP_MAX_WORLD; ++r)
          if (r < A.world) v += __uint_as_float((unsigned)w[r][u]);
        const int64_t t = e / A.n, j = e - t * A.n;
        float* dst = A.y_out + t * A.y_ld + j;
        *dst = A.accumulate ? *dst + v : v;
      }
    }
  }
}

}  // namespace

cudaError_t launch_tp_allreduce(const TpArgs& a, int blocks, cudaStream_t s) {
  if (a.world < 1 || a.world > TP_MAX_WORLD || blocks < 1) return cudaErrorInvalidValue;
  return launch_pdl(tp_allreduce_kernel, dim3(blocks), dim3(512), 0, s, a);
}

cudaError_t launch_tp_allgather(const TpArgs& a, int blocks, cudaStream_t s) {
  if (a.world < 1 || a.world > TP_MAX_WORLD || blocks < 1) return cudaErrorInvalidValue;
  return launch_pdl(tp_allgather_kernel, dim3(blocks), dim3(512), 0, s, a);
}

}  // namespace kq
