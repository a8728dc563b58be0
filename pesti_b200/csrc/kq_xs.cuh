// kq_xs.cuh -- building blocks of the single-token (decode) GEMV kernels:
// the bounded mbarrier waits and bulk copies of the TMA weight ring, the
// 8-byte exchange words of the tensor-parallel path, the per-superblock
// activation quantization (15-bit integers split into hi / lo bytes) and the
// dp4a forms the integer dot products use.  Shared by kq_dp4a.cu (one
// kernel per linear) and kq_step.cu (the persistent decode step).
#pragma once

#include "kq_common.cuh"

namespace kq {
namespace {

__device__ __forceinline__ int dp4a_s(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }
__device__ __forceinline__ int dp4a_u(uint32_t a, uint32_t b, int c) {
  return (int)__dp4a(a, b, (unsigned)c);
}
// unsigned bytes of a times signed bytes of b
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// signed bytes of a times unsigned bytes of b
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void xs_bar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void xs_bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(b)) : "memory");
}
__device__ __forceinline__ void xs_bar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)), "r"(bytes) : "memory");
}
// Bounded wait for the phase of parity `par`; on giving up sets *err (first
// code wins) and returns false.
__device__ __forceinline__ bool xs_bar_wait(uint64_t* b, uint32_t par, int* err, int code) {
  const uint32_t a = smem_addr(b);
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(par)
        : "memory");
    if (done) return true;
    if ((i & 1023u) == 1023u && *(volatile int*)err) return false;
  }
  atomicCAS(err, 0, code);
  return false;
}
// Global -> shared bulk copy completing on mbarrier b (no multicast), with an
// L2 eviction policy (the weights are read once per call: evict first).
__device__ __forceinline__ void xs_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(b)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void xs_bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(b))
               : "memory");
}
// 8-byte exchange words {f32 bits, epoch}: single 64-bit accesses
__device__ __forceinline__ void st_word(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void ld_words2(const unsigned long long* p, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ void xs_named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Per-superblock activation scale shared by the 8 lanes staging a
// superblock: max|x| * inv in [2^13, 2^14) so that rint(x * inv) fits 15 bits.
struct XScale {
  float inv, factor;  // 2^-e, 2^e (NaN: the block holds a non-finite value)
};
__device__ __forceinline__ XScale xs_scale(float amax) {
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
  XScale s;
  if (!(amax <= 3.4e38f)) {
    s.inv = 0.f;
    s.factor = __int_as_float(0x7fc00000);
    return s;
  }
  int e = 0;
  if (amax > 0.f) e = (int)((__float_as_uint(amax) >> 23) & 0xff) - 127 - 13;
  e = max(-126, min(126, e));
  s.inv = __uint_as_float((uint32_t)(127 - e) << 23);
  s.factor = __uint_as_float((uint32_t)(127 + e) << 23);
  return s;
}
// Four activations -> {hi bytes, lo bytes} of rint(v * inv) (|.| <= 2^14).
__device__ __forceinline__ void xs_pack4(float v0, float v1, float v2, float v3, float inv, uint32_t& hi,
                                         uint32_t& lo) {
  constexpr float M = 12582912.0f;  // 1.5 * 2^23: the sum's low 16 bits are rint(v * inv)
  const uint32_t f0 = __float_as_uint(fmaf(v0, inv, M)), f1 = __float_as_uint(fmaf(v1, inv, M));
  const uint32_t f2 = __float_as_uint(fmaf(v2, inv, M)), f3 = __float_as_uint(fmaf(v3, inv, M));
  const uint32_t p01 = prmt(f0, f1, 0x5140u), p23 = prmt(f2, f3, 0x5140u);  // {lo0, lo1, hi0, hi1}
  lo = prmt(p01, p23, 0x5410u);
  hi = prmt(p01, p23, 0x7632u);
}

__device__ __forceinline__ int xs_swz(int kb, int u) { return (u + 4 * (kb & 1)) & 7; }

}  // namespace
}  // namespace kq
