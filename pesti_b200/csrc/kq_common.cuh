// kq_common.cuh -- shared device helpers for the K-quant kernels (sm_100a).
//
// Block formats decoded here (all little-endian):
//   GGUF Q4_K  144 B / 256 weights: d f16 | dmin f16 | scales[12] | qs[128]
//   GGUF Q6_K  210 B / 256 weights: ql[128] | qh[64] | int8 scales[16] | d f16
//   Q6_K on the device is re-laid at upload time into two arrays so that every
//   vector load is 16-byte aligned: q6 "body" [rows][sb][208] = ql|qh|scales
//   and q6 "d" [rows][sb] f16.  The byte count is unchanged (208 + 2 = 210).
//   pesti-legacy Q4_K / Q6_K (28 B / 42 B per 16 weights) stay as uploaded.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kq_kernels.h"

namespace kq {

// Device Q6_K body: where GGUF byte b (0..207: ql[128] | qh[64] | scales[16])
// of a superblock is stored.  The 32 columns l of each 32-weight group are
// split into four slots c = l/8; slot c's 48 bytes are contiguous at 48c:
// pieces 0..3 = ql[64h + 32gg + 8c .. +8] (piece 2h+gg), pieces 4..5 =
// qh[32h + 8c .. +8].  Scales stay at 192.  Slot c is what one lane of the
// decode kernel reads with three 16-byte loads.
__host__ __device__ __forceinline__ int q6k_body_offset(int b) {
  if (b < 128) {
    const int h = b >> 6, gg = (b >> 5) & 1, l = b & 31;
    return 48 * (l >> 3) + 8 * (2 * h + gg) + (l & 7);
  }
  if (b < 192) {
    const int i = b - 128, h = i >> 5, l = i & 31;
    return 48 * (l >> 3) + 8 * (4 + h) + (l & 7);
  }
  return b;
}

// Exact f16 bits -> f32 (the hardware conversion is exact for every input).
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

// 6-bit (scale, min) pair j of a Q4_K superblock, from its 12 packed bytes.
// Bytes 0..3: low 6 bits = sc[0..3], top 2 bits = high bits of sc[4..7];
// bytes 4..7: low 6 bits = m[0..3], top 2 bits = high bits of m[4..7];
// bytes 8..11: low nibble = low 4 bits of sc[4..7], high nibble = of m[4..7].
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// Same, from the three little-endian words of the 12 packed bytes.
__device__ __forceinline__ void q4k_scale_min_w(uint32_t s0, uint32_t s1, uint32_t s2, int j,
                                                int& sc, int& m) {
  if (j < 4) {
    sc = (s0 >> (8 * j)) & 63;
    m = (s1 >> (8 * j)) & 63;
  } else {
    const int b = 8 * (j - 4);
    sc = ((s2 >> b) & 0x0f) | (((s0 >> (b + 6)) & 3) << 4);
    m = ((s2 >> (b + 4)) & 0x0f) | (((s1 >> (b + 6)) & 3) << 4);
  }
}

// Float whose value is 0.5 + q/256 for the byte q (q < 128) held in byte SEL
// of w: one PRMT assembles the bits 0x3F, q, 0x00, 0x00 (high to low byte).
// Exact for every q in [0, 127].
template <int SEL>
__device__ __forceinline__ float magic_byte(uint32_t w) {
  uint32_t r;
  // result bytes: [0] = 0x00, [1] = 0x00, [2] = w.byte[SEL], [3] = 0x3F
  constexpr uint32_t sel = 0x7054u | (uint32_t(SEL) << 8);
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0x3F000000u), "n"(sel));
  return __uint_as_float(r);
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float4 ldg_f4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

// Gate activation of the SwiGLU FFN: act(g) * u with act(g) = s(g) * g.
// mode 1: s is the logistic sigmoid (SiLU).  mode 0 follows pesti-runner's
// layer.rs:16-29 as written: for g < 0 it uses g / (1 + e^g) in place of the
// sigmoid.  Both kernels that apply it (the SwiGLU kernel and the fused
// single-token GEMV) call this one function.  It uses the hardware
// exponential and reciprocal (__expf, __frcp_rn): a few ulp from the exact
// function, far inside the decode tolerance, and an order of magnitude
// cheaper on the fused GEMV's critical path.  Large |g| saturate as the exact
// function does (e^g = inf gives s = 0).
__device__ __forceinline__ float swiglu_gate(float g, int mode) {
  const bool pos = g >= 0.f || mode == 1;
  const float e = __expf(pos ? -g : g);
  const float r = __frcp_rn(1.f + e);
  return (pos ? r : g * r) * g;
}

}  // namespace kq
