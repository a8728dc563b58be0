// kq_dequant.cu -- bit-exact dequantization, the Q6_K upload re-layout, and
// the pesti-legacy block kernels.
//
// Dequantized values are computed with explicitly rounded f32 operations
// (__fmul_rn / __fadd_rn / __fsub_rn) in the same association as the
// CPU definitions they must match bit for bit:
//   GGUF Q4_K  (d*sc)*q - (dmin*m)                         (gguf-py / ggml)
//   GGUF Q6_K  (d*sc)*(q-32)                                (gguf-py / ggml)
//   legacy Q4_K ((delta*h)*(q-4)) + d     pesti-runner/src/tile_dequant.rs:261
//   legacy Q6_K (d*(q-32))*scale          pesti-runner/src/tile_dequant.rs:373
#include "kq_common.cuh"
#include "kq_kernels.h"

namespace kq {

namespace {

__device__ __forceinline__ float gguf_q4k_value(const uint8_t* blk, int e) {
  const float d = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
  const float dmin = f16_bits_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
  const int c = e >> 6, p = e & 63;
  const int j = 2 * c + (p >> 5);
  int sc, m;
  q4k_scale_min(blk + 4, j, sc, m);
  const uint8_t byte = blk[16 + 32 * c + (p & 31)];
  const int q = (p < 32) ? (byte & 0x0f) : (byte >> 4);
  const float d1 = __fmul_rn(d, (float)sc);
  const float m1 = __fmul_rn(dmin, (float)m);
  return __fsub_rn(__fmul_rn(d1, (float)q), m1);
}

// Device Q6_K body (see q6k_body_offset): element e = 128h + 32g + l.
__device__ __forceinline__ float gguf_q6k_value(const uint8_t* body, uint16_t dbits, int e) {
  const int h = e >> 7, g = (e >> 5) & 3, l = e & 31;
  const uint8_t qlb = body[q6k_body_offset(64 * h + l + 32 * (g & 1))];
  const int lo = (g < 2) ? (qlb & 0x0f) : (qlb >> 4);
  const int hi = (body[q6k_body_offset(128 + 32 * h + l)] >> (2 * g)) & 3;
  const int q = (lo | (hi << 4)) - 32;
  const int sc = (int)(int8_t)body[192 + (e >> 4)];
  const float d = f16_bits_to_f32(dbits);
  return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

__device__ __forceinline__ uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// Legacy Q4_K: tile_dequant.rs:238-290.  Element i of a row.
__device__ __forceinline__ float legacy_q4k_value(const uint8_t* row, int64_t k, int64_t i) {
  const int64_t nfull = k / 16;
  const int64_t b = i / 16;
  if (b >= nfull) {  // trailing 4-byte partial block: value = d
    return f16_bits_to_f32(rd16(row + nfull * 28));
  }
  const uint8_t* p = row + b * 28;
  const int e = (int)(i & 15);
  const float d = f16_bits_to_f32(rd16(p));
  const float delta = f16_bits_to_f32(rd16(p + 2));
  const uint8_t* qsrc = p + 4 + (e >> 3) * 4;  // qs_low for e<8, qs_high for e>=8
  const int ei = e & 7;
  const int q = (qsrc[ei >> 1] >> (4 * (ei & 1))) & 0x0f;
  const float h = f16_bits_to_f32(rd16(p + 12 + 2 * (e >> 3)));
  float t = __fmul_rn(delta, h);
  t = __fmul_rn(t, __fsub_rn((float)q, 4.0f));
  return __fadd_rn(t, d);
}

// Legacy Q6_K: tile_dequant.rs:347-374.
__device__ __forceinline__ float legacy_q6k_value(const uint8_t* row, int64_t i) {
  const uint8_t* p = row + (i / 16) * 42;
  const int e = (int)(i & 15);
  const float d = f16_bits_to_f32(rd16(p));
  const float sc = f16_bits_to_f32(rd16(p + 2 + 2 * (e >> 2)));
  const int qlow = (p[10 + (e >> 2)] >> ((e & 3) * 2)) & 3;
  const int flag = (p[18 + (e >> 2)] >> ((e & 3) * 2)) & 3;
  const int qhigh = flag == 0 ? 0 : flag - 1;
  const int q = qlow + 4 * qhigh;
  const float t = __fmul_rn(d, __fsub_rn((float)q, 32.0f));
  return __fmul_rn(t, sc);
}

__global__ void dequant_kernel(DevWeight w, int64_t row0, int64_t nrows, float* __restrict__ out) {
  const int64_t total = nrows * w.k;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = row0 + idx / w.k;
    const int64_t i = idx - (idx / w.k) * w.k;
    float v;
    switch (w.type) {
      case GGUF_Q4_K:
        v = gguf_q4k_value(w.q + ((size_t)r * w.sb + i / QK) * Q4K_BYTES, (int)(i % QK));
        break;
      case GGUF_Q6_K: {
        const int64_t kb = i / QK;
        const size_t g = (size_t)r * w.sb + kb;
        v = gguf_q6k_value(w.q + g * Q6K_BODY, w.d[r * w.d_ld + kb], (int)(i % QK));
        break;
      }
      case LEGACY_Q4_K:
      case LEGACY_Q5_K:  // quantized_linear.rs:170-173: Q5_K rows go through the Q4_K tile decoder
        v = legacy_q4k_value(w.q + r * w.row_bytes, w.k, i);
        break;
      default:
        v = legacy_q6k_value(w.q + r * w.row_bytes, i);
        break;
    }
    out[idx] = v;
  }
}

__global__ void q6k_relayout_kernel(const uint8_t* __restrict__ raw, int64_t n, int64_t sb,
                                    uint8_t* __restrict__ body, uint16_t* __restrict__ d) {
  const int64_t total = n * sb * Q6K_BYTES;
  const int64_t ld = q6k_d_ld(sb);
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = idx / Q6K_BYTES;  // row * sb + kb
    const int b = (int)(idx - g * Q6K_BYTES);
    if (b < Q6K_BODY) {
      body[g * Q6K_BODY + q6k_body_offset(b)] = raw[idx];
    } else if (b == Q6K_BODY) {
      const int64_t row = g / sb, kb = g - row * sb;
      d[row * ld + kb] = (uint16_t)(raw[idx] | (raw[idx + 1] << 8));
    }
  }
}

// Legacy linear: one warp per output row; lane l takes 16-weight blocks l,
// l + 32, ... and loads each block's fields once (Q4_K: d, delta, the two
// nibble words and h0 / h1 as four 32-bit words; Q6_K: d, the four scales,
// the low-bit and flag words as 16-bit pieces -- its blocks start on 2-byte
// boundaries), decodes its 16 values in registers with the CPU association,
// and multiplies them with the activations (f32 accumulate).  A warp's 32
// blocks are one contiguous run of the row, so the loads are coalesced.
__device__ __forceinline__ void legacy_q4k_block(const uint8_t* p, float (&v)[16]) {
  const uint32_t w0 = *reinterpret_cast<const uint32_t*>(p);       // d | delta
  const uint32_t lo = *reinterpret_cast<const uint32_t*>(p + 4);   // elements 0..7
  const uint32_t hi = *reinterpret_cast<const uint32_t*>(p + 8);   // elements 8..15
  const uint32_t hh = *reinterpret_cast<const uint32_t*>(p + 12);  // h0 | h1
  const float d = f16_bits_to_f32((uint16_t)(w0 & 0xffff)), delta = f16_bits_to_f32((uint16_t)(w0 >> 16));
  const float t0 = __fmul_rn(delta, f16_bits_to_f32((uint16_t)(hh & 0xffff)));
  const float t1 = __fmul_rn(delta, f16_bits_to_f32((uint16_t)(hh >> 16)));
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    v[e] = __fadd_rn(__fmul_rn(t0, __fsub_rn((float)((lo >> (4 * e)) & 15u), 4.0f)), d);
    v[8 + e] = __fadd_rn(__fmul_rn(t1, __fsub_rn((float)((hi >> (4 * e)) & 15u), 4.0f)), d);
  }
}
__device__ __forceinline__ void legacy_q6k_block(const uint8_t* p, float (&v)[16]) {
  const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
  const float d = f16_bits_to_f32(h[0]);
  float sc[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) sc[s] = f16_bits_to_f32(h[1 + s]);
  const uint32_t ql = (uint32_t)h[5] | ((uint32_t)h[6] << 16);  // bytes 10..13: 2 low bits per element
  const uint32_t fl = (uint32_t)h[9] | ((uint32_t)h[10] << 16); // bytes 18..21: 2 flag bits per element
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int qlow = (ql >> (2 * e)) & 3, flag = (fl >> (2 * e)) & 3;
    const int q = qlow + 4 * (flag == 0 ? 0 : flag - 1);
    v[e] = __fmul_rn(__fmul_rn(d, __fsub_rn((float)q, 32.0f)), sc[e >> 2]);
  }
}

template <int M>
__global__ void __launch_bounds__(256) legacy_gemv_kernel(DevWeight w, const float* __restrict__ x,
                                                          const float* __restrict__ bias,
                                                          float* __restrict__ y, int64_t ldy) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= w.n) return;
  const uint8_t* rp = w.q + row * w.row_bytes;
  const bool q6 = w.type == LEGACY_Q6_K;
  const int bs = q6 ? 42 : 28;
  float acc[M];
#pragma unroll
  for (int mi = 0; mi < M; ++mi) acc[mi] = 0.f;
  const int64_t nfull = w.k / 16;
  const bool x4 = (w.k & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (int64_t b = lane; b < nfull; b += 32) {
    float v[16];
    if (q6) legacy_q6k_block(rp + b * bs, v);
    else legacy_q4k_block(rp + b * bs, v);
#pragma unroll
    for (int mi = 0; mi < M; ++mi) {
      const float* xr = x + mi * w.k + b * 16;
      if (x4) {  // rows of x start on 16-byte boundaries
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 xv = __ldg(reinterpret_cast<const float4*>(xr) + j);
          acc[mi] = fmaf(v[4 * j], xv.x, acc[mi]);
          acc[mi] = fmaf(v[4 * j + 1], xv.y, acc[mi]);
          acc[mi] = fmaf(v[4 * j + 2], xv.z, acc[mi]);
          acc[mi] = fmaf(v[4 * j + 3], xv.w, acc[mi]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[mi] = fmaf(v[e], __ldg(xr + e), acc[mi]);
      }
    }
  }
  if (lane == 0 && nfull * 16 < w.k) {  // trailing partial block (element-wise decode)
    for (int64_t i = nfull * 16; i < w.k; ++i) {
      const float v = q6 ? legacy_q6k_value(rp, i) : legacy_q4k_value(rp, w.k, i);
#pragma unroll
      for (int mi = 0; mi < M; ++mi) acc[mi] = fmaf(v, x[mi * w.k + i], acc[mi]);
    }
  }
#pragma unroll
  for (int mi = 0; mi < M; ++mi)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc[mi] += __shfl_xor_sync(0xffffffffu, acc[mi], off);
  if (lane == 0) {
    const float bv = bias ? bias[row] : 0.f;
#pragma unroll
    for (int mi = 0; mi < M; ++mi) y[mi * ldy + row] = acc[mi] + bv;
  }
}

}  // namespace

cudaError_t launch_dequant_f32(const DevWeight& w, int64_t row0, int64_t nrows, float* out,
                               cudaStream_t s) {
  const int64_t total = nrows * w.k;
  if (total <= 0) return cudaSuccess;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  dequant_kernel<<<(unsigned)blocks, 256, 0, s>>>(w, row0, nrows, out);
  return cudaGetLastError();
}

cudaError_t launch_q6k_relayout(const uint8_t* raw, int64_t n, int64_t sb, uint8_t* body, uint16_t* d,
                                cudaStream_t s) {
  const int64_t total = n * sb * Q6K_BYTES;
  if (total <= 0) return cudaSuccess;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  q6k_relayout_kernel<<<(unsigned)blocks, 256, 0, s>>>(raw, n, sb, body, d);
  return cudaGetLastError();
}

cudaError_t launch_gemv_legacy(const DevWeight& w, const float* x, int64_t m, const float* bias,
                               float* y, cudaStream_t s, int* launches, Bracket br) {
  const unsigned grid = (unsigned)((w.n + 7) / 8);
  bracket_record(br.start, s);
  for (int64_t m0 = 0; m0 < m; m0 += 4) {
    const int mc = (int)((m - m0) < 4 ? (m - m0) : 4);
    const float* xc = x + m0 * w.k;
    float* yc = y + m0 * w.n;
    switch (mc) {
      case 1: legacy_gemv_kernel<1><<<grid, 256, 0, s>>>(w, xc, bias, yc, w.n); break;
      case 2: legacy_gemv_kernel<2><<<grid, 256, 0, s>>>(w, xc, bias, yc, w.n); break;
      case 3: legacy_gemv_kernel<3><<<grid, 256, 0, s>>>(w, xc, bias, yc, w.n); break;
      default: legacy_gemv_kernel<4><<<grid, 256, 0, s>>>(w, xc, bias, yc, w.n); break;
    }
    if (launches) ++*launches;
  }
  bracket_record(br.stop, s);
  return cudaGetLastError();
}

}  // namespace kq
