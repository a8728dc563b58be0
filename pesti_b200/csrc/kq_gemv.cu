// kq_gemv.cu -- decode-shaped (small m) K-quant linear on CUDA cores.
//
// y[m][n] = sum_k x[m][k] * W[n][k] for GGUF Q4_K / Q6_K weights, f32 in and
// out.  The weight stream is the only large input, so the kernel is HBM-bound
// and is organised around reading each superblock exactly once with 16-byte
// loads while keeping the per-weight instruction count low:
//
//  * 8 lanes ("an octet") share one superblock; each lane owns 32 weights in
//    two runs of 16 that share one sub-block scale ("run a" / "run b").
//  * Quants are turned into floats with one PRMT each: the byte q lands in
//    bits 16..23 of 0x3F000000, i.e. the exact float 0.5 + q/256.  The
//    accumulated 0.5*sum(x) is removed per run with a precomputed sum of the
//    run's activations, so each weight costs one PRMT and one FFMA.
//  * A warp handles two rows at a time so every activation it loads feeds two
//    weights; activations are pre-permuted once per call (kq_prep_x) so that
//    the 8 lanes of an octet read 128 contiguous bytes (one L1 line).
//  * The next superblock step's weights are loaded before the current step is
//    computed, keeping two steps of loads in flight per warp.
//  * Partial sums are combined with warp shuffles.
//
// Reference semantics: QuantizedLinear::forward (pesti-runner/src/
// quantized_linear.rs:101-143) computes the same product after a full f32
// dequantization; here the dequantized value d*sc*q - dmin*m (Q4_K) or
// d*sc*(q-32) (Q6_K) is never materialised, the sum is regrouped per run.
#include "kq_common.cuh"
#include "kq_kernels.h"

namespace kq {

namespace {

template <int QT>
struct Geo;
template <>
struct Geo<GGUF_Q4_K> {
  static constexpr int DELTA = 32;  // run b starts 32 weights after run a
  __host__ __device__ static int run_a(int t) { return 64 * (t >> 1) + 16 * (t & 1); }
};
template <>
struct Geo<GGUF_Q6_K> {
  static constexpr int DELTA = 64;
  __host__ __device__ static int run_a(int t) {
    return 128 * (t >> 2) + 32 * ((t >> 1) & 1) + 16 * (t & 1);
  }
};

// ---- per-call activation prep --------------------------------------------
// xp[m][kb][j][t][4]: lane t's 8 float4 of superblock kb (j 0..3 run a,
// 4..7 run b).  sx[m][kb][t] = (sum run a, sum run b), sequential f32.
template <int QT>
__global__ void __launch_bounds__(256) prep_x_kernel(const float* __restrict__ x, int64_t m,
                                                     int64_t k, float4* __restrict__ xp,
                                                     float2* __restrict__ sx) {
  const int64_t sb = k / QK;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= m * sb * 8) return;
  const int t = (int)(idx & 7);
  const int64_t mkb = idx >> 3;  // m*sb + kb
  const int64_t mi = mkb / sb, kb = mkb - mi * sb;
  const float* src = x + mi * k + kb * QK + Geo<QT>::run_a(t);
  float4 v[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = ldg_f4(src + 4 * j);
#pragma unroll
  for (int j = 0; j < 4; ++j) v[4 + j] = ldg_f4(src + Geo<QT>::DELTA + 4 * j);
  float sa = 0.f, sb2 = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sa = __fadd_rn(sa, v[j].x);
    sa = __fadd_rn(sa, v[j].y);
    sa = __fadd_rn(sa, v[j].z);
    sa = __fadd_rn(sa, v[j].w);
    sb2 = __fadd_rn(sb2, v[4 + j].x);
    sb2 = __fadd_rn(sb2, v[4 + j].y);
    sb2 = __fadd_rn(sb2, v[4 + j].z);
    sb2 = __fadd_rn(sb2, v[4 + j].w);
  }
  float4* dst = xp + mkb * 64 + t;
#pragma unroll
  for (int j = 0; j < 8; ++j) dst[8 * j] = v[j];
  sx[mkb * 8 + t] = make_float2(sa, sb2);
}

// ---- raw superblock data a lane needs -------------------------------------
struct RawQ4 {
  uint4 hdr;  // d | dmin | scales[12]
  uint4 qs;   // 16 of the 128 quant bytes
};
struct RawQ6 {
  uint4 ql, qh, sc;
  uint32_t d;
};

__device__ __forceinline__ RawQ4 load_q4(const uint8_t* __restrict__ wq, int64_t row, int sb,
                                         int kb, int t) {
  const uint8_t* blk = wq + ((size_t)row * sb + kb) * Q4K_BYTES;
  RawQ4 r;
  r.hdr = ldg_nc_v4(blk);
  r.qs = ldg_nc_v4(blk + 16 + 16 * t);
  return r;
}

__device__ __forceinline__ RawQ6 load_q6(const uint8_t* __restrict__ wq,
                                         const uint16_t* __restrict__ wd, int64_t row, int sb,
                                         int kb, int t) {
  const size_t g = (size_t)row * sb + kb;
  const uint8_t* body = wq + g * Q6K_BODY;
  const int n = t >> 2, jj = (t >> 1) & 1, v = t & 1;
  RawQ6 r;
  r.ql = ldg_nc_v4(body + 64 * n + 32 * jj + 16 * v);
  r.qh = ldg_nc_v4(body + 128 + 32 * n + 16 * v);
  r.sc = ldg_nc_v4(body + 192);
  r.d = __ldg(wd + g);
  return r;
}

// Run coefficients: the run contributes A*acc - B*sum(x_run), where acc is the
// sum of (0.5 + q/256) * x over the run.
struct RunCoef {
  float A, B;
};

__device__ __forceinline__ void q4_coefs(const RawQ4& r, int t, RunCoef& a, RunCoef& b) {
  const float d = f16_bits_to_f32((uint16_t)(r.hdr.x & 0xffff));
  const float dmin = f16_bits_to_f32((uint16_t)(r.hdr.x >> 16));
  const int c = t >> 1;
  int sca, ma, scb, mb;
  q4k_scale_min_w(r.hdr.y, r.hdr.z, r.hdr.w, 2 * c, sca, ma);
  q4k_scale_min_w(r.hdr.y, r.hdr.z, r.hdr.w, 2 * c + 1, scb, mb);
  const float d1a = __fmul_rn(d, (float)sca), m1a = __fmul_rn(dmin, (float)ma);
  const float d1b = __fmul_rn(d, (float)scb), m1b = __fmul_rn(dmin, (float)mb);
  a.A = 256.f * d1a;
  a.B = __fadd_rn(128.f * d1a, m1a);
  b.A = 256.f * d1b;
  b.B = __fadd_rn(128.f * d1b, m1b);
}

__device__ __forceinline__ int sbyte(const uint4& v, int i) {
  const uint32_t w = (i < 4) ? v.x : (i < 8) ? v.y : (i < 12) ? v.z : v.w;
  return (int)(int8_t)((w >> (8 * (i & 3))) & 0xff);
}

__device__ __forceinline__ void q6_coefs(const RawQ6& r, int t, RunCoef& a, RunCoef& b) {
  const float d = f16_bits_to_f32((uint16_t)r.d);
  const int s = 8 * (t >> 2) + 2 * ((t >> 1) & 1) + (t & 1);
  const float dsa = __fmul_rn(d, (float)sbyte(r.sc, s));
  const float dsb = __fmul_rn(d, (float)sbyte(r.sc, s + 4));
  a.A = 256.f * dsa;
  a.B = 160.f * dsa;  // (q-32) = 256*f - 128 - 32
  b.A = 256.f * dsb;
  b.B = 160.f * dsb;
}

// The 16 magic floats of run a (RUN=0) or run b (RUN=1) of a lane.
template <int RUN>
__device__ __forceinline__ void q4_floats(const RawQ4& r, float f[16]) {
  const uint32_t w[4] = {r.qs.x, r.qs.y, r.qs.z, r.qs.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t q = RUN == 0 ? (w[i] & 0x0F0F0F0Fu) : ((w[i] >> 4) & 0x0F0F0F0Fu);
    f[4 * i + 0] = magic_byte<0>(q);
    f[4 * i + 1] = magic_byte<1>(q);
    f[4 * i + 2] = magic_byte<2>(q);
    f[4 * i + 3] = magic_byte<3>(q);
  }
}

template <int RUN>
__device__ __forceinline__ void q6_floats(const RawQ6& r, int t, float f[16]) {
  const uint32_t ql[4] = {r.ql.x, r.ql.y, r.ql.z, r.ql.w};
  const uint32_t qh[4] = {r.qh.x, r.qh.y, r.qh.z, r.qh.w};
  const int sh = 2 * ((t >> 1) & 1);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t hm = (qh[i] >> sh) & 0x33333333u;  // bits 0-1 run a, 4-5 run b
    const uint32_t q = RUN == 0 ? ((ql[i] & 0x0F0F0F0Fu) | ((hm << 4) & 0x30303030u))
                                : (((ql[i] >> 4) & 0x0F0F0F0Fu) | (hm & 0x30303030u));
    f[4 * i + 0] = magic_byte<0>(q);
    f[4 * i + 1] = magic_byte<1>(q);
    f[4 * i + 2] = magic_byte<2>(q);
    f[4 * i + 3] = magic_byte<3>(q);
  }
}

__device__ __forceinline__ float dot16(const float f[16], const float4 x[4]) {
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc = fmaf(f[4 * j + 0], x[j].x, acc);
    acc = fmaf(f[4 * j + 1], x[j].y, acc);
    acc = fmaf(f[4 * j + 2], x[j].z, acc);
    acc = fmaf(f[4 * j + 3], x[j].w, acc);
  }
  return acc;
}

template <int QT>
struct RawT;
template <>
struct RawT<GGUF_Q4_K> {
  using type = RawQ4;
};
template <>
struct RawT<GGUF_Q6_K> {
  using type = RawQ6;
};

template <int QT>
__device__ __forceinline__ typename RawT<QT>::type load_raw(const uint8_t* wq, const uint16_t* wd,
                                                            int64_t row, int sb, int kb, int t) {
  if constexpr (QT == GGUF_Q4_K)
    return load_q4(wq, row, sb, kb, t);
  else
    return load_q6(wq, wd, row, sb, kb, t);
}

template <int QT>
__device__ __forceinline__ void coefs(const typename RawT<QT>::type& r, int t, RunCoef& a,
                                      RunCoef& b) {
  if constexpr (QT == GGUF_Q4_K)
    q4_coefs(r, t, a, b);
  else
    q6_coefs(r, t, a, b);
}

template <int QT, int RUN>
__device__ __forceinline__ void run_floats(const typename RawT<QT>::type& r, int t, float f[16]) {
  if constexpr (QT == GGUF_Q4_K)
    q4_floats<RUN>(r, f);
  else
    q6_floats<RUN>(r, t, f);
}

// One warp = two rows; lane = (octet sbi 0..3, slot t 0..7).  The warp walks
// superblocks kb = sbi, sbi+4, ... of both rows.
template <int QT, int M>
__global__ void __launch_bounds__(256) gemv_kernel(const uint8_t* __restrict__ wq,
                                                   const uint16_t* __restrict__ wd, int64_t n,
                                                   int sb, const float4* __restrict__ xp,
                                                   const float2* __restrict__ sx,
                                                   const float* __restrict__ bias,
                                                   float* __restrict__ y, int64_t ldy) {
  using Raw = typename RawT<QT>::type;
  const int lane = threadIdx.x & 31;
  const int t = lane & 7, sbi = lane >> 3;
  const int64_t r0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 2;
  if (r0 >= n) return;
  const bool two = r0 + 1 < n;
  const int64_t r1 = two ? r0 + 1 : r0;

  float tot0[M], tot1[M];
#pragma unroll
  for (int mi = 0; mi < M; ++mi) tot0[mi] = tot1[mi] = 0.f;

  int kb = sbi;
  Raw c0, c1;
  if (kb < sb) {
    c0 = load_raw<QT>(wq, wd, r0, sb, kb, t);
    c1 = load_raw<QT>(wq, wd, r1, sb, kb, t);
  }
  for (; kb < sb; kb += 4) {
    Raw n0, n1;
    const int kn = kb + 4;
    if (kn < sb) {
      n0 = load_raw<QT>(wq, wd, r0, sb, kn, t);
      n1 = load_raw<QT>(wq, wd, r1, sb, kn, t);
    }
    RunCoef a0, b0, a1, b1;
    coefs<QT>(c0, t, a0, b0);
    coefs<QT>(c1, t, a1, b1);
    {
      float f0[16], f1[16];
      run_floats<QT, 0>(c0, t, f0);
      run_floats<QT, 0>(c1, t, f1);
#pragma unroll
      for (int mi = 0; mi < M; ++mi) {
        const size_t mkb = (size_t)mi * sb + kb;
        const float4* xr = xp + mkb * 64 + t;
        float4 xv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = __ldg(xr + 8 * j);
        const float s = __ldg(&sx[mkb * 8 + t].x);
        tot0[mi] += fmaf(a0.A, dot16(f0, xv), -a0.B * s);
        tot1[mi] += fmaf(a1.A, dot16(f1, xv), -a1.B * s);
      }
    }
    {
      float f0[16], f1[16];
      run_floats<QT, 1>(c0, t, f0);
      run_floats<QT, 1>(c1, t, f1);
#pragma unroll
      for (int mi = 0; mi < M; ++mi) {
        const size_t mkb = (size_t)mi * sb + kb;
        const float4* xr = xp + mkb * 64 + 32 + t;
        float4 xv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = __ldg(xr + 8 * j);
        const float s = __ldg(&sx[mkb * 8 + t].y);
        tot0[mi] += fmaf(b0.A, dot16(f0, xv), -b0.B * s);
        tot1[mi] += fmaf(b1.A, dot16(f1, xv), -b1.B * s);
      }
    }
    c0 = n0;
    c1 = n1;
  }

#pragma unroll
  for (int mi = 0; mi < M; ++mi) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      tot0[mi] += __shfl_xor_sync(0xffffffffu, tot0[mi], off);
      tot1[mi] += __shfl_xor_sync(0xffffffffu, tot1[mi], off);
    }
  }
  if (lane == 0) {
    const float b0v = bias ? bias[r0] : 0.f;
    const float b1v = (bias && two) ? bias[r1] : 0.f;
#pragma unroll
    for (int mi = 0; mi < M; ++mi) {
      y[mi * ldy + r0] = tot0[mi] + b0v;
      if (two) y[mi * ldy + r1] = tot1[mi] + b1v;
    }
  }
}

template <int QT>
cudaError_t launch_typed(const DevWeight& w, const float* x, int64_t m, const float* bias,
                         float* y, void* ws, cudaStream_t s, int* launches, Bracket br) {
  const int64_t sb = w.sb;
  float4* xp = reinterpret_cast<float4*>(ws);
  float2* sx = reinterpret_cast<float2*>(reinterpret_cast<char*>(ws) + (size_t)m * w.k * 4);
  {
    const int64_t threads = m * sb * 8;
    const int bs = 256;
    prep_x_kernel<QT><<<(unsigned)((threads + bs - 1) / bs), bs, 0, s>>>(x, m, w.k, xp, sx);
    if (launches) ++*launches;
  }
  const int64_t pairs = (w.n + 1) / 2;
  const int warps = 8;
  const unsigned grid = (unsigned)((pairs + warps - 1) / warps);
  bracket_record(br.start, s);
  for (int64_t m0 = 0; m0 < m; m0 += 4) {
    const int mc = (int)((m - m0) < 4 ? (m - m0) : 4);
    const float4* xpc = xp + (size_t)m0 * sb * 64;
    const float2* sxc = sx + (size_t)m0 * sb * 8;
    float* yc = y + m0 * w.n;
    switch (mc) {
      case 1:
        gemv_kernel<QT, 1><<<grid, warps * 32, 0, s>>>(w.q, w.d, w.n, (int)sb, xpc, sxc, bias, yc, w.n);
        break;
      case 2:
        gemv_kernel<QT, 2><<<grid, warps * 32, 0, s>>>(w.q, w.d, w.n, (int)sb, xpc, sxc, bias, yc, w.n);
        break;
      case 3:
        gemv_kernel<QT, 3><<<grid, warps * 32, 0, s>>>(w.q, w.d, w.n, (int)sb, xpc, sxc, bias, yc, w.n);
        break;
      default:
        gemv_kernel<QT, 4><<<grid, warps * 32, 0, s>>>(w.q, w.d, w.n, (int)sb, xpc, sxc, bias, yc, w.n);
        break;
    }
    if (launches) ++*launches;
  }
  bracket_record(br.stop, s);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemv_gguf(const DevWeight& w, const float* x, int64_t m, const float* bias,
                             float* y, void* ws, cudaStream_t s, int* launches, Bracket br) {
  if (w.type == GGUF_Q4_K) return launch_typed<GGUF_Q4_K>(w, x, m, bias, y, ws, s, launches, br);
  return launch_typed<GGUF_Q6_K>(w, x, m, bias, y, ws, s, launches, br);
}

size_t gemv_gguf_workspace_bytes(int64_t m, int64_t k) {
  // xp: m*k floats; sx: m*(k/256)*8 float2
  return (size_t)m * k * 4 + (size_t)m * (k / QK) * 8 * 8 + 256;
}

}  // namespace kq
