// kq_dp4a.cu -- decode dequant-GEMV for small batches (M <= 4 tokens) on the
// CUDA cores, built to keep HBM busy.
//
// Work split: one warp streams one weight row at a time (rows are dealt out
// grid-stride, so every SM gets the same number of rows within one), in
// "iterations" of 32 lane units:
//   GGUF Q4_K: 4 superblocks per iteration; lane i takes superblock 4it+i/8,
//              16-byte quant chunk c = i%8 (32 weights: 16 of sub-block 2(c/2)
//              in the low nibbles, 16 of sub-block 2(c/2)+1 in the high ones)
//              plus the superblock's 16-byte header (d, dmin, 6-bit scales).
//   GGUF Q6_K: 8 superblocks per iteration; lane i takes superblock 8it+i/4,
//              slot c = i%4 of the device body (48 bytes = 64 weights, see
//              q6k_body_offset), the 16 scale bytes and d.
// Every lane keeps D iterations of raw weights in flight in registers
// (coalesced 128-bit loads that bypass L1), so an SM has ~16-24 warps x D
// iterations of loads outstanding -- the memory-level parallelism HBM needs.
//
// Products: the activations are prepared once per call (prep kernel) as
// 16-bit integers x_int = rint(x * 2^-e), one power-of-two scale 2^e per
// (token, superblock) chosen so that max|x| * 2^-e is in [2^14, 2^15), split
// into a signed high byte and an unsigned low byte (x_int = 256 hi + lo).
// The quants are non-negative bytes, so two dp4a per 4 weights give exact
// integer partial sums; sub-block scales are applied in integer (Q4_K) or in
// f32 per 8-weight group (Q6_K), the superblock factor d * 2^e in f32.  The
// only approximation is the 16-bit activation rounding (relative 2^-15 of
// each superblock's largest activation); the Q4_K min term uses exact f32
// activation sums.  Partial sums are added with warp shuffles.
//
// The prepared activations are laid out in the order lanes read them
// (x[token][iteration][j][lane] in 16-byte units), so each activation load of
// a warp is one contiguous 512-byte run (L1-resident: every warp of an SM
// reads the same activations).
#include "kq_common.cuh"
#include "kq_kernels.h"
#include "kq_xs.cuh"

#include <algorithm>
#include <map>
#include <utility>

namespace kq {
namespace {

constexpr int WARPS = 8;  // per CTA

template <int QT>
struct Dp4aFmt;
template <>
struct Dp4aFmt<GGUF_Q4_K> {
  static constexpr int SPI = 4;   // superblocks per iteration
  static constexpr int XJ = 4;    // 16-byte activation units per lane per iteration
  static constexpr int SUMJ = 1;  // 8-byte f32 sums (2 floats) per lane per iteration
  static constexpr int D = 4;     // iterations in flight
  static constexpr int CPS = 3;   // CTAs per SM
};
template <>
struct Dp4aFmt<GGUF_Q6_K> {
  static constexpr int SPI = 8;
  static constexpr int XJ = 8;
  static constexpr int SUMJ = 2;  // 16-byte int sums (4 ints) per lane per iteration
  static constexpr int D = 3;
  static constexpr int CPS = 2;
};

// Scratch layout for m tokens (offsets in bytes, each 256-aligned).
struct Dp4aLayout {
  int64_t iters;
  size_t xq, sums, xs, end;
};
template <int QT>
Dp4aLayout dp4a_layout(int64_t m, int64_t sb) {
  using F = Dp4aFmt<QT>;
  Dp4aLayout L;
  L.iters = (sb + F::SPI - 1) / F::SPI;
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t per_it = 32 * 16;  // one 16-byte unit per lane
  L.xq = 0;
  L.sums = up(L.xq + (size_t)m * L.iters * F::XJ * per_it);
  const size_t sum_bytes = QT == GGUF_Q4_K ? 8 : 16;
  L.xs = up(L.sums + (size_t)m * L.iters * F::SUMJ * 32 * sum_bytes);
  L.end = up(L.xs + (size_t)m * L.iters * F::SPI * sizeof(float));
  return L;
}

struct Dp4aParams {
  const uint8_t* q;
  const uint16_t* d;
  int64_t d_ld;
  int n, sb, iters, m;
  const uint4* xq;     // [m][iters][XJ][32] 16-byte units
  const void* sums;    // Q4_K: float2 [m][iters][32]; Q6_K: int4 [m][iters][2][32]
  const float* xs;     // [m][iters * SPI] superblock factors 2^e (NaN: non-finite block)
  const float* bias;
  float* y;
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t ldg_nc_u16(const uint16_t* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// ---- activation prep ------------------------------------------------------------
// Quantize one superblock's activations: the block maximum over the `group`
// lanes that share superblock kb (consecutive lanes), then 2^-e scaling.
struct BlockScale {
  float inv;     // 2^-e
  float factor;  // 2^e, or NaN when the block holds a non-finite value
};
__device__ __forceinline__ BlockScale block_scale(float amax_lane, int group) {
  float amax = amax_lane;
  for (int o = 1; o < group; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  BlockScale s;
  if (!(amax <= 3.4e38f)) {  // inf or NaN somewhere in the block
    s.inv = 0.f;
    s.factor = __int_as_float(0x7fc00000);
    return s;
  }
  int e = 0;
  if (amax > 0.f) e = (int)((__float_as_uint(amax) >> 23) & 0xff) - 127 - 14;
  e = max(-126, min(126, e));
  s.inv = __uint_as_float((uint32_t)(127 - e) << 23);
  s.factor = __uint_as_float((uint32_t)(127 + e) << 23);
  return s;
}
__device__ __forceinline__ int quant16(float v, float inv) {
  const float r = rintf(v * inv);
  return (int)fminf(fmaxf(r, -32768.f), 32767.f);
}
// Four 16-bit activations -> (hi bytes, lo bytes) words, byte i = activation i.
__device__ __forceinline__ void split4(const int (&v)[4], uint32_t& hi, uint32_t& lo) {
  hi = 0;
  lo = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    hi |= (uint32_t)((v[i] >> 8) & 0xff) << (8 * i);
    lo |= (uint32_t)(v[i] & 0xff) << (8 * i);
  }
}

// One thread per (token, iteration, lane unit); blockDim = 128 (4 iterations).
template <int QT>
__global__ void __launch_bounds__(128) dp4a_prep_kernel(const float* __restrict__ x, int m, int k, int sb,
                                                        int iters, uint4* __restrict__ xq,
                                                        void* __restrict__ sums, float* __restrict__ xs) {
  using F = Dp4aFmt<QT>;
  pdl_trigger();  // let the GEMV kernel start streaming weights now
  const int lane = threadIdx.x & 31;
  const int it = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int t = blockIdx.y;
  if (it >= iters) return;  // whole warp
  const float* xr = x + (int64_t)t * k;
  uint4* xo = xq + ((int64_t)t * iters + it) * F::XJ * 32 + lane;
  if constexpr (QT == GGUF_Q4_K) {
    const int kb = 4 * it + (lane >> 3), c = lane & 7;
    const bool live = kb < sb;
    const int base = kb * 256 + 64 * (c >> 1) + 16 * (c & 1);  // sub-block A run; B run = base + 32
    float a[16], b[16];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
      if (live) {
        va = ldg_f4(xr + base + i);
        vb = ldg_f4(xr + base + 32 + i);
      }
      a[i] = va.x; a[i + 1] = va.y; a[i + 2] = va.z; a[i + 3] = va.w;
      b[i] = vb.x; b[i + 1] = vb.y; b[i + 2] = vb.z; b[i + 3] = vb.w;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fmaxf(fabsf(a[i]), fabsf(b[i])));
    const BlockScale s = block_scale(amax, 8);
    float sa = 0.f, sbm = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      int qa[4], qb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        qa[i] = quant16(a[4 * w + i], s.inv);
        qb[i] = quant16(b[4 * w + i], s.inv);
        sa += a[4 * w + i];
        sbm += b[4 * w + i];
      }
      uint4 u;
      split4(qa, u.x, u.y);
      split4(qb, u.z, u.w);
      xo[w * 32] = u;
    }
    reinterpret_cast<float2*>(sums)[((int64_t)t * iters + it) * 32 + lane] = make_float2(sa, sbm);
    if (c == 0) xs[(int64_t)t * iters * F::SPI + kb] = live ? s.factor : 0.f;
  } else {
    const int kb = 8 * it + (lane >> 2), c = lane & 3;
    const bool live = kb < sb;
    // group (h, g, w): weights 128h + 32g + 8c + 4w + [0, 4)
    float v[2][4][2][4];
    float amax = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int g = 0; g < 4; ++g)
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
          if (live) f = ldg_f4(xr + kb * 256 + 128 * h + 32 * g + 8 * c + 4 * w);
          v[h][g][w][0] = f.x; v[h][g][w][1] = f.y; v[h][g][w][2] = f.z; v[h][g][w][3] = f.w;
          amax = fmaxf(amax, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
        }
    const BlockScale s = block_scale(amax, 4);
    int4* so = reinterpret_cast<int4*>(sums) + ((int64_t)t * iters + it) * 2 * 32 + lane;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int gs[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        gs[g] = 0;
        uint32_t hw[2], lw[2];
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          int qv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            qv[i] = quant16(v[h][g][w][i], s.inv);
            gs[g] += qv[i];
          }
          split4(qv, hw[w], lw[w]);
        }
        // unit j = 4h + 2w + g/2 holds {hi, lo} of g even then g odd
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          uint32_t* u = reinterpret_cast<uint32_t*>(xo + (4 * h + 2 * w + (g >> 1)) * 32);
          u[2 * (g & 1)] = hw[w];
          u[2 * (g & 1) + 1] = lw[w];
        }
      }
      so[h * 32] = make_int4(-32 * gs[0], -32 * gs[1], -32 * gs[2], -32 * gs[3]);
    }
    if (c == 0) xs[(int64_t)t * iters * F::SPI + kb] = live ? s.factor : 0.f;
  }
}

// ---- GEMV -----------------------------------------------------------------------
template <int QT>
struct Raw;
template <>
struct Raw<GGUF_Q4_K> {
  uint4 qs, hdr;
};
template <>
struct Raw<GGUF_Q6_K> {
  uint4 p0, p1, p2, sc;
  uint32_t d;
};

template <int QT>
__device__ __forceinline__ void load_raw(Raw<QT>& r, const Dp4aParams& P, int row, int it, int lane, bool valid) {
  if constexpr (QT == GGUF_Q4_K) {
    const int kb = 4 * it + (lane >> 3), c = lane & 7;
    if (valid && kb < P.sb) {
      const uint8_t* blk = P.q + ((int64_t)row * P.sb + kb) * Q4K_BYTES;
      r.qs = ldg_nc_v4(blk + 16 + 16 * c);
      r.hdr = ldg_nc_v4(blk);
    } else {
      r.qs = make_uint4(0, 0, 0, 0);
      r.hdr = r.qs;
    }
  } else {
    const int kb = 8 * it + (lane >> 2), c = lane & 3;
    if (valid && kb < P.sb) {
      const uint8_t* blk = P.q + ((int64_t)row * P.sb + kb) * Q6K_BODY;
      r.p0 = ldg_nc_v4(blk + 48 * c);
      r.p1 = ldg_nc_v4(blk + 48 * c + 16);
      r.p2 = ldg_nc_v4(blk + 48 * c + 32);
      r.sc = ldg_nc_v4(blk + 192);
      r.d = ldg_nc_u16(P.d + (int64_t)row * P.d_ld + kb);
    } else {
      r.p0 = make_uint4(0, 0, 0, 0);
      r.p1 = r.p0;
      r.p2 = r.p0;
      r.sc = r.p0;
      r.d = 0;
    }
  }
}

// acc[t] += this lane's share of row . x_t for iteration `it`.
template <int MT>
__device__ __forceinline__ void compute_q4(const Raw<GGUF_Q4_K>& r, const Dp4aParams& P, int it, int lane,
                                           float (&acc)[MT]) {
  const int c = lane & 7, j2 = 2 * (c >> 1);
  const float d = f16_bits_to_f32((uint16_t)(r.hdr.x & 0xffff));
  const float dmin = f16_bits_to_f32((uint16_t)(r.hdr.x >> 16));
  int sca, ma, scb, mb;
  q4k_scale_min_w(r.hdr.y, r.hdr.z, r.hdr.w, j2, sca, ma);
  q4k_scale_min_w(r.hdr.y, r.hdr.z, r.hdr.w, j2 + 1, scb, mb);
  uint32_t qa[4], qb[4];
  const uint32_t W[4] = {r.qs.x, r.qs.y, r.qs.z, r.qs.w};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    qa[w] = W[w] & 0x0F0F0F0Fu;
    qb[w] = (W[w] >> 4) & 0x0F0F0F0Fu;
  }
  const int kb = 4 * it + (lane >> 3);
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int64_t ti = (int64_t)t * P.iters + it;
    const uint4* xv = P.xq + ti * 4 * 32 + lane;
    int ahi = 0, alo = 0, bhi = 0, blo = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint4 u = __ldg(xv + w * 32);
      ahi = dp4a_s(qa[w], u.x, ahi);
      alo = dp4a_u(qa[w], u.y, alo);
      bhi = dp4a_s(qb[w], u.z, bhi);
      blo = dp4a_u(qb[w], u.w, blo);
    }
    const float2 s = __ldg(reinterpret_cast<const float2*>(P.sums) + ti * 32 + lane);
    const float f = __ldg(P.xs + (int64_t)t * P.iters * 4 + kb);
    const int da = ahi * 256 + alo, db = bhi * 256 + blo;
    const int iv = sca * da + scb * db;  // |iv| < 2^30
    acc[t] = fmaf(d * f, (float)iv, acc[t]);
    acc[t] = fmaf(-dmin, fmaf((float)ma, s.x, (float)mb * s.y), acc[t]);
  }
}

__device__ __forceinline__ float sbyte(uint32_t w, int b) { return (float)(int)(int8_t)((w >> (8 * b)) & 0xff); }

template <int MT>
__device__ __forceinline__ void compute_q6(const Raw<GGUF_Q6_K>& r, const Dp4aParams& P, int it, int lane,
                                           float (&acc)[MT]) {
  const int c = lane & 3;
  const int kb = 8 * it + (lane >> 2);
  // q[h][g][w]: the 4 six-bit quants of group (h, g, w) as bytes
  uint32_t q[2][4][2];
  const uint32_t ql[2][2][2] = {{{r.p0.x, r.p0.y}, {r.p0.z, r.p0.w}}, {{r.p1.x, r.p1.y}, {r.p1.z, r.p1.w}}};
  const uint32_t qh[2][2] = {{r.p2.x, r.p2.y}, {r.p2.z, r.p2.w}};
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const uint32_t H = qh[h][w];
      q[h][0][w] = (ql[h][0][w] & 0x0F0F0F0Fu) | ((H << 4) & 0x30303030u);
      q[h][1][w] = (ql[h][1][w] & 0x0F0F0F0Fu) | ((H << 2) & 0x30303030u);
      q[h][2][w] = ((ql[h][0][w] >> 4) & 0x0F0F0F0Fu) | (H & 0x30303030u);
      q[h][3][w] = ((ql[h][1][w] >> 4) & 0x0F0F0F0Fu) | ((H >> 2) & 0x30303030u);
    }
  // scale of group (h, g): byte 8h + 2g + c/2 of the 16 scale bytes
  float scf[2][4];
  const uint32_t S[4] = {r.sc.x, r.sc.y, r.sc.z, r.sc.w};
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int si = 8 * h + 2 * g;  // + c/2
      const uint32_t word = S[si >> 2];
      scf[h][g] = sbyte(word, (si & 3) + (c >> 1));
    }
  const float d = f16_bits_to_f32((uint16_t)r.d);
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int64_t ti = (int64_t)t * P.iters + it;
    const uint4* xv = P.xq + ti * 8 * 32 + lane;
    const int4* sv = reinterpret_cast<const int4*>(P.sums) + ti * 2 * 32 + lane;
    float part = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int4 sg = __ldg(sv + h * 32);
      const int sgv[4] = {sg.x, sg.y, sg.z, sg.w};
      uint4 u[2][2];
#pragma unroll
      for (int w = 0; w < 2; ++w)
#pragma unroll
        for (int gp = 0; gp < 2; ++gp) u[w][gp] = __ldg(xv + (4 * h + 2 * w + gp) * 32);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int gp = g >> 1, od = g & 1;
        int hi = 0, lo = 0;
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const uint32_t xh = od ? u[w][gp].z : u[w][gp].x;
          const uint32_t xl = od ? u[w][gp].w : u[w][gp].y;
          hi = dp4a_s(q[h][g][w], xh, hi);
          lo = dp4a_u(q[h][g][w], xl, lo);
        }
        const int v = hi * 256 + lo + sgv[g];  // sum of (q - 32) * x_int, |v| < 2^24
        part = fmaf((float)v, scf[h][g], part);
      }
    }
    const float f = __ldg(P.xs + (int64_t)t * P.iters * 8 + kb);
    acc[t] = fmaf(part, d * f, acc[t]);
  }
}

template <int QT, int MT>
__global__ void __launch_bounds__(32 * WARPS, Dp4aFmt<QT>::CPS) dp4a_gemv_kernel(const Dp4aParams P) {
  using F = Dp4aFmt<QT>;
  constexpr int D = F::D;
  const int lane = threadIdx.x & 31;
  const int slot = (threadIdx.x >> 5) * gridDim.x + blockIdx.x;  // warp slot: rows slot, slot + stride, ...
  const int stride = WARPS * gridDim.x;
  if (slot >= P.n) {
    pdl_wait();
    return;
  }
  // load cursor (row, iteration) runs D iterations ahead of the compute cursor
  int lrow = slot, lit = 0;
  Raw<QT> buf[D];
#pragma unroll
  for (int j = 0; j < D; ++j) {
    load_raw<QT>(buf[j], P, lrow, lit, lane, lrow < P.n);
    if (++lit == P.iters) { lit = 0; lrow += stride; }
  }
  pdl_wait();  // activations are ready from here on
  int crow = slot, cit = 0;
  float acc[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) acc[t] = 0.f;
  bool more = true;
  while (more) {
#pragma unroll
    for (int j = 0; j < D; ++j) {
      if (more) {
        if constexpr (QT == GGUF_Q4_K) compute_q4<MT>(buf[j], P, cit, lane, acc);
        else compute_q6<MT>(buf[j], P, cit, lane, acc);
        load_raw<QT>(buf[j], P, lrow, lit, lane, lrow < P.n);
        if (++lit == P.iters) { lit = 0; lrow += stride; }
        if (++cit == P.iters) {
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            float v = acc[t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && t < P.m) P.y[(int64_t)t * P.n + crow] = v + (P.bias ? P.bias[crow] : 0.f);
            acc[t] = 0.f;
          }
          cit = 0;
          crow += stride;
          more = crow < P.n;
        }
      }
    }
  }
}

template <int QT, int MT>
cudaError_t launch_main(const Dp4aParams& P, int num_sms, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(num_sms * Dp4aFmt<QT>::CPS));
  cfg.blockDim = dim3(32 * WARPS);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, dp4a_gemv_kernel<QT, MT>, P);
}

template <int QT>
cudaError_t launch_typed(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y, void* ws,
                         int num_sms, cudaStream_t s, int* launches, Bracket br) {
  using F = Dp4aFmt<QT>;
  const Dp4aLayout L = dp4a_layout<QT>(m, w.sb);
  uint8_t* base = static_cast<uint8_t*>(ws);
  Dp4aParams P;
  P.q = w.q;
  P.d = w.d;
  P.d_ld = w.d_ld;
  P.n = (int)w.n;
  P.sb = (int)w.sb;
  P.iters = (int)L.iters;
  P.m = (int)m;
  P.xq = reinterpret_cast<const uint4*>(base + L.xq);
  P.sums = base + L.sums;
  P.xs = reinterpret_cast<const float*>(base + L.xs);
  P.bias = bias;
  P.y = y;
  dim3 pg((unsigned)((L.iters + 3) / 4), (unsigned)m);
  dp4a_prep_kernel<QT><<<pg, 128, 0, s>>>(x, (int)m, (int)w.k, (int)w.sb, (int)L.iters,
                                         reinterpret_cast<uint4*>(base + L.xq), base + L.sums,
                                         reinterpret_cast<float*>(base + L.xs));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (launches) ++*launches;
  bracket_record(br.start, s);
  switch (m) {
    case 1: e = launch_main<QT, 1>(P, num_sms, s); break;
    case 2: e = launch_main<QT, 2>(P, num_sms, s); break;
    case 3: e = launch_main<QT, 3>(P, num_sms, s); break;
    case 4: e = launch_main<QT, 4>(P, num_sms, s); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  if (launches) ++*launches;
  bracket_record(br.stop, s);
  (void)F::SPI;
  return cudaSuccess;
}

// ---- one token: TMA-streamed rows, activation-stationary warps -------------------
// For a single token the activations of an 8-superblock K-slice fit in a
// warp's registers (64 weights per lane -> 32 registers of hi/lo bytes), so
// each compute warp owns one K-slice and applies it to every row of its CTA.
// The weights reach shared memory by bulk TMA copies (cp.async.bulk) issued
// by one producer warp: each CTA owns a contiguous block of rows and streams
// it through a ring of S stages of 2G rows each (rows are contiguous in
// memory, Q6_K d rows too), so up to ~100 KB per CTA are in flight without
// tying up registers or L1 miss slots.  Compute warps: nk K-slices x G row
// groups; warp (s, g) takes rows g and g + G of every stage and reduces the
// two partials together with shuffles into shared memory; the CTA adds the
// nk partials in slice order at the end (deterministic).  Bulk copies carry a
// fixed cost each, so stages are large (tens of KB).
//
// One CTA per SM (up to 15 compute warps + the producer).  The ring holds
// about XS_INFLIGHT bytes: streaming-read measurements on B200 peak near
// 64-128 KB in flight per SM with 16-32 KB bulk copies; much deeper rings
// lose bandwidth.  The kernel triggers its dependents at once, so the next
// GEMV's CTAs can start streaming on an SM as soon as ours retires there.
//
// Lane i of slice s works on superblock kb = 8s + i/4, unit u = i%4:
//   Q4_K: qs bytes 32u .. 32u+31 (sub-blocks 2u and 2u+1 complete) + header
//   Q6_K: body slot u (48 bytes, 64 weights) + the scale bytes + d
// Each lane quantizes its own 64 activations once (per superblock 2^e with
// max|x| * 2^-e in [2^13, 2^14), rounding by the 1.5 * 2^23 float addition,
// so the low 16 bits of the float are the two's-complement integer).
// Q6_K sub-block scales are applied in exact int32: the hi- and lo-limb
// products are accumulated separately (each sum of 8 (q-32) x products is
// < 2^17 in size), the -32 x corrections are the accumulators' start values.
// Every mbarrier wait is bounded: a stalled pipeline ends the kernel with an
// error code in *err instead of hanging, and the producer always waits for
// its issued copies to land before the CTA may exit.
constexpr int XS_SPW = 8;          // superblocks per warp slice
constexpr int XS_MAX_COMPUTE = 15;  // compute warps (+ 1 producer = 512 threads)
constexpr int XS_MAX_SMEM = 227 * 1024;
constexpr int64_t XS_INFLIGHT = 144 * 1024;  // ring bytes in flight per CTA
constexpr int64_t XS_STAGE_MAX = 64 * 1024;  // bytes of one ring stage (unless one row group exceeds it)

enum : int { XS_ERR_FULL = 21, XS_ERR_EMPTY = 22, XS_ERR_DRAIN = 23, XS_ERR_TP = 32 };
constexpr int64_t XS_PF_CHUNK = 64 * 1024;  // bytes per L2 prefetch instruction

// Device bytes of one superblock within a row (Q6_K: the body; its d values
// are a separate array), and a row's stride: its superblocks rounded up to a
// whole number of 16-byte units (the same stride the upload gives each type).
__host__ __device__ constexpr int xs_stride(int qt) {
  return qt == GGUF_Q4_K     ? Q4K_BYTES
         : qt == GGUF_Q6_K   ? Q6K_BODY
         : qt == GGUF_Q5_K   ? Q5K_BYTES
         : qt == GGUF_Q3_K   ? Q3K_DEV
         : qt == LEGACY_Q4_K ? 16 * 28  // the reference's blocks: 16 per 256 weights
         : qt == LEGACY_Q6_K ? 16 * 42
                             : Q2K_DEV;
}
// The reference's own 16-weight blocks (rows of k % 256 == 0 weights, so a
// row is whole 256-weight spans of 448 / 672 bytes).
__host__ __device__ constexpr bool xs_legacy(int qt) { return qt == LEGACY_Q4_K || qt == LEGACY_Q6_K; }
__host__ __device__ constexpr int64_t xs_row_bytes(int qt, int64_t sb) { return (sb * xs_stride(qt) + 15) & ~int64_t(15); }
// Types whose sub-blocks hold 16 weights (Q2_K, Q3_K) instead of 32 (Q4_K, Q5_K).
__host__ __device__ constexpr bool xs_g16(int qt) { return qt == GGUF_Q2_K || qt == GGUF_Q3_K; }
// Activation sums kept per 64-weight unit: Q4_K / Q5_K float2 (the unit's two
// 32-weight sub-blocks), Q2_K / Q3_K float4 (four 16-weight sub-blocks),
// Q6_K int4[4] (the -32 corrections of its 8-weight groups).
// Legacy Q4_K: eight floats per unit (the sums of each block half); legacy Q6_K none (16 kept for alignment).
__host__ __device__ constexpr int xs_sum_bytes(int qt) {
  return qt == GGUF_Q6_K ? 64 : qt == LEGACY_Q4_K ? 32 : (xs_g16(qt) || qt == LEGACY_Q6_K) ? 16 : 8;
}

struct XsParams {
  const uint8_t* q;     // [n][row_bytes]
  // (tensor-parallel fields last)
  const uint16_t* d;    // Q6_K: [n][d_row_bytes / 2]
  int64_t row_bytes;    // weight bytes per row
  int d_row_bytes;      // Q6_K: d bytes per row (a multiple of 16); Q4_K: 0
  int n, sb, nk, G, S;  // rows, superblocks per row, K-slices, rows per stage, ring stages
  int rows_max;         // most rows any CTA owns (shared-memory sizing)
  int64_t stage_bytes;  // 2G * (row_bytes + d_row_bytes)
  const float* x;
  const float* bias;  // may alias y (residual update)
  float* y;
  int* err;
  // activation source: XS_X_NORM x / sqrt(mean(x[0:dim]^2) + eps) * nw (zero past dim);
  // XS_X_SWIGLU act(x) * x2 with the decoder's gate activation `act`
  const float* x2;
  const float* nw;
  int dim;
  float eps;
  int act;
  // L2 prefetch of the weight the next kernel reads: two byte ranges, split over the CTAs
  const uint8_t* pf[2];
  int64_t pf_bytes[2];
  // tensor parallel (XsTp): XS_Y_PEERS sends y to every rank's exchange image;
  // XS_X_REDUCE* stage x = h_in + the ranks' partials (and write it to h_out)
  XsTp tp;
  int64_t xr_floats;  // XS_X_REDUCE*: floats of the reduced vector kept in shared memory
  int64_t nw_floats;  // NORM modes: norm weights copied to shared memory at kernel start
};

// Dynamic shared memory: ring | staged x: words uint4 [sb8 * 4 units][8]
// (swizzled), sums (Q4_K float2 / Q6_K int4[4] per unit), 2^e per superblock
// | row partials [rows_max][nk] | 32 reduction floats | reduced x (tensor
// parallel consumers) | norm weights | full[S], empty[S], aux.
struct XsSmem {
  size_t ring, xw, sums, xsf, part, red, xr, nw, bar, end;
  __host__ __device__ XsSmem(int qt, int nk, int64_t stage_bytes, int S, int rows_max, int64_t xr_floats,
                             int64_t nw_floats) {
    const size_t units = (size_t)XS_SPW * nk * 4;
    ring = 0;
    xw = ring + (size_t)S * (size_t)stage_bytes;
    sums = xw + units * 128;
    xsf = sums + units * xs_sum_bytes(qt);
    part = xsf + units;  // one float per superblock = units / 4 floats
    red = (part + (size_t)rows_max * nk * 4 + 15) & ~size_t(15);
    xr = red + 32 * 4;
    nw = xr + (size_t)xr_floats * 4;
    bar = (nw + (size_t)nw_floats * 4 + 7) & ~size_t(7);
    end = bar + (size_t)(2 * S + 1) * 8;
  }
};

// This CTA's share of the next weight's bytes into L2 (16-byte units only:
// nothing past the end of a range is touched).
__device__ __forceinline__ void xs_prefetch(const XsParams& P, int b, int C) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!P.pf[r] || P.pf_bytes[r] < 16) continue;
    const int64_t units = P.pf_bytes[r] / 16;
    const int64_t u0 = units * b / C, u1 = units * (b + 1) / C;
    for (int64_t u = u0; u < u1; u += XS_PF_CHUNK / 16) {
      const uint32_t bytes = (uint32_t)((XS_PF_CHUNK / 16 < u1 - u ? XS_PF_CHUNK / 16 : u1 - u) * 16);
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(P.pf[r] + u * 16), "r"(bytes) : "memory");
    }
  }
}
// Quantize x into shared memory: half-unit hu = 8 kb + 2 u + hf (32 weights)
// per thread of the `nthreads` compute threads, the 8 half-units of a
// superblock on consecutive lanes, written in the order lanes read them.
// XS_X_NORM first reduces sum(x^2) over the CTA (every CTA does it: the
// vector is small and L2-resident); XS_X_SWIGLU applies the gate per element.
template <int QT, int XM>
__device__ __forceinline__ void xs_stage_x(const XsParams& P, const XsSmem& L, uint8_t* smem, int nthreads) {
  uint4* xw = reinterpret_cast<uint4*>(smem + L.xw);
  float* xsf = reinterpret_cast<float*>(smem + L.xsf);
  const int lane = threadIdx.x & 31;
  constexpr bool REDUCE = XM == XS_X_REDUCE || XM == XS_X_REDUCE_NORM;
  float* xr = reinterpret_cast<float*>(smem + L.xr);
  if constexpr (REDUCE) {
    // every rank's partial of the last exchange (sent by the previous kernel
    // on every rank): x = h_in + sum_r p_r in rank order into shared memory,
    // each value taken once its word carries that exchange's epoch; this
    // CTA's slice also goes to h_out
    const XsTp& T = P.tp;
    const unsigned epoch = *reinterpret_cast<volatile unsigned*>(T.epoch);
    const unsigned long long* img = T.exch[T.rank] + (size_t)(epoch & 1u) * (size_t)T.slot_elems;
    const int q4 = P.dim / 4, C = gridDim.x, b = blockIdx.x;
    const int lo = (int)((int64_t)q4 * b / C) * 4, hi = (int)((int64_t)q4 * (b + 1) / C) * 4;
    bool ok = true;
    for (int i = 4 * threadIdx.x; i < P.dim; i += 4 * nthreads) {
      float4 v = __ldcg(reinterpret_cast<const float4*>(T.h_in + i));
      // all ranks' words of these 4 elements in flight at once; re-read only
      // while some word still carries an older epoch
      unsigned long long w[TP_MAX_WORLD][4];
      for (uint32_t it = 0;; ++it) {
#pragma unroll
        for (int r = 0; r < TP_MAX_WORLD; ++r)
          if (r < T.world) {
            const unsigned long long* wp = img + (size_t)r * P.dim + i;
            ld_words2(wp, w[r][0], w[r][1]);
            ld_words2(wp + 2, w[r][2], w[r][3]);
          }
        bool ready = true;
#pragma unroll
        for (int r = 0; r < TP_MAX_WORLD; ++r)
          if (r < T.world)
#pragma unroll
            for (int c = 0; c < 4; ++c) ready = ready && (unsigned)(w[r][c] >> 32) == epoch;
        if (ready || !ok) break;
        if (it >= (1u << 22) || ((it & 255u) == 255u && *(volatile int*)P.err)) {
          atomicCAS(P.err, 0, XS_ERR_TP);  // the output is invalid; the kernel still runs to its end
          ok = false;
          break;
        }
        __nanosleep(32);
      }
#pragma unroll
      for (int r = 0; r < TP_MAX_WORLD; ++r)
        if (r < T.world) {  // rank order: every rank sums the same way
          v.x += __uint_as_float((unsigned)w[r][0]);
          v.y += __uint_as_float((unsigned)w[r][1]);
          v.z += __uint_as_float((unsigned)w[r][2]);
          v.w += __uint_as_float((unsigned)w[r][3]);
        }
      *reinterpret_cast<float4*>(xr + i) = v;
      if (i >= lo && i < hi) *reinterpret_cast<float4*>(T.h_out + i) = v;
    }
    xs_named_sync(1, nthreads);
  }
  // RMSNorm: the staged values are x * w and the kernel scales each output
  // row by 1 / rms at the end (the product is linear in x; each superblock's
  // power-of-two quantization scale absorbs the constant), so sum(x^2) is
  // gathered here, in the same pass, and reduced after the staging barrier
  constexpr bool NORM = XM == XS_X_NORM || XM == XS_X_REDUCE_NORM;
  float ss = 0.f;
  const float* nws = reinterpret_cast<const float*>(smem + L.nw);
  if constexpr (NORM) {
    // the norm weights were bulk-copied at kernel start (they do not depend on the previous kernel)
    uint64_t* aux = reinterpret_cast<uint64_t*>(smem + L.bar) + 2 * P.S;
    xs_bar_wait(aux, 0, P.err, XS_ERR_FULL);
  }
  const int total = XS_SPW * P.nk * 8;  // multiple of 64
  for (int base = (threadIdx.x & ~31); base < total; base += nthreads) {
    const int hu = base + lane;
    const int kb = hu >> 3, u = (hu >> 1) & 3, hf = hu & 1;
    const bool live = kb < P.sb;
    const float* xrow = P.x + (int64_t)kb * 256;
    float v[32];  // Q4: [0,16) sub-block 2u run, [16,32) sub-block 2u+1 run; Q6: group (g, w) at 8g + 4w
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int off;
      if constexpr (xs_legacy(QT)) off = 64 * u + 32 * hf + 4 * i;  // contiguous: blocks 4u + 2hf, +1
      else if constexpr (QT != GGUF_Q6_K) off = 64 * u + 16 * hf + (i < 4 ? 4 * i : 32 + 4 * (i - 4));
      else off = 128 * hf + 32 * (i >> 1) + 8 * u + 4 * (i & 1);
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (XM == XS_X_PLAIN) {
        if (live) f = ldg_f4(xrow + off);
      } else if constexpr (REDUCE) {
        const int64_t gi = (int64_t)kb * 256 + off;
        if (live && gi < P.dim) {
          f = *reinterpret_cast<const float4*>(xr + gi);
          if constexpr (XM == XS_X_REDUCE_NORM) {
            const float4 wv = *reinterpret_cast<const float4*>(nws + gi);
            ss = fmaf(f.x, f.x, fmaf(f.y, f.y, fmaf(f.z, f.z, fmaf(f.w, f.w, ss))));
            f.x *= wv.x;
            f.y *= wv.y;
            f.z *= wv.z;
            f.w *= wv.w;
          }
        }
      } else if constexpr (XM == XS_X_NORM) {
        const int64_t gi = (int64_t)kb * 256 + off;
        if (live && gi < P.dim) {
          f = ldg_f4(xrow + off);
          const float4 wv = *reinterpret_cast<const float4*>(nws + gi);
          ss = fmaf(f.x, f.x, fmaf(f.y, f.y, fmaf(f.z, f.z, fmaf(f.w, f.w, ss))));
          f.x *= wv.x;
          f.y *= wv.y;
          f.z *= wv.z;
          f.w *= wv.w;
        }
      } else {
        if (live) {
          const float4 g = ldg_f4(xrow + off), uu = ldg_f4(P.x2 + (int64_t)kb * 256 + off);
          f.x = swiglu_gate(g.x, P.act) * uu.x;
          f.y = swiglu_gate(g.y, P.act) * uu.y;
          f.z = swiglu_gate(g.z, P.act) * uu.z;
          f.w = swiglu_gate(g.w, P.act) * uu.w;  // fast exp: see swiglu_gate
        }
      }
      v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const XScale sc = xs_scale(amax);
    uint4* unit = xw + (size_t)(kb * 4 + u) * 8;
    const int sw = xs_swz(kb, u);
    if constexpr (xs_legacy(QT)) {
      // word 4 hf + j covers elements 8j .. 8j + 7 of this half-unit (block 4u + 2hf + j/2,
      // its half j % 2).  Legacy Q6_K: {hi, lo} of the scale group 8j..8j+3, then of 8j+4..;
      // legacy Q4_K: {hi, lo} of the even elements 8j, +2, +4, +6, then of the odd ones
      // (the low and high nibbles of the block's code bytes), and the half's exact sum.
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 o;
        const float* q = v + 8 * j;
        if constexpr (QT == LEGACY_Q6_K) {
          xs_pack4(q[0], q[1], q[2], q[3], sc.inv, o.x, o.y);
          xs_pack4(q[4], q[5], q[6], q[7], sc.inv, o.z, o.w);
        } else {
          xs_pack4(q[0], q[2], q[4], q[6], sc.inv, o.x, o.y);
          xs_pack4(q[1], q[3], q[5], q[7], sc.inv, o.z, o.w);
          float hs = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) hs += q[e];
          reinterpret_cast<float*>(smem + L.sums)[(size_t)(kb * 4 + u) * 8 + 4 * hf + j] = hs;
        }
        unit[(4 * hf + j) ^ sw] = o;
      }
    } else if constexpr (QT != GGUF_Q6_K) {
      // word 4 hf + j: {hi, lo} of A elements 4j.., then of B elements 4j..
      // (A: unit elements 0-31, B: 32-63; this half-unit holds 16 hf .. 16 hf + 15 of each)
      float sa = 0.f, sbb = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        sa += v[i];
        sbb += v[16 + i];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 o;
        xs_pack4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3], sc.inv, o.x, o.y);
        xs_pack4(v[16 + 4 * j], v[17 + 4 * j], v[18 + 4 * j], v[19 + 4 * j], sc.inv, o.z, o.w);
        unit[(4 * hf + j) ^ sw] = o;
      }
      if constexpr (xs_g16(QT)) {
        // a half-unit's A and B runs are whole 16-weight sub-blocks: 4u + hf and 4u + 2 + hf
        float* s4 = reinterpret_cast<float*>(smem + L.sums) + (size_t)(kb * 4 + u) * 4;
        s4[hf] = sa;
        s4[2 + hf] = sbb;
      } else {
        sa += __shfl_xor_sync(0xffffffffu, sa, 1);  // the unit's other half
        sbb += __shfl_xor_sync(0xffffffffu, sbb, 1);
        if (hf == 0) reinterpret_cast<float2*>(smem + L.sums)[kb * 4 + u] = make_float2(sa, sbb);
      }
    } else {
      // h = hf; word 4h + 2w + gp holds {hi, lo} of group (h, 2gp, w), then of (h, 2gp + 1, w)
      int shs[4], sls[4];
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        shs[g] = 0;
        sls[g] = 0;
      }
#pragma unroll
      for (int w = 0; w < 2; ++w)
#pragma unroll
        for (int gp = 0; gp < 2; ++gp) {
          uint4 o;
          const int g0 = 2 * gp, g1 = 2 * gp + 1;
          xs_pack4(v[8 * g0 + 4 * w], v[8 * g0 + 4 * w + 1], v[8 * g0 + 4 * w + 2], v[8 * g0 + 4 * w + 3], sc.inv,
                   o.x, o.y);
          xs_pack4(v[8 * g1 + 4 * w], v[8 * g1 + 4 * w + 1], v[8 * g1 + 4 * w + 2], v[8 * g1 + 4 * w + 3], sc.inv,
                   o.z, o.w);
          shs[g0] = __dp4a((int)o.x, 0x01010101, shs[g0]);
          sls[g0] = (int)__dp4a(o.y, 0x01010101u, (unsigned)sls[g0]);
          shs[g1] = __dp4a((int)o.z, 0x01010101, shs[g1]);
          sls[g1] = (int)__dp4a(o.w, 0x01010101u, (unsigned)sls[g1]);
          unit[(4 * hf + 2 * w + gp) ^ sw] = o;
        }
      int4* so = reinterpret_cast<int4*>(smem + L.sums) + (size_t)(kb * 4 + u) * 4 + 2 * hf;
      so[0] = make_int4(-32 * shs[0], -32 * shs[1], -32 * shs[2], -32 * shs[3]);
      so[1] = make_int4(-32 * sls[0], -32 * sls[1], -32 * sls[2], -32 * sls[3]);
    }
    if ((hu & 7) == 0) xsf[kb] = live ? sc.factor : 0.f;
  }
  if constexpr (NORM) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) reinterpret_cast<float*>(smem + L.red)[threadIdx.x >> 5] = ss;  // read after the staging barrier
  }
}

template <int QT, int XM, int YM>
__global__ void __launch_bounds__(32 * (XS_MAX_COMPUTE + 1), 1) xs_gemv_kernel(const XsParams P) {
  extern __shared__ __align__(128) uint8_t xs_smem[];
  pdl_trigger();  // the next kernel's CTAs may start on each SM as ours retire there
  const int C = gridDim.x, b = blockIdx.x;
  // XS_Y_SWIGLU: rows come in (gate, up) pairs that must stay in one CTA
  const int64_t r0 = YM == XS_Y_SWIGLU ? 2 * ((int64_t)(P.n / 2) * b / C) : (int64_t)P.n * b / C;
  const int64_t r1 = YM == XS_Y_SWIGLU ? 2 * ((int64_t)(P.n / 2) * (b + 1) / C) : (int64_t)P.n * (b + 1) / C;
  const int rows = (int)(r1 - r0);  // this CTA's rows r0 .. r1-1
  const int R = 2 * P.G;  // rows per stage: each compute warp takes two of them
  const int T = (rows + R - 1) / R;
  const int NC = P.nk * P.G;
  const XsSmem L(QT, P.nk, P.stage_bytes, P.S, P.rows_max, P.xr_floats, P.nw_floats);
  uint64_t* full = reinterpret_cast<uint64_t*>(xs_smem + L.bar);
  uint64_t* empty = full + P.S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.S; ++i) {
      xs_bar_init(&full[i], 1);
      xs_bar_init(&empty[i], NC);
    }
    xs_bar_init(empty + P.S, 1);  // aux: the norm weights
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == NC) {
    // ---------------- producer: the weights do not depend on the previous kernel ----------------
    if (lane == 0) {
      if constexpr (XM == XS_X_NORM || XM == XS_X_REDUCE_NORM) {
        const uint32_t nb = (uint32_t)(P.dim * 4);  // a multiple of 16 (dim % 4 == 0)
        xs_bar_expect(empty + P.S, nb);
        xs_bulk_g2s_plain(xs_smem + L.nw, P.nw, nb, empty + P.S);
      }
      uint64_t pol;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
      // the next weight is prefetched once the ring's first fill is issued
      const int fill = min(T, P.S);
      int t = 0;
      for (; t < T; ++t) {
        if (t == fill) xs_prefetch(P, b, C);
        const int st = t % P.S;
        if (t >= P.S && !xs_bar_wait(&empty[st], ((t / P.S) - 1) & 1, P.err, XS_ERR_EMPTY)) break;
        const int nr = min(R, rows - t * R);
        const int64_t row = r0 + (int64_t)t * R;
        uint8_t* dst = xs_smem + L.ring + (size_t)st * (size_t)P.stage_bytes;
        const uint32_t wb = (uint32_t)(nr * P.row_bytes), db = (uint32_t)(nr * P.d_row_bytes);
        xs_bar_expect(&full[st], wb + db);
        xs_bulk_g2s(dst, P.q + row * P.row_bytes, wb, &full[st], pol);
        if constexpr (QT == GGUF_Q6_K)
          xs_bulk_g2s(dst + (size_t)R * P.row_bytes, reinterpret_cast<const uint8_t*>(P.d) + row * P.d_row_bytes,
                      db, &full[st], pol);
      }
      if (t == fill && t == T) xs_prefetch(P, b, C);
      // the CTA must not retire while a copy into its shared memory is in flight
      for (int v = max(0, t - P.S); v < t; ++v) xs_bar_wait(&full[v % P.S], (v / P.S) & 1, P.err, XS_ERR_DRAIN);
      if constexpr (XM == XS_X_NORM || XM == XS_X_REDUCE_NORM) xs_bar_wait(empty + P.S, 0, P.err, XS_ERR_DRAIN);
    }
    return;
  }

  // ---------------- compute warps ----------------
  const int s = warp % P.nk, g = warp / P.nk;
  const int kb = XS_SPW * s + (lane >> 2), u = lane & 3;
  const bool live = kb < P.sb;
  pdl_wait();  // x may be the previous kernel's output
  xs_stage_x<QT, XM>(P, L, xs_smem, NC * 32);
  xs_named_sync(1, NC * 32);
  float yscale = 1.f;  // RMSNorm: 1 / sqrt(mean(x^2) + eps), applied to every output row
  if constexpr (XM == XS_X_NORM || XM == XS_X_REDUCE_NORM) {
    const float* red = reinterpret_cast<const float*>(xs_smem + L.red);
    float t = 0.f;
    for (int w = 0; w < NC; ++w) t += red[w];
    yscale = 1.f / sqrtf(t / (float)P.dim + P.eps);
  }

  // this lane's 64 activations, from the staged copy
  uint4 X[8];
  {
    const uint4* unit = reinterpret_cast<const uint4*>(xs_smem + L.xw) + (size_t)(kb * 4 + u) * 8;
    const int sw = xs_swz(kb, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) X[j] = unit[j ^ sw];
  }
  const float xf = reinterpret_cast<const float*>(xs_smem + L.xsf)[kb];
  float sa = 0.f, sbb = 0.f;   // Q4_K / Q5_K: exact sums of the sub-block 2u / 2u+1 activations
  float4 s16 = make_float4(0.f, 0.f, 0.f, 0.f);  // Q2_K / Q3_K: exact sums of sub-blocks 4u .. 4u+3
  int Sh[2][4], Sl[2][4];      // Q6_K: -32 * (sum of hi / lo bytes) of group (h, g)
  uint32_t sel_lo = 0, sel_hi = 0;  // Q6_K: PRMT selectors of this lane's scale bytes
  float lsum[8];               // legacy Q4_K: exact sums of the unit's eight block halves
  if constexpr (QT == GGUF_Q4_K || QT == GGUF_Q5_K) {
    const float2 t = reinterpret_cast<const float2*>(xs_smem + L.sums)[kb * 4 + u];
    sa = t.x;
    sbb = t.y;
  } else if constexpr (xs_g16(QT)) {
    s16 = reinterpret_cast<const float4*>(xs_smem + L.sums)[kb * 4 + u];
  } else if constexpr (xs_legacy(QT)) {
    if constexpr (QT == LEGACY_Q4_K) {
      const float4* t = reinterpret_cast<const float4*>(xs_smem + L.sums) + (size_t)(kb * 4 + u) * 2;
      const float4 a = t[0], b = t[1];
      lsum[0] = a.x; lsum[1] = a.y; lsum[2] = a.z; lsum[3] = a.w;
      lsum[4] = b.x; lsum[5] = b.y; lsum[6] = b.z; lsum[7] = b.w;
    }
  } else {
    const int4* si = reinterpret_cast<const int4*>(xs_smem + L.sums) + (size_t)(kb * 4 + u) * 4;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int4 a = si[2 * h], c = si[2 * h + 1];
      Sh[h][0] = a.x; Sh[h][1] = a.y; Sh[h][2] = a.z; Sh[h][3] = a.w;
      Sl[h][0] = c.x; Sl[h][1] = c.y; Sl[h][2] = c.z; Sl[h][3] = c.w;
    }
    // scale byte of group (h, g) = byte 8h + 2g + u/2: byte (u/2) of word 2h + g/2 for even g,
    // byte 2 + u/2 for odd g; sign-extended by PRMT (selector nibble | 8 replicates the sign)
    const uint32_t b0 = (uint32_t)(u >> 1), b2 = b0 + 2;
    sel_lo = b0 | ((b0 | 8) << 4) | ((b0 | 8) << 8) | ((b0 | 8) << 12);
    sel_hi = b2 | ((b2 | 8) << 4) | ((b2 | 8) << 8) | ((b2 | 8) << 12);
  }
  float* part = reinterpret_cast<float*>(xs_smem + L.part);
  const bool hi4 = u >= 2;  // Q4_K / Q5_K: sub-blocks 2u, 2u+1 take the packed high scale/min bits
  const int sh = 16 * (u & 1);
  // Q5_K: left rotations moving bit 2u / 2u+1 of every qh byte to bit 4;
  // Q3_K: moving bit 2u / 2u+1 of every hmask byte to bit 2
  const int r5a = (4 - 2 * u) & 31, r5b = (3 - 2 * u) & 31;
  const int r3a = (2 - 2 * u) & 31, r3b = (1 - 2 * u) & 31;
  const int sh2 = 4 * (u & 1);  // Q2_K / Q3_K: bit offset of the unit's 2-bit codes in its qs bytes

  // one row of this warp's slice: returns the lane's partial (0 for lanes past the row's end)
  auto row_partial = [&](const uint8_t* rowp, const uint8_t* drow) -> float {
    float v = 0.f;
    if (live) {
      if constexpr (QT == GGUF_Q4_K) {
        const uint8_t* blk = rowp + kb * Q4K_BYTES;
        const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * u);
        const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * u);
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint32_t W[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        // high nibbles are used in place (16 x the value, no shift per word);
        // the B sums are divided by 16 once, exactly
        int ahi = 0, alo = 0, bhi = 0, blo = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const uint32_t qa4 = W[w] & 0x0F0F0F0Fu, qb16 = W[w] & 0xF0F0F0F0u;
          ahi = dp4a_s(qa4, X[w].x, ahi);
          alo = dp4a_u(qa4, X[w].y, alo);
          bhi = dp4a_us(qb16, X[w].z, bhi);
          blo = dp4a_u(qb16, X[w].w, blo);
        }
        const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
        uint32_t scp, mp;
        if (!hi4) {
          scp = (s0 >> sh) & 0x3F3Fu;
          mp = (s1 >> sh) & 0x3F3Fu;
        } else {
          scp = ((s2 >> sh) & 0x0F0Fu) | ((s0 >> (sh + 2)) & 0x3030u);
          mp = ((s2 >> (sh + 4)) & 0x0F0Fu) | ((s1 >> (sh + 2)) & 0x3030u);
        }
        const int da = ahi * 256 + alo, db = (bhi * 256 + blo) >> 4;  // |.| < 2^23 (16 | bhi, blo)
        const int iv = (int)(scp & 0xffu) * da + (int)(scp >> 8) * db;  // |iv| < 2^30
        const float d = f16_bits_to_f32((uint16_t)(hdr.x & 0xffff));
        const float dmin = f16_bits_to_f32((uint16_t)(hdr.x >> 16));
        const float msum = fmaf((float)(mp & 0xffu), sa, (float)(mp >> 8) * sbb);
        v = fmaf(d * xf, (float)iv, -dmin * msum);
      } else if constexpr (QT == GGUF_Q5_K) {
        // d | dmin | 12 scale bytes (as Q4_K) | qh[32] | qs[128]; this lane's
        // qs bytes 32u .. 32u+31 hold sub-blocks 2u (low nibbles) and 2u+1
        // (high nibbles), whose fifth bits are bits 2u and 2u+1 of qh[0..31]
        const uint8_t* blk = rowp + kb * Q5K_BYTES;
        const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
        const uint4 h0 = *reinterpret_cast<const uint4*>(blk + 16);
        const uint4 h1 = *reinterpret_cast<const uint4*>(blk + 32);
        const uint4 qa = *reinterpret_cast<const uint4*>(blk + 48 + 32 * u);
        const uint4 qb = *reinterpret_cast<const uint4*>(blk + 64 + 32 * u);
        const uint32_t W[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const uint32_t H[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        int ahi = 0, alo = 0, bhi = 0, blo = 0;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const uint32_t qA = (W[w] & 0x0F0F0F0Fu) | (__funnelshift_l(H[w], H[w], r5a) & 0x10101010u);
          const uint32_t qB = ((W[w] >> 4) & 0x0F0F0F0Fu) | (__funnelshift_l(H[w], H[w], r5b) & 0x10101010u);
          ahi = dp4a_s(qA, X[w].x, ahi);
          alo = dp4a_u(qA, X[w].y, alo);
          bhi = dp4a_s(qB, X[w].z, bhi);
          blo = dp4a_u(qB, X[w].w, blo);
        }
        const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
        uint32_t scp, mp;
        if (!hi4) {
          scp = (s0 >> sh) & 0x3F3Fu;
          mp = (s1 >> sh) & 0x3F3Fu;
        } else {
          scp = ((s2 >> sh) & 0x0F0Fu) | ((s0 >> (sh + 2)) & 0x3030u);
          mp = ((s2 >> (sh + 4)) & 0x0F0Fu) | ((s1 >> (sh + 2)) & 0x3030u);
        }
        // |da|, |db| <= 32 * 31 * 2^14 < 2^24; |iv| <= 2 * 63 * 32 * 31 * 2^14 < 2^31
        const int da = ahi * 256 + alo, db = bhi * 256 + blo;
        const int iv = (int)(scp & 0xffu) * da + (int)(scp >> 8) * db;
        const float d = f16_bits_to_f32((uint16_t)(hdr.x & 0xffff));
        const float dmin = f16_bits_to_f32((uint16_t)(hdr.x >> 16));
        const float msum = fmaf((float)(mp & 0xffu), sa, (float)(mp >> 8) * sbb);
        v = fmaf(d * xf, (float)iv, -dmin * msum);
      } else if constexpr (QT == GGUF_Q3_K) {
        // device superblock (112 bytes): hmask[32] | qs[64] | scales[12] | d | 2 zero bytes.
        // This lane's elements: 2-bit codes at bits sh2 (A) / sh2 + 2 (B) of
        // qs bytes 32(u/2) .. + 31, third bits 2u / 2u+1 of hmask[0..31]; the
        // code q + 4 = lo | h << 2 is in [0, 7] and the -4 goes through the sums
        const uint8_t* blk = rowp + kb * Q3K_DEV;
        const uint4 m0 = *reinterpret_cast<const uint4*>(blk);
        const uint4 m1 = *reinterpret_cast<const uint4*>(blk + 16);
        const uint4 qa = *reinterpret_cast<const uint4*>(blk + 32 + 32 * (u >> 1));
        const uint4 qb = *reinterpret_cast<const uint4*>(blk + 48 + 32 * (u >> 1));
        const uint4 sd = *reinterpret_cast<const uint4*>(blk + 96);  // scales 0-11 | d
        const uint32_t W[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const uint32_t H[8] = {m0.x, m0.y, m0.z, m0.w, m1.x, m1.y, m1.z, m1.w};
        int gh[4] = {0, 0, 0, 0}, gl[4] = {0, 0, 0, 0};  // sub-blocks 4u .. 4u+3
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const uint32_t t = W[w] >> sh2;
          const uint32_t qA = (t & 0x03030303u) | (__funnelshift_l(H[w], H[w], r3a) & 0x04040404u);
          const uint32_t qB = ((t >> 2) & 0x03030303u) | (__funnelshift_l(H[w], H[w], r3b) & 0x04040404u);
          const int a = w >> 2, bb = 2 + (w >> 2);
          gh[a] = dp4a_s(qA, X[w].x, gh[a]);
          gl[a] = dp4a_u(qA, X[w].y, gl[a]);
          gh[bb] = dp4a_s(qB, X[w].z, gh[bb]);
          gl[bb] = dp4a_u(qB, X[w].w, gl[bb]);
        }
        // six-bit scale of sub-block 4u + i (byte i): low nibble of scale
        // byte 4u + i (u < 2) or high nibble of byte 4(u-2) + i, and bits 2u
        // of byte 8 + i on top; minus 32
        const uint32_t sc4 = (((u & 1) ? sd.y : sd.x) >> (4 * (u >> 1)) & 0x0F0F0F0Fu) |
                             (((sd.z >> (2 * u)) & 0x03030303u) << 4);
        const float S[4] = {s16.x, s16.y, s16.z, s16.w};
        int iv = 0;  // |.| <= 4 * 32 * 16 * 7 * 2^14 < 2^28
        float fs = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int sc = (int)((sc4 >> (8 * i)) & 63u) - 32;
          iv += sc * (gh[i] * 256 + gl[i]);
          fs = fmaf((float)sc, S[i], fs);
        }
        v = f16_bits_to_f32((uint16_t)(sd.w & 0xffff)) * fmaf(xf, (float)iv, -4.f * fs);
      } else if constexpr (QT == LEGACY_Q4_K) {
        // four 28-byte blocks (pesti-runner/src/tile_dequant.rs:238-290): d | delta,
        // the code nibbles of elements 0-7 and 8-15, h0 | h1; value = delta * h * (q - 4) + d.
        // Per block half: sum q x from the even / odd nibbles (exact int32), then
        // delta * h * (x-scale * that - 4 * sum x) + d * sum x
        const uint8_t* unitp = rowp + kb * (16 * 28) + u * 112;
#pragma unroll
        for (int bl = 0; bl < 4; ++bl) {
          const uint32_t* bw = reinterpret_cast<const uint32_t*>(unitp + 28 * bl);  // 4-byte aligned
          const uint32_t w0 = bw[0], hh = bw[3];
          const float d = f16_bits_to_f32((uint16_t)(w0 & 0xffff)), delta = f16_bits_to_f32((uint16_t)(w0 >> 16));
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            const uint32_t word = bw[1 + hb];
            const uint32_t ev = word & 0x0F0F0F0Fu, od = (word >> 4) & 0x0F0F0F0Fu;
            const uint4 xw = X[2 * bl + hb];
            const int hi = dp4a_us(od, xw.z, dp4a_us(ev, xw.x, 0));
            const int lo = dp4a_u(od, xw.w, dp4a_u(ev, xw.y, 0));
            const float hs = lsum[2 * bl + hb];
            const float t = delta * f16_bits_to_f32((uint16_t)(hb ? hh >> 16 : hh & 0xffff));
            v = fmaf(t, fmaf(xf, (float)(hi * 256 + lo), -4.f * hs), fmaf(d, hs, v));  // |hi*256+lo| < 2^21
          }
        }
      } else if constexpr (QT == LEGACY_Q6_K) {
        // four 42-byte blocks (tile_dequant.rs:347-374, 2-byte aligned): d, four f16 group
        // scales, 2-bit low codes (bytes 10-13), 2-bit flags (bytes 18-21); q = low + 4 *
        // (flag ? flag - 1 : 0) and value = d * (q - 32) * scale of its group of four.
        // Byte-parallel: word C_j holds position j of the four groups; a 4x4 byte
        // transpose gives each group's four codes, OR 0xE0 makes q - 32 a signed byte
        const uint16_t* unitp = reinterpret_cast<const uint16_t*>(rowp + kb * (16 * 42) + u * 168);
#pragma unroll
        for (int bl = 0; bl < 4; ++bl) {
          const uint16_t* h = unitp + 21 * bl;
          const float d = f16_bits_to_f32(h[0]);
          const uint32_t ql = (uint32_t)h[5] | ((uint32_t)h[6] << 16);
          const uint32_t fl = (uint32_t)h[9] | ((uint32_t)h[10] << 16);
          uint32_t C[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t lq = (ql >> (2 * j)) & 0x03030303u, f = (fl >> (2 * j)) & 0x03030303u;
            const uint32_t qh = f - ((f | (f >> 1)) & 0x01010101u);  // per byte: flag ? flag - 1 : 0
            C[j] = lq + (qh << 2);                                     // per byte <= 11: no carries
          }
          const uint32_t T0 = prmt(C[0], C[1], 0x5140u), T1 = prmt(C[0], C[1], 0x7362u);
          const uint32_t T2 = prmt(C[2], C[3], 0x5140u), T3 = prmt(C[2], C[3], 0x7362u);
          const uint32_t G[4] = {prmt(T0, T2, 0x5410u), prmt(T0, T2, 0x7632u), prmt(T1, T3, 0x5410u),
                                 prmt(T1, T3, 0x7632u)};
          float acc = 0.f;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint32_t sq = G[g] | 0xE0E0E0E0u;  // q - 32 as signed bytes
            const uint4 xw = X[2 * bl + (g >> 1)];
            const uint32_t xh = (g & 1) ? xw.z : xw.x, xl = (g & 1) ? xw.w : xw.y;
            const int D = dp4a_s(sq, xh, 0) * 256 + dp4a_su(sq, xl, 0);  // |.| < 2^21
            acc = fmaf(f16_bits_to_f32(h[1 + g]), (float)D, acc);
          }
          v = fmaf(d * xf, acc, v);
        }
      } else if constexpr (QT == GGUF_Q2_K) {
        // scales[16] | qs[64] | d | dmin at the 96-byte device stride (32-bit
        // loads).  Codes at bits sh2 (A) / sh2 + 2 (B) of qs bytes
        // 32(u/2) .. + 31; the B codes are used in place (4x) and their sums
        // divided by 4, exactly
        const uint32_t* blk = reinterpret_cast<const uint32_t*>(rowp + kb * Q2K_DEV);
        const uint32_t scw = blk[u];  // scale / min nibbles of sub-blocks 4u .. 4u+3
        const uint32_t dd = blk[20];  // d | dmin
        const uint32_t* qs = blk + 4 + 8 * (u >> 1);
        int gh[4] = {0, 0, 0, 0}, gl[4] = {0, 0, 0, 0};
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const uint32_t t = qs[w] >> sh2;
          const uint32_t qA = t & 0x03030303u, qB4 = t & 0x0C0C0C0Cu;
          const int a = w >> 2, bb = 2 + (w >> 2);
          gh[a] = dp4a_s(qA, X[w].x, gh[a]);
          gl[a] = dp4a_u(qA, X[w].y, gl[a]);
          gh[bb] = dp4a_s(qB4, X[w].z, gh[bb]);
          gl[bb] = dp4a_u(qB4, X[w].w, gl[bb]);
        }
        const float S[4] = {s16.x, s16.y, s16.z, s16.w};
        int iv = 0;  // |.| <= 4 * 15 * 16 * 3 * 2^14 < 2^26
        float msum = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int D = (gh[i] * 256 + gl[i]) >> (i >= 2 ? 2 : 0);
          iv += (int)((scw >> (8 * i)) & 15u) * D;
          msum = fmaf((float)((scw >> (8 * i + 4)) & 15u), S[i], msum);
        }
        const float d = f16_bits_to_f32((uint16_t)(dd & 0xffff)), dmin = f16_bits_to_f32((uint16_t)(dd >> 16));
        v = fmaf(d * xf, (float)iv, -dmin * msum);
      } else {
        const uint8_t* blk = rowp + kb * Q6K_BODY;
        const uint4 p0 = *reinterpret_cast<const uint4*>(blk + 48 * u);
        const uint4 p1 = *reinterpret_cast<const uint4*>(blk + 48 * u + 16);
        const uint4 p2 = *reinterpret_cast<const uint4*>(blk + 48 * u + 32);
        const uint4 scw = *reinterpret_cast<const uint4*>(blk + 192);
        const uint16_t dbits = reinterpret_cast<const uint16_t*>(drow)[kb];
        const uint32_t ql[2][2][2] = {{{p0.x, p0.y}, {p0.z, p0.w}}, {{p1.x, p1.y}, {p1.z, p1.w}}};
        const uint32_t qh[2][2] = {{p2.x, p2.y}, {p2.z, p2.w}};
        const uint32_t SCW[4] = {scw.x, scw.y, scw.z, scw.w};
        int ih = 0, il = 0;  // sum over groups of scale * (hi-limb / lo-limb products)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int hi[4], lo[4];
#pragma unroll
          for (int gg = 0; gg < 4; ++gg) {
            hi[gg] = Sh[h][gg];
            lo[gg] = Sl[h][gg];
          }
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            // six-bit quants: low nibble | two high bits << 4 (Hm: fields g0, g2; Hn: g1, g3)
            const uint32_t H = qh[h][w];
            const uint32_t Hm = H & 0x33333333u, Hn = (H >> 2) & 0x33333333u;
            const uint32_t A0 = ql[h][0][w], A1 = ql[h][1][w];
            const uint32_t q0 = (A0 & 0x0F0F0F0Fu) | ((Hm << 4) & 0xF0F0F0F0u);
            const uint32_t q1 = (A1 & 0x0F0F0F0Fu) | ((Hn << 4) & 0xF0F0F0F0u);
            const uint32_t q2 = ((A0 >> 4) & 0x0F0F0F0Fu) | (Hm & 0xF0F0F0F0u);
            const uint32_t q3 = ((A1 >> 4) & 0x0F0F0F0Fu) | (Hn & 0xF0F0F0F0u);
            const uint4 x01 = X[4 * h + 2 * w], x23 = X[4 * h + 2 * w + 1];
            hi[0] = dp4a_s(q0, x01.x, hi[0]);
            lo[0] = dp4a_u(q0, x01.y, lo[0]);
            hi[1] = dp4a_s(q1, x01.z, hi[1]);
            lo[1] = dp4a_u(q1, x01.w, lo[1]);
            hi[2] = dp4a_s(q2, x23.x, hi[2]);
            lo[2] = dp4a_u(q2, x23.y, lo[2]);
            hi[3] = dp4a_s(q3, x23.z, hi[3]);
            lo[3] = dp4a_u(q3, x23.w, lo[3]);
          }
#pragma unroll
          for (int gg = 0; gg < 4; ++gg) {
            // scale byte 8h + 2gg + u/2: word 2h + gg/2, byte 2(gg%2) + u/2
            const int scv = (int)prmt(SCW[2 * h + (gg >> 1)], 0u, (gg & 1) ? sel_hi : sel_lo);
            ih += scv * hi[gg];  // |.| < 2^24 in total
            il += scv * lo[gg];  // |.| < 2^26 in total
          }
        }
        v = fmaf(256.f, (float)ih, (float)il) * (f16_bits_to_f32(dbits) * xf);
      }
    }
    return v;
  };

  // each warp takes rows g and g + G of every stage
  for (int t = 0; t < T; ++t) {
    const int st = t % P.S;
    if (!__all_sync(0xffffffffu, xs_bar_wait(&full[st], (t / P.S) & 1, P.err, XS_ERR_FULL))) break;
    const uint8_t* stage = xs_smem + L.ring + (size_t)st * (size_t)P.stage_bytes;
    const uint8_t* dstage = stage + (size_t)R * P.row_bytes;
    const int q0 = t * R + g, q1 = q0 + P.G;  // local rows of this warp
    const float v0 = q0 < rows ? row_partial(stage + (size_t)g * P.row_bytes, dstage + (size_t)g * P.d_row_bytes) : 0.f;
    const float v1 = q1 < rows ? row_partial(stage + (size_t)(g + P.G) * P.row_bytes,
                                             dstage + (size_t)(g + P.G) * P.d_row_bytes)
                               : 0.f;
    // reduce both rows at once: lanes 0-15 end with row q0's sum, lanes 16-31 with q1's
    const bool upper = lane & 16;
    float keep = upper ? v1 : v0;
    keep += __shfl_xor_sync(0xffffffffu, upper ? v0 : v1, 16);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
    if (lane == 0 && q0 < rows) part[q0 * P.nk + s] = keep;
    if (lane == 16 && q1 < rows) part[q1 * P.nk + s] = keep;
    __syncwarp();
    if (lane == 0) xs_bar_arrive(&empty[st]);
  }
  xs_named_sync(1, NC * 32);
  if constexpr (YM == XS_Y_SWIGLU) {
    // rows (2j, 2j + 1) = (gate, up) of output j = r0 / 2 + j
    for (int j = threadIdx.x; 2 * j < rows; j += NC * 32) {
      float g = 0.f, u = 0.f;
      for (int t = 0; t < P.nk; ++t) {
        g += part[(2 * j) * P.nk + t];
        u += part[(2 * j + 1) * P.nk + t];
      }
      const int64_t row = r0 + 2 * j;
      g = fmaf(g, yscale, P.bias ? P.bias[row] : 0.f);
      u = fmaf(u, yscale, P.bias ? P.bias[row + 1] : 0.f);
      P.y[r0 / 2 + j] = swiglu_gate(g, P.act) * u;
    }
  } else if constexpr (YM == XS_Y_LOCAL) {
    for (int q = threadIdx.x; q < rows; q += NC * 32) {
      float acc = 0.f;
      for (int t = 0; t < P.nk; ++t) acc += part[q * P.nk + t];
      const int64_t row = r0 + q;
      P.y[row] = fmaf(acc, yscale, P.bias ? P.bias[row] : 0.f);
    }
  } else {
    // this exchange's epoch: one past the last; the last CTA to arrive
    // advances the counter, after every CTA has read it here
    const XsTp& T = P.tp;
    const unsigned epoch = *reinterpret_cast<volatile unsigned*>(T.epoch) + 1u;
    const unsigned long long tag = (unsigned long long)epoch << 32;
    const size_t at = (size_t)(epoch & 1u) * (size_t)T.slot_elems + (size_t)T.rank * P.n + r0;
    for (int q = threadIdx.x; q < rows; q += NC * 32) {
      float acc = 0.f;
      for (int t = 0; t < P.nk; ++t) acc += part[q * P.nk + t];
      const float v = acc + (P.bias ? P.bias[r0 + q] : 0.f);
      for (int p = 0; p < T.world; ++p) st_word(T.exch[p] + at + q, tag | __float_as_uint(v));  // over NVLink
    }
    xs_named_sync(1, NC * 32);
    if (threadIdx.x == 0 && atomicAdd(T.ctr, 1u) == gridDim.x - 1) {
      *T.ctr = 0u;
      *T.epoch = epoch;
    }
  }
}

struct XsLaunch {
  bool ok = false;
  int64_t xr_floats = 0, nw_floats = 0;
  int threads = 0, grid = 0, G = 0, S = 0, rows_max = 0;
  int64_t stage_bytes = 0;
  size_t smem = 0;
};

// Launch shape of the single-token kernel, or ok = false when it does not
// apply (more than XS_MAX_COMPUTE slices, or a ring of fewer than 2 stages).
XsLaunch xs_shape(int qt, int64_t n, int64_t sb, int num_sms, int64_t xr_floats = 0, int64_t nw_floats = 0) {
  XsLaunch r;
  r.xr_floats = xr_floats;
  r.nw_floats = nw_floats;
  const int nk = (int)((sb + XS_SPW - 1) / XS_SPW);
  if (n < 1 || nk < 1 || nk > XS_MAX_COMPUTE) return r;
  // the most row groups whose two-row-per-group stages stay within
  // XS_STAGE_MAX and still give a ring of two (only rows of KBs, the
  // reference's blocks, need fewer groups: bulk copies stream best at tens of KB)
  for (int G = XS_MAX_COMPUTE / nk; G >= 1; --G) {
    if (G > 1 && 2 * G * xs_row_bytes(qt, sb) > XS_STAGE_MAX) continue;
    r.G = G;
    r.threads = 32 * (nk * r.G + 1);
    r.grid = (int)std::min<int64_t>(n, num_sms);
    r.rows_max = (int)((n + r.grid - 1) / r.grid);
    const int64_t row_bytes = xs_row_bytes(qt, sb);
    const int64_t d_row_bytes = qt == GGUF_Q6_K ? q6k_d_ld(sb) * 2 : 0;
    r.stage_bytes = 2 * r.G * (row_bytes + d_row_bytes);  // 2G rows per stage
    const int T = (r.rows_max + 2 * r.G - 1) / (2 * r.G);
    const size_t fixed = XsSmem(qt, nk, r.stage_bytes, 0, r.rows_max, xr_floats, nw_floats).end + 64;
    if (fixed >= (size_t)XS_MAX_SMEM) continue;
    const int64_t fit = (int64_t)((XS_MAX_SMEM - fixed) / (size_t)(r.stage_bytes + 16));
    const int64_t want = std::max<int64_t>(2, (XS_INFLIGHT + r.stage_bytes / 2) / r.stage_bytes);
    const int S = (int)std::min<int64_t>(std::min<int64_t>(T, fit), want);
    if (S < std::min(T, 2)) continue;
    r.S = S;
    r.smem = XsSmem(qt, nk, r.stage_bytes, S, r.rows_max, xr_floats, nw_floats).end;
    r.ok = r.smem <= (size_t)XS_MAX_SMEM;
    if (r.ok) return r;
  }
  r.ok = false;
  return r;
}

template <int QT>
cudaError_t launch_xs(const DevWeight& w, const XsInput& in, const float* bias, float* y, int* err,
                      const Prefetch* pf, cudaStream_t s, const XsLaunch& sh) {
  XsParams P;
  P.q = w.q;
  P.d = w.d;
  P.row_bytes = xs_row_bytes(QT, w.sb);
  P.d_row_bytes = QT == GGUF_Q6_K ? (int)(w.d_ld * 2) : 0;
  P.n = (int)w.n;
  P.sb = (int)w.sb;
  P.nk = (int)((w.sb + XS_SPW - 1) / XS_SPW);
  P.G = sh.G;
  P.S = sh.S;
  P.rows_max = sh.rows_max;
  P.stage_bytes = sh.stage_bytes;
  P.x = in.x;
  P.bias = bias;
  P.y = y;
  P.err = err;
  P.x2 = in.x2;
  P.nw = in.nw;
  P.dim = in.dim;
  P.eps = in.eps;
  P.act = in.act;
  for (int r = 0; r < 2; ++r) {
    P.pf[r] = pf ? static_cast<const uint8_t*>(pf->p[r]) : nullptr;
    P.pf_bytes[r] = pf && pf->p[r] ? pf->bytes[r] : 0;
  }
  P.tp = in.tp;
  P.xr_floats = sh.xr_floats;
  P.nw_floats = sh.nw_floats;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sh.grid);
  cfg.blockDim = dim3((unsigned)sh.threads);
  cfg.dynamicSmemBytes = sh.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if constexpr (QT != GGUF_Q4_K && QT != GGUF_Q6_K) {  // the other types: plain linears only
    if (in.mode != XS_X_PLAIN || in.ymode != XS_Y_LOCAL) return cudaErrorNotSupported;
    return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_PLAIN, XS_Y_LOCAL>, P);
  } else {
  if (in.ymode == XS_Y_SWIGLU) {
    switch (in.mode) {
      case XS_X_PLAIN: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_PLAIN, XS_Y_SWIGLU>, P);
      case XS_X_NORM: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_NORM, XS_Y_SWIGLU>, P);
      case XS_X_REDUCE_NORM: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_REDUCE_NORM, XS_Y_SWIGLU>, P);
    }
    return cudaErrorInvalidValue;
  }
  if (in.ymode == XS_Y_PEERS) {
    switch (in.mode) {
      case XS_X_PLAIN: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_PLAIN, XS_Y_PEERS>, P);
      case XS_X_SWIGLU: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_SWIGLU, XS_Y_PEERS>, P);
    }
    return cudaErrorInvalidValue;
  }
  switch (in.mode) {
    case XS_X_PLAIN: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_PLAIN, XS_Y_LOCAL>, P);
    case XS_X_NORM: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_NORM, XS_Y_LOCAL>, P);
    case XS_X_SWIGLU: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_SWIGLU, XS_Y_LOCAL>, P);
    case XS_X_REDUCE: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_REDUCE, XS_Y_LOCAL>, P);
    case XS_X_REDUCE_NORM: return cudaLaunchKernelEx(&cfg, xs_gemv_kernel<QT, XS_X_REDUCE_NORM, XS_Y_LOCAL>, P);
  }
  return cudaErrorInvalidValue;
  }
}

}  // namespace

// ---- fixed scratch for the no-allocation entry ----------------------------------
// Some callers cannot allocate device memory on the call path: a serving
// engine that has handed all of HBM to weights and KV cache up front, or a
// loop whose latency budget cannot absorb cudaMalloc (which may synchronise
// the device and stall every stream).  For them the batched dp4a kernels can
// take their scratch (the prepared activations) from this file-scope array
// instead of the context's grow-on-demand buffer.  Nothing in it needs to
// start at zero: the prep kernel writes every byte the GEMV kernel reads.
// There is one array per device, shared by every context: calls that use it
// concurrently (different streams or contexts on one device without
// ordering between them) race on its contents.
static __device__ __align__(256) uint8_t g_dp4a_static_scratch[DP4A_STATIC_SCRATCH];

// The array's device address, looked up with the device current.  The lookup
// is repeated on every call (a host-side table read once the module is
// loaded): a cached address would dangle after cudaDeviceReset or a torn-down
// primary context, and the next kernel would write through it.  The first
// lookup on a device may load this file's module, which is why the first
// call on a device should come before any stream capture.
cudaError_t dp4a_static_scratch(void** ptr) {
  *ptr = nullptr;
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_dp4a_static_scratch);
  if (e != cudaSuccess) return e;
  *ptr = p;
  return cudaSuccess;
}

cudaError_t launch_gemv_dp4a_batched(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y,
                                     void* ws, int num_sms, cudaStream_t s, int* launches) {
  if (m < 1 || m > DP4A_MAX_M) return cudaErrorInvalidValue;
  if (w.type == GGUF_Q4_K) return launch_typed<GGUF_Q4_K>(w, x, m, bias, y, ws, num_sms, s, launches, Bracket());
  if (w.type == GGUF_Q6_K) return launch_typed<GGUF_Q6_K>(w, x, m, bias, y, ws, num_sms, s, launches, Bracket());
  return cudaErrorInvalidValue;
}

template <typename K>
static cudaError_t xs_attr(K kernel) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, XS_MAX_SMEM);
}

template <int QT>
static cudaError_t xs_attrs() {
  cudaError_t e = xs_attr(xs_gemv_kernel<QT, XS_X_PLAIN, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_NORM, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_SWIGLU, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_REDUCE, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_REDUCE_NORM, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_PLAIN, XS_Y_PEERS>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_SWIGLU, XS_Y_PEERS>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_PLAIN, XS_Y_SWIGLU>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_NORM, XS_Y_SWIGLU>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<QT, XS_X_REDUCE_NORM, XS_Y_SWIGLU>);
  return e;
}

cudaError_t dp4a_init_device() {
  cudaError_t e = xs_attrs<GGUF_Q4_K>();
  if (e == cudaSuccess) e = xs_attrs<GGUF_Q6_K>();
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<GGUF_Q2_K, XS_X_PLAIN, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<GGUF_Q3_K, XS_X_PLAIN, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<GGUF_Q5_K, XS_X_PLAIN, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<LEGACY_Q4_K, XS_X_PLAIN, XS_Y_LOCAL>);
  if (e == cudaSuccess) e = xs_attr(xs_gemv_kernel<LEGACY_Q6_K, XS_X_PLAIN, XS_Y_LOCAL>);
  return e;
}

cudaError_t launch_gemv_xs(const DevWeight& w, const XsInput& in, const float* bias, float* y, int num_sms, int* err,
                           const Prefetch* pf, cudaStream_t s, int* launches, Bracket br) {
  if (w.type != GGUF_Q4_K && w.type != GGUF_Q6_K && w.type != GGUF_Q2_K && w.type != GGUF_Q3_K &&
      w.type != GGUF_Q5_K && !xs_legacy(w.type))
    return cudaErrorNotSupported;
  if (in.mode < XS_X_PLAIN || in.mode > XS_X_REDUCE_NORM) return cudaErrorInvalidValue;
  // Q2_K / Q3_K / Q5_K and the legacy blocks: plain linears, rows laid out at
  // the stride the kernel streams (legacy: whole 256-weight spans, sb = k / 256)
  if (w.type != GGUF_Q4_K && w.type != GGUF_Q6_K) {
    if (in.mode != XS_X_PLAIN || in.ymode != XS_Y_LOCAL) return cudaErrorNotSupported;
    if (xs_legacy(w.type) && (w.sb < 1 || w.sb * 256 != w.k)) return cudaErrorNotSupported;
    if (w.row_bytes != xs_row_bytes(w.type, w.sb)) return cudaErrorInvalidValue;
  }
  const bool reduce = in.mode == XS_X_REDUCE || in.mode == XS_X_REDUCE_NORM;
  const bool norm = in.mode == XS_X_NORM || in.mode == XS_X_REDUCE_NORM;
  if (in.ymode == XS_Y_SWIGLU && (w.n & 1)) return cudaErrorInvalidValue;
  const int64_t vec = (int64_t)((in.dim + 3) & ~3);
  const XsLaunch sh = xs_shape(w.type, w.n, w.sb, num_sms, reduce ? vec : 0, norm ? vec : 0);
  if (!sh.ok) return cudaErrorNotSupported;
  bracket_record(br.start, s);
  cudaError_t e;
  switch (w.type) {
    case GGUF_Q4_K: e = launch_xs<GGUF_Q4_K>(w, in, bias, y, err, pf, s, sh); break;
    case GGUF_Q6_K: e = launch_xs<GGUF_Q6_K>(w, in, bias, y, err, pf, s, sh); break;
    case GGUF_Q5_K: e = launch_xs<GGUF_Q5_K>(w, in, bias, y, err, pf, s, sh); break;
    case GGUF_Q3_K: e = launch_xs<GGUF_Q3_K>(w, in, bias, y, err, pf, s, sh); break;
    case LEGACY_Q4_K: e = launch_xs<LEGACY_Q4_K>(w, in, bias, y, err, pf, s, sh); break;
    case LEGACY_Q6_K: e = launch_xs<LEGACY_Q6_K>(w, in, bias, y, err, pf, s, sh); break;
    default: e = launch_xs<GGUF_Q2_K>(w, in, bias, y, err, pf, s, sh); break;
  }
  if (e != cudaSuccess) return e;
  if (launches) ++*launches;
  bracket_record(br.stop, s);
  return cudaSuccess;
}

size_t dp4a_workspace_bytes(int type, int64_t m, int64_t sb) {
  if (type == GGUF_Q4_K) return dp4a_layout<GGUF_Q4_K>(m, sb).end;
  if (type == GGUF_Q6_K) return dp4a_layout<GGUF_Q6_K>(m, sb).end;
  return 0;
}

cudaError_t launch_gemv_dp4a(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y, void* ws,
                             int num_sms, int* err, cudaStream_t s, int* launches, Bracket br, const Prefetch* pf) {
  if (m < 1 || m > DP4A_MAX_M) return cudaErrorInvalidValue;
  if (m == 1) {
    XsInput in;
    in.x = x;
    const cudaError_t e = launch_gemv_xs(w, in, bias, y, num_sms, err, pf, s, launches, br);
    if (e != cudaErrorNotSupported) return e;
  }
  if (w.type == GGUF_Q4_K) return launch_typed<GGUF_Q4_K>(w, x, m, bias, y, ws, num_sms, s, launches, br);
  if (w.type == GGUF_Q6_K) return launch_typed<GGUF_Q6_K>(w, x, m, bias, y, ws, num_sms, s, launches, br);
  return cudaErrorInvalidValue;
}

}  // namespace kq
