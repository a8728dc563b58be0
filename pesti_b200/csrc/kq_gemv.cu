// kq_gemv.cu -- decode-shaped (m <= 32) K-quant linear: y[m][n] = x[m][k] . W[n][k].
//
// The weight stream is the only large input, so the kernel is built to read
// every superblock exactly once with 16-byte loads and to spend as few
// integer instructions per weight as possible (the integer pipe runs at half
// the rate of the FMA pipe and is what bounds a CUDA-core dequant-GEMV):
//
//  * Weights are unpacked in registers straight into f16 tensor-core
//    fragments.  The A operand is the exact integer sc*q (Q4_K, <= 945) or
//    sc*(q-32) (Q6_K), so the per-superblock factors d / dmin are the only
//    floating-point scales left; they are applied in f32 once per superblock.
//    Two nibbles become one f16x2 with one LOP3 (the bits 0x6400 make the
//    exact value 1024+q) and one HFMA2 removes the offset and applies sc.
//  * The activations are converted once per call (prep_kernel) into the
//    matching B fragments: per (token, superblock) a power-of-two scale keeps
//    them in f16 range, and each value is split into f16 hi + lo parts so the
//    product keeps ~22 significant bits.  For m <= 8 the hi and lo parts sit in
//    the 8 columns of one n8 tile (4 tokens x 2), so m <= 4 costs one MMA per
//    16 weights per row; for m > 8 only the hi part is used.
//  * A warp owns a 16-row tile and a stride of superblocks; the 8 warps of a
//    CTA split K, the next superblock's weights are loaded before the current
//    one is computed, and partial sums are combined in shared memory.
//  * The main kernel is launched as a programmatic dependent of prep_kernel:
//    it starts streaming weights while the activation prep finishes.
//
// Reference semantics: QuantizedLinear::forward (pesti-runner/src/
// quantized_linear.rs:101-143), y = x . W^T (+ bias), computed there after a
// full f32 dequantization.
#include "kq_common.cuh"
#include "kq_kernels.h"

namespace kq {

namespace {

constexpr int KSPLIT_WARPS = 8;  // warps per CTA, splitting K

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;");
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// First of the 4 consecutive weights (k = e, e+1, e+2, e+3) that lane slot c
// feeds to MMA step s of a superblock.  In every step the slot's four
// weights enter the MMA as k-columns (2c, 2c+8, 2c+1, 2c+9) <- (e, e+1, e+2, e+3).
//  Q4_K: slot c owns chunk c (qs[32c..32c+31]); step s takes qs word s>>1,
//        low nibbles (s even, sub-block 2c) or high nibbles (sub-block 2c+1).
//  Q6_K: slot c owns l in [8c, 8c+8) of every 32-group; step s reads ql piece
//        p = s>>2 (half h = p>>1, group pair gg = p&1), word (s>>1)&1, low
//        nibbles (group g = gg) or high nibbles (g = gg+2).
template <int QT>
__host__ __device__ __forceinline__ int step_elem(int s, int c) {
  if (QT == GGUF_Q4_K) {
    return 64 * c + 32 * (s & 1) + 4 * (s >> 1);
  } else {
    const int p = s >> 2, h = p >> 1, gg = p & 1;
    const int w = (s >> 1) & 1, g = gg + 2 * (s & 1);
    return 128 * h + 32 * g + 8 * c + 4 * w;
  }
}

// ---- per-call activation prep ---------------------------------------------
// Tokens per n8 tile: 4 with hi/lo split (columns 0-3 hi, 4-7 lo), else 8.
// bf[((nt*sb + kb)*8 + s/2)*32 + lane] = {b0(s), b1(s), b0(s+1), b1(s+1)}
// for the lane's column g = lane>>2 and slot c = lane&3.
// scl[kb*32 + t] = 2^e, the power of two token t's superblock kb was divided by.
template <int QT, bool HILO>
__global__ void __launch_bounds__(256) prep_kernel(const float* __restrict__ x, int m, int64_t k,
                                                   int ntiles, uint4* __restrict__ bf,
                                                   float* __restrict__ scl) {
  pdl_launch_dependents();
  const int sb = (int)(k / QK);
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wid >= (int64_t)ntiles * sb) return;
  const int nt = (int)(wid / sb), kb = (int)(wid - (int64_t)nt * sb);
  constexpr int TPT = HILO ? 4 : 8;
  const int t = nt * TPT + (HILO ? (g & 3) : g);
  const bool lo = HILO && g >= 4;
  const bool live = t < m;
  float4 v[16];
  float amax = 0.f;
  const float* xr = x + (int64_t)(live ? t : 0) * k + (int64_t)kb * QK;
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    v[s] = live ? ldg_f4(xr + step_elem<QT>(s, c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[s].x), fabsf(v[s].y)), fmaxf(fabsf(v[s].z), fabsf(v[s].w))));
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  // power of two 2^e with amax / 2^e in [2^13, 2^14): no f16 overflow, and
  // small activations are scaled up instead of becoming f16 subnormals
  int e = 0;
  if (amax > 0.f && isfinite(amax)) e = ((__float_as_uint(amax) >> 23) & 0xff) - 127 - 13;
  e = max(-120, min(120, e));
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e
  uint4* dst = bf + ((int64_t)(nt * sb + kb) * 8) * 32 + lane;
#pragma unroll
  for (int s2 = 0; s2 < 8; ++s2) {
    uint32_t r[4];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float4 a = v[2 * s2 + u];
      const float a0 = a.x * inv, a1 = a.y * inv, a2 = a.z * inv, a3 = a.w * inv;
      __half2 p02 = __floats2half2_rn(a0, a2), p13 = __floats2half2_rn(a1, a3);
      if (lo) {
        p02 = __floats2half2_rn(a0 - __low2float(p02), a2 - __high2float(p02));
        p13 = __floats2half2_rn(a1 - __low2float(p13), a3 - __high2float(p13));
      }
      r[2 * u] = h2_bits(p02);
      r[2 * u + 1] = h2_bits(p13);
    }
    dst[s2 * 32] = make_uint4(r[0], r[1], r[2], r[3]);
  }
  if (live && c == 0 && !lo) scl[(int64_t)kb * 32 + t] = __uint_as_float((uint32_t)(127 + e) << 23);
}

// ---- weights --------------------------------------------------------------
struct RawQ4 {
  uint4 hdr;     // d | dmin | scales[12]
  uint4 q0, q1;  // qs[32c .. 32c+31]
};
struct RawQ6 {
  uint4 p01, p23, p45;  // the slot's 48 body bytes: ql pieces 0-3, qh pieces 4-5
  uint4 sc;             // int8 scales[16]
  uint32_t d;
};

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

// ---- shared-memory staging of the weight stream ------------------------------
// Each warp keeps a ring of STAGES slots; a slot holds what the warp needs of
// one superblock of its 16 rows.  Every lane copies (cp.async) exactly the
// bytes it will read itself, plus one row's header/scales for the whole warp,
// so a slot is ready once every lane has passed cp.async.wait_group and the
// warp has synchronised.  Per-lane areas are padded to an odd number of
// 16-byte units so the 8 lanes of a quarter-warp hit distinct banks.
//  Q4_K slot: lane area [32][80]  = row a qs[32c..+32] | row b qs[32c..+32] | pad
//             header area [16 rows][16] (d, dmin, scales)           -> 2816 B
//  Q6_K slot: lane area [32][112] = row a slot bytes(48) | row b (48) |
//             d pair of row a (4) | d pair of row b (4) | pad
//             scale area [16 rows][16]                              -> 3840 B
template <int QT>
struct Stage;
template <>
struct Stage<GGUF_Q4_K> {
  static constexpr int LANE = 80, HDR = 32 * 80, BYTES = HDR + 16 * 16;
};
template <>
struct Stage<GGUF_Q6_K> {
  static constexpr int LANE = 112, HDR = 32 * 112, BYTES = HDR + 16 * 16;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copy superblock kb of rows ra (= tile row g) and rb (= g + 8) into `slot`.
template <int QT>
__device__ __forceinline__ void stage_issue(uint8_t* slot, const uint8_t* __restrict__ wq,
                                            const uint16_t* __restrict__ wd, int64_t n, int64_t ra,
                                            int64_t rb, int sb, int kb, int g, int c, int lane) {
  using S = Stage<QT>;
  const size_t ga = (size_t)ra * sb + kb, gb = (size_t)rb * sb + kb;
  uint8_t* la = slot + lane * S::LANE;
  if constexpr (QT == GGUF_Q4_K) {
    const uint8_t* A = wq + ga * Q4K_BYTES;
    const uint8_t* B = wq + gb * Q4K_BYTES;
    cp_async16(la, A + 16 + 32 * c);
    cp_async16(la + 16, A + 32 + 32 * c);
    cp_async16(la + 32, B + 16 + 32 * c);
    cp_async16(la + 48, B + 32 + 32 * c);
    if (c == 0) cp_async16(slot + S::HDR + 16 * g, A);
    if (c == 1) cp_async16(slot + S::HDR + 16 * (g + 8), B);
  } else {
    const uint8_t* A = wq + ga * Q6K_BODY;
    const uint8_t* B = wq + gb * Q6K_BODY;
    cp_async16(la, A + 48 * c);
    cp_async16(la + 16, A + 48 * c + 16);
    cp_async16(la + 32, A + 48 * c + 32);
    cp_async16(la + 48, B + 48 * c);
    cp_async16(la + 64, B + 48 * c + 16);
    cp_async16(la + 80, B + 48 * c + 32);
    // d is row-major [n][d_ld]: copy the aligned pair holding d(row, kb)
    const size_t dld = (size_t)q6k_d_ld(sb);
    cp_async4(la + 96, wd + (size_t)ra * dld + (size_t)(kb & ~1));
    cp_async4(la + 100, wd + (size_t)rb * dld + (size_t)(kb & ~1));
    if (c == 0) cp_async16(slot + S::HDR + 16 * g, A + 192);
    if (c == 1) cp_async16(slot + S::HDR + 16 * (g + 8), B + 192);
  }
}

template <int QT>
__device__ __forceinline__ void stage_read(const uint8_t* slot, int kb,
                                           int g, int lane, typename RawT<QT>::type& a,
                                           typename RawT<QT>::type& b) {
  using S = Stage<QT>;
  const uint8_t* la = slot + lane * S::LANE;
  const uint4* l4 = reinterpret_cast<const uint4*>(la);
  if constexpr (QT == GGUF_Q4_K) {
    a.q0 = l4[0];
    a.q1 = l4[1];
    b.q0 = l4[2];
    b.q1 = l4[3];
    a.hdr = *reinterpret_cast<const uint4*>(slot + S::HDR + 16 * g);
    b.hdr = *reinterpret_cast<const uint4*>(slot + S::HDR + 16 * (g + 8));
  } else {
    a.p01 = l4[0];
    a.p23 = l4[1];
    a.p45 = l4[2];
    b.p01 = l4[3];
    b.p23 = l4[4];
    b.p45 = l4[5];
    const uint2 dd = *reinterpret_cast<const uint2*>(la + 96);
    a.d = (kb & 1) ? (dd.x >> 16) : (dd.x & 0xffff);
    b.d = (kb & 1) ? (dd.y >> 16) : (dd.y & 0xffff);
    a.sc = *reinterpret_cast<const uint4*>(slot + S::HDR + 16 * g);
    b.sc = *reinterpret_cast<const uint4*>(slot + S::HDR + 16 * (g + 8));
  }
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// (v, v) as f16x2 for the byte v (0..255) held in byte `b` of w, without an
// int->half conversion: the bits 0x64 | v make 1024 + v exactly.
__device__ __forceinline__ __half2 byte_h2(uint32_t w, int b) {
  const uint32_t sel = (uint32_t)b | 0x0070u | ((uint32_t)b << 8) | 0x7000u;  // v,0x64,v,0x64
  return __hsub2(bits_h2(prmt(w, 0x64646464u, sel)), __float2half2_rn(1024.f));
}

// Per-row constants for one superblock.
struct RowQ4 {
  __half2 mul[2], add[2];  // step lohi 0 / 1: A = t*mul + add = sc*q
  __half2 mmin[2];         // (m, m) of sub-blocks 2c, 2c+1
  float d, dmin;
};
struct RowQ6 {
  __half2 sc[8], off[8];  // (sc, sc), (-288sc, -288sc) per scale group, index 2*piece + lohi
  float d;
};

__device__ __forceinline__ RowQ4 row_q4(const RawQ4& r, int c) {
  RowQ4 o;
  o.d = f16_bits_to_f32((uint16_t)(r.hdr.x & 0xffff));
  o.dmin = f16_bits_to_f32((uint16_t)(r.hdr.x >> 16));
  int sca, ma, scb, mb;
  q4k_scale_min_w(r.hdr.y, r.hdr.z, r.hdr.w, 2 * c, sca, ma);
  q4k_scale_min_w(r.hdr.y, r.hdr.z, r.hdr.w, 2 * c + 1, scb, mb);
  const uint32_t packed = (uint32_t)sca | ((uint32_t)scb << 8) | ((uint32_t)ma << 16) | ((uint32_t)mb << 24);
  const __half2 sa = byte_h2(packed, 0), sb = byte_h2(packed, 1);
  // low nibbles: (1024+q)*sc - 1024*sc; high nibbles hold 16q: (1024+16q)*(sc/16) - 64*sc
  o.mul[0] = sa;
  o.add[0] = __hmul2(sa, __float2half2_rn(-1024.f));
  o.mul[1] = __hmul2(sb, __float2half2_rn(0.0625f));
  o.add[1] = __hmul2(sb, __float2half2_rn(-64.f));
  o.mmin[0] = byte_h2(packed, 2);
  o.mmin[1] = byte_h2(packed, 3);
  return o;
}

__device__ __forceinline__ RowQ6 row_q6(const RawQ6& r, int c) {
  RowQ6 o;
  o.d = f16_bits_to_f32((uint16_t)r.d);
  // int8 scales: flip the sign bit to get s + 128 in 0..255, convert, subtract 128
  const __half2 k128 = __float2half2_rn(128.f), km288 = __float2half2_rn(-288.f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // i = 2*piece + lohi: piece p = i>>1 (half h = p>>1), group g = (p&1) + 2*lohi
    const int p = i >> 1, h = p >> 1, g = (p & 1) + 2 * (i & 1);
    const int si = 8 * h + 2 * g + (c >> 1);
    const __half2 v = __hsub2(byte_h2(word_of(r.sc, si >> 2) ^ 0x80808080u, si & 3), k128);
    o.sc[i] = v;
    o.off[i] = __hmul2(v, km288);
  }
  return o;
}

// A fragment halves for one row, step s: (k 2c,2c+1) <- (e, e+2), (k 2c+8,2c+9) <- (e+1, e+3).
__device__ __forceinline__ void a_q4(const RawQ4& r, const RowQ4& k, int s, uint32_t& lo02,
                                     uint32_t& lo13) {
  const int w = s >> 1, lohi = s & 1;
  const uint32_t W = word_of(w < 4 ? r.q0 : r.q1, w & 3);
  const uint32_t mask = lohi ? 0x00F000F0u : 0x000F000Fu;
  const uint32_t t02 = (W & mask) | 0x64006400u;
  const uint32_t t13 = ((W >> 8) & mask) | 0x64006400u;
  lo02 = h2_bits(__hfma2(bits_h2(t02), k.mul[lohi], k.add[lohi]));
  lo13 = h2_bits(__hfma2(bits_h2(t13), k.mul[lohi], k.add[lohi]));
}

// Q6_K: the four 6-bit codes of the step are first assembled as bytes 4q
// (nibble in bits 2-5, high pair in bits 6-7, one LOP3), then PRMT pairs them
// with 0x5C into f16 lanes of value 256 + q, and one HFMA2 gives (q-32)*sc.
__device__ __forceinline__ void a_q6(const RawQ6& r, const RowQ6& k, int s, uint32_t& lo02,
                                     uint32_t& lo13) {
  const int p = s >> 2, h = p >> 1, gg = p & 1, w = (s >> 1) & 1, lohi = s & 1;
  const uint32_t W = word_of(p < 2 ? r.p01 : r.p23, 2 * (p & 1) + w);
  const uint32_t H = word_of(r.p45, 2 * h + w);
  const uint32_t hm = (H >> (2 * gg)) & 0x33333333u;  // bits 0-1: group gg, 4-5: gg+2
  const uint32_t a = lohi ? (W >> 2) : (W << 2);     // nibble -> bits 2-5
  const uint32_t b = lohi ? (hm << 2) : (hm << 6);   // its high pair -> bits 6-7
  const uint32_t q4 = (a & 0x3C3C3C3Cu) | (b & 0xC3C3C3C3u);
  const int i = 2 * p + lohi;
  lo02 = h2_bits(__hfma2(bits_h2(prmt(q4, 0x5C5C5C5Cu, 0x7250u)), k.sc[i], k.off[i]));
  lo13 = h2_bits(__hfma2(bits_h2(prmt(q4, 0x5C5C5C5Cu, 0x7351u)), k.sc[i], k.off[i]));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Superblocks each warp keeps in flight in its ring.  With B staging (m <= 4)
// a slot also carries the superblock's activation fragments of the live
// columns and the per-token scales, so fewer slots fit.
template <int QT>
__host__ __device__ constexpr int stages() {
  return QT == GGUF_Q4_K ? 4 : 3;
}
constexpr int STAGES_WITH_B = 2;

// Slot layout with B staging: weights | scl[4] (16 B) | B of the 8m live
// lanes, 128 B each (8 uint4, one per step pair).
__host__ __device__ inline int slot_bytes(int qt, bool stageb, int m) {
  const int w = qt == GGUF_Q4_K ? Stage<GGUF_Q4_K>::BYTES : Stage<GGUF_Q6_K>::BYTES;
  return stageb ? w + 16 + 1024 * m : w;
}

// Copies of the activation side of superblock kb into a slot (B staging).
__device__ __forceinline__ void stage_issue_b(uint8_t* sx, const uint4* __restrict__ bf,
                                              const float* __restrict__ scl, int kb, int m, int g,
                                              int c, int lane) {
  if ((g & 3) < m) {
    const int compact = ((g >> 2) * m + (g & 3)) * 4 + c;
    const uint4* src = bf + (size_t)kb * 8 * 32 + lane;
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2) cp_async16(sx + 16 + compact * 128 + 16 * s2, src + s2 * 32);
  }
  if (lane == 0) cp_async16(sx, scl + (size_t)kb * 32);
}

// One CTA = one 16-row tile; warp w takes superblocks w, w+8, ...
// Lane (g = lane>>2, c = lane&3) feeds rows g and g+8 and holds C columns 2c, 2c+1.
template <int QT, int NT, bool HILO, int ST, bool STAGEB>
__global__ void __launch_bounds__(32 * KSPLIT_WARPS)
    gemv_kernel(const uint8_t* __restrict__ wq, const uint16_t* __restrict__ wd, int64_t n, int sb,
                int m, const uint4* __restrict__ bf, const float* __restrict__ scl,
                const float* __restrict__ bias, float* __restrict__ y, int slot) {
  static_assert(!STAGEB || (NT == 1 && HILO), "B staging is for the m <= 4 tile");
  using Raw = typename RawT<QT>::type;
  constexpr int TPT = HILO ? 4 : 8;
  __shared__ float red[KSPLIT_WARPS][NT][4][32];
  __shared__ uint4 zeros[8];  // B fragments of columns without a token
  extern __shared__ __align__(16) uint8_t ring[];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x < 8) zeros[threadIdx.x] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  const int g = lane >> 2, c = lane & 3;
  const int64_t r0 = (int64_t)blockIdx.x * 16;
  const int64_t ra = min(r0 + g, n - 1), rb = min(r0 + g + 8, n - 1);
  uint8_t* wring = ring + warp * ST * slot;

  float tot[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) tot[i][0] = tot[i][1] = tot[i][2] = tot[i][3] = 0.f;

  // prologue: the weights of the first ST-1 superblocks of this warp.  The
  // activation side may only be read after the prep kernel has finished.
#pragma unroll
  for (int j = 0; j < ST - 1; ++j) {
    const int kj = warp + j * KSPLIT_WARPS;
    if (kj < sb) stage_issue<QT>(wring + j * slot, wq, wd, n, ra, rb, sb, kj, g, c, lane);
    if (!STAGEB) cp_async_commit();
  }
  pdl_wait();  // activation fragments are written by the preceding prep kernel
  if (STAGEB) {
#pragma unroll
    for (int j = 0; j < ST - 1; ++j) {
      const int kj = warp + j * KSPLIT_WARPS;
      if (kj < sb) stage_issue_b(wring + j * slot + Stage<QT>::BYTES, bf, scl, kj, m, g, c, lane);
      cp_async_commit();
    }
  }

  // which of this lane's B columns carry a token (skip loads of empty columns)
  bool bcol[NT];
#pragma unroll
  for (int i = 0; i < NT; ++i) bcol[i] = i * TPT + (HILO ? (g & 3) : g) < m;
  const int compact = ((g >> 2) * m + (g & 3)) * 4 + c;

  int it = 0;
  for (int kb = warp; kb < sb; kb += KSPLIT_WARPS, ++it) {
    {
      const int kn = kb + (ST - 1) * KSPLIT_WARPS;
      if (kn < sb) {
        uint8_t* sl = wring + ((it + ST - 1) % ST) * slot;
        stage_issue<QT>(sl, wq, wd, n, ra, rb, sb, kn, g, c, lane);
        if (STAGEB) stage_issue_b(sl + Stage<QT>::BYTES, bf, scl, kn, m, g, c, lane);
      }
      cp_async_commit();
    }
    cp_async_wait<ST - 1>();
    __syncwarp();
    const uint8_t* cur = wring + (it % ST) * slot;
    Raw ca, cb;
    stage_read<QT>(cur, kb, g, lane, ca, cb);
    // B fragments of this superblock, from the slot or (m > 4) from L2
    const uint4* bs = bcol[0] ? reinterpret_cast<const uint4*>(cur + Stage<QT>::BYTES + 16 +
                                                               compact * 128)
                              : zeros;
    auto bload = [&](int i, int s2) -> uint4 {
      if constexpr (STAGEB)
        return bs[s2];
      else
        return bcol[i] ? __ldg(bf + ((int64_t)(i * sb + kb) * 8 + s2) * 32 + lane)
                       : make_uint4(0, 0, 0, 0);
    };
    auto sload = [&](int t) -> float {
      if constexpr (STAGEB)
        return reinterpret_cast<const float*>(cur + Stage<QT>::BYTES)[t];
      else
        return __ldg(scl + (int64_t)kb * 32 + t);
    };
    float acc[NT][4], amin[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = amin[i][j] = 0.f;

    float da, db, dma = 0.f, dmb = 0.f;
    if constexpr (QT == GGUF_Q4_K) {
      const RowQ4 ka = row_q4(ca, c), kb4 = row_q4(cb, c);
      da = ka.d;
      db = kb4.d;
      dma = ka.dmin;
      dmb = kb4.dmin;
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        uint4 bv[NT];
#pragma unroll
        for (int i = 0; i < NT; ++i) bv[i] = bload(i, s2);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int s = 2 * s2 + u;
          uint32_t a0, a2, a1, a3;
          a_q4(ca, ka, s, a0, a2);
          a_q4(cb, kb4, s, a1, a3);
          const uint32_t m0 = h2_bits(ka.mmin[u]), m1 = h2_bits(kb4.mmin[u]);
#pragma unroll
          for (int i = 0; i < NT; ++i) {
            const uint32_t b0 = u ? bv[i].z : bv[i].x, b1 = u ? bv[i].w : bv[i].y;
            mma16816(acc[i], a0, a1, a2, a3, b0, b1);
            mma16816(amin[i], m0, m1, m0, m1, b0, b1);
          }
        }
      }
    } else {
      const RowQ6 ka = row_q6(ca, c), kb6 = row_q6(cb, c);
      da = ka.d;
      db = kb6.d;
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        uint4 bv[NT];
#pragma unroll
        for (int i = 0; i < NT; ++i) bv[i] = bload(i, s2);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int s = 2 * s2 + u;
          uint32_t a0, a2, a1, a3;
          a_q6(ca, ka, s, a0, a2);
          a_q6(cb, kb6, s, a1, a3);
#pragma unroll
          for (int i = 0; i < NT; ++i) {
            const uint32_t b0 = u ? bv[i].z : bv[i].x, b1 = u ? bv[i].w : bv[i].y;
            mma16816(acc[i], a0, a1, a2, a3, b0, b1);
          }
        }
      }
    }
    // scale this superblock's partial sums: d per row, 2^e per token column
#pragma unroll
    for (int i = 0; i < NT; ++i) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int col = 2 * c + j;
        const int t = i * TPT + (HILO ? (col & 3) : col);
        const float sc = t < m ? sload(t) : 0.f;
        tot[i][j] += (da * sc) * acc[i][j];
        tot[i][2 + j] += (db * sc) * acc[i][2 + j];
        if constexpr (QT == GGUF_Q4_K) {
          tot[i][j] -= (dma * sc) * amin[i][j];
          tot[i][2 + j] -= (dmb * sc) * amin[i][2 + j];
        }
      }
    }
    __syncwarp();  // every lane is done with this slot before it is refilled
  }
  cp_async_wait<0>();  // nothing may be left in flight into the ring at exit

  // combine the K-split warps in a fixed order
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) red[warp][i][j][lane] = tot[i][j];
  __syncthreads();
  if (warp != 0) return;
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v = red[0][i][j][lane];
#pragma unroll
      for (int w = 1; w < KSPLIT_WARPS; ++w) v += red[w][i][j][lane];
      tot[i][j] = v;
    }
  const int64_t rowa = r0 + g, rowb = r0 + g + 8;
  const float ba = (bias && rowa < n) ? bias[rowa] : 0.f;
  const float bb = (bias && rowb < n) ? bias[rowb] : 0.f;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    if constexpr (HILO) {
      // columns 4..7 (lanes with c >= 2) hold the lo parts of tokens 0..3
#pragma unroll
      for (int j = 0; j < 4; ++j) tot[i][j] += __shfl_xor_sync(0xffffffffu, tot[i][j], 2);
      if (c >= 2) continue;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int t = i * TPT + 2 * c + j;
      if (t < m) {
        if (rowa < n) y[(int64_t)t * n + rowa] = tot[i][j] + ba;
        if (rowb < n) y[(int64_t)t * n + rowb] = tot[i][2 + j] + bb;
      }
    }
  }
}

int tiles_for(int m, bool& hilo) {
  hilo = m <= 8;
  return hilo ? (m + 3) / 4 : (m + 7) / 8;
}

template <int QT, int NT, bool HILO, int ST, bool STAGEB>
cudaError_t launch_main(const DevWeight& w, int m, const uint4* bf, const float* scl,
                        const float* bias, float* y, cudaStream_t s) {
  const int slot = slot_bytes(QT, STAGEB, m);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((w.n + 15) / 16));
  cfg.blockDim = dim3(32 * KSPLIT_WARPS);
  cfg.dynamicSmemBytes = (size_t)KSPLIT_WARPS * ST * slot;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<QT, NT, HILO, ST, STAGEB>, w.q, w.d, w.n, (int)w.sb,
                            m, bf, scl, bias, y, slot);
}

template <int QT>
cudaError_t launch_typed(const DevWeight& w, const float* x, int64_t m64, const float* bias,
                         float* y, void* ws, cudaStream_t s, int* launches, Bracket br) {
  const int sb = (int)w.sb;
  for (int64_t m0 = 0; m0 < m64; m0 += 32) {
    const int m = (int)((m64 - m0) < 32 ? (m64 - m0) : 32);
    bool hilo;
    const int nt = tiles_for(m, hilo);
    uint4* bf = reinterpret_cast<uint4*>(ws);
    float* scl = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + (size_t)nt * sb * 4096);
    const float* xc = x + m0 * w.k;
    float* yc = y + m0 * w.n;
    {
      const int64_t warps = (int64_t)nt * sb;
      const unsigned grid = (unsigned)((warps + 7) / 8);
      if (hilo)
        prep_kernel<QT, true><<<grid, 256, 0, s>>>(xc, m, w.k, nt, bf, scl);
      else
        prep_kernel<QT, false><<<grid, 256, 0, s>>>(xc, m, w.k, nt, bf, scl);
      if (launches) ++*launches;
    }
    bracket_record(br.start, s);
    cudaError_t e;
    constexpr int ST = stages<QT>();
    if (hilo) {
      e = nt == 1 ? launch_main<QT, 1, true, STAGES_WITH_B, true>(w, m, bf, scl, bias, yc, s)
                  : launch_main<QT, 2, true, ST, false>(w, m, bf, scl, bias, yc, s);
    } else {
      e = nt <= 2 ? launch_main<QT, 2, false, ST, false>(w, m, bf, scl, bias, yc, s)
          : nt == 3 ? launch_main<QT, 3, false, ST, false>(w, m, bf, scl, bias, yc, s)
                    : launch_main<QT, 4, false, ST, false>(w, m, bf, scl, bias, yc, s);
    }
    bracket_record(br.stop, s);
    br = Bracket();  // only the first chunk is bracketed
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
  }
  return cudaGetLastError();
}

template <int QT, int NT, bool HILO, int ST, bool STAGEB>
cudaError_t set_smem_attr() {
  const int most = KSPLIT_WARPS * ST * slot_bytes(QT, STAGEB, 4);
  return cudaFuncSetAttribute(gemv_kernel<QT, NT, HILO, ST, STAGEB>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, most);
}

template <int QT>
cudaError_t set_attrs_typed() {
  constexpr int ST = stages<QT>();
  cudaError_t e = cudaSuccess, r;
  if ((r = set_smem_attr<QT, 1, true, STAGES_WITH_B, true>()) != cudaSuccess) e = r;
  if ((r = set_smem_attr<QT, 2, true, ST, false>()) != cudaSuccess) e = r;
  if ((r = set_smem_attr<QT, 2, false, ST, false>()) != cudaSuccess) e = r;
  if ((r = set_smem_attr<QT, 3, false, ST, false>()) != cudaSuccess) e = r;
  if ((r = set_smem_attr<QT, 4, false, ST, false>()) != cudaSuccess) e = r;
  return e;
}

}  // namespace

cudaError_t gemv_init_device() {
  cudaError_t e = set_attrs_typed<GGUF_Q4_K>();
  cudaError_t e2 = set_attrs_typed<GGUF_Q6_K>();
  return e != cudaSuccess ? e : e2;
}

cudaError_t launch_gemv_gguf(const DevWeight& w, const float* x, int64_t m, const float* bias,
                             float* y, void* ws, cudaStream_t s, int* launches, Bracket br) {
  if (w.type == GGUF_Q4_K) return launch_typed<GGUF_Q4_K>(w, x, m, bias, y, ws, s, launches, br);
  return launch_typed<GGUF_Q6_K>(w, x, m, bias, y, ws, s, launches, br);
}

size_t gemv_gguf_workspace_bytes(int64_t m, int64_t k) {
  // per chunk of up to 32 tokens: B fragments (nt <= 4 tiles x sb x 4 KB)
  // and per-(token, superblock) scales
  const int64_t mc = m < 32 ? m : 32;
  bool hilo;
  const int nt = tiles_for((int)(mc > 0 ? mc : 1), hilo);
  const int64_t sb = k / QK;
  return (size_t)nt * sb * 4096 + (size_t)32 * sb * 4 + 256;
}

}  // namespace kq
