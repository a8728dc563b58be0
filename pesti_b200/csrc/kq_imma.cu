// kq_imma.cu -- batched decode linear (2..32 tokens per chunk) for GGUF Q4_K,
// Q5_K and Q6_K on the integer tensor-core path: y[m][n] = x[m][k] . W[n][k] (+ bias).
//
// A Q4_K sub-block is 32 weights with one 6-bit scale and one 6-bit min, so it
// is exactly one k32 step of mma.sync.m16n8k32 with 8-bit operands:
//  * A = the raw codes: the qs bytes of a row hold sub-blocks 2p (low
//    nibbles) and 2p+1 (high nibbles) of pair p, so one 32-bit load and one
//    mask give a lane its four codes of an A fragment;
//  * B = the activations as in the single-token kernel: per (token,
//    superblock) a power of two 2^e with max|x| 2^-e in [2^13, 2^14), the
//    15-bit integer split into a signed high byte and an unsigned low byte,
//    so two MMAs (u8 x s8, u8 x u8) give exact int32 sums of q x;
//  * per sub-block the int32 result is scaled by sc (f32 accumulate) and the
//    min term dmin m_j sum(x) uses exact int32 sums of the quantized
//    activations; d, dmin and 2^e are applied once per superblock.
// Q5_K is Q4_K with a fifth bit per weight: its codes (nibble | qh bit << 4,
// at most 31) are the A fragment of the same k32 steps, the rest as Q4_K.
// Q6_K's scale groups are 16 weights (elements 16s .. 16s+15 of a
// superblock), so a group is one k16 step of mma.sync.m16n8k16 with 8-bit
// operands: in the device body layout a lane's four codes of a group are one
// 32-bit ql word and one 32-bit qh word per row (nibble | 2 high bits << 4 by
// four bit operations), the -32 offset is applied with exact int32 group sums
// of the quantized activations, the int8 group scale per group, d per
// superblock.
// Only the 15-bit activation rounding approximates, as in the single-token
// kernel.
//
// Data movement: one CTA = 128 weight rows x a contiguous range of
// superblocks (split-K across CTAs when there are few row tiles).  A producer
// warp streams one superblock of all 128 rows per stage with one 2D TMA copy
// (the weight's tensor map: box = one superblock x 128 rows), plus the
// superblock's activation fragments, sums and scales (bulk copies), through a ring of
// shared-memory stages; eight MMA warps each own a 16-row tile of every
// stage.  Partials of the K-splits are added in split order by the last CTA of
// each row tile (deterministic).  Every wait is bounded.
//
// Reference semantics: QuantizedLinear::forward (pesti-runner/src/
// quantized_linear.rs:101-143).
#include "kq_common.cuh"
#include "kq_kernels.h"
#include "kq_sm100.cuh"

#include <algorithm>

namespace kq {
namespace {

constexpr int IM_WARPS = 8;
constexpr int IM_ROWS = 16 * IM_WARPS;    // the weight maps' box height
constexpr int IM_MAX_SMEM = 226 * 1024;   // dynamic; room for the static bytes
constexpr int IM_HALF_SMEM = 112 * 1024;  // two CTAs per SM
// CTAs per SM: one or two token tiles leave registers and shared memory for two
constexpr int im_ctas_per_sm(int nt) { return nt <= 2 ? 2 : 1; }
// MMA warps per CTA and token tiles per MMA warp: up to two tiles, 8 warps
// (one per 16-row group); three or four, 16 warps (two per 16-row group, two
// tiles each), so one CTA per SM still has 16 warps issuing
constexpr int im_mma_warps(int nt) { return nt > 2 ? 16 : 8; }
constexpr int im_tiles_per_warp(int nt) { return nt > 2 ? 2 : nt; }
constexpr int IM_ERR_FULL = 27, IM_ERR_EMPTY = 28;

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Four 15-bit integers -> their signed high bytes and unsigned low bytes.
__device__ __forceinline__ void split4(int v0, int v1, int v2, int v3, uint32_t& hi, uint32_t& lo) {
  hi = ((uint32_t)(v0 >> 8) & 0xffu) | (((uint32_t)(v1 >> 8) & 0xffu) << 8) | (((uint32_t)(v2 >> 8) & 0xffu) << 16) |
       (((uint32_t)(v3 >> 8) & 0xffu) << 24);
  lo = ((uint32_t)v0 & 0xffu) | (((uint32_t)v1 & 0xffu) << 8) | (((uint32_t)v2 & 0xffu) << 16) |
       (((uint32_t)v3 & 0xffu) << 24);
}

// One warp per (token slot t, superblock kb); lane = (sub-block j = lane/4, c = lane%4).
// Token slots t >= m (the rest of the last 8-token tile) get zero fragments.
//   bq[((tile * sb + kb) * 8 + j) * 32 + 4 * (t % 8) + c] = {hi(k 4c..4c+3), hi(k 16+4c..), lo(..), lo(..)}
//   ssum[(kb * 32 + t) * 8 + j] = sum of the 32 quantized values of sub-block j
//   scl[kb * 32 + t] = 2^e (NaN when the superblock holds a non-finite value)
// Q6_K: lane = (group s0 = lane/4, c = lane%4) handles groups s0 and s0 + 8:
//   bq[((tile * sb + kb) * 16 + s) * 32 + 4 * (t % 8) + c] = uint2 {hi(k 4c..4c+3), lo(..)} of group s
//   ssum as int2 [(kb * 16 + s) * 32 + t] = {-32 x the sum of the 16 high bytes of group s,
//                                            -32 x the sum of its 16 low bytes}
//   (the code offset of sum (q - 32) x, applied to each limb's product)
// Where one (token slot t, superblock) job of the preparation writes: the
// activation fragments of its 8-token tile, its sums and its 2^e.  The
// preparation kernel points these into the scratch workspace, the fused
// kernel into its shared-memory copy of its K range (the same per-superblock
// layout the ring stages receive).
struct ImPrepDst {
  uint4* frag;  // Q4_K / Q5_K: [8 j][32] uint4 of this tile; Q6_K: [16 s][32] uint2 (as uint4*: reinterpreted)
  int* sum;     // Q4_K / Q5_K: [32 t][8 j] int; Q6_K: [16 s][32 t] int2 (as int*: reinterpreted)
  float* scale; // [32 t]
};

// This lane's two runs of four activations of job (t, superblock): Q4_K:
// sub-block j = lane / 4, elements 32j + 4c.. and 32j + 16 + 4c..; Q6_K: groups
// j and j + 8, elements 16j + 4c.. and 16(j + 8) + 4c.. (c = lane % 4).
template <int QT>
__device__ __forceinline__ void im_prep_offsets(int lane, int& ea, int& eb) {
  const int j = lane >> 2, c = lane & 3;
  constexpr bool Q4 = QT == GGUF_Q4_K;
  ea = Q4 ? 32 * j + 4 * c : 16 * j + 4 * c;
  eb = Q4 ? ea + 16 : ea + 128;
}

// RMSNorm scaling of the two runs (global element offsets ga, gb; dim % 4 ==
// 0 so each float4 is wholly inside or past dim, where the result is zero).
__device__ __forceinline__ void im_prep_norm(float4& a, float4& b, int64_t ga, int64_t gb, const float* nw, int dim,
                                             float rinv) {
  const float4 wa = ga < dim ? ldg_f4(nw + ga) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 wb = gb < dim ? ldg_f4(nw + gb) : make_float4(0.f, 0.f, 0.f, 0.f);
  a = ga < dim ? make_float4(a.x * rinv * wa.x, a.y * rinv * wa.y, a.z * rinv * wa.z, a.w * rinv * wa.w) : wa;
  b = gb < dim ? make_float4(b.x * rinv * wb.x, b.y * rinv * wb.y, b.z * rinv * wb.z, b.w * rinv * wb.w) : wb;
}

// 1 / sqrt(mean(row[0:dim]^2) + eps), reduced over the warp.
__device__ __forceinline__ float im_row_rinv(const float* row, int dim, float eps, int lane) {
  float ss = 0.f;
#pragma unroll 4
  for (int i = 4 * lane; i < dim; i += 128) {
    const float4 v = ldg_f4(row + i);
    ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return 1.f / sqrtf(ss / (float)dim + eps);
}

// Quantize one job's activations (this lane's runs a, b; the whole warp
// takes part) and write its fragments (token slot position tt = t % 8 in the
// tile), sums (slot t) and scale.
template <int QT>
__device__ __forceinline__ void im_prep_store(float4 a, float4 b, int lane, int t, const ImPrepDst& d) {
  constexpr bool Q4 = QT == GGUF_Q4_K;
  const int j = lane >> 2, c = lane & 3, tt = t & 7;
  float amax = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
  amax = fmaxf(amax, fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float inv = 0.f, factor = __int_as_float(0x7fc00000);
  if (amax <= 3.4e38f) {  // finite (NaN compares false)
    int e = 0;
    if (amax > 0.f) e = (int)((__float_as_uint(amax) >> 23) & 0xff) - 127 - 13;
    e = max(-126, min(126, e));
    inv = __uint_as_float((uint32_t)(127 - e) << 23);
    factor = __uint_as_float((uint32_t)(127 + e) << 23);
  }
  const int v0 = __float2int_rn(a.x * inv), v1 = __float2int_rn(a.y * inv), v2 = __float2int_rn(a.z * inv),
            v3 = __float2int_rn(a.w * inv);
  const int v4 = __float2int_rn(b.x * inv), v5 = __float2int_rn(b.y * inv), v6 = __float2int_rn(b.z * inv),
            v7 = __float2int_rn(b.w * inv);
  uint4 o;
  split4(v0, v1, v2, v3, o.x, o.z);
  split4(v4, v5, v6, v7, o.y, o.w);
  if constexpr (Q4) {
    d.frag[j * 32 + 4 * tt + c] = o;
    int s = v0 + v1 + v2 + v3 + v4 + v5 + v6 + v7;
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (c == 0) d.sum[t * 8 + j] = s;
  } else {
    uint2* f2 = reinterpret_cast<uint2*>(d.frag);
    f2[j * 32 + 4 * tt + c] = make_uint2(o.x, o.z);
    f2[(j + 8) * 32 + 4 * tt + c] = make_uint2(o.y, o.w);
    // limb sums of groups j (v0..v3) and j + 8 (v4..v7): high bytes v >> 8, low bytes v & 255
    int ha = (v0 >> 8) + (v1 >> 8) + (v2 >> 8) + (v3 >> 8), la = (v0 & 255) + (v1 & 255) + (v2 & 255) + (v3 & 255);
    int hb = (v4 >> 8) + (v5 >> 8) + (v6 >> 8) + (v7 >> 8), lb = (v4 & 255) + (v5 & 255) + (v6 & 255) + (v7 & 255);
#pragma unroll
    for (int o2 = 1; o2 <= 2; o2 <<= 1) {
      ha += __shfl_xor_sync(0xffffffffu, ha, o2);
      la += __shfl_xor_sync(0xffffffffu, la, o2);
      hb += __shfl_xor_sync(0xffffffffu, hb, o2);
      lb += __shfl_xor_sync(0xffffffffu, lb, o2);
    }
    if (c == 0) {  // times the code offset 32, negated: the MMAs' start values
      int2* s2 = reinterpret_cast<int2*>(d.sum);
      s2[j * 32 + t] = make_int2(-32 * ha, -32 * la);
      s2[(j + 8) * 32 + t] = make_int2(-32 * hb, -32 * lb);
    }
  }
  if (lane == 0) d.scale[t] = factor;
}

// Zero fragments for a token slot past m (the rest of the last 8-token tile);
// its sums and scale are written as zero too.
template <int QT>
__device__ __forceinline__ void im_prep_zero(int lane, int t, const ImPrepDst& d) {
  const int j = lane >> 2, c = lane & 3, tt = t & 7;
  if constexpr (QT == GGUF_Q4_K) {
    d.frag[j * 32 + 4 * tt + c] = make_uint4(0u, 0u, 0u, 0u);
    if (c == 0) d.sum[t * 8 + j] = 0;
  } else {
    uint2* f2 = reinterpret_cast<uint2*>(d.frag);
    f2[j * 32 + 4 * tt + c] = make_uint2(0u, 0u);
    f2[(j + 8) * 32 + 4 * tt + c] = make_uint2(0u, 0u);
    if (c == 0) {
      int2* s2 = reinterpret_cast<int2*>(d.sum);
      s2[j * 32 + t] = make_int2(0, 0);
      s2[(j + 8) * 32 + t] = make_int2(0, 0);
    }
  }
  if (lane == 0) d.scale[t] = 0.f;
}

// Workspace layout per superblock kb: fragments [tile][kb] 4096 bytes each,
// sums [kb] (Q4_K 1024 / Q6_K 4096 bytes), scales [kb] 128 bytes.
template <int QT>
__device__ __forceinline__ ImPrepDst im_ws_dst(uint4* bq, int* ssum, float* scl, int sb, int kb, int t) {
  ImPrepDst d;
  d.frag = bq + (size_t)((t >> 3) * sb + kb) * 256;
  d.sum = ssum + (size_t)kb * (QT == GGUF_Q4_K ? 256 : 1024);
  d.scale = scl + (size_t)kb * 32;
  return d;
}

// With a norm (nw != nullptr) the quantized activations are RMSNorm(x) =
// x / sqrt(mean(x[0:dim]^2) + eps) * nw, zero past dim: each warp first
// reduces its token's sum of squares over the whole row (the row is small and
// L2-resident, so the redundant reads across a token's superblocks are cheap).
// Q5_K uses the Q4_K form (the same 32-weight sub-blocks).
template <int QT>
__global__ void __launch_bounds__(256) imma_prep_kernel(const float* __restrict__ x, int64_t x_ld, int m, int slots,
                                                        int64_t k, int sb, uint4* __restrict__ bq,
                                                        int* __restrict__ ssum, float* __restrict__ scl,
                                                        const float* __restrict__ nw, int dim, float eps) {
  pdl_trigger();
  pdl_wait();  // x may be the previous kernel's output
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (wid >= (int64_t)slots * sb) return;
  const int t = (int)(wid / sb), kb = (int)(wid - (int64_t)t * sb);
  const ImPrepDst d = im_ws_dst<QT>(bq, ssum, scl, sb, kb, t);
  if (t >= m) {
    im_prep_zero<QT>(lane, t, d);
    return;
  }
  int ea, eb;
  im_prep_offsets<QT>(lane, ea, eb);
  const float* xs = x + (int64_t)t * x_ld + (int64_t)kb * 256;
  float4 a = ldg_f4(xs + ea), b = ldg_f4(xs + eb);
  if (nw) {
    const float rinv = im_row_rinv(x + (int64_t)t * x_ld, dim, eps, lane);
    im_prep_norm(a, b, (int64_t)kb * 256 + ea, (int64_t)kb * 256 + eb, nw, dim, rinv);
  }
  im_prep_store<QT>(a, b, lane, t, d);
}

// Device bytes of one superblock in the weight's tensor map box.
constexpr int im_block_bytes(int qt) {
  return qt == GGUF_Q4_K   ? Q4K_BYTES
         : qt == GGUF_Q5_K ? Q5K_BYTES
         : qt == GGUF_Q3_K ? Q3K_DEV
         : qt == GGUF_Q2_K ? Q2K_DEV
                           : Q6K_BODY;
}
// Types whose scale groups are 16 weights (one k16 step each): Q6_K, Q3_K and
// Q2_K; they share the Q6_K activation preparation (groups j and j + 8 per lane).
constexpr bool im_k16(int qt) { return qt == GGUF_Q6_K || qt == GGUF_Q3_K || qt == GGUF_Q2_K; }

// Bytes of one ring stage for type qt and nt 8-token tiles: the weight box,
// Q6_K's d box, the activation fragments, the activation sums of the 32 token
// slots (Q4_K / Q5_K: one int per sub-block; Q6_K: two limb sums per group)
// and the 32 slots' 2^e.  The kernel's stage layout (ImStage) and the launch's
// shared-memory size (im_shape) both come from here.
constexpr int im_stage_w(int qt) { return IM_ROWS * im_block_bytes(qt); }
constexpr int im_stage_d(int qt) { return qt == GGUF_Q6_K ? IM_ROWS * 16 : 0; }
constexpr int im_stage_s(int qt) { return im_k16(qt) ? 32 * 16 * 8 : 32 * 8 * 4; }
constexpr int im_stage_bytes(int qt, int nt) { return im_stage_w(qt) + im_stage_d(qt) + nt * 4096 + im_stage_s(qt) + 32 * 4; }

template <int QT, int NT>
struct ImStage {
  static constexpr int W = im_stage_w(QT);     // 18432 / 22528 / 26624
  static constexpr int D = im_stage_d(QT);     // Q6_K: d of 8 superblocks per row
  static constexpr int B = NT * 4096;          // activation fragments, 8 tokens per tile
  static constexpr int S = im_stage_s(QT);     // activation sums of the 32 token slots
  static constexpr int F = 32 * 4;             // 2^e of the 32 token slots
  static constexpr int BYTES = W + D + B + S + F;
  static_assert(BYTES == im_stage_bytes(QT, NT) && BYTES % 128 == 0, "stage layout");
};

struct ImParams {
  const uint4* bq;
  const int* ssum;
  const float* scl;
  const float* bias;
  float* y;     // [m][n]
  float* part;  // [splits][m][n] (splits > 1)
  unsigned* ctr;
  int64_t n;
  int sb, m, splits, kb_per, S;
  int accumulate;  // y += the product instead of y = (the residual update)
  int* err;
  // shared-memory plan: ring stages stage_bytes apart, the fused form's
  // prepared K range at xp_off (xp_stride bytes per superblock), barriers at bar_off
  int stage_bytes, xp_off, xp_stride, bar_off;
  // fused form: the activations (rows x_ld floats apart), optional RMSNorm
  const float* x;
  int64_t x_ld;
  const float* nw;
  int dim;
  float eps;
};

// Hand a ring stage back to the producer.  The warp's shared-memory reads of
// the stage (generic proxy) are fenced against the TMA / bulk copies that
// refill it (async proxy) before the release: without the fence a refill was
// seen to overtake reads still queued behind the arrive.
__device__ __forceinline__ void stage_release(uint64_t* empty, int lane) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) sm100::mbar_arrive(empty);
}
__device__ __forceinline__ void mbar_expect_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(sm100::smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_u8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// k16 forms (Q6_K groups): A = a0 (row g, k 4c..4c+3), a1 (row g + 8); B = b0 (k 4c..4c+3, column g)
__device__ __forceinline__ void mma16_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
               : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
               : "r"(a0), "r"(a1), "r"(b0));
}
__device__ __forceinline__ void mma16_u8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
               : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
               : "r"(a0), "r"(a1), "r"(b0));
}

// FUSED: the CTA prepares the activation fragments, sums and scales of its
// own K range itself (its MMA warps, into shared memory, while the producer's
// first weight copies are in flight) instead of a preparation kernel writing
// them to the workspace for the producer to copy per stage; chosen where that
// range fits beside the ring.
template <int QT, int NT, bool FUSED>
__global__ void __launch_bounds__(32 * (im_mma_warps(NT) + 1), im_ctas_per_sm(NT))
    imma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap dmap, const ImParams P) {
  using St = ImStage<QT, NT>;
  // MMA warps: 16 for three or four token tiles (warps w and w + 8 share a
  // 16-row group and take two tiles each), 8 otherwise
  constexpr int MW = im_mma_warps(NT), NTW = im_tiles_per_warp(NT);
  constexpr bool Q4 = !im_k16(QT);  // Q4_K and Q5_K: 32-weight sub-blocks
  constexpr bool Q5 = QT == GGUF_Q5_K;
  constexpr bool Q6 = QT == GGUF_Q6_K;  // the only type with a separate d box
  constexpr int BPS = im_block_bytes(QT);
  constexpr int QS = Q5 ? 48 : 16;  // offset of the qs bytes in the superblock
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_trigger();
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.bar_off);
  uint64_t* empty = full + P.S;
  __shared__ int last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = (int64_t)blockIdx.x * IM_ROWS;
  const int sp = blockIdx.y;
  const int kb0 = sp * P.kb_per;
  const int T = max(0, min(P.sb, kb0 + P.kb_per) - kb0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.S; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], MW);
    }
    sm100::mbar_fence_init();
  }
  __syncthreads();

  if (warp == MW) {
    // ---- producer: the weights first (they do not depend on the previous kernel)
    if (lane == 0) {
      sm100::tma_prefetch(&wmap);
      if constexpr (Q6) sm100::tma_prefetch(&dmap);
      auto weights = [&](int t) {
        const int st = t % P.S, kb = kb0 + t;
        uint8_t* dst = smem + (size_t)st * P.stage_bytes;
        // fused: the weights are the whole stage, so this is the stage's arrival
        if constexpr (FUSED) sm100::mbar_expect_tx(&full[st], St::W + St::D);
        else mbar_expect_only(&full[st], St::W + St::D);
        sm100::tma_load_2d(dst, &wmap, kb * BPS, (int)row0, &full[st]);
        if constexpr (Q6) sm100::tma_load_2d(dst + St::W, &dmap, kb & ~7, (int)row0, &full[st]);
      };
      const int pre = min(T, P.S);
      for (int t = 0; t < pre; ++t) weights(t);
      if constexpr (!FUSED) pdl_wait();  // activation fragments and sums come from the prep kernel
      int t = 0;
      for (; t < T; ++t) {
        const int st = t % P.S, kb = kb0 + t;
        if (t >= pre) {
          if (!sm100::mbar_wait(&empty[st], ((t / P.S) - 1) & 1, P.err, IM_ERR_EMPTY)) break;
          weights(t);
        }
        if constexpr (FUSED) continue;
        uint8_t* dst = smem + (size_t)st * P.stage_bytes + St::W + St::D;
        sm100::mbar_expect_tx(&full[st], St::B + St::S + St::F);  // the stage's arrival
#pragma unroll
        for (int i = 0; i < NT; ++i)
          sm100::bulk_load(dst + i * 4096, P.bq + ((size_t)i * P.sb + kb) * 8 * 32, 4096, &full[st]);
        sm100::bulk_load(dst + St::B, P.ssum + (size_t)kb * St::S / 4, St::S, &full[st]);
        sm100::bulk_load(dst + St::B + St::S, P.scl + (size_t)kb * 32, St::F, &full[st]);
      }
      // no copy may still be in flight into the ring when the CTA retires
      for (int v = max(0, t - P.S); v < t; ++v) sm100::mbar_wait(&full[v % P.S], (v / P.S) & 1, P.err, IM_ERR_FULL);
    }
    return;
  }

  // ---- MMA warps: warp w owns tile rows 16w + g (C rows 0-7) and 16w + g + 8
  pdl_wait();  // x, or the per-(superblock, token) fragments and scales the prep kernel wrote
  if constexpr (FUSED) {
    // this CTA's K range [kb0, kb0 + T) for every token slot: job (t, i) =
    // slot t, local superblock i, one warp each, JB jobs' loads in flight per warp
    constexpr int PQT = im_k16(QT) ? GGUF_Q6_K : GGUF_Q4_K;  // Q5_K: the Q4_K preparation, Q3_K the Q6_K one
    constexpr int JB = 4;
    __shared__ float rinv_s[32];
    if (P.nw) {
      for (int t = warp; t < P.m; t += MW) {
        const float r = im_row_rinv(P.x + (int64_t)t * P.x_ld, P.dim, P.eps, lane);
        if (lane == 0) rinv_s[t] = r;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(32 * MW) : "memory");
    }
    int ea, eb;
    im_prep_offsets<PQT>(lane, ea, eb);
    const int jobs = NT * 8 * T;
    for (int j0 = warp; j0 < jobs; j0 += MW * JB) {
      float4 a[JB], b[JB];
#pragma unroll
      for (int u = 0; u < JB; ++u) {
        const int job = j0 + u * MW, t = job / max(T, 1), i = job - t * max(T, 1);
        a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (job < jobs && t < P.m) {
          const float* xs = P.x + (int64_t)t * P.x_ld + (int64_t)(kb0 + i) * 256;
          a[u] = ldg_f4(xs + ea);
          b[u] = ldg_f4(xs + eb);
        }
      }
#pragma unroll
      for (int u = 0; u < JB; ++u) {
        const int job = j0 + u * MW, t = job / max(T, 1), i = job - t * max(T, 1);
        if (job >= jobs) continue;  // uniform across the warp
        uint8_t* blk = smem + P.xp_off + (size_t)i * P.xp_stride;
        ImPrepDst d;
        d.frag = reinterpret_cast<uint4*>(blk) + (t >> 3) * 256;
        d.sum = reinterpret_cast<int*>(blk + St::B);
        d.scale = reinterpret_cast<float*>(blk + St::B + St::S);
        if (t >= P.m) {
          im_prep_zero<PQT>(lane, t, d);
        } else {
          if (P.nw) {
            const int64_t base = (int64_t)(kb0 + i) * 256;
            im_prep_norm(a[u], b[u], base + ea, base + eb, P.nw, P.dim, rinv_s[t]);
          }
          im_prep_store<PQT>(a[u], b[u], lane, t, d);
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(32 * MW) : "memory");
  }
  const int g = lane >> 2, c = lane & 3;
  const int i0 = (warp / 8) * NTW;  // this warp's first token tile
  const int ra = 16 * (warp % 8) + g, rb = ra + 8;
  float tot[NTW][4];
#pragma unroll
  for (int i = 0; i < NTW; ++i) tot[i][0] = tot[i][1] = tot[i][2] = tot[i][3] = 0.f;

  for (int t = 0; t < T; ++t) {
    const int st = t % P.S, kb = kb0 + t;
    if (!sm100::mbar_wait_warp(&full[st], (t / P.S) & 1, P.err, IM_ERR_FULL)) break;
    const uint8_t* stage = smem + (size_t)st * P.stage_bytes;
    // fragments | sums | scales of this superblock: the stage's copies, or the fused preparation's
    const uint8_t* bsf = FUSED ? smem + P.xp_off + (size_t)t * P.xp_stride : stage + St::W + St::D;
    if constexpr (Q4) {
      const uint8_t* pa = stage + ra * BPS;
      const uint8_t* pb = stage + rb * BPS;
      const uint4 ha = *reinterpret_cast<const uint4*>(pa), hb = *reinterpret_cast<const uint4*>(pb);
      // the eight 6-bit scales / mins of each row as bytes: [0..3] and [4..7]
      const uint32_t sca_lo = ha.y & 0x3F3F3F3Fu, ma_lo = ha.z & 0x3F3F3F3Fu;
      const uint32_t sca_hi = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
      const uint32_t ma_hi = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
      const uint32_t scb_lo = hb.y & 0x3F3F3F3Fu, mb_lo = hb.z & 0x3F3F3F3Fu;
      const uint32_t scb_hi = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
      const uint32_t mb_hi = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
      const uint4* bs = reinterpret_cast<const uint4*>(bsf);
      const int* ss = reinterpret_cast<const int*>(bsf + St::B);
      // sum over sub-blocks of scale x limb product, exact in int32: a
      // sub-block's high-limb sum is < 2^16 in size, its low-limb one < 2^18
      // (codes up to 31), so 8 six-bit scales keep them below 2^25 / 2^27
      int aH[NTW][4], aL[NTW][4], ma[NTW][4];
#pragma unroll
      for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          aH[i][e] = aL[i][e] = 0;
          ma[i][e] = 0;
        }
      // Q5_K: the qh bytes of this lane's k (bit j of byte l is the fifth bit
      // of element l of sub-block j), the same for every pair
      uint32_t ha0 = 0, ha1 = 0, hb0 = 0, hb1 = 0;
      if constexpr (Q5) {
        ha0 = *reinterpret_cast<const uint32_t*>(pa + 16 + 4 * c);
        ha1 = *reinterpret_cast<const uint32_t*>(pa + 32 + 4 * c);
        hb0 = *reinterpret_cast<const uint32_t*>(pb + 16 + 4 * c);
        hb1 = *reinterpret_cast<const uint32_t*>(pb + 32 + 4 * c);
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        // qs of pair p: bytes QS + 32p ..; this lane's k = 4c..4c+3 and 16+4c..
        const uint32_t wa0 = *reinterpret_cast<const uint32_t*>(pa + QS + 32 * p + 4 * c);
        const uint32_t wa1 = *reinterpret_cast<const uint32_t*>(pa + QS + 16 + 32 * p + 4 * c);
        const uint32_t wb0 = *reinterpret_cast<const uint32_t*>(pb + QS + 32 * p + 4 * c);
        const uint32_t wb1 = *reinterpret_cast<const uint32_t*>(pb + QS + 16 + 32 * p + 4 * c);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = 2 * p + h;
          uint32_t a0 = (h ? wa0 >> 4 : wa0) & 0x0F0F0F0Fu, a1 = (h ? wb0 >> 4 : wb0) & 0x0F0F0F0Fu;
          uint32_t a2 = (h ? wa1 >> 4 : wa1) & 0x0F0F0F0Fu, a3 = (h ? wb1 >> 4 : wb1) & 0x0F0F0F0Fu;
          if constexpr (Q5) {  // bit j of every qh byte to bit 4: a left rotation by 4 - j
            a0 |= __funnelshift_l(ha0, ha0, (4 - j) & 31) & 0x10101010u;
            a1 |= __funnelshift_l(hb0, hb0, (4 - j) & 31) & 0x10101010u;
            a2 |= __funnelshift_l(ha1, ha1, (4 - j) & 31) & 0x10101010u;
            a3 |= __funnelshift_l(hb1, hb1, (4 - j) & 31) & 0x10101010u;
          }
          const int sh = 8 * (j & 3);
          const int sca = (int)(((j < 4 ? sca_lo : sca_hi) >> sh) & 0xffu);
          const int scb = (int)(((j < 4 ? scb_lo : scb_hi) >> sh) & 0xffu);
          const int mina = (int)(((j < 4 ? ma_lo : ma_hi) >> sh) & 0xffu);
          const int minb = (int)(((j < 4 ? mb_lo : mb_hi) >> sh) & 0xffu);
#pragma unroll
          for (int i = 0; i < NTW; ++i) {
            const int ti = i0 + i;  // token tile
            if (ti >= NT) break;    // uniform across the warp
            const uint4 bv = bs[(ti * 8 + j) * 32 + lane];
            int ch[4] = {0, 0, 0, 0}, cl[4] = {0, 0, 0, 0};
            mma_u8s8(ch, a0, a1, a2, a3, bv.x, bv.y);
            mma_u8u8(cl, a0, a1, a2, a3, bv.z, bv.w);
            // C: [0], [1] row g, tokens 8i + 2c, +1; [2], [3] row g + 8
            aH[i][0] += sca * ch[0];
            aH[i][1] += sca * ch[1];
            aH[i][2] += scb * ch[2];
            aH[i][3] += scb * ch[3];
            aL[i][0] += sca * cl[0];
            aL[i][1] += sca * cl[1];
            aL[i][2] += scb * cl[2];
            aL[i][3] += scb * cl[3];
            const int s0 = ss[(8 * ti + 2 * c) * 8 + j], s1 = ss[(8 * ti + 2 * c + 1) * 8 + j];
            ma[i][0] += mina * s0;
            ma[i][1] += mina * s1;
            ma[i][2] += minb * s0;
            ma[i][3] += minb * s1;
          }
        }
      }
      const float* fsc = reinterpret_cast<const float*>(bsf + St::B + St::S);
      float f[NTW][2];
#pragma unroll
      for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = 8 * (i0 + i) + 2 * c + e;
          f[i][e] = tk < P.m ? fsc[tk] : 0.f;
        }
      stage_release(&empty[st], lane);
      const float da = f16_bits_to_f32((uint16_t)(ha.x & 0xffff)), dma = f16_bits_to_f32((uint16_t)(ha.x >> 16));
      const float db = f16_bits_to_f32((uint16_t)(hb.x & 0xffff)), dmb = f16_bits_to_f32((uint16_t)(hb.x >> 16));
#pragma unroll
      for (int i = 0; i < NTW; ++i) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float va = fmaf(256.f, (float)aH[i][e], (float)aL[i][e]);
          const float vb = fmaf(256.f, (float)aH[i][2 + e], (float)aL[i][2 + e]);
          tot[i][e] = fmaf(f[i][e], fmaf(da, va, -dma * (float)ma[i][e]), tot[i][e]);
          tot[i][2 + e] = fmaf(f[i][e], fmaf(db, vb, -dmb * (float)ma[i][2 + e]), tot[i][2 + e]);
        }
      }
    } else if constexpr (QT == GGUF_Q2_K) {
      // device superblock (96 bytes): scales[16] | qs[64] | d | dmin | 12 zero bytes.
      // Group s = 8h + 2G + b (elements 16s..16s+15): this lane's four 2-bit codes are
      // bits 2G of qs word (h, b) (bytes 16 + 32h + 16b + 4c..); scale byte s holds the
      // group's scale (low nibble) and min (high nibble); value = d sc q - dmin m.  The
      // min term takes the group's activation sum from the Q6_K preparation's limb sums:
      // sum x = -(256 S_hi + S_lo) / 32, exactly
      const uint8_t* pa = stage + ra * Q2K_DEV;
      const uint8_t* pb = stage + rb * Q2K_DEV;
      const uint4 sca4 = *reinterpret_cast<const uint4*>(pa), scb4 = *reinterpret_cast<const uint4*>(pb);
      const uint32_t dda = *reinterpret_cast<const uint32_t*>(pa + 80);
      const uint32_t ddb = *reinterpret_cast<const uint32_t*>(pb + 80);
      const uint2* bs = reinterpret_cast<const uint2*>(bsf);
      const int4* ss4 = reinterpret_cast<const int4*>(bsf + St::B);
      int aH[NTW][4], aL[NTW][4], ma[NTW][4];
#pragma unroll
      for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) aH[i][e] = aL[i][e] = ma[i][e] = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int b2 = 0; b2 < 2; ++b2) {
          const uint32_t qsa = *reinterpret_cast<const uint32_t*>(pa + 16 + 32 * h + 16 * b2 + 4 * c);
          const uint32_t qsb = *reinterpret_cast<const uint32_t*>(pb + 16 + 32 * h + 16 * b2 + 4 * c);
#pragma unroll
          for (int G = 0; G < 4; ++G) {
            const int sg = 8 * h + 2 * G + b2;
            const uint32_t a0 = (qsa >> (2 * G)) & 0x03030303u, a1 = (qsb >> (2 * G)) & 0x03030303u;
            const uint32_t wa = (sg < 4 ? sca4.x : sg < 8 ? sca4.y : sg < 12 ? sca4.z : sca4.w) >> (8 * (sg & 3));
            const uint32_t wb = (sg < 4 ? scb4.x : sg < 8 ? scb4.y : sg < 12 ? scb4.z : scb4.w) >> (8 * (sg & 3));
            const int sca = (int)(wa & 15u), mina = (int)((wa >> 4) & 15u);
            const int scb = (int)(wb & 15u), minb = (int)((wb >> 4) & 15u);
#pragma unroll
            for (int i = 0; i < NTW; ++i) {
              const int ti = i0 + i;  // token tile
              if (ti >= NT) break;    // uniform across the warp
              const uint2 bv = bs[(ti * 16 + sg) * 32 + lane];
              const int4 sv = ss4[sg * 16 + 4 * ti + c];
              int ch[4] = {0, 0, 0, 0}, cl[4] = {0, 0, 0, 0};
              mma16_u8s8(ch, a0, a1, bv.x);
              mma16_u8u8(cl, a0, a1, bv.y);
              aH[i][0] += sca * ch[0];
              aH[i][1] += sca * ch[1];
              aH[i][2] += scb * ch[2];
              aH[i][3] += scb * ch[3];
              aL[i][0] += sca * cl[0];
              aL[i][1] += sca * cl[1];
              aL[i][2] += scb * cl[2];
              aL[i][3] += scb * cl[3];
              const int s0 = -((sv.x * 256 + sv.y) >> 5), s1 = -((sv.z * 256 + sv.w) >> 5);  // tokens 2c, 2c+1
              ma[i][0] += mina * s0;
              ma[i][1] += mina * s1;
              ma[i][2] += minb * s0;
              ma[i][3] += minb * s1;
            }
          }
        }
      const float da = f16_bits_to_f32((uint16_t)(dda & 0xffff)), dma = f16_bits_to_f32((uint16_t)(dda >> 16));
      const float db = f16_bits_to_f32((uint16_t)(ddb & 0xffff)), dmb = f16_bits_to_f32((uint16_t)(ddb >> 16));
      const float* fsc = reinterpret_cast<const float*>(bsf + St::B + St::S);
      float f[NTW][2];
#pragma unroll
      for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = 8 * (i0 + i) + 2 * c + e;
          f[i][e] = tk < P.m ? fsc[tk] : 0.f;
        }
      stage_release(&empty[st], lane);
#pragma unroll
      for (int i = 0; i < NTW; ++i) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float va = fmaf(256.f, (float)aH[i][e], (float)aL[i][e]);
          const float vb = fmaf(256.f, (float)aH[i][2 + e], (float)aL[i][2 + e]);
          tot[i][e] = fmaf(f[i][e], fmaf(da, va, -dma * (float)ma[i][e]), tot[i][e]);
          tot[i][2 + e] = fmaf(f[i][e], fmaf(db, vb, -dmb * (float)ma[i][2 + e]), tot[i][2 + e]);
        }
      }
    } else if constexpr (QT == GGUF_Q3_K) {
      // device superblock (112 bytes): hmask[32] | qs[64] | scales[12] | d.  Group
      // s = 8h + 2G + b (elements 16s..16s+15): this lane's four codes are bits 2G of
      // qs word (h, b) (bytes 32h + 16b + 4c..) and bit 4h + G of hmask word b (bytes
      // 16b + 4c..) as bit 2: q + 4 in [0, 7], the -4 through the limb sums (the
      // preparation's -32 sums divided by 8, exactly)
      const uint8_t* pa = stage + ra * Q3K_DEV;
      const uint8_t* pb = stage + rb * Q3K_DEV;
      const uint4 sda = *reinterpret_cast<const uint4*>(pa + 96), sdb = *reinterpret_cast<const uint4*>(pb + 96);
      const uint2* bs = reinterpret_cast<const uint2*>(bsf);
      const int4* ss4 = reinterpret_cast<const int4*>(bsf + St::B);
      int aH[NTW][4], aL[NTW][4];
#pragma unroll
      for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) aH[i][e] = aL[i][e] = 0;
#pragma unroll
      for (int b2 = 0; b2 < 2; ++b2) {
        const uint32_t hma = *reinterpret_cast<const uint32_t*>(pa + 16 * b2 + 4 * c);
        const uint32_t hmb = *reinterpret_cast<const uint32_t*>(pb + 16 * b2 + 4 * c);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t qsa = *reinterpret_cast<const uint32_t*>(pa + 32 + 32 * h + 16 * b2 + 4 * c);
          const uint32_t qsb = *reinterpret_cast<const uint32_t*>(pb + 32 + 32 * h + 16 * b2 + 4 * c);
#pragma unroll
          for (int G = 0; G < 4; ++G) {
            const int sg = 8 * h + 2 * G + b2;
            const uint32_t a0 = ((qsa >> (2 * G)) & 0x03030303u) | (((hma >> (4 * h + G)) & 0x01010101u) << 2);
            const uint32_t a1 = ((qsb >> (2 * G)) & 0x03030303u) | (((hmb >> (4 * h + G)) & 0x01010101u) << 2);
            // six-bit scale of group sg, minus 32: low nibble of scale byte sg (sg < 8)
            // or high nibble of byte sg - 8, bits 2(sg/4) of byte 8 + sg%4 on top
            const uint32_t wlo_a = (sg & 4) ? sda.y : sda.x, wlo_b = (sg & 4) ? sdb.y : sdb.x;
            const int sh = 8 * (sg & 3), hs = 2 * (sg >> 2);
            const int sca = (int)(((wlo_a >> (sh + ((sg & 8) ? 4 : 0))) & 15u) | (((sda.z >> (sh + hs)) & 3u) << 4)) - 32;
            const int scb = (int)(((wlo_b >> (sh + ((sg & 8) ? 4 : 0))) & 15u) | (((sdb.z >> (sh + hs)) & 3u) << 4)) - 32;
#pragma unroll
            for (int i = 0; i < NTW; ++i) {
              const int ti = i0 + i;  // token tile
              if (ti >= NT) break;    // uniform across the warp
              const uint2 bv = bs[(ti * 16 + sg) * 32 + lane];
              const int4 sv = ss4[sg * 16 + 4 * ti + c];
              int ch[4] = {sv.x >> 3, sv.z >> 3, sv.x >> 3, sv.z >> 3};
              int cl[4] = {sv.y >> 3, sv.w >> 3, sv.y >> 3, sv.w >> 3};
              mma16_u8s8(ch, a0, a1, bv.x);
              mma16_u8u8(cl, a0, a1, bv.y);
              aH[i][0] += sca * ch[0];
              aH[i][1] += sca * ch[1];
              aH[i][2] += scb * ch[2];
              aH[i][3] += scb * ch[3];
              aL[i][0] += sca * cl[0];
              aL[i][1] += sca * cl[1];
              aL[i][2] += scb * cl[2];
              aL[i][3] += scb * cl[3];
            }
          }
        }
      }
      const float da = f16_bits_to_f32((uint16_t)(sda.w & 0xffff)), db = f16_bits_to_f32((uint16_t)(sdb.w & 0xffff));
      const float* fsc = reinterpret_cast<const float*>(bsf + St::B + St::S);
      float f[NTW][2];
#pragma unroll
      for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = 8 * (i0 + i) + 2 * c + e;
          f[i][e] = tk < P.m ? fsc[tk] : 0.f;
        }
      stage_release(&empty[st], lane);
#pragma unroll
      for (int i = 0; i < NTW; ++i) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float va = fmaf(256.f, (float)aH[i][e], (float)aL[i][e]);
          const float vb = fmaf(256.f, (float)aH[i][2 + e], (float)aL[i][2 + e]);
          tot[i][e] = fmaf(f[i][e] * da, va, tot[i][e]);
          tot[i][2 + e] = fmaf(f[i][e] * db, vb, tot[i][2 + e]);
        }
      }
    } else {
      const uint8_t* pa = stage + ra * Q6K_BODY;
      const uint8_t* pb = stage + rb * Q6K_BODY;
      const uint16_t* dtile = reinterpret_cast<const uint16_t*>(stage + St::W);
      const uint4 sca4 = *reinterpret_cast<const uint4*>(pa + 192), scb4 = *reinterpret_cast<const uint4*>(pb + 192);
      const uint2* bs = reinterpret_cast<const uint2*>(bsf);
      // {-32 sum hi, -32 sum lo} of tokens 8i + 2c and 8i + 2c + 1 for group sg: int4 [sg][4i + c]
      const int4* ss4 = reinterpret_cast<const int4*>(bsf + St::B);
      // sum over groups of scale x limb product, exact in int32: a group's
      // high-limb sum (q - 32) hi is < 2^15 in size, its low-limb one < 2^17,
      // so 16 groups of int8 scales stay below 2^26 / 2^28
      int aH[NTW][4], aL[NTW][4];
#pragma unroll
      for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) aH[i][e] = aL[i][e] = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int l16 = 0; l16 < 2; ++l16) {
          // this lane's 4 columns of the groups: slot 2 l16 + c/2, bytes 4 (c % 2) ..
          const int off = 48 * (2 * l16 + (c >> 1)) + 4 * (c & 1);
          const uint32_t qha = *reinterpret_cast<const uint32_t*>(pa + off + 8 * (4 + h));
          const uint32_t qhb = *reinterpret_cast<const uint32_t*>(pb + off + 8 * (4 + h));
#pragma unroll
          for (int gg = 0; gg < 2; ++gg) {
            const uint32_t qla = *reinterpret_cast<const uint32_t*>(pa + off + 8 * (2 * h + gg));
            const uint32_t qlb = *reinterpret_cast<const uint32_t*>(pb + off + 8 * (2 * h + gg));
#pragma unroll
            for (int nib = 0; nib < 2; ++nib) {
              const int G = gg + 2 * nib, sg = 8 * h + 2 * G + l16;
              // six-bit codes: nibble | two high bits << 4
              const uint32_t a0 = ((nib ? qla >> 4 : qla) & 0x0F0F0F0Fu) | (((qha >> (2 * G)) & 0x03030303u) << 4);
              const uint32_t a1 = ((nib ? qlb >> 4 : qlb) & 0x0F0F0F0Fu) | (((qhb >> (2 * G)) & 0x03030303u) << 4);
              const uint32_t wsa = sg < 4 ? sca4.x : sg < 8 ? sca4.y : sg < 12 ? sca4.z : sca4.w;
              const uint32_t wsb = sg < 4 ? scb4.x : sg < 8 ? scb4.y : sg < 12 ? scb4.z : scb4.w;
              const int sca = (int)(int8_t)(wsa >> (8 * (sg & 3)));
              const int scb = (int)(int8_t)(wsb >> (8 * (sg & 3)));
#pragma unroll
              for (int i = 0; i < NTW; ++i) {
                const int ti = i0 + i;  // token tile
                if (ti >= NT) break;    // uniform across the warp
                const uint2 bv = bs[(ti * 16 + sg) * 32 + lane];
                // sum (q - 32) x per limb: each product starts from -32 x its limb sum
                const int4 sv = ss4[sg * 16 + 4 * ti + c];
                int ch[4] = {sv.x, sv.z, sv.x, sv.z}, cl[4] = {sv.y, sv.w, sv.y, sv.w};
                mma16_u8s8(ch, a0, a1, bv.x);
                mma16_u8u8(cl, a0, a1, bv.y);
                aH[i][0] += sca * ch[0];
                aH[i][1] += sca * ch[1];
                aH[i][2] += scb * ch[2];
                aH[i][3] += scb * ch[3];
                aL[i][0] += sca * cl[0];
                aL[i][1] += sca * cl[1];
                aL[i][2] += scb * cl[2];
                aL[i][3] += scb * cl[3];
              }
            }
          }
        }
      // the superblock scales leave the stage before it is released
      const float da = f16_bits_to_f32(dtile[ra * 8 + (kb & 7)]), db = f16_bits_to_f32(dtile[rb * 8 + (kb & 7)]);
      const float* fsc = reinterpret_cast<const float*>(bsf + St::B + St::S);
      float f[NTW][2];
#pragma unroll
      for (int i = 0; i < NTW; ++i)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tk = 8 * (i0 + i) + 2 * c + e;
          f[i][e] = tk < P.m ? fsc[tk] : 0.f;
        }
      stage_release(&empty[st], lane);
#pragma unroll
      for (int i = 0; i < NTW; ++i) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float va = fmaf(256.f, (float)aH[i][e], (float)aL[i][e]);
          const float vb = fmaf(256.f, (float)aH[i][2 + e], (float)aL[i][2 + e]);
          tot[i][e] = fmaf(f[i][e] * da, va, tot[i][e]);
          tot[i][2 + e] = fmaf(f[i][e] * db, vb, tot[i][2 + e]);
        }
      }
    }
  }

  // ---- this CTA's result for its 128 rows and K range
  const int64_t rowa = row0 + ra, rowb = row0 + rb;
  float* dst = P.splits == 1 ? P.y : P.part + (size_t)sp * P.m * P.n;
  const bool add_bias = P.splits == 1 && P.bias;
#pragma unroll
  for (int i = 0; i < NTW; ++i)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int tk = 8 * (i0 + i) + 2 * c + e;
      if (tk < P.m) {
        // one writer per output; the residual form adds to what y holds (only the last write, splits == 1)
        if (rowa < P.n) {
          float* d = dst + (int64_t)tk * P.n + rowa;
          const float v = tot[i][e] + (add_bias ? P.bias[rowa] : 0.f);
          *d = P.splits == 1 && P.accumulate ? *d + v : v;
        }
        if (rowb < P.n) {
          float* d = dst + (int64_t)tk * P.n + rowb;
          const float v = tot[i][2 + e] + (add_bias ? P.bias[rowb] : 0.f);
          *d = P.splits == 1 && P.accumulate ? *d + v : v;
        }
      }
    }
  if (P.splits == 1) return;
  // split-K: the last CTA of this row tile adds the splits in order
  __threadfence();
  asm volatile("bar.sync 1, %0;" ::"r"(32 * MW) : "memory");
  if (threadIdx.x == 0) last = atomicAdd(P.ctr + blockIdx.x, 1u) == (unsigned)P.splits - 1;
  asm volatile("bar.sync 1, %0;" ::"r"(32 * MW) : "memory");
  if (!last) return;
  __threadfence();
  // a full tile (128 rows, n a multiple of 4): each thread owns up to four
  // 4-row groups of the <= 32 x 128 outputs and reads a split's partials for
  // all of them at once (one memory round trip per split); summation order as
  // in the scalar form (bias, then the splits in order)
  const int rows = (int)(P.n - row0 < IM_ROWS ? P.n - row0 : IM_ROWS);
  if (rows == IM_ROWS && (P.n & 3) == 0 && P.m * (IM_ROWS / 4) <= 32 * MW) {
    // up to 8 tokens: one 4-row group per thread, eight splits' loads in
    // flight per round trip (the same summation order as below)
    const int e = threadIdx.x;
    if (e < P.m * (IM_ROWS / 4)) {
      const int r = 4 * (e & (IM_ROWS / 4 - 1));
      const int64_t off = (int64_t)(e / (IM_ROWS / 4)) * P.n + row0 + r;
      float4 v = P.bias ? make_float4(P.bias[row0 + r], P.bias[row0 + r + 1], P.bias[row0 + r + 2],
                                      P.bias[row0 + r + 3])
                        : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int q = 0; q < P.splits; ++q) {
        const float4 t = __ldcg(reinterpret_cast<const float4*>(P.part + (size_t)q * P.m * P.n + off));
        v.x += t.x;
        v.y += t.y;
        v.z += t.z;
        v.w += t.w;
      }
      float* yo = P.y + off;
      if (P.accumulate) {
        yo[0] += v.x;
        yo[1] += v.y;
        yo[2] += v.z;
        yo[3] += v.w;
      } else {
        yo[0] = v.x;
        yo[1] = v.y;
        yo[2] = v.z;
        yo[3] = v.w;
      }
    }
  } else if (rows == IM_ROWS && (P.n & 3) == 0) {
    constexpr int U = 32 * (IM_ROWS / 4) / (32 * MW);
    const int total4 = P.m * (IM_ROWS / 4);
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = threadIdx.x + u * 32 * MW, r = 4 * (e & (IM_ROWS / 4 - 1));
      v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < total4 && P.bias)
        v[u] = make_float4(P.bias[row0 + r], P.bias[row0 + r + 1], P.bias[row0 + r + 2], P.bias[row0 + r + 3]);
    }
#pragma unroll 2
    for (int q = 0; q < P.splits; ++q) {
      const float* pq = P.part + (size_t)q * P.m * P.n + row0;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int e = threadIdx.x + u * 32 * MW;
        if (e < total4) {
          const float4 t = __ldcg(reinterpret_cast<const float4*>(pq + (int64_t)(e / (IM_ROWS / 4)) * P.n +
                                                                  4 * (e & (IM_ROWS / 4 - 1))));
          v[u].x += t.x;
          v[u].y += t.y;
          v[u].z += t.z;
          v[u].w += t.w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = threadIdx.x + u * 32 * MW;
      if (e < total4) {
        float* yo = P.y + (int64_t)(e / (IM_ROWS / 4)) * P.n + row0 + 4 * (e & (IM_ROWS / 4 - 1));
        if (P.accumulate) {
          yo[0] += v[u].x;
          yo[1] += v[u].y;
          yo[2] += v[u].z;
          yo[3] += v[u].w;
        } else {
          yo[0] = v[u].x;
          yo[1] = v[u].y;
          yo[2] = v[u].z;
          yo[3] = v[u].w;
        }
      }
    }
  } else {
    for (int e = threadIdx.x; e < P.m * rows; e += 32 * MW) {
      const int tk = e / rows, r = e - tk * rows;
      const int64_t idx = (int64_t)tk * P.n + row0 + r;
      float v = P.bias ? P.bias[row0 + r] : 0.f;
      for (int q = 0; q < P.splits; ++q) v += __ldcg(P.part + (size_t)q * P.m * P.n + idx);
      P.y[idx] = P.accumulate ? P.y[idx] + v : v;
    }
  }
  if (threadIdx.x == 0) P.ctr[blockIdx.x] = 0u;  // ready for the next call (stream-ordered)
}

// Ring stages and K-splits: about one CTA per SM, at least 2 superblocks per CTA.
struct ImShape {
  int S, splits, kb_per;
  int stage_bytes, xp_off, xp_stride, bar_off;
  bool ok = true;  // fused: the CTA's prepared K range fits beside a ring of at least two stages
  size_t smem;
};
ImShape im_shape(int qt, int nt, int64_t n, int sb, int num_sms, bool fused = false) {
  ImShape r;
  const int64_t tiles = (n + IM_ROWS - 1) / IM_ROWS;
  const int per_sm = im_ctas_per_sm(nt);
  const int64_t slots = (int64_t)per_sm * num_sms;
  // split-K count: the fewest waves of CTAs x (superblocks per CTA + one for
  // a CTA's fixed start-up) plus the merge (one round trip per 8 splits), fewer
  // splits on a tie
  r.splits = 1;
  r.kb_per = sb;
  int64_t best = INT64_MAX;
  for (int s = 1; s <= sb; ++s) {
    const int per = (sb + s - 1) / s, sp = (sb + per - 1) / per;
    if (sp != s) continue;  // the same split as a smaller count
    const int64_t cost = (tiles * sp + slots - 1) / slots * (per + 1) + (sp + 7) / 8;
    if (cost < best) {
      best = cost;
      r.splits = sp;
      r.kb_per = per;
    }
    if (tiles * sp >= 2 * slots) break;
  }
  const int budget = (per_sm == 2 ? IM_HALF_SMEM : IM_MAX_SMEM) - 2 * 8 * 8;
  if (!fused) {
    const int stage = im_stage_bytes(qt, nt);
    const int fit = budget / (stage + 16);
    r.S = std::max(2, std::min(std::min(fit, 6), r.kb_per));
    r.stage_bytes = stage;
    r.xp_off = r.xp_stride = 0;
    r.bar_off = r.S * stage;
  } else {
    // ring stages hold the weights (and Q6_K's d box) only; the prepared
    // fragments | sums | scales of the CTA's kb_per superblocks sit after them
    const int stage = im_stage_w(qt) + im_stage_d(qt);
    r.xp_stride = nt * 4096 + im_stage_s(qt) + 32 * 4;
    const int xp = r.kb_per * r.xp_stride;
    const int fit = xp < budget ? (budget - xp) / (stage + 16) : 0;
    // and the preparation stays short: one token tile (a 32-token chunk's RMSNorm pass
    // alone reads 32 rows per CTA; measured slower at 8 GPUs, batch 32), at most 8 jobs
    // (token slot x superblock) per MMA warp
    r.ok = fit >= 2 && nt == 1 && r.kb_per <= 8;
    r.S = std::max(2, std::min(std::min(fit, 6), r.kb_per));
    r.stage_bytes = stage;
    r.xp_off = r.S * stage;
    r.bar_off = r.xp_off + xp;
  }
  r.smem = (size_t)r.bar_off + (size_t)2 * r.S * 8;
  return r;
}

struct ImWs {
  size_t bq, ssum, scl, part, end;
};
ImWs im_ws(int64_t m, int64_t n, int64_t k, int num_sms) {
  const int64_t mc = m < 32 ? m : 32;
  const int nt = (int)((mc + 7) / 8);
  const int64_t sb = k / QK;
  ImWs L;
  L.bq = 0;
  L.ssum = (size_t)nt * sb * 4096;
  L.scl = L.ssum + (size_t)sb * 32 * 16 * 8;  // room for Q6_K's 16 groups x two limb sums
  L.part = (L.scl + (size_t)sb * 32 * 4 + 255) & ~size_t(255);
  // partials of the largest chunk: a full 32-token chunk and the tail chunk
  // can split K differently (one or two CTAs per SM); the split count does
  // not depend on the weight type
  size_t part = 0;
  for (const int64_t c : {mc, m > 32 ? m % 32 : (int64_t)0}) {
    if (c <= 0) continue;
    const ImShape sh = im_shape(GGUF_Q4_K, (int)((c + 7) / 8), n, (int)sb, num_sms);
    if (sh.splits > 1) part = std::max(part, (size_t)sh.splits * c * n * 4);
  }
  L.end = L.part + part + 256;
  return L;
}

template <int QT, int NT, bool FUSED>
cudaError_t launch_im(const DevWeight& w, int m, const ImWs& L, void* ws, const float* bias, float* y, unsigned* ctr,
                      int num_sms, int* err, cudaStream_t s, const float* x, const ImOpts& op) {
  const ImShape sh = im_shape(QT, NT, w.n, (int)w.sb, num_sms, FUSED);
  char* base = static_cast<char*>(ws);
  ImParams P;
  P.bq = reinterpret_cast<const uint4*>(base + L.bq);
  P.ssum = reinterpret_cast<const int*>(base + L.ssum);
  P.scl = reinterpret_cast<const float*>(base + L.scl);
  P.bias = bias;
  P.y = y;
  P.part = reinterpret_cast<float*>(base + L.part);
  P.ctr = ctr;
  P.n = w.n;
  P.sb = (int)w.sb;
  P.m = m;
  P.splits = sh.splits;
  P.kb_per = sh.kb_per;
  P.S = sh.S;
  P.accumulate = op.accumulate ? 1 : 0;
  P.err = err;
  P.stage_bytes = sh.stage_bytes;
  P.xp_off = sh.xp_off;
  P.xp_stride = sh.xp_stride;
  P.bar_off = sh.bar_off;
  P.x = x;
  P.x_ld = op.x_ld ? op.x_ld : w.k;
  P.nw = op.nw;
  P.dim = op.dim;
  P.eps = op.eps;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((w.n + IM_ROWS - 1) / IM_ROWS), (unsigned)sh.splits);
  cfg.blockDim = dim3(32 * (im_mma_warps(NT) + 1));
  cfg.dynamicSmemBytes = sh.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, imma_kernel<QT, NT, FUSED>, w.wmap, w.dmap, P);
}

// One chunk of up to 32 tokens: the fused kernel where its shared-memory plan
// fits, else the preparation kernel and the plain one.
template <int QT, int NT>
cudaError_t launch_chunk(const DevWeight& w, int m, const ImWs& L, void* ws, const float* bias, float* y,
                         unsigned* ctr, int num_sms, int* err, cudaStream_t s, const float* x, const ImOpts& op,
                         int* launches, Bracket br) {
  if (im_shape(QT, NT, w.n, (int)w.sb, num_sms, true).ok) {
    bracket_record(br.start, s);
    const cudaError_t e = launch_im<QT, NT, true>(w, m, L, ws, bias, y, ctr, num_sms, err, s, x, op);
    if (e == cudaSuccess && launches) ++*launches;
    bracket_record(br.stop, s);
    return e;
  }
  constexpr int PQT = im_k16(QT) ? GGUF_Q6_K : GGUF_Q4_K;  // Q5_K: the Q4_K preparation, Q3_K the Q6_K one
  const int sb = (int)w.sb, nt = NT;
  const int64_t warps = (int64_t)nt * 8 * sb;
  const int64_t x_ld = op.x_ld ? op.x_ld : w.k;
  char* base = static_cast<char*>(ws);
  cudaError_t e = launch_pdl(imma_prep_kernel<PQT>, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s, x, x_ld, m,
                             nt * 8, w.k, sb, reinterpret_cast<uint4*>(base + L.bq),
                             reinterpret_cast<int*>(base + L.ssum), reinterpret_cast<float*>(base + L.scl), op.nw,
                             op.dim, op.eps);
  if (e != cudaSuccess) return e;
  if (launches) ++*launches;
  bracket_record(br.start, s);
  e = launch_im<QT, NT, false>(w, m, L, ws, bias, y, ctr, num_sms, err, s, x, op);
  if (e == cudaSuccess && launches) ++*launches;
  bracket_record(br.stop, s);
  return e;
}

}  // namespace

template <typename K>
static cudaError_t im_attr(K kernel) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, IM_MAX_SMEM);
}

template <int QT>
static cudaError_t im_attrs() {
  cudaError_t e = cudaSuccess, r;
  if ((r = im_attr(imma_kernel<QT, 1, false>))) e = r;
  if ((r = im_attr(imma_kernel<QT, 2, false>))) e = r;
  if ((r = im_attr(imma_kernel<QT, 3, false>))) e = r;
  if ((r = im_attr(imma_kernel<QT, 4, false>))) e = r;
  if ((r = im_attr(imma_kernel<QT, 1, true>))) e = r;
  if ((r = im_attr(imma_kernel<QT, 2, true>))) e = r;
  if ((r = im_attr(imma_kernel<QT, 3, true>))) e = r;
  if ((r = im_attr(imma_kernel<QT, 4, true>))) e = r;
  return e;
}

cudaError_t imma_init_device() {
  cudaError_t e = im_attrs<GGUF_Q4_K>();
  if (e == cudaSuccess) e = im_attrs<GGUF_Q5_K>();
  if (e == cudaSuccess) e = im_attrs<GGUF_Q3_K>();
  if (e == cudaSuccess) e = im_attrs<GGUF_Q2_K>();
  if (e == cudaSuccess) e = im_attrs<GGUF_Q6_K>();
  return e;
}

size_t imma_workspace_bytes(int64_t m, int64_t n, int64_t k, int num_sms) { return im_ws(m, n, k, num_sms).end; }
size_t imma_counter_bytes(int64_t n) { return (size_t)((n + IM_ROWS - 1) / IM_ROWS) * 4 + 256; }

cudaError_t launch_gemv_imma(const DevWeight& w, const float* x, int64_t m64, const float* bias, float* y, void* ws,
                             unsigned* ctr, int num_sms, int* err, cudaStream_t s, int* launches, Bracket br,
                             const ImOpts& op) {
  if (w.type != GGUF_Q4_K && w.type != GGUF_Q5_K && w.type != GGUF_Q6_K && w.type != GGUF_Q3_K &&
      w.type != GGUF_Q2_K)
    return cudaErrorNotSupported;
  const int64_t x_ld = op.x_ld ? op.x_ld : w.k;
  const ImWs L = im_ws(m64, w.n, w.k, num_sms);
  for (int64_t m0 = 0; m0 < m64; m0 += 32) {
    const int m = (int)((m64 - m0) < 32 ? (m64 - m0) : 32);
    const int nt = (m + 7) / 8;
    const float* xc = x + m0 * x_ld;
    float* yc = y + m0 * w.n;
    cudaError_t e;
#define KQ_IM_CHUNK(QT)                                                                                          \
  switch (nt) {                                                                                                  \
    case 1: e = launch_chunk<QT, 1>(w, m, L, ws, bias, yc, ctr, num_sms, err, s, xc, op, launches, br); break;  \
    case 2: e = launch_chunk<QT, 2>(w, m, L, ws, bias, yc, ctr, num_sms, err, s, xc, op, launches, br); break;  \
    case 3: e = launch_chunk<QT, 3>(w, m, L, ws, bias, yc, ctr, num_sms, err, s, xc, op, launches, br); break;  \
    default: e = launch_chunk<QT, 4>(w, m, L, ws, bias, yc, ctr, num_sms, err, s, xc, op, launches, br); break; \
  }
    if (w.type == GGUF_Q4_K) {
      KQ_IM_CHUNK(GGUF_Q4_K)
    } else if (w.type == GGUF_Q5_K) {
      KQ_IM_CHUNK(GGUF_Q5_K)
    } else if (w.type == GGUF_Q3_K) {
      KQ_IM_CHUNK(GGUF_Q3_K)
    } else if (w.type == GGUF_Q2_K) {
      KQ_IM_CHUNK(GGUF_Q2_K)
    } else {
      KQ_IM_CHUNK(GGUF_Q6_K)
    }
#undef KQ_IM_CHUNK
    br = Bracket();  // only the first chunk is bracketed
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace kq
