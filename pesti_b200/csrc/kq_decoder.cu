// kq_decoder.cu -- the small kernels of a decoder step around the quantized
// linears: RMSNorm, rotary embedding with KV-cache append, decode attention
// over an f16 KV cache, SwiGLU, residual add and embedding lookup.
//
// Semantics follow pesti-runner's CPU decoder (transformer/rms_norm.rs:24-43,
// rope.rs:36-77, layer.rs:16-29,169-244, kv_cache.rs:57-80); the KV cache is
// kept in f16 (values are rounded when appended).  All activations are f32,
// batch-major: x[b][dim].
#include "kq_common.cuh"
#include "kq_kernels.h"
#include "kq_sm100.cuh"

#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>

namespace kq {
namespace {

// Each kernel lets the next one launch at once and waits for its own
// predecessor only before touching memory (programmatic dependent launch).
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// cos / sin of the rotary angle of pair i at position pos (rope.rs:36-77).
__device__ __forceinline__ void rope_cs(int64_t pos, int i, int half, float theta, float& c, float& s) {
  const float freq = powf(theta, -(float)i / (float)half);
  const float angle = (float)pos * freq;
  c = cosf(angle);
  s = sinf(angle);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// out = x / sqrt(mean(x^2) + eps) * w, one CTA per row (rms_norm.rs:24-43).
__global__ void __launch_bounds__(512) rmsnorm_kernel(const float* __restrict__ x, int64_t x_ld,
                                                      const float* __restrict__ w, float* __restrict__ out,
                                                      int64_t out_ld, int dim, float eps) {
  pdl_enter();
  const float* xr = x + (int64_t)blockIdx.x * x_ld;
  float* orow = out + (int64_t)blockIdx.x * out_ld;
  float s = 0.f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
  __shared__ float red[32];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rms = sqrtf(red[0] / (float)dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) orow[i] = xr[i] / rms * w[i];
}

// Rotary embedding (pairs i, i + hd/2; angle = pos * base^(-i/(hd/2)), rope.rs:36-77)
// of the q heads in place and of the k heads, then k and v appended to the f16
// caches at `pos`.  Token b's row qkv + b*ld holds q (hq heads), k (hkv), v (hkv).
// One thread per (head, i < hd/2) of q heads then kv heads; grid.y = batch.
__global__ void __launch_bounds__(256) rope_append_kernel(float* __restrict__ qkv, int64_t ld,
                                                          __half* __restrict__ kc, __half* __restrict__ vc, int hq,
                                                          int hkv, int hd, int64_t pos, int64_t max_seq,
                                                          float theta) {
  pdl_enter();
  const int half = hd / 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (idx >= (hq + hkv) * half) return;
  const int head = idx / half, i = idx - head * half;
  float c, s;
  rope_cs(pos, i, half, theta, c, s);
  float* row = qkv + (int64_t)b * ld;
  if (head < hq) {
    float* p = row + (int64_t)head * hd;
    const float a = p[i], bb = p[i + half];
    p[i] = a * c - bb * s;
    p[i + half] = a * s + bb * c;
  } else {
    const int h = head - hq;
    const float* kp = row + (int64_t)(hq + h) * hd;
    const float* vp = row + (int64_t)(hq + hkv + h) * hd;
    const float a = kp[i], bb = kp[i + half];
    const int64_t o = (((int64_t)b * hkv + h) * max_seq + pos) * hd;
    kc[o + i] = __float2half_rn(a * c - bb * s);
    kc[o + i + half] = __float2half_rn(a * s + bb * c);
    vc[o + i] = __float2half_rn(vp[i]);
    vc[o + i + half] = __float2half_rn(vp[i + half]);
  }
}

// Decode attention, split over the sequence (flash-decoding), in one kernel.
// CTA = (kv head, split, token), 256 threads, about two CTAs per SM.  The
// split's K and V rows arrive in tiles of AT_TILE positions through a
// two-stage shared-memory ring filled with 16-byte cp.async copies (all
// threads; tile j + 2 is issued once tile j is consumed), into rows padded to
// HD * 2 + 16 bytes so that the eight rows a warp's fragment loads touch sit
// on different banks.  Both products run on the tensor cores
// (mma.sync.m16n8k16, f16 inputs, f32 accumulate) with the group's query
// heads as the M rows (G <= 8 of 16; the other rows are zero):
//  * scores: warp w takes positions 8w .. 8w+7 of the tile; A = q, B = K^T
//    read straight from the K rows.  q enters as two f16 parts (hi, and the
//    f16 rounding of q - hi) after scaling each head by a power of two that
//    puts its largest |q| in [2^14, 2^15), so the f16 products carry q to
//    about 2^-22 of that head's largest element;
//  * online softmax: one warp per query head over the tile, as before;
//  * P.V: warp w takes head dims 16w .. 16w+15; A = the probabilities (hi and
//    lo f16 parts again), B = V through ldmatrix.trans.
// With ROPE the kernel also rotates the group's query heads (in shared
// memory: qkv is not written back) and the split holding `pos` appends the
// rotated k and v of the new token to the f16 caches; that row is patched
// into its tile in shared memory (the copies skip it), so it is read as the
// same f16 values every later step reads.  Each CTA writes one partial (max,
// sum, acc[HD]) per query head; the last CTA of a (token, kv head) to finish
// -- an arrival counter in the scratch, reset by that CTA -- merges the
// splits' partials into `out`.  No wait in the kernel spins: the ring is
// ordered by cp.async groups and block barriers.
constexpr int AT_THREADS = 256;
constexpr int AT_TILE = 64;  // positions per ring stage
constexpr int AT_STAGES = 2;  // ring stages: one tile in flight while one is multiplied
constexpr int ATT_MAX_GROUP = 8;  // query heads per kv head
constexpr int ATT_MAX_SPLITS = 64;

struct AttnArgs {
  const float* q;     // token b's query heads at q + b * q_ld (ROPE: the fused qkv row)
  int64_t q_ld;
  __half* kc;         // [batch][hkv][max_seq][HD]
  __half* vc;
  float* part;        // [batch][hq][splits][HD + 4]: max, sum, 2 pad, acc[HD]
  unsigned* ctr;      // [batch][hkv] arrival counters, zero between calls
  float* out;         // token b's heads at out + b * out_ld
  int64_t out_ld;
  int hq, hkv;
  int64_t len, max_seq;  // positions [0, len); ROPE: the new token sits at len - 1
  int splits;
  float theta, scale;
  int* err;
};

// Dynamic shared memory of the decode-attention kernel (bytes).
template <int HD, int G>
struct AttnSmem {
  static constexpr int PITCH = HD * 2 + 16;        // bytes per K / V row in shared memory
  static constexpr int TILE_B = AT_TILE * PITCH;   // one K or V tile
  static constexpr int STAGE = 2 * TILE_B;
  static constexpr int Q = AT_STAGES * STAGE;               // q [G][HD] f32
  static constexpr int SP = AT_TILE + 8;                    // score row pitch (floats): rows 8 banks apart
  static constexpr int S = Q + G * HD * 4;                  // scores / probabilities [G][SP]
  static constexpr int ML = S + G * SP * 4;                 // running max, sum, tile correction, q scale [4][G]
  static constexpr int NEW = ML + ((4 * G * 4 + 15) / 16) * 16;  // appended k | v row, f16
  static constexpr int END = NEW + 2 * HD * 2;
  // after the last tile the ring is reused by the split merge
  static constexpr int CF = 0;                              // weights [G][ATT_MAX_SPLITS]
  static constexpr int CL = CF + G * ATT_MAX_SPLITS * 4;    // sums [G][ATT_MAX_SPLITS]
  static constexpr int CI = CL + G * ATT_MAX_SPLITS * 4;    // 1 / total sum [G]
  static constexpr int CR = CI + ((G * 4 + 15) / 16) * 16;  // per-warp sums [AT_THREADS / 32][G * HD]
  static_assert(CR + (AT_THREADS / 32) * G * HD * 4 <= AT_STAGES * STAGE, "merge scratch exceeds the ring");
  static_assert(HD / 16 <= AT_THREADS / 32 && AT_TILE == 8 * (AT_THREADS / 32), "warp roles");
};

__device__ __forceinline__ void at_cp16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sm100::smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void at_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// this thread's copies of the oldest pending tile have landed (the AT_STAGES - 1 newer groups may be in flight)
__device__ __forceinline__ void at_wait_tile() {
  asm volatile("cp.async.wait_group %0;" ::"n"(AT_STAGES - 1) : "memory");
}

// f16 pair {hi(a), hi(b)} and the pair of remainders {a - hi(a), b - hi(b)}, low half = a
__device__ __forceinline__ void at_split(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const __half2 l = __floats2half2_rn(a - __low2float(h), b - __high2float(h));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// D = A . B + D, m16n8k16, f16 inputs, f32 accumulate; A rows 8..15 are zero here
__device__ __forceinline__ void at_mma(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void at_ldm_x4_trans(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(sm100::smem_u32(p))
               : "memory");
}

template <int HD, int G, bool ROPE>
__global__ void __launch_bounds__(AT_THREADS, 2) attn_decode_kernel(const AttnArgs A) {
  using L = AttnSmem<HD, G>;
  constexpr int HALF = HD / 2, CH = HD / 8, KS = HD / 16, PITCH = L::PITCH;
  extern __shared__ __align__(128) uint8_t sm[];
  pdl_enter();
  const int hk = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;  // fragment row (query head) and column pair
  const int64_t chunk = (A.len + A.splits - 1) / A.splits;
  const int64_t t0 = min(A.len, (int64_t)sp * chunk), t1 = min(A.len, t0 + chunk);
  const int64_t pos = A.len - 1;
  const bool has_new = ROPE && pos >= t0 && pos < t1;
  const int ntiles = (int)((t1 - t0 + AT_TILE - 1) / AT_TILE);
  const float* row = A.q + (int64_t)b * A.q_ld;
  const int64_t base = ((int64_t)b * A.hkv + hk) * A.max_seq * HD;
  float* q_s = reinterpret_cast<float*>(sm + L::Q);
  float* s_s = reinterpret_cast<float*>(sm + L::S);
  float* m_s = reinterpret_cast<float*>(sm + L::ML);
  float* l_s = m_s + G;
  float* c_s = l_s + G;
  float* x_s = c_s + G;  // 2^e of each head's q scaling
  __half* new_s = reinterpret_cast<__half*>(sm + L::NEW);

  // tile j into stage j % AT_STAGES (every thread issues its share, then one group);
  // rows past the split and the appended row are zero-filled (the latter is
  // patched in from new_s)
  auto issue = [&](int j) {
    const int64_t r0 = t0 + (int64_t)j * AT_TILE;
    uint8_t* st = sm + (j % AT_STAGES) * L::STAGE;
    for (int e = tid; e < 2 * AT_TILE * CH; e += AT_THREADS) {
      const int kv = e / (AT_TILE * CH), rem = e - kv * (AT_TILE * CH);
      const int r = rem / CH, ch = rem - r * CH;
      const int64_t t = r0 + r;
      const bool live = t < t1 && !(has_new && t == pos);
      const __half* src = (kv ? A.vc : A.kc) + base + (live ? t : t0) * HD + ch * 8;
      at_cp16(st + kv * L::TILE_B + r * PITCH + ch * 16, src, live ? 16u : 0u);
    }
    at_commit();
  };
#pragma unroll
  for (int j = 0; j < AT_STAGES; ++j) {
    if (j < ntiles) issue(j); else at_commit();  // one group per stage, empty past the split
  }

  for (int e = tid; e < G * HALF; e += AT_THREADS) {
    const int gg = e / HALF, i = e - gg * HALF;
    const float* p = row + (int64_t)(hk * G + gg) * HD;
    if constexpr (ROPE) {
      float cs, sn;
      rope_cs(pos, i, HALF, A.theta, cs, sn);
      const float a = p[i], bb = p[i + HALF];
      q_s[gg * HD + i] = (a * cs - bb * sn) * A.scale;
      q_s[gg * HD + i + HALF] = (a * sn + bb * cs) * A.scale;
    } else {
      q_s[gg * HD + i] = p[i] * A.scale;
      q_s[gg * HD + i + HALF] = p[i + HALF] * A.scale;
    }
  }
  if (has_new) {
    const float* kp = row + (int64_t)(A.hq + hk) * HD;
    const float* vp = row + (int64_t)(A.hq + A.hkv + hk) * HD;
    const int64_t o = base + pos * HD;
    for (int i = tid; i < HALF; i += AT_THREADS) {
      float cs, sn;
      rope_cs(pos, i, HALF, A.theta, cs, sn);
      const float a = kp[i], bb = kp[i + HALF];
      const __half k0 = __float2half_rn(a * cs - bb * sn), k1 = __float2half_rn(a * sn + bb * cs);
      const __half v0 = __float2half_rn(vp[i]), v1 = __float2half_rn(vp[i + HALF]);
      A.kc[o + i] = k0;
      A.kc[o + i + HALF] = k1;
      A.vc[o + i] = v0;
      A.vc[o + i + HALF] = v1;
      new_s[i] = k0;
      new_s[i + HALF] = k1;
      new_s[HD + i] = v0;
      new_s[HD + i + HALF] = v1;
    }
  }
  if (tid < G) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  __syncthreads();
  // each head's power-of-two q scale: largest |q| 2^-e in [2^14, 2^15)
  if (warp < G) {
    float mx = 0.f;
    for (int i = lane; i < HD; i += 32) mx = fmaxf(mx, fabsf(q_s[warp * HD + i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) {
      int e = 0;
      if (mx > 0.f && mx <= 3.4e38f) e = (int)((__float_as_uint(mx) >> 23) & 0xff) - 127 - 14;
      e = max(-126, min(126, e));
      x_s[warp] = __uint_as_float((uint32_t)(127 + e) << 23);
    }
  }
  __syncthreads();
  // q as A fragments (rows = query heads): hi and lo f16 parts, 2 registers per k16 step
  uint32_t qh[KS][2], ql[KS][2];
  {
    const float inv = g < G ? 1.f / x_s[g] : 0.f;  // a power of two: exact
#pragma unroll
    for (int kk = 0; kk < KS; ++kk)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int d = 16 * kk + 8 * h + 2 * c;
        const float v0 = g < G ? q_s[g * HD + d] * inv : 0.f, v1 = g < G ? q_s[g * HD + d + 1] * inv : 0.f;
        at_split(v0, v1, qh[kk][h], ql[kk][h]);
      }
  }
  float o[2][4];  // P.V accumulators: head g, dims 16 warp + 8 t + 2c, +1
#pragma unroll
  for (int t = 0; t < 2; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;

  for (int j = 0; j < ntiles; ++j) {
    const int64_t r0 = t0 + (int64_t)j * AT_TILE;
    const int rows = (int)(t1 - r0 < AT_TILE ? t1 - r0 : AT_TILE);
    uint8_t* Ks = sm + (j % AT_STAGES) * L::STAGE;
    uint8_t* Vs = Ks + L::TILE_B;
    at_wait_tile();  // this thread's copies of tile j have landed (later tiles may be in flight)
    __syncthreads();
    if (has_new && pos >= r0 && pos < r0 + rows) {
      const int r = (int)(pos - r0);
      for (int i = tid; i < HD; i += AT_THREADS) {
        reinterpret_cast<__half*>(Ks + r * PITCH)[i] = new_s[i];
        reinterpret_cast<__half*>(Vs + r * PITCH)[i] = new_s[HD + i];
      }
      __syncthreads();
    }
    // scores of (query head g, positions 8 warp + 2c, +1)
    {
      const uint8_t* kt = Ks + (8 * warp + g) * PITCH + 4 * c;
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kt + 32 * kk);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kt + 32 * kk + 16);
        at_mma(sc, qh[kk][0], qh[kk][1], b0, b1);
        at_mma(sc, ql[kk][0], ql[kk][1], b0, b1);
      }
      if (g < G) {
        const float xs = x_s[g];
        *reinterpret_cast<float2*>(s_s + g * L::SP + 8 * warp + 2 * c) = make_float2(sc[0] * xs, sc[1] * xs);
      }
    }
    __syncthreads();
    // online softmax: warp gg updates query head gg
    for (int gg = warp; gg < G; gg += AT_THREADS / 32) {
      const float v0 = lane < rows ? s_s[gg * L::SP + lane] : -INFINITY;
      const float v1 = lane + 32 < rows ? s_s[gg * L::SP + lane + 32] : -INFINITY;
      float mx = fmaxf(v0, v1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mold = m_s[gg], mnew = fmaxf(mold, mx);
      const float p0 = lane < rows ? __expf(v0 - mnew) : 0.f;
      const float p1 = lane + 32 < rows ? __expf(v1 - mnew) : 0.f;
      s_s[gg * L::SP + lane] = p0;
      s_s[gg * L::SP + lane + 32] = p1;
      float ps = p0 + p1;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
      if (lane == 0) {
        const float corr = __expf(mold - mnew);  // 0 while mold is -inf
        c_s[gg] = corr;
        l_s[gg] = l_s[gg] * corr + ps;
        m_s[gg] = mnew;
      }
    }
    __syncthreads();
    // P.V: warp w owns head dims 16w .. 16w+15 (two n8 tiles)
    if (warp < HD / 16) {
      const float corr = g < G ? c_s[g] : 0.f;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        o[t][0] *= corr;
        o[t][1] *= corr;
      }
      const int mat = lane >> 3, rr = lane & 7;
      const uint8_t* va = Vs + ((mat & 1) * 8 + rr) * PITCH + (16 * warp + (mat >> 1) * 8) * 2;
#pragma unroll
      for (int kk = 0; kk < AT_TILE / 16; ++kk) {
        const float2 pa = g < G ? *reinterpret_cast<const float2*>(s_s + g * L::SP + 16 * kk + 2 * c)
                                : make_float2(0.f, 0.f);
        const float2 pb = g < G ? *reinterpret_cast<const float2*>(s_s + g * L::SP + 16 * kk + 8 + 2 * c)
                                : make_float2(0.f, 0.f);
        uint32_t ph0, pl0, ph2, pl2;
        at_split(pa.x, pa.y, ph0, pl0);
        at_split(pb.x, pb.y, ph2, pl2);
        uint32_t v0, v1, v2, v3;
        at_ldm_x4_trans(va + 16 * kk * PITCH, v0, v1, v2, v3);
        at_mma(o[0], ph0, ph2, v0, v1);
        at_mma(o[0], pl0, pl2, v0, v1);
        at_mma(o[1], ph0, ph2, v2, v3);
        at_mma(o[1], pl0, pl2, v2, v3);
      }
    }
    __syncthreads();  // the stage and the scores are free again
    if (j + AT_STAGES < ntiles) issue(j + AT_STAGES); else at_commit();
  }

  // this split's partial per query head
  constexpr int PS = HD + 4;  // partial row: max, sum, 2 pad, acc[HD] (16-byte aligned)
  float* pb = A.part + ((int64_t)b * A.hq + hk * G) * A.splits * PS;
  if (warp < HD / 16 && g < G) {
#pragma unroll
    for (int t = 0; t < 2; ++t)
      *reinterpret_cast<float2*>(pb + ((int64_t)g * A.splits + sp) * PS + 4 + 16 * warp + 8 * t + 2 * c) =
          make_float2(o[t][0], o[t][1]);
  }
  if (tid < G) *reinterpret_cast<float2*>(pb + ((int64_t)tid * A.splits + sp) * PS) = make_float2(m_s[tid], l_s[tid]);
  // the last CTA of (token, kv head) merges the splits
  __shared__ int last;
  __threadfence();
  __syncthreads();
  unsigned* ctr = A.ctr + (int64_t)b * A.hkv + hk;
  if (tid == 0) last = atomicAdd(ctr, 1u) == (unsigned)A.splits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  float* f_s = reinterpret_cast<float*>(sm + L::CF);
  float* l2 = reinterpret_cast<float*>(sm + L::CL);
  float* inv_l = reinterpret_cast<float*>(sm + L::CI);
  float* red = reinterpret_cast<float*>(sm + L::CR);
  // (1) every split's max and sum
  for (int e = tid; e < G * A.splits; e += AT_THREADS) {
    const int g = e / A.splits, s2 = e - g * A.splits;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(pb + ((int64_t)g * A.splits + s2) * PS));
    f_s[g * ATT_MAX_SPLITS + s2] = ml.x;
    l2[g * ATT_MAX_SPLITS + s2] = ml.y;
  }
  __syncthreads();
  // (2) warp g: the splits' weights e^(m_s - M) and 1 / sum_s l_s e^(m_s - M)
  for (int g = warp; g < G; g += AT_THREADS / 32) {
    float* fg = f_s + g * ATT_MAX_SPLITS;
    const float* lg = l2 + g * ATT_MAX_SPLITS;
    const bool v0 = lane < A.splits, v1 = lane + 32 < A.splits;
    const float a0 = v0 ? fg[lane] : -INFINITY, a1 = v1 ? fg[lane + 32] : -INFINITY;
    float mx = fmaxf(a0, a1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float f0 = a0 == -INFINITY ? 0.f : __expf(a0 - mx), f1 = a1 == -INFINITY ? 0.f : __expf(a1 - mx);
    if (v0) fg[lane] = f0;
    if (v1) fg[lane + 32] = f1;
    float ls = (v0 ? f0 * lg[lane] : 0.f) + (v1 ? f1 * lg[lane + 32] : 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    if (lane == 0) inv_l[g] = 1.f / ls;
  }
  __syncthreads();
  // (3) warp w sums splits w, w + 8, ...; lane c takes float4 columns c, c + 32, ... of [G][HD]
  constexpr int C4 = G * HD / 4, PER = (C4 + 31) / 32;
  float4 a[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) a[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 2
  for (int s2 = warp; s2 < A.splits; s2 += AT_THREADS / 32) {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int c = lane + 32 * k;
      if (c < C4) {
        const int g = c / (HD / 4), d4 = c - g * (HD / 4);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(pb + ((int64_t)g * A.splits + s2) * PS + 4) + d4);
        const float f = f_s[g * ATT_MAX_SPLITS + s2];
        a[k].x = fmaf(v.x, f, a[k].x);
        a[k].y = fmaf(v.y, f, a[k].y);
        a[k].z = fmaf(v.z, f, a[k].z);
        a[k].w = fmaf(v.w, f, a[k].w);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = lane + 32 * k;
    if (c < C4) reinterpret_cast<float4*>(red + warp * G * HD)[c] = a[k];
  }
  __syncthreads();
  for (int e = tid; e < G * HD; e += AT_THREADS) {
    const int g = e / HD, d = e - g * HD;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < AT_THREADS / 32; ++w) v += red[w * G * HD + e];
    A.out[(int64_t)b * A.out_ld + (int64_t)(hk * G + g) * HD + d] = v * inv_l[g];
  }
  if (tid == 0) *ctr = 0u;  // ready for the next call (stream-ordered)
}

// SwiGLU over a fused [gate | up] row per token.  mode 0 is pesti's CPU
// function (layer.rs:16-29): for gate < 0 its "sigmoid" is g / (1 + e^g), so
// out = (g / (1 + e^g)) * g * u; mode 1 is SiLU, sigmoid(g) * g * u.
__global__ void swiglu_kernel(const float* __restrict__ gu, float* __restrict__ out, int64_t ffn, int64_t total,
                              int mode) {
  pdl_enter();
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = e / ffn, i = e - b * ffn;
    const float g = gu[b * 2 * ffn + i], u = gu[b * 2 * ffn + ffn + i];
    out[e] = swiglu_gate(g, mode) * u;
  }
}

// h[r][c] += y[r][c] for c < cols.
__global__ void add_kernel(float* __restrict__ h, int64_t h_ld, const float* __restrict__ y, int64_t y_ld,
                           int64_t rows, int64_t cols) {
  pdl_enter();
  const int64_t n = rows * cols;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / cols, c = e - r * cols;
    h[r * h_ld + c] += y[r * y_ld + c];
  }
}

__global__ void embed_kernel(const float* __restrict__ table, const int* __restrict__ tokens,
                             float* __restrict__ out, int64_t out_ld, int64_t dim) {
  pdl_enter();
  const int64_t tok = tokens[blockIdx.y];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += (int64_t)gridDim.x * blockDim.x)
    out[(int64_t)blockIdx.y * out_ld + i] = table[tok * dim + i];
}

template <int HD, int G>
cudaError_t launch_attn_g(const AttnArgs& a, bool rope, int64_t batch, cudaStream_t s) {
  dim3 grid((unsigned)a.hkv, (unsigned)a.splits, (unsigned)batch);
  constexpr size_t smem = AttnSmem<HD, G>::END;
  return rope ? launch_pdl(attn_decode_kernel<HD, G, true>, grid, dim3(AT_THREADS), smem, s, a)
              : launch_pdl(attn_decode_kernel<HD, G, false>, grid, dim3(AT_THREADS), smem, s, a);
}

template <int HD, int G>
cudaError_t attn_attrs() {
  constexpr int smem = AttnSmem<HD, G>::END;
  cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<HD, G, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_decode_kernel<HD, G, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  return e;
}

template <int HD>
cudaError_t attn_attrs_hd() {
  cudaError_t e = attn_attrs<HD, 1>();
  if (e == cudaSuccess) e = attn_attrs<HD, 2>();
  if (e == cudaSuccess) e = attn_attrs<HD, 4>();
  if (e == cudaSuccess) e = attn_attrs<HD, 7>();
  if (e == cudaSuccess) e = attn_attrs<HD, 8>();
  return e;
}

template <int HD>
cudaError_t launch_attn_hd(const AttnArgs& a, bool rope, int64_t batch, cudaStream_t s) {
  switch (a.hq / a.hkv) {
    case 1: return launch_attn_g<HD, 1>(a, rope, batch, s);
    case 2: return launch_attn_g<HD, 2>(a, rope, batch, s);
    case 4: return launch_attn_g<HD, 4>(a, rope, batch, s);
    case 7: return launch_attn_g<HD, 7>(a, rope, batch, s);
    case 8: return launch_attn_g<HD, 8>(a, rope, batch, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t dec_rmsnorm(const float* x, int64_t x_ld, const float* w, float* out, int64_t out_ld, int64_t rows,
                        int64_t dim, float eps, cudaStream_t s) {
  if (rows < 1 || dim < 1) return cudaSuccess;
  return launch_pdl(rmsnorm_kernel, dim3((unsigned)rows), dim3(512), 0, s, x, x_ld, w, out, out_ld, (int)dim, eps);
}

cudaError_t dec_rope_append(float* qkv, int64_t ld, void* kc, void* vc, int64_t batch, int hq, int hkv, int hd,
                            int64_t pos, int64_t max_seq, float theta, cudaStream_t s) {
  const int work = (hq + hkv) * (hd / 2);
  dim3 grid((unsigned)((work + 255) / 256), (unsigned)batch);
  return launch_pdl(rope_append_kernel, grid, dim3(256), 0, s, qkv, ld, static_cast<__half*>(kc),
                    static_cast<__half*>(vc), hq, hkv, hd, pos, max_seq, theta);
}

cudaError_t dec_init_device() {
  cudaError_t e = attn_attrs_hd<128>();
  if (e == cudaSuccess) e = attn_attrs_hd<64>();
  return e;
}

// About two CTAs per SM over all (token, kv head) pairs, at least 16
// positions per split.
int dec_attention_splits(int64_t batch, int hkv, int64_t len, int num_sms) {
  const int64_t ctas = batch * hkv;
  int64_t sp = 2 * (int64_t)num_sms / ctas;
  sp = std::min<int64_t>(sp, (len + 15) / 16);
  return (int)std::max<int64_t>(1, std::min<int64_t>(sp, ATT_MAX_SPLITS));
}

// Scratch: the arrival counters [batch][hkv] u32 (zero before the first
// call; every call leaves them zero), then from a 256-byte boundary the
// partials [batch][hq][splits][hd + 4] f32.  The counters' place does not
// depend on the split count, which grows with the sequence length.
static size_t attn_part_offset(int64_t batch, int hkv) {
  return ((size_t)batch * hkv * sizeof(unsigned) + 255) & ~size_t(255);
}

size_t dec_attention_scratch_bytes(int64_t batch, int hq, int hkv, int hd, int splits) {
  return attn_part_offset(batch, hkv) + (size_t)batch * hq * splits * (hd + 4) * sizeof(float);
}

cudaError_t dec_attention(const float* q, int64_t q_ld, void* kc, void* vc, float* out, int64_t out_ld,
                          int64_t batch, int hq, int hkv, int hd, int64_t len, int64_t max_seq, void* scratch,
                          int splits, bool rope, float theta, int* err, cudaStream_t s) {
  if ((hd != 64 && hd != 128) || hkv < 1 || hq % hkv || hq / hkv > ATT_MAX_GROUP || len < 1 || splits < 1 ||
      splits > ATT_MAX_SPLITS)
    return cudaErrorInvalidValue;
  AttnArgs a;
  a.q = q;
  a.q_ld = q_ld;
  a.kc = static_cast<__half*>(kc);
  a.vc = static_cast<__half*>(vc);
  a.ctr = static_cast<unsigned*>(scratch);
  a.part = reinterpret_cast<float*>(static_cast<char*>(scratch) + attn_part_offset(batch, hkv));
  a.out = out;
  a.out_ld = out_ld;
  a.hq = hq;
  a.hkv = hkv;
  a.len = len;
  a.max_seq = max_seq;
  a.splits = splits;
  a.theta = theta;
  a.scale = 1.f / sqrtf((float)hd);
  a.err = err;
  return hd == 128 ? launch_attn_hd<128>(a, rope, batch, s) : launch_attn_hd<64>(a, rope, batch, s);
}

cudaError_t dec_swiglu(const float* gu, float* out, int64_t batch, int64_t ffn, int mode, cudaStream_t s) {
  const int64_t total = batch * ffn;
  if (total < 1) return cudaSuccess;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 4096);
  return launch_pdl(swiglu_kernel, dim3(blocks), dim3(256), 0, s, gu, out, ffn, total, mode);
}

cudaError_t dec_add(float* h, int64_t h_ld, const float* y, int64_t y_ld, int64_t rows, int64_t cols,
                    cudaStream_t s) {
  const int64_t n = rows * cols;
  if (n < 1) return cudaSuccess;
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 4096);
  return launch_pdl(add_kernel, dim3(blocks), dim3(256), 0, s, h, h_ld, y, y_ld, rows, cols);
}

cudaError_t dec_embed(const float* table, const int* tokens, float* out, int64_t out_ld, int64_t batch, int64_t dim,
                      cudaStream_t s) {
  dim3 grid((unsigned)std::min<int64_t>((dim + 255) / 256, 64), (unsigned)batch);
  return launch_pdl(embed_kernel, grid, dim3(256), 0, s, table, tokens, out, out_ld, dim);
}

}  // namespace kq
