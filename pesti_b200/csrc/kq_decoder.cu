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
// split's K and V rows are contiguous in the cache, so they arrive by bulk
// copies (cp.async.bulk) in tiles of AT_TILE positions through a two-stage
// shared-memory ring: tile j + 1 lands while tile j is computed.  Per tile:
// one thread per (query head, position) score -- a 16-byte-chunk walk along
// the K row, rotated by the position so 8 neighbouring threads read 8
// different chunks (no bank conflicts) -- then one warp per query head for
// the online-softmax update, then one thread per (query head, 2 dims) for
// P.V.  With ROPE the kernel also rotates the group's query heads (in shared
// memory: qkv is not written back) and the split holding `pos` appends the
// rotated k and v of the new token to the f16 caches; that row is patched
// into its tile in shared memory (the bulk copies stop before it), so it is
// read as the same f16 values every later step reads.  Each CTA writes one
// partial (max, sum, acc[HD]) per query head; the last CTA of a (token, kv
// head) to finish -- an arrival counter in the scratch, reset by that CTA --
// merges the splits' partials into `out`.
constexpr int AT_THREADS = 256;
constexpr int AT_TILE = 64;  // positions per ring stage
constexpr int ATT_MAX_GROUP = 8;  // query heads per kv head
constexpr int ATT_MAX_SPLITS = 64;
constexpr int ERR_ATT_WAIT = 24;

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
  static constexpr int TILE_B = AT_TILE * HD * 2;  // one K or V tile (f16)
  static constexpr int STAGE = 2 * TILE_B;
  static constexpr int Q = 2 * STAGE;                       // q [G][HD] f32
  static constexpr int S = Q + G * HD * 4;                  // scores / probabilities [G][AT_TILE]
  static constexpr int ML = S + G * AT_TILE * 4;            // running max, sum, tile correction [3][G]
  static constexpr int NEW = ML + ((3 * G * 4 + 15) / 16) * 16;  // appended k | v row, f16
  static constexpr int BAR = NEW + 2 * HD * 2;
  static constexpr int END = BAR + 16;
  // after the last tile the ring is reused by the split merge
  static constexpr int CF = 0;                              // weights [G][ATT_MAX_SPLITS]
  static constexpr int CL = CF + G * ATT_MAX_SPLITS * 4;    // sums [G][ATT_MAX_SPLITS]
  static constexpr int CI = CL + G * ATT_MAX_SPLITS * 4;    // 1 / total sum [G]
  static constexpr int CR = CI + ((G * 4 + 15) / 16) * 16;  // per-warp sums [AT_THREADS / 32][G * HD]
  static_assert(CR + (AT_THREADS / 32) * G * HD * 4 <= 2 * STAGE, "merge scratch exceeds the ring");
};

template <int HD, int G, bool ROPE>
__global__ void __launch_bounds__(AT_THREADS, 2) attn_decode_kernel(const AttnArgs A) {
  using L = AttnSmem<HD, G>;
  constexpr int HALF = HD / 2, C8 = HD / 8;  // C8: 16-byte chunks per f16 row
  constexpr int NPAIR = (G * HALF + AT_THREADS - 1) / AT_THREADS;
  extern __shared__ __align__(128) uint8_t sm[];
  pdl_enter();
  const int hk = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t chunk = (A.len + A.splits - 1) / A.splits;
  const int64_t t0 = min(A.len, (int64_t)sp * chunk), t1 = min(A.len, t0 + chunk);
  const int64_t pos = A.len - 1;
  const bool has_new = ROPE && pos >= t0 && pos < t1;
  const int64_t copy_end = has_new ? pos : t1;  // the bulk copies stop before the appended row
  const int ntiles = (int)((t1 - t0 + AT_TILE - 1) / AT_TILE);
  const float* row = A.q + (int64_t)b * A.q_ld;
  const int64_t base = ((int64_t)b * A.hkv + hk) * A.max_seq * HD;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::BAR);
  float* q_s = reinterpret_cast<float*>(sm + L::Q);
  float* s_s = reinterpret_cast<float*>(sm + L::S);
  float* m_s = reinterpret_cast<float*>(sm + L::ML);
  float* l_s = m_s + G;
  float* c_s = l_s + G;
  __half* new_s = reinterpret_cast<__half*>(sm + L::NEW);

  auto issue = [&](int j) {  // tile j into stage j % 2 (one thread)
    const int64_t r0 = t0 + (int64_t)j * AT_TILE;
    const int64_t r1 = min(copy_end, r0 + AT_TILE);
    const uint32_t bytes = r1 > r0 ? (uint32_t)((r1 - r0) * HD * 2) : 0u;
    sm100::mbar_expect_tx(&bar[j & 1], 2 * bytes);
    if (bytes) {
      uint8_t* st = sm + (j & 1) * L::STAGE;
      sm100::bulk_load(st, A.kc + base + r0 * HD, bytes, &bar[j & 1]);
      sm100::bulk_load(st + L::TILE_B, A.vc + base + r0 * HD, bytes, &bar[j & 1]);
    }
  };
  if (tid == 0) {
    sm100::mbar_init(&bar[0], 1);
    sm100::mbar_init(&bar[1], 1);
    sm100::mbar_fence_init();
    if (ntiles > 0) issue(0);
    if (ntiles > 1) issue(1);
  }
  for (int e = tid; e < G * HALF; e += AT_THREADS) {
    const int g = e / HALF, i = e - g * HALF;
    const float* p = row + (int64_t)(hk * G + g) * HD;
    if constexpr (ROPE) {
      float c, s;
      rope_cs(pos, i, HALF, A.theta, c, s);
      const float a = p[i], bb = p[i + HALF];
      q_s[g * HD + i] = (a * c - bb * s) * A.scale;
      q_s[g * HD + i + HALF] = (a * s + bb * c) * A.scale;
    } else {
      q_s[g * HD + i] = p[i] * A.scale;
      q_s[g * HD + i + HALF] = p[i + HALF] * A.scale;
    }
  }
  if (has_new) {
    const float* kp = row + (int64_t)(A.hq + hk) * HD;
    const float* vp = row + (int64_t)(A.hq + A.hkv + hk) * HD;
    const int64_t o = base + pos * HD;
    for (int i = tid; i < HALF; i += AT_THREADS) {
      float c, s;
      rope_cs(pos, i, HALF, A.theta, c, s);
      const float a = kp[i], bb = kp[i + HALF];
      const __half k0 = __float2half_rn(a * c - bb * s), k1 = __float2half_rn(a * s + bb * c);
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
  float2 acc[NPAIR];
#pragma unroll
  for (int k = 0; k < NPAIR; ++k) acc[k] = make_float2(0.f, 0.f);
  __syncthreads();

  for (int j = 0; j < ntiles; ++j) {
    const int64_t r0 = t0 + (int64_t)j * AT_TILE;
    const int rows = (int)(t1 - r0 < AT_TILE ? t1 - r0 : AT_TILE);
    __half* Ks = reinterpret_cast<__half*>(sm + (j & 1) * L::STAGE);
    __half* Vs = Ks + AT_TILE * HD;
    const bool ok = sm100::mbar_wait(&bar[j & 1], (j >> 1) & 1, A.err, ERR_ATT_WAIT);
    if (!__syncthreads_and(ok)) {
      // give up: let the copies already issued land before the CTA exits
      if (tid == 0 && j + 1 < ntiles) sm100::mbar_wait(&bar[(j + 1) & 1], ((j + 1) >> 1) & 1, A.err, ERR_ATT_WAIT);
      return;
    }
    if (has_new && pos >= r0 && pos < r0 + rows) {
      const int r = (int)(pos - r0);
      for (int i = tid; i < HD; i += AT_THREADS) {
        Ks[r * HD + i] = new_s[i];
        Vs[r * HD + i] = new_s[HD + i];
      }
      __syncthreads();
    }
    // scores of (query head g, position t)
    for (int e = tid; e < G * AT_TILE; e += AT_THREADS) {
      const int g = e / AT_TILE, t = e - g * AT_TILE;
      if (t < rows) {
        const uint4* kr = reinterpret_cast<const uint4*>(Ks + t * HD);
        const float4* qg = reinterpret_cast<const float4*>(q_s + g * HD);
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < C8; ++c) {
          const int cc = (c + t) & (C8 - 1);
          const uint4 kw = kr[cc];
          const float4 qa = qg[2 * cc], qb = qg[2 * cc + 1];
          const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kw.x));
          const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kw.y));
          const float2 k2 = __half22float2(*reinterpret_cast<const __half2*>(&kw.z));
          const float2 k3 = __half22float2(*reinterpret_cast<const __half2*>(&kw.w));
          d = fmaf(qa.x, k0.x, d);
          d = fmaf(qa.y, k0.y, d);
          d = fmaf(qa.z, k1.x, d);
          d = fmaf(qa.w, k1.y, d);
          d = fmaf(qb.x, k2.x, d);
          d = fmaf(qb.y, k2.y, d);
          d = fmaf(qb.z, k3.x, d);
          d = fmaf(qb.w, k3.y, d);
        }
        s_s[g * AT_TILE + t] = d;
      }
    }
    __syncthreads();
    // online softmax: warp g updates query head g
    for (int g = warp; g < G; g += AT_THREADS / 32) {
      const float v0 = lane < rows ? s_s[g * AT_TILE + lane] : -INFINITY;
      const float v1 = lane + 32 < rows ? s_s[g * AT_TILE + lane + 32] : -INFINITY;
      float mx = fmaxf(v0, v1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = m_s[g], mnew = fmaxf(mold, mx);
      const float p0 = lane < rows ? __expf(v0 - mnew) : 0.f;
      const float p1 = lane + 32 < rows ? __expf(v1 - mnew) : 0.f;
      s_s[g * AT_TILE + lane] = p0;
      s_s[g * AT_TILE + lane + 32] = p1;
      float ps = p0 + p1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      if (lane == 0) {
        const float corr = __expf(mold - mnew);  // 0 while mold is -inf
        c_s[g] = corr;
        l_s[g] = l_s[g] * corr + ps;
        m_s[g] = mnew;
      }
    }
    __syncthreads();
    // P.V: thread = (query head g, dims 2 d2, 2 d2 + 1)
#pragma unroll
    for (int k = 0; k < NPAIR; ++k) {
      const int e = tid + k * AT_THREADS;
      if (e < G * HALF) {
        const int g = e / HALF, d2 = e - g * HALF;
        const __half2* vcol = reinterpret_cast<const __half2*>(Vs) + d2;
        const float* pg = s_s + g * AT_TILE;
        const float corr = c_s[g];
        float2 a = make_float2(acc[k].x * corr, acc[k].y * corr);
#pragma unroll 8
        for (int t = 0; t < rows; ++t) {
          const float2 v = __half22float2(vcol[t * HALF]);
          const float p = pg[t];
          a.x = fmaf(p, v.x, a.x);
          a.y = fmaf(p, v.y, a.y);
        }
        acc[k] = a;
      }
    }
    __syncthreads();  // the stage and the scores are free again
    if (tid == 0 && j + 2 < ntiles) issue(j + 2);
  }

  // this split's partial per query head
  constexpr int PS = HD + 4;  // partial row: max, sum, 2 pad, acc[HD] (16-byte aligned)
  float* pb = A.part + ((int64_t)b * A.hq + hk * G) * A.splits * PS;
#pragma unroll
  for (int k = 0; k < NPAIR; ++k) {
    const int e = tid + k * AT_THREADS;
    if (e < G * HALF) {
      const int g = e / HALF, d2 = e - g * HALF;
      *reinterpret_cast<float2*>(pb + ((int64_t)g * A.splits + sp) * PS + 4 + 2 * d2) = acc[k];
    }
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
