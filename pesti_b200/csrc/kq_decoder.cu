// kq_decoder.cu -- the small kernels of a decoder step around the quantized
// linears: RMSNorm, rotary embedding with KV-cache append, decode attention
// over an f16 KV cache, SwiGLU, residual add and embedding lookup.
//
// Semantics follow pesti-runner's CPU decoder (transformer/rms_norm.rs:24-43,
// rope.rs:36-77, layer.rs:16-29,169-244, kv_cache.rs:57-80); the KV cache is
// kept in f16 (values are rounded when appended).  All activations are f32,
// batch-major: x[b][dim].
#include "kq_kernels.h"

#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>

namespace kq {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// out = x / sqrt(mean(x^2) + eps) * w, one CTA per row (rms_norm.rs:24-43).
__global__ void __launch_bounds__(512) rmsnorm_kernel(const float* __restrict__ x, int64_t x_ld,
                                                      const float* __restrict__ w, float* __restrict__ out,
                                                      int64_t out_ld, int dim, float eps) {
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
  const int half = hd / 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y;
  if (idx >= (hq + hkv) * half) return;
  const int head = idx / half, i = idx - head * half;
  const float freq = powf(theta, -(float)i / (float)half);
  const float angle = (float)pos * freq;
  const float c = cosf(angle), s = sinf(angle);
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

// Decode attention, split over the sequence (flash-decoding).  CTA = (kv head,
// split, batch), 4 warps; a warp walks positions of the split, each lane holds
// HD/32 of the head elements of the group's query heads, K/V rows are read as
// coalesced f16 vectors.  Online softmax per query head; the partial (max,
// sum, acc[HD]) per (query head, split) goes to `part`.
constexpr int ATT_WARPS = 4;
constexpr int ATT_MAX_GROUP = 8;  // query heads per kv head

template <int HD>
struct KvQuad;  // HD/32 f16 per lane
template <>
struct KvQuad<128> {
  static constexpr int E = 4;
  __device__ static void load(const __half* p, float (&o)[4]) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  }
};
template <>
struct KvQuad<64> {
  static constexpr int E = 2;
  __device__ static void load(const __half* p, float (&o)[2]) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(p));
    o[0] = a.x; o[1] = a.y;
  }
};

template <int HD, int G>
__global__ void __launch_bounds__(32 * ATT_WARPS) attn_partial_kernel(const float* __restrict__ q, int64_t q_ld,
                                                                      const __half* __restrict__ kc,
                                                                      const __half* __restrict__ vc,
                                                                      float* __restrict__ part, int hq, int hkv,
                                                                      int64_t len, int64_t max_seq, int splits,
                                                                      float scale) {
  using KV = KvQuad<HD>;
  constexpr int E = KV::E;
  const int hk = blockIdx.x, sp = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t chunk = (len + splits - 1) / splits;
  const int64_t t0 = sp * chunk, t1 = min(len, t0 + chunk);
  float qr[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < E; ++j) qr[g][j] = q[(int64_t)b * q_ld + (int64_t)(hk * G + g) * HD + E * lane + j] * scale;
  float m[G], l[G], acc[G][E];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) acc[g][j] = 0.f;
  }
  const int64_t base = ((int64_t)b * hkv + hk) * max_seq * HD;
  for (int64_t t = t0 + warp; t < t1; t += ATT_WARPS) {
    float kv[E], vv[E];
    KV::load(kc + base + t * HD + E * lane, kv);
    KV::load(vc + base + t * HD + E * lane, vv);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sc = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) sc = fmaf(qr[g][j], kv[j], sc);
      sc = warp_sum(sc);
      const float mn = fmaxf(m[g], sc);
      const float corr = __expf(m[g] - mn), p = __expf(sc - mn);
      l[g] = l[g] * corr + p;
#pragma unroll
      for (int j = 0; j < E; ++j) acc[g][j] = acc[g][j] * corr + p * vv[j];
      m[g] = mn;
    }
  }
  // combine the 4 warps through shared memory, then one partial per query head
  __shared__ float sm_m[ATT_WARPS][G], sm_l[ATT_WARPS][G];
  __shared__ float sm_acc[ATT_WARPS][G][HD];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      sm_m[warp][g] = m[g];
      sm_l[warp][g] = l[g];
    }
#pragma unroll
    for (int j = 0; j < E; ++j) sm_acc[warp][g][E * lane + j] = acc[g][j];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
    const int g = e / HD, d = e - g * HD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) mx = fmaxf(mx, sm_m[w][g]);
    float ls = 0.f, as = 0.f;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) {
      const float f = sm_m[w][g] == -INFINITY ? 0.f : __expf(sm_m[w][g] - mx);
      ls += sm_l[w][g] * f;
      as += sm_acc[w][g][d] * f;
    }
    float* pp = part + ((((int64_t)b * hq + hk * G + g) * splits + sp) * (HD + 2));
    pp[2 + d] = as;
    if (d == 0) {
      pp[0] = mx;
      pp[1] = ls;
    }
  }
}

// out[b][h][d] = sum_s acc_s[d] e^(m_s - M) / sum_s l_s e^(m_s - M).
// Grid b * hq + h, HD threads.
__global__ void attn_combine_kernel(const float* __restrict__ part, float* __restrict__ out, int64_t out_ld, int hq,
                                    int hd, int splits) {
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / hq, h = bh - b * hq;
  const int d = threadIdx.x;
  const float* pp = part + bh * splits * (hd + 2);
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, pp[s * (hd + 2)]);
  float ls = 0.f, as = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = pp[s * (hd + 2)];
    const float f = ms == -INFINITY ? 0.f : __expf(ms - mx);
    ls += pp[s * (hd + 2) + 1] * f;
    as += pp[s * (hd + 2) + 2 + d] * f;
  }
  out[b * out_ld + h * hd + d] = as / ls;
}

// SwiGLU over a fused [gate | up] row per token.  mode 0 is pesti's CPU
// function (layer.rs:16-29): for gate < 0 its "sigmoid" is g / (1 + e^g), so
// out = (g / (1 + e^g)) * g * u; mode 1 is SiLU, sigmoid(g) * g * u.
__global__ void swiglu_kernel(const float* __restrict__ gu, float* __restrict__ out, int64_t ffn, int64_t total,
                              int mode) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = e / ffn, i = e - b * ffn;
    const float g = gu[b * 2 * ffn + i], u = gu[b * 2 * ffn + ffn + i];
    float sg;
    if (g >= 0.f || mode == 1) sg = 1.f / (1.f + expf(-g));
    else sg = g / (1.f + expf(g));
    out[e] = sg * g * u;
  }
}

// h[r][c] += y[r][c] for c < cols.
__global__ void add_kernel(float* __restrict__ h, int64_t h_ld, const float* __restrict__ y, int64_t y_ld,
                           int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / cols, c = e - r * cols;
    h[r * h_ld + c] += y[r * y_ld + c];
  }
}

__global__ void embed_kernel(const float* __restrict__ table, const int* __restrict__ tokens,
                             float* __restrict__ out, int64_t out_ld, int64_t dim) {
  const int64_t tok = tokens[blockIdx.y];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += (int64_t)gridDim.x * blockDim.x)
    out[(int64_t)blockIdx.y * out_ld + i] = table[tok * dim + i];
}

template <int HD, int G>
cudaError_t launch_attn_g(const float* q, int64_t q_ld, const __half* kc, const __half* vc, float* part, int hq,
                          int hkv, int64_t len, int64_t max_seq, int splits, int64_t batch, cudaStream_t s) {
  dim3 grid((unsigned)hkv, (unsigned)splits, (unsigned)batch);
  attn_partial_kernel<HD, G><<<grid, 32 * ATT_WARPS, 0, s>>>(q, q_ld, kc, vc, part, hq, hkv, len, max_seq, splits,
                                                              1.f / sqrtf((float)HD));
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_attn_hd(const float* q, int64_t q_ld, const __half* kc, const __half* vc, float* part, int hq,
                           int hkv, int64_t len, int64_t max_seq, int splits, int64_t batch, cudaStream_t s) {
  switch (hq / hkv) {
    case 1: return launch_attn_g<HD, 1>(q, q_ld, kc, vc, part, hq, hkv, len, max_seq, splits, batch, s);
    case 2: return launch_attn_g<HD, 2>(q, q_ld, kc, vc, part, hq, hkv, len, max_seq, splits, batch, s);
    case 4: return launch_attn_g<HD, 4>(q, q_ld, kc, vc, part, hq, hkv, len, max_seq, splits, batch, s);
    case 7: return launch_attn_g<HD, 7>(q, q_ld, kc, vc, part, hq, hkv, len, max_seq, splits, batch, s);
    case 8: return launch_attn_g<HD, 8>(q, q_ld, kc, vc, part, hq, hkv, len, max_seq, splits, batch, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t dec_rmsnorm(const float* x, int64_t x_ld, const float* w, float* out, int64_t out_ld, int64_t rows,
                        int64_t dim, float eps, cudaStream_t s) {
  if (rows < 1 || dim < 1) return cudaSuccess;
  rmsnorm_kernel<<<(unsigned)rows, 512, 0, s>>>(x, x_ld, w, out, out_ld, (int)dim, eps);
  return cudaGetLastError();
}

cudaError_t dec_rope_append(float* qkv, int64_t ld, void* kc, void* vc, int64_t batch, int hq, int hkv, int hd,
                            int64_t pos, int64_t max_seq, float theta, cudaStream_t s) {
  const int work = (hq + hkv) * (hd / 2);
  dim3 grid((unsigned)((work + 255) / 256), (unsigned)batch);
  rope_append_kernel<<<grid, 256, 0, s>>>(qkv, ld, static_cast<__half*>(kc), static_cast<__half*>(vc), hq, hkv, hd,
                                         pos, max_seq, theta);
  return cudaGetLastError();
}

int dec_attention_splits(int64_t batch, int hkv, int64_t len, int num_sms) {
  const int64_t ctas = batch * hkv;
  int64_t sp = (2 * (int64_t)num_sms + ctas - 1) / ctas;
  sp = std::min<int64_t>(sp, (len + 31) / 32);
  return (int)std::max<int64_t>(1, std::min<int64_t>(sp, 64));
}

size_t dec_attention_scratch_bytes(int64_t batch, int hq, int hd, int splits) {
  return (size_t)batch * hq * splits * (hd + 2) * sizeof(float);
}

cudaError_t dec_attention(const float* q, int64_t q_ld, const void* kc, const void* vc, float* out, int64_t out_ld,
                          int64_t batch, int hq, int hkv, int hd, int64_t len, int64_t max_seq, float* scratch,
                          int splits, cudaStream_t s) {
  if ((hd != 64 && hd != 128) || hkv < 1 || hq % hkv || hq / hkv > ATT_MAX_GROUP || len < 1 || splits < 1)
    return cudaErrorInvalidValue;
  const __half* k = static_cast<const __half*>(kc);
  const __half* v = static_cast<const __half*>(vc);
  cudaError_t e = hd == 128 ? launch_attn_hd<128>(q, q_ld, k, v, scratch, hq, hkv, len, max_seq, splits, batch, s)
                            : launch_attn_hd<64>(q, q_ld, k, v, scratch, hq, hkv, len, max_seq, splits, batch, s);
  if (e != cudaSuccess) return e;
  attn_combine_kernel<<<(unsigned)(batch * hq), hd, 0, s>>>(scratch, out, out_ld, hq, hd, splits);
  return cudaGetLastError();
}

cudaError_t dec_swiglu(const float* gu, float* out, int64_t batch, int64_t ffn, int mode, cudaStream_t s) {
  const int64_t total = batch * ffn;
  if (total < 1) return cudaSuccess;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 4096);
  swiglu_kernel<<<blocks, 256, 0, s>>>(gu, out, ffn, total, mode);
  return cudaGetLastError();
}

cudaError_t dec_add(float* h, int64_t h_ld, const float* y, int64_t y_ld, int64_t rows, int64_t cols,
                    cudaStream_t s) {
  const int64_t n = rows * cols;
  if (n < 1) return cudaSuccess;
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 4096);
  add_kernel<<<blocks, 256, 0, s>>>(h, h_ld, y, y_ld, rows, cols);
  return cudaGetLastError();
}

cudaError_t dec_embed(const float* table, const int* tokens, float* out, int64_t out_ld, int64_t batch, int64_t dim,
                      cudaStream_t s) {
  dim3 grid((unsigned)std::min<int64_t>((dim + 255) / 256, 64), (unsigned)batch);
  embed_kernel<<<grid, 256, 0, s>>>(table, tokens, out, out_ld, dim);
  return cudaGetLastError();
}

}  // namespace kq
