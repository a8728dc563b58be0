// kq_step.cu -- one batch-1 decode step as a single persistent kernel.
//
// A step program is a list of stages, built once per model on the host
// (kq_step_* in include/pesti_decoder.h):
//   GEMV  y = act(x) . W^T for a GGUF Q4_K / Q6_K weight, with the work split
//         and integer arithmetic of the single-token kernel (kq_dp4a.cu).
//         x is staged PLAIN, NORM (RMSNorm folded into a per-row output
//         scale) or REDUCE(_NORM): x = the sum, in rank order, of the parts
//         every rank sent in the pending exchange (the new residual), also
//         written to h_out.  y is written STORE, SWIGLU ((gate, up) row pairs)
//         or PARTIAL: this rank's part of a residual update, stored as
//         exchange words into every rank's buffer; rank 0's part carries the
//         residual being updated, so the parts sum to the new residual.
//   ATTN  RoPE of the new token's q and k, the KV append, and split-sequence
//         GQA attention over the f16 cache, merged per KV head by the last
//         CTA to finish it.
// One CTA per SM runs every stage (cooperative launch: all CTAs are resident).
// A producer warp streams the bytes every stage of this CTA reads -- weight
// rows, then its KV tile -- through one shared-memory ring, in program order.
// Weights and the cache prefix do not depend on the step's activations, so
// the producer runs ahead of the compute warps across stage boundaries: while
// the compute warps wait on a dependency, the next stages' bytes are landing.
// Dependencies:
//   * a stage that reads a vector other CTAs produced in this launch (qkv ->
//     attention, attention -> output projection, SwiGLU -> down projection)
//     starts after a grid barrier (arrival counter, bounded acquire spin);
//   * a REDUCE stage waits only on the exchange words it reads: each word
//     carries its exchange's epoch.  The residual itself travels in rank 0's
//     words: the CTA that adds residual element i into its part is the one
//     that wrote element i to h_out in the REDUCE before (both stages split
//     the vector by the same 4-aligned partition), so no CTA reads another
//     CTA's residual slice.
// Ring slots hold 2G rows of a GEMV stage (as the single-token kernel) or one
// KV tile, and are released with a proxy fence before the producer's next
// bulk copy overwrites them.  Every wait is bounded and reports through the
// error word; the producer drains its copies before the CTA exits.
#include "kq_common.cuh"
#include "kq_kernels.h"
#include "kq_xs.cuh"

#include <cuda_fp16.h>
#include <math.h>

#include <algorithm>

namespace kq {
namespace {

constexpr int SP_NC = STEP_COMPUTE_WARPS;  // compute warps
constexpr int SP_CT = 32 * SP_NC;          // compute threads
constexpr int SP_SPW = 8;                  // superblocks per warp K-slice
constexpr uint32_t SP_SPIN = 1u << 22;     // bound of the barrier / exchange spins
enum : int { SP_ERR_FULL = 41, SP_ERR_EMPTY = 42, SP_ERR_DRAIN = 43, SP_ERR_BAR = 44, SP_ERR_TP = 45 };

__device__ __forceinline__ void sp_sync() { xs_named_sync(1, SP_CT); }

// Optional trace (a profiling hook): global timer stamps per CTA and stage,
// STEP_TRACE_POINTS of them: before the barrier, after it, after the input
// staging (attention: the query rotation), after the weight loop
// (attention: once the first KV tile has landed), after the outputs
// (attention: after the KV loop), at the stage's end.
__device__ __forceinline__ void sp_stamp(const StepArgs& A, int si, int k) {
  if (A.trace && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    A.trace[((size_t)blockIdx.x * A.nstages + si) * STEP_TRACE_POINTS + k] = t;
  }
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool err_set(const int* err) { return *(const volatile int*)err != 0; }

// All compute threads: this CTA's writes so far are published, then wait for
// every CTA to arrive `target` times in total.
__device__ void sp_grid_sync(unsigned* ctr, unsigned target, int* err) {
  sp_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ctr, 1u);
    for (uint32_t i = 0;; ++i) {  // one poller per CTA: no back-off
      if (ld_acquire(ctr) >= target) break;
      if (i >= SP_SPIN || ((i & 255u) == 255u && err_set(err))) {
        atomicCAS(err, 0, SP_ERR_BAR);
        break;
      }
    }
    __threadfence();
  }
  sp_sync();
}

// Rows [r0, r1) of a GEMV stage owned by CTA b of C: a contiguous block;
// SWIGLU keeps (gate, up) pairs together, PARTIAL uses the 4-aligned split
// that the REDUCE staging uses for its slice of h_out.
__device__ __forceinline__ void sp_rows(const StepStage& S, int b, int C, int64_t& r0, int64_t& r1) {
  if (S.ymode == SY_SWIGLU) {
    r0 = 2 * ((int64_t)(S.n / 2) * b / C);
    r1 = 2 * ((int64_t)(S.n / 2) * (b + 1) / C);
  } else if (S.ymode == SY_PARTIAL) {
    r0 = 4 * ((int64_t)(S.n / 4) * b / C);
    r1 = b == C - 1 ? S.n : 4 * ((int64_t)(S.n / 4) * (b + 1) / C);
  } else {
    r0 = (int64_t)S.n * b / C;
    r1 = (int64_t)S.n * (b + 1) / C;
  }
}

// Splits of each KV head's positions: at least SP_ATT_MIN positions each (a
// split is one CTA's work; fewer, longer splits keep the merge short), at most
// the stage's bound (the CTAs per KV head).
constexpr int SP_ATT_MIN = 64;
__device__ __forceinline__ int sp_attn_splits(const StepStage& S, int64_t len) {
  return (int)max((int64_t)1, min((int64_t)S.splits, (len + SP_ATT_MIN - 1) / SP_ATT_MIN));
}
// Attention item of CTA b: (kv head, split) and its positions [t0, t1).
__device__ __forceinline__ bool sp_attn_item(const StepStage& S, int b, int64_t len, int& hk, int64_t& t0,
                                             int64_t& t1) {
  const int splits = sp_attn_splits(S, len);
  if (b >= S.hkv * splits) return false;
  hk = b / splits;
  const int sp = b - hk * splits;
  const int64_t chunk = (len + splits - 1) / splits;
  t0 = min(len, (int64_t)sp * chunk);
  t1 = min(len, t0 + chunk);
  return true;
}

// ---------------------------------------------------------------------------
// producer: every stage's bytes for this CTA, in program order
// ---------------------------------------------------------------------------
constexpr int64_t SP_PF_CHUNK = 64 * 1024;     // bytes per L2 prefetch instruction
constexpr int64_t SP_PF_MAX = 384 * 1024;      // at most this much of a stage per CTA

__device__ __forceinline__ void sp_prefetch_range(const uint8_t* p, int64_t bytes) {
  bytes &= ~int64_t(15);  // whole 16-byte units only: nothing past the range is touched
  for (int64_t o = 0; o < bytes; o += SP_PF_CHUNK) {
    const uint32_t n = (uint32_t)min(SP_PF_CHUNK, bytes - o);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + o), "r"(n) : "memory");
  }
}

// L2 prefetch of the bytes CTA b will copy for stage S (its rows, or its KV
// tile), up to SP_PF_MAX bytes.
__device__ void sp_prefetch_l2(const StepStage& S, const StepArgs& A, int b, int C) {
  if (S.kind == STEP_GEMV) {
    int64_t r0, r1;
    sp_rows(S, b, C, r0, r1);
    const int64_t rows = r1 - r0;
    sp_prefetch_range(S.q + r0 * S.row_bytes, min(rows * S.row_bytes, SP_PF_MAX));
    if (S.d_row_bytes)
      sp_prefetch_range(reinterpret_cast<const uint8_t*>(S.d) + r0 * S.d_row_bytes, rows * S.d_row_bytes);
  } else {
    int hk;
    int64_t t0, t1;
    if (!sp_attn_item(S, b, A.pos + 1, hk, t0, t1)) return;
    const int64_t rowb = (int64_t)S.hd * 2, off = ((int64_t)hk * S.max_seq + t0) * rowb;
    const int64_t bytes = min((t1 - t0) * rowb, SP_PF_MAX / 2);
    sp_prefetch_range(static_cast<const uint8_t*>(S.kc) + off, bytes);
    sp_prefetch_range(static_cast<const uint8_t*>(S.vc) + off, bytes);
  }
}
__device__ void sp_produce(const StepArgs& A, const StepSmem& L, uint8_t* sm) {
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint64_t* empty = full + A.S;
  const int b = blockIdx.x, C = gridDim.x;
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  uint32_t seq = 0;
  bool ok = true;
  auto take = [&](uint32_t bytes) -> uint8_t* {  // the next slot, once free; expects `bytes`
    const int st = (int)(seq % (uint32_t)A.S);
    if (seq >= (uint32_t)A.S && !xs_bar_wait(&empty[st], ((seq / A.S) - 1) & 1, A.err, SP_ERR_EMPTY)) {
      ok = false;  // the consumers gave up: issue nothing more
      return nullptr;
    }
    xs_bar_expect(&full[st], bytes);
    return sm + L.ring + (size_t)st * A.slot_bytes;
  };
  for (int si = 0; si < A.nstages && ok; ++si) {
    const StepStage& S = A.stages[si];
    // the next stage's bytes of this CTA into L2 now, so HBM keeps streaming
    // while the compute warps wait on this stage's dependencies
    if (si + 1 < A.nstages) sp_prefetch_l2(A.stages[si + 1], A, b, C);
    if (S.kind == STEP_GEMV) {
      int64_t r0, r1;
      sp_rows(S, b, C, r0, r1);
      const int rows = (int)(r1 - r0), R = 2 * S.G;
      for (int t = 0; t * R < rows && ok; ++t) {
        const int nr = min(R, rows - t * R);
        const int64_t row = r0 + (int64_t)t * R;
        const uint32_t wb = (uint32_t)(nr * S.row_bytes), db = (uint32_t)(nr * S.d_row_bytes);
        uint8_t* dst = take(wb + db);
        if (!dst) break;
        const int st = (int)(seq % (uint32_t)A.S);
        xs_bulk_g2s(dst, S.q + row * S.row_bytes, wb, &full[st], pol);
        if (db) xs_bulk_g2s(dst + (size_t)R * S.row_bytes, reinterpret_cast<const uint8_t*>(S.d) + row * S.d_row_bytes,
                            db, &full[st], pol);
        ++seq;
      }
    } else {
      int hk;
      int64_t t0, t1;
      if (!sp_attn_item(S, b, A.pos + 1, hk, t0, t1)) continue;
      const int64_t rowb = (int64_t)S.hd * 2;
      for (int64_t p0 = t0; p0 < t1 && ok; p0 += S.tile) {
        const int np = (int)min((int64_t)S.tile, t1 - p0);
        const uint32_t bytes = (uint32_t)(np * rowb);
        const int64_t off = ((int64_t)hk * S.max_seq + p0) * rowb;
        for (int kv = 0; kv < 2; ++kv) {  // the K tile, then the V tile
          uint8_t* dst = take(bytes);
          if (!dst) break;
          const int st = (int)(seq % (uint32_t)A.S);
          xs_bulk_g2s_plain(dst, static_cast<const uint8_t*>(kv ? S.vc : S.kc) + off, bytes, &full[st]);
          ++seq;
        }
      }
    }
  }
  // the CTA must not retire while a copy into its shared memory is in flight
  for (uint32_t v = seq > (uint32_t)A.S ? seq - A.S : 0; v < seq; ++v)
    xs_bar_wait(&full[v % A.S], (v / A.S) & 1, A.err, SP_ERR_DRAIN);
}

// Consumer side of one ring slot: wait until it is full (every compute warp).
__device__ __forceinline__ bool sp_wait_full(const StepArgs& A, uint64_t* full, uint32_t seq) {
  return __all_sync(0xffffffffu, xs_bar_wait(&full[seq % A.S], (seq / A.S) & 1, A.err, SP_ERR_FULL));
}
// Release a slot (one arrival per compute warp): generic reads of it are
// ordered before the producer's next bulk copy into it.
__device__ __forceinline__ void sp_release(const StepArgs& A, uint64_t* empty, uint32_t seq) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if ((threadIdx.x & 31) == 0) xs_bar_arrive(&empty[seq % A.S]);
}

// ---------------------------------------------------------------------------
// GEMV stage
// ---------------------------------------------------------------------------

// Stage x of a GEMV stage into shared memory as the single-token kernel does
// (15-bit hi / lo bytes per superblock, swizzled in the order lanes read
// them; Q4_K exact f32 sub-block sums, Q6_K -32 * byte sums).  REDUCE first
// sums the exchange's parts (rank order) into xr and writes this CTA's slice
// to h_out.  NORM copies the norm weights to shared memory first and leaves
// per-warp sum(x^2) in red.
template <int QT>
__device__ void sp_stage_x(const StepStage& S, const StepArgs& A, const StepSmem& L, uint8_t* sm, unsigned ep0) {
  uint4* xw = reinterpret_cast<uint4*>(sm + L.xw);
  float* xsf = reinterpret_cast<float*>(sm + L.xsf);
  float* xr = reinterpret_cast<float*>(sm + L.xr);
  const int lane = threadIdx.x & 31;
  const bool reduce = S.xmode == SX_REDUCE || S.xmode == SX_REDUCE_NORM;
  const bool norm = S.xmode == SX_NORM || S.xmode == SX_REDUCE_NORM;
  float* nws = reinterpret_cast<float*>(sm + L.nw);
  if (norm && !reduce)  // the norm weights are read-only: their copy does not wait on anything
    for (int i = 4 * threadIdx.x; i < S.dim; i += 4 * SP_CT)
      *reinterpret_cast<float4*>(nws + i) = __ldg(reinterpret_cast<const float4*>(S.nw + i));
  if (reduce) {
    const unsigned epoch = ep0 + 1u + (unsigned)S.exch;
    const unsigned long long* img = A.exch[A.rank] + (size_t)(epoch & 1u) * (size_t)A.slot_elems;
    const int q4 = S.dim / 4, C = gridDim.x, b = blockIdx.x;
    const int lo = 4 * (int)((int64_t)q4 * b / C), hi = b == C - 1 ? S.dim : 4 * (int)((int64_t)q4 * (b + 1) / C);
    bool ok = !err_set(A.err);
    // every rank's parts of this thread's 8-element groups (one per thread for
    // vectors up to 3840 elements), summed in rank order (every rank sums the
    // same way); a rank's eight words are re-read only while one still
    // carries an older epoch
    for (int i = 8 * threadIdx.x; i < S.dim; i += 8 * SP_CT) {
      // the norm weights of these elements are loaded while the words are polled
      float4 nw0 = make_float4(0.f, 0.f, 0.f, 0.f), nw1 = nw0;
      if (norm) {
        nw0 = __ldg(reinterpret_cast<const float4*>(S.nw + i));
        nw1 = __ldg(reinterpret_cast<const float4*>(S.nw + i + 4));
      }
      float p[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < A.world; ++r) {
        const unsigned long long* wp = img + (size_t)r * S.dim + i;
        unsigned long long w[8];
        for (uint32_t it = 0;; ++it) {
#pragma unroll
          for (int c = 0; c < 8; c += 2) ld_words2(wp + c, w[c], w[c + 1]);
          bool ready = true;
#pragma unroll
          for (int c = 0; c < 8; ++c) ready = ready && (unsigned)(w[c] >> 32) == epoch;
          if (ready || !ok) break;
          if (it >= SP_SPIN || ((it & 255u) == 255u && err_set(A.err))) {
            atomicCAS(A.err, 0, SP_ERR_TP);  // the output is invalid; the kernel still runs to its end
            ok = false;
            break;
          }
          if (it >= 64) __nanosleep(64);
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) p[c] += __uint_as_float((unsigned)w[c]);
      }
      const float4 a = make_float4(p[0], p[1], p[2], p[3]), b4 = make_float4(p[4], p[5], p[6], p[7]);
      *reinterpret_cast<float4*>(xr + i) = a;
      *reinterpret_cast<float4*>(xr + i + 4) = b4;
      if (norm) {
        *reinterpret_cast<float4*>(nws + i) = nw0;
        *reinterpret_cast<float4*>(nws + i + 4) = nw1;
      }
      if (i >= lo && i < hi) *reinterpret_cast<float4*>(S.h_out + i) = a;
      if (i + 4 >= lo && i + 4 < hi) *reinterpret_cast<float4*>(S.h_out + i + 4) = b4;
    }
  }
  if (reduce || norm) sp_sync();
  float ss = 0.f;
  const int total = SP_SPW * S.nk * 8;  // half-units (32 weights each), a multiple of 64
  for (int base = (threadIdx.x & ~31); base < total; base += SP_CT) {
    const int hu = base + lane;
    const int kb = hu >> 3, u = (hu >> 1) & 3, hf = hu & 1;
    const bool live = kb < S.sb;
    float v[32];  // Q4: [0,16) sub-block 2u run, [16,32) sub-block 2u+1 run; Q6: group (g, w) at 8g + 4w
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int off;
      if constexpr (QT == GGUF_Q4_K) off = 64 * u + 16 * hf + (i < 4 ? 4 * i : 32 + 4 * (i - 4));
      else off = 128 * hf + 32 * (i >> 1) + 8 * u + 4 * (i & 1);
      const int64_t gi = (int64_t)kb * 256 + off;
      float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
      if (live && (!norm && !reduce || gi < S.dim)) {
        f = reduce ? *reinterpret_cast<const float4*>(xr + gi) : __ldcg(reinterpret_cast<const float4*>(S.x + gi));
        if (norm) {
          const float4 wv = *reinterpret_cast<const float4*>(nws + gi);
          ss = fmaf(f.x, f.x, fmaf(f.y, f.y, fmaf(f.z, f.z, fmaf(f.w, f.w, ss))));
          f.x *= wv.x;
          f.y *= wv.y;
          f.z *= wv.z;
          f.w *= wv.w;
        }
      }
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const XScale sc = xs_scale(amax);
    uint4* unit = xw + (size_t)(kb * 4 + u) * 8;
    const int sw = xs_swz(kb, u);
    if constexpr (QT == GGUF_Q4_K) {
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
      sa += __shfl_xor_sync(0xffffffffu, sa, 1);
      sbb += __shfl_xor_sync(0xffffffffu, sbb, 1);
      if (hf == 0) reinterpret_cast<float2*>(sm + L.sums)[kb * 4 + u] = make_float2(sa, sbb);
    } else {
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
      int4* so = reinterpret_cast<int4*>(sm + L.sums) + (size_t)(kb * 4 + u) * 4 + 2 * hf;
      so[0] = make_int4(-32 * shs[0], -32 * shs[1], -32 * shs[2], -32 * shs[3]);
      so[1] = make_int4(-32 * sls[0], -32 * sls[1], -32 * sls[2], -32 * sls[3]);
    }
    if ((hu & 7) == 0) xsf[kb] = live ? sc.factor : 0.f;
  }
  if (norm) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) reinterpret_cast<float*>(sm + L.red)[threadIdx.x >> 5] = ss;
  }
}

// One row of a warp's K-slice (lane's unit of superblock kb), as the
// single-token kernel computes it; 0 for lanes past the row's end.
template <int QT>
__device__ __forceinline__ float sp_row_partial(const uint8_t* rowp, const uint8_t* drow, int kb, int u, bool live,
                                                const uint4 (&X)[8], float xf, float sa, float sbb,
                                                const int (&Sh)[2][4], const int (&Sl)[2][4], uint32_t sel_lo,
                                                uint32_t sel_hi) {
  if (!live) return 0.f;
  if constexpr (QT == GGUF_Q4_K) {
    const uint8_t* blk = rowp + kb * Q4K_BYTES;
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * u);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * u);
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const uint32_t W[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int ahi = 0, alo = 0, bhi = 0, blo = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t qa4 = W[w] & 0x0F0F0F0Fu, qb16 = W[w] & 0xF0F0F0F0u;
      ahi = dp4a_s(qa4, X[w].x, ahi);
      alo = dp4a_u(qa4, X[w].y, alo);
      bhi = dp4a_us(qb16, X[w].z, bhi);
      blo = dp4a_u(qb16, X[w].w, blo);
    }
    const bool hi4 = u >= 2;
    const int sh = 16 * (u & 1);
    const uint32_t s0 = hdr.y, s1 = hdr.z, s2 = hdr.w;
    uint32_t scp, mp;
    if (!hi4) {
      scp = (s0 >> sh) & 0x3F3Fu;
      mp = (s1 >> sh) & 0x3F3Fu;
    } else {
      scp = ((s2 >> sh) & 0x0F0Fu) | ((s0 >> (sh + 2)) & 0x3030u);
      mp = ((s2 >> (sh + 4)) & 0x0F0Fu) | ((s1 >> (sh + 2)) & 0x3030u);
    }
    const int da = ahi * 256 + alo, db = (bhi * 256 + blo) >> 4;
    const int iv = (int)(scp & 0xffu) * da + (int)(scp >> 8) * db;
    const float d = f16_bits_to_f32((uint16_t)(hdr.x & 0xffff));
    const float dmin = f16_bits_to_f32((uint16_t)(hdr.x >> 16));
    const float msum = fmaf((float)(mp & 0xffu), sa, (float)(mp >> 8) * sbb);
    return fmaf(d * xf, (float)iv, -dmin * msum);
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
    int ih = 0, il = 0;
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
        const int scv = (int)prmt(SCW[2 * h + (gg >> 1)], 0u, (gg & 1) ? sel_hi : sel_lo);
        ih += scv * hi[gg];
        il += scv * lo[gg];
      }
    }
    return fmaf(256.f, (float)ih, (float)il) * (f16_bits_to_f32(dbits) * xf);
  }
}

template <int QT>
__device__ void sp_gemv(const StepStage& S, const StepArgs& A, const StepSmem& L, uint8_t* sm, uint32_t& seq,
                        unsigned ep0, int si) {
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint64_t* empty = full + A.S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t r0, r1;
  sp_rows(S, blockIdx.x, gridDim.x, r0, r1);
  const int rows = (int)(r1 - r0), R = 2 * S.G, T = (rows + R - 1) / R, NC = S.nk * S.G;
  const bool norm = S.xmode == SX_NORM || S.xmode == SX_REDUCE_NORM;

  sp_stage_x<QT>(S, A, L, sm, ep0);
  sp_sync();
  sp_stamp(A, si, 2);
  float yscale = 1.f;  // RMSNorm: 1 / sqrt(mean(x^2) + eps), applied to every output row
  if (norm) {
    const float* red = reinterpret_cast<const float*>(sm + L.red);
    float t = 0.f;
    for (int w = 0; w < SP_NC; ++w) t += red[w];
    yscale = 1.f / sqrtf(t / (float)S.dim + S.eps);
  }
  float* part = reinterpret_cast<float*>(sm + L.part);
  if (warp < NC) {
    const int s = warp % S.nk, g = warp / S.nk;
    const int kb = SP_SPW * s + (lane >> 2), u = lane & 3;
    const bool live = kb < S.sb;
    uint4 X[8];
    {
      const uint4* unit = reinterpret_cast<const uint4*>(sm + L.xw) + (size_t)(kb * 4 + u) * 8;
      const int sw = xs_swz(kb, u);
#pragma unroll
      for (int j = 0; j < 8; ++j) X[j] = unit[j ^ sw];
    }
    const float xf = reinterpret_cast<const float*>(sm + L.xsf)[kb];
    float sa = 0.f, sbb = 0.f;
    int Sh[2][4] = {}, Sl[2][4] = {};
    uint32_t sel_lo = 0, sel_hi = 0;
    if constexpr (QT == GGUF_Q4_K) {
      const float2 t = reinterpret_cast<const float2*>(sm + L.sums)[kb * 4 + u];
      sa = t.x;
      sbb = t.y;
    } else {
      const int4* si = reinterpret_cast<const int4*>(sm + L.sums) + (size_t)(kb * 4 + u) * 4;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int4 a = si[2 * h], c = si[2 * h + 1];
        Sh[h][0] = a.x; Sh[h][1] = a.y; Sh[h][2] = a.z; Sh[h][3] = a.w;
        Sl[h][0] = c.x; Sl[h][1] = c.y; Sl[h][2] = c.z; Sl[h][3] = c.w;
      }
      const uint32_t b0 = (uint32_t)(u >> 1), b2 = b0 + 2;
      sel_lo = b0 | ((b0 | 8) << 4) | ((b0 | 8) << 8) | ((b0 | 8) << 12);
      sel_hi = b2 | ((b2 | 8) << 4) | ((b2 | 8) << 8) | ((b2 | 8) << 12);
    }
    for (int t = 0; t < T; ++t) {
      if (!sp_wait_full(A, full, seq + t)) break;
      const uint8_t* stage = sm + L.ring + (size_t)((seq + t) % A.S) * A.slot_bytes;
      const uint8_t* dstage = stage + (size_t)R * S.row_bytes;
      const int q0 = t * R + g, q1 = q0 + S.G;
      const float v0 = q0 < rows ? sp_row_partial<QT>(stage + (size_t)g * S.row_bytes, dstage + (size_t)g * S.d_row_bytes,
                                                      kb, u, live, X, xf, sa, sbb, Sh, Sl, sel_lo, sel_hi)
                                 : 0.f;
      const float v1 = q1 < rows ? sp_row_partial<QT>(stage + (size_t)(g + S.G) * S.row_bytes,
                                                      dstage + (size_t)(g + S.G) * S.d_row_bytes, kb, u, live, X, xf,
                                                      sa, sbb, Sh, Sl, sel_lo, sel_hi)
                                 : 0.f;
      const bool upper = lane & 16;
      float keep = upper ? v1 : v0;
      keep += __shfl_xor_sync(0xffffffffu, upper ? v0 : v1, 16);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
      if (lane == 0 && q0 < rows) part[q0 * S.nk + s] = keep;
      if (lane == 16 && q1 < rows) part[q1 * S.nk + s] = keep;
      sp_release(A, empty, seq + t);
    }
  } else {
    for (int t = 0; t < T; ++t) {  // idle in this stage: release each slot once it has landed
      if (!sp_wait_full(A, full, seq + t)) break;
      sp_release(A, empty, seq + t);
    }
  }
  seq += (uint32_t)T;
  sp_sync();
  sp_stamp(A, si, 3);
  const int tid = threadIdx.x;
  if (S.ymode == SY_SWIGLU) {
    for (int j = tid; 2 * j < rows; j += SP_CT) {
      float gv = 0.f, uv = 0.f;
      for (int t = 0; t < S.nk; ++t) {
        gv += part[(2 * j) * S.nk + t];
        uv += part[(2 * j + 1) * S.nk + t];
      }
      S.y[r0 / 2 + j] = swiglu_gate(gv * yscale, S.act) * (uv * yscale);
    }
  } else if (S.ymode == SY_STORE) {
    for (int q = tid; q < rows; q += SP_CT) {
      float acc = 0.f;
      for (int t = 0; t < S.nk; ++t) acc += part[q * S.nk + t];
      S.y[r0 + q] = acc * yscale;
    }
  } else {
    // this rank's partial: rows [r0, r1) of the exchange's rank block, to every rank
    const unsigned epoch = ep0 + 1u + (unsigned)S.exch;
    const unsigned long long tag = (unsigned long long)epoch << 32;
    const size_t at = (size_t)(epoch & 1u) * (size_t)A.slot_elems + (size_t)A.rank * S.n + r0;
    // rank 0 adds the residual being updated; its rows [r0, r1) are the slice
    // this CTA itself wrote (or the launch's input)
    const float* res = A.rank == 0 ? S.h_in : nullptr;
    for (int q = tid; q < rows; q += SP_CT) {
      float acc = 0.f;
      for (int t = 0; t < S.nk; ++t) acc += part[q * S.nk + t];
      float v = acc * yscale;
      if (res) v = __ldcg(res + r0 + q) + v;
      const unsigned long long wv = tag | __float_as_uint(v);
      for (int p = 0; p < A.world; ++p) st_word(A.exch[p] + at + q, wv);
    }
  }
  sp_stamp(A, si, 4);
}

// ---------------------------------------------------------------------------
// attention stage (batch 1, f32 arithmetic on f16 K / V)
// ---------------------------------------------------------------------------

// cos / sin of the rotary angle of pair i at position pos (rope.rs:36-77)
__device__ __forceinline__ void sp_rope_cs(int64_t pos, int i, int half, float theta, float& c, float& s) {
  const float freq = powf(theta, -(float)i / (float)half);
  const float angle = (float)pos * freq;
  c = cosf(angle);
  s = sinf(angle);
}

// Scores q_g . k_p of one KV tile into s_s[g][p] (G <= GP query heads, GP a
// power of two <= 8).  A warp pass takes 32 / GP positions: lane l holds its
// HD / 32 dims of every head's q in registers and accumulates its part of all
// 32 (head, position) products; one transpose-reduction (31 shuffles) then
// leaves the total of pair l in lane l.  K rows are read with the lanes
// across the row (conflict-free).
template <int HD, int GP>
__device__ __forceinline__ void sp_scores(const uint8_t* Ks, const float* q_s, float* s_s, int G, int np, int TP) {
  constexpr int DPL = HD / 32, NP = 32 / GP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float qr[GP][DPL];
#pragma unroll
  for (int g = 0; g < GP; ++g)
#pragma unroll
    for (int j = 0; j < DPL; ++j) qr[g][j] = g < G ? q_s[g * HD + DPL * lane + j] : 0.f;
  for (int p0 = warp * NP; p0 < np; p0 += SP_NC * NP) {
    float v[32];  // index g * NP + pi
#pragma unroll
    for (int pi = 0; pi < NP; ++pi) {
      float kf[DPL];
      const int p = p0 + pi;
      if (p < np) {
        const __half2* kr = reinterpret_cast<const __half2*>(Ks + (size_t)p * HD * 2) + (DPL / 2) * lane;
#pragma unroll
        for (int j = 0; j < DPL / 2; ++j) {
          const float2 f = __half22float2(kr[j]);
          kf[2 * j] = f.x;
          kf[2 * j + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < DPL; ++j) kf[j] = 0.f;
      }
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        float d = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) d = fmaf(qr[g][j], kf[j], d);
        v[g * NP + pi] = d;
      }
    }
#pragma unroll
    for (int st = 0; st < 5; ++st) {  // halves of 16, 8, 4, 2, 1 values
      const int off = 16 >> st;
      const bool up = lane & off;
#pragma unroll
      for (int i = 0; i < (16 >> st); ++i) {
        const float send = up ? v[i] : v[i + (16 >> st)];
        const float keep = up ? v[i + (16 >> st)] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
    const int g = lane / NP, p = p0 + lane % NP;
    if (g < G && p < np) s_s[g * (TP + 4) + p] = v[0];
  }
}

template <int HD>
__device__ void sp_attention(const StepStage& S, const StepArgs& A, const StepSmem& L, uint8_t* sm, uint32_t& seq,
                             int si) {
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint64_t* empty = full + A.S;
  constexpr int HALF = HD / 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = S.hq / S.hkv;
  const int64_t pos = A.pos;
  int hk;
  int64_t t0, t1;
  if (!sp_attn_item(S, blockIdx.x, pos + 1, hk, t0, t1)) return;
  const int TP = S.tile;
  const int splits = sp_attn_splits(S, pos + 1);
  float* q_s = reinterpret_cast<float*>(sm + L.attn);             // [G][HD], scaled by 1/sqrt(HD)
  float* s_s = q_s + G * HD;                                      // [G][TP + 4] scores / probabilities
  float* st_s = s_s + G * (TP + 4);                               // [3][G]: running max, sum, tile correction
  float* w_s = st_s + 3 * STEP_ATTN_MAX_GROUP;                    // [G][splits] merge weights
  __half* new_s = reinterpret_cast<__half*>(w_s + G * S.splits);  // the new k | v row
  const bool has_new = pos >= t0 && pos < t1;
  const float* row = S.qkv;
  const float scale = rsqrtf((float)HD);
  for (int e = tid; e < G * HALF; e += SP_CT) {
    const int g = e / HALF, i = e - g * HALF;
    const float* p = row + (int64_t)(hk * G + g) * HD;
    float cs, sn;
    sp_rope_cs(pos, i, HALF, S.theta, cs, sn);
    const float a = __ldcg(p + i), bb = __ldcg(p + i + HALF);
    q_s[g * HD + i] = (a * cs - bb * sn) * scale;
    q_s[g * HD + i + HALF] = (a * sn + bb * cs) * scale;
  }
  if (has_new) {
    __half* kc = static_cast<__half*>(S.kc);
    __half* vc = static_cast<__half*>(S.vc);
    const float* kp = row + (int64_t)(S.hq + hk) * HD;
    const float* vp = row + (int64_t)(S.hq + S.hkv + hk) * HD;
    const int64_t o = ((int64_t)hk * S.max_seq + pos) * HD;
    for (int i = tid; i < HALF; i += SP_CT) {
      float cs, sn;
      sp_rope_cs(pos, i, HALF, S.theta, cs, sn);
      const float a = __ldcg(kp + i), bb = __ldcg(kp + i + HALF);
      const __half k0 = __float2half_rn(a * cs - bb * sn), k1 = __float2half_rn(a * sn + bb * cs);
      const __half v0 = __float2half_rn(__ldcg(vp + i)), v1 = __float2half_rn(__ldcg(vp + i + HALF));
      kc[o + i] = k0;
      kc[o + i + HALF] = k1;
      vc[o + i] = v0;
      vc[o + i + HALF] = v1;
      new_s[i] = k0;
      new_s[i + HALF] = k1;
      new_s[HD + i] = v0;
      new_s[HD + i + HALF] = v1;
    }
  }
  if (tid < G) {
    st_s[tid] = -INFINITY;
    st_s[STEP_ATTN_MAX_GROUP + tid] = 0.f;
  }
  sp_sync();
  sp_stamp(A, si, 2);
  // P.V accumulators: thread (g, pair) for g < G, pair < HALF
  const int pg = tid / HALF, pd = tid - pg * HALF;
  const bool pv = pg < G;
  float acc0 = 0.f, acc1 = 0.f;
  for (int64_t p0 = t0; p0 < t1; p0 += TP) {
    const int np = (int)min((int64_t)TP, t1 - p0);
    bool ok = sp_wait_full(A, full, seq);
    ok = sp_wait_full(A, full, seq + 1) && ok;
    if (p0 == t0) sp_stamp(A, si, 3);
    uint8_t* Ks = sm + L.ring + (size_t)(seq % A.S) * A.slot_bytes;
    uint8_t* Vs = sm + L.ring + (size_t)((seq + 1) % A.S) * A.slot_bytes;
    if (has_new && pos >= p0 && pos < p0 + np) {  // the copied row is the stale cache entry: use the new one
      const int r = (int)(pos - p0);
      for (int i = tid; i < HD; i += SP_CT) {
        reinterpret_cast<__half*>(Ks)[r * HD + i] = new_s[i];
        reinterpret_cast<__half*>(Vs)[r * HD + i] = new_s[HD + i];
      }
    }
    sp_sync();
    if (ok) {
      if (G == 1) sp_scores<HD, 1>(Ks, q_s, s_s, G, np, TP);
      else if (G == 2) sp_scores<HD, 2>(Ks, q_s, s_s, G, np, TP);
      else if (G <= 4) sp_scores<HD, 4>(Ks, q_s, s_s, G, np, TP);
      else sp_scores<HD, 8>(Ks, q_s, s_s, G, np, TP);
    }
    sp_sync();
    // online softmax per head: warp g
    if (warp < G) {
      float* sg = s_s + warp * (TP + 4);
      float mx = -INFINITY;
      for (int p = lane; p < np; p += 32) mx = fmaxf(mx, sg[p]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = st_s[warp];
      const float mnew = fmaxf(mold, mx);
      float sum = 0.f;
      for (int p = lane; p < np; p += 32) {
        const float e = __expf(sg[p] - mnew);
        sg[p] = e;
        sum += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        const float corr = __expf(mold - mnew);  // 0 on the first tile (mold = -inf)
        st_s[warp] = mnew;
        st_s[STEP_ATTN_MAX_GROUP + warp] = st_s[STEP_ATTN_MAX_GROUP + warp] * corr + sum;
        st_s[2 * STEP_ATTN_MAX_GROUP + warp] = corr;
      }
    }
    sp_sync();
    if (pv) {
      const float corr = st_s[2 * STEP_ATTN_MAX_GROUP + pg];
      acc0 *= corr;
      acc1 *= corr;
      const float* pr = s_s + pg * (TP + 4);
      const __half2* vr = reinterpret_cast<const __half2*>(Vs) + pd;
#pragma unroll 4
      for (int p = 0; p < np; ++p) {
        const float2 v = __half22float2(vr[p * HALF]);
        acc0 = fmaf(pr[p], v.x, acc0);
        acc1 = fmaf(pr[p], v.y, acc1);
      }
    }
    sp_sync();  // every read of the two slots is done
    sp_release(A, empty, seq);
    sp_release(A, empty, seq + 1);
    seq += 2;
  }
  sp_stamp(A, si, 4);
  // this split's partial (max, sum, acc[HD]) per query head
  const int sp = blockIdx.x - hk * splits;
  const int64_t pstride = HD + 4;
  float* part = A.attn_part + ((int64_t)hk * splits + sp) * G * pstride;
  if (pv) {
    part[pg * pstride + 4 + 2 * pd] = acc0;
    part[pg * pstride + 4 + 2 * pd + 1] = acc1;
  }
  if (tid < G) {
    part[tid * pstride] = st_s[tid];
    part[tid * pstride + 1] = st_s[STEP_ATTN_MAX_GROUP + tid];
  }
  __threadfence();
  sp_sync();
  __shared__ int last;
  if (tid == 0) {
    unsigned* ctr = A.sync + STEP_SYNC_ATTN + hk;
    last = atomicAdd(ctr, 1u) == (unsigned)splits - 1;
    if (last) {
      *ctr = 0u;  // ready for the next attention stage
      __threadfence();
    }
  }
  sp_sync();
  if (!last) return;
  // the last split of this KV head merges every split's partial into the
  // output: per head (warp g) the weights e^(m_j - M) / L of the splits, then
  // per output element the weighted sum of the splits' accumulators
  const float* base = A.attn_part + (int64_t)hk * splits * G * pstride;
  if (warp < G) {
    float M = -INFINITY;
    for (int j = lane; j < splits; j += 32) M = fmaxf(M, __ldcg(base + ((int64_t)j * G + warp) * pstride));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float lsum = 0.f;
    for (int j = lane; j < splits; j += 32) {
      const float* pj = base + ((int64_t)j * G + warp) * pstride;
      const float w = __expf(__ldcg(pj) - M);  // empty splits: exp(-inf) = 0
      w_s[warp * S.splits + j] = w;
      lsum = fmaf(__ldcg(pj + 1), w, lsum);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    const float inv = 1.f / lsum;
    for (int j = lane; j < splits; j += 32) w_s[warp * S.splits + j] *= inv;
  }
  sp_sync();
  for (int e = tid; e < G * HD; e += SP_CT) {
    const int g = e / HD, d = e - g * HD;
    const float* wg = w_s + g * S.splits;
    const float* pd0 = base + (int64_t)g * pstride + 4 + d;
    float o = 0.f;
#pragma unroll 8
    for (int j = 0; j < splits; ++j) o = fmaf(wg[j], __ldcg(pd0 + (int64_t)j * G * pstride), o);
    S.out[(int64_t)(hk * G + g) * HD + d] = o;
  }
}

__global__ void __launch_bounds__(STEP_THREADS, 1) step_kernel(const StepArgs A) {
  extern __shared__ __align__(128) uint8_t sm[];
  const StepSmem L(A.S, A.slot_bytes, A.nk_max, A.rows_max, A.xr_floats, A.nw_floats, A.attn_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint64_t* empty = full + A.S;
  if (threadIdx.x == 0) {
    for (int i = 0; i < A.S; ++i) {
      xs_bar_init(&full[i], 1);
      xs_bar_init(&empty[i], SP_NC);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  if (warp == SP_NC) {
    if ((threadIdx.x & 31) == 0) sp_produce(A, L, sm);
    return;
  }
  const unsigned ep0 = *reinterpret_cast<const volatile unsigned*>(A.epoch);
  uint32_t seq = 0;
  unsigned nbar = 0;
  const unsigned C = gridDim.x;
  for (int si = 0; si < A.nstages; ++si) {
    const StepStage& S = A.stages[si];
    sp_stamp(A, si, 0);
    if (S.barrier) sp_grid_sync(A.sync + STEP_SYNC_BAR, ++nbar * C, A.err);
    sp_stamp(A, si, 1);
    if (S.kind == STEP_GEMV) {
      if (S.qt == GGUF_Q4_K) sp_gemv<GGUF_Q4_K>(S, A, L, sm, seq, ep0, si);
      else sp_gemv<GGUF_Q6_K>(S, A, L, sm, seq, ep0, si);
    } else {
      if (S.hd == 128) sp_attention<128>(S, A, L, sm, seq, si);
      else sp_attention<64>(S, A, L, sm, seq, si);
    }
    sp_sync();
    sp_stamp(A, si, 5);
  }
  // the last CTA out resets the barrier counters and publishes the epoch
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(A.sync + STEP_SYNC_EXIT, 1u) == C - 1) {
      A.sync[STEP_SYNC_BAR] = 0u;
      A.sync[STEP_SYNC_EXIT] = 0u;
      *A.epoch = ep0 + (unsigned)A.nexch;
      __threadfence();
    }
  }
}

}  // namespace

cudaError_t step_init_device() {
  return cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, STEP_MAX_SMEM);
}

cudaError_t launch_step(const StepArgs& a, int grid, cudaStream_t s) {
  const StepSmem L(a.S, a.slot_bytes, a.nk_max, a.rows_max, a.xr_floats, a.nw_floats, a.attn_bytes);
  if (L.end > (size_t)STEP_MAX_SMEM) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(STEP_THREADS);
  cfg.dynamicSmemBytes = L.end;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers rely on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel, a);
}

}  // namespace kq
