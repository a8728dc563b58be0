// kq_kx.cu -- the other GGUF K-quants: Q2_K (84 B / 256 weights), Q3_K
// (110 B) and Q5_K (176 B).  Bit-exact dequantization and a fused
// dequant-GEMV / small-batch GEMM on the CUDA cores.
//
// Superblock formats (little-endian; the same layouts gguf-py decodes):
//   Q2_K  scales[16] | qs[64] | d f16 | dmin f16
//         element e: 2-bit q = bits 2*((e%128)/32) of qs[32*(e/128) + e%32];
//         sub-block s = e/16 has scale = low nibble, min = high nibble of
//         scales[s]; value = (d*scale)*q - (dmin*min)
//   Q3_K  hmask[32] | qs[64] | scales[12] | d f16
//         two low bits as Q2_K (from qs); bit e/32 of hmask[e%32] is the third
//         bit, and a clear bit means q -= 4 (q in [-4, 3]); the 6-bit scale of
//         sub-block s is the low (s < 8) / high (s >= 8) nibble of byte s%8
//         with bits 2*(s/4) of byte 8 + s%4 on top, minus 32;
//         value = (d*scale)*q
//   Q5_K  d f16 | dmin f16 | 12 scale/min bytes (packed as in Q4_K) | qh[32]
//         | qs[128]; element e: nibble of qs[32*(e/64) + e%32] (low for
//         e%64 < 32) plus bit e/32 of qh[e%32] as bit 4; sub-block e/32;
//         value = (d*sc)*q - (dmin*m)
// Every product is rounded on its own (__fmul_rn / __fsub_rn), in this
// association, so the decode matches the CPU definition bit for bit.
//
// Device layout: Q5_K rows as uploaded (176-byte superblocks, 16-byte
// multiples); Q3_K and Q2_K superblocks at a 112 / 96-byte stride (zero bytes
// after each), so that every one starts on a 16-byte boundary for vector loads
// and tensor-map boxes.
//
// GEMV: a CTA owns KX_RB rows (two per warp) and walks K in chunks of CH
// superblocks.  Each chunk's activations (up to MT tokens) and the CTA's
// weight bytes are copied into shared memory with 16-byte cp.async, double
// buffered, so the next chunk streams while this one is multiplied.  Lane l
// of a warp takes elements l + 32i (i = 0..7) of every superblock: activation
// reads are consecutive across the warp (no bank conflicts) and the quant
// bytes a lane needs are bytes l and 32 + l of its plane.  The dequantized
// weight multiplies the f32 activations directly (f32 accumulation, no
// activation rounding); partial sums are reduced with warp shuffles.  The
// per-weight decode costs a few instructions, so at one token these types
// are issue-bound rather than HBM-bound on this kernel.  Waits are cp.async
// group waits only (no spin loops).
#include "kq_common.cuh"
#include "kq_kernels.h"

#include <algorithm>

namespace kq {
namespace {

constexpr int KX_THREADS = 256;  // 8 warps
constexpr int KX_RB = 16;        // rows per CTA: two per warp

template <int QT>
struct KxFmt;
// BS: bytes of a superblock in the file; DS: device stride between the
// superblocks of a row; CH: superblocks per chunk (CH * DS is a multiple of 16)
template <>
struct KxFmt<GGUF_Q2_K> {
  static constexpr int BS = Q2K_BYTES, DS = Q2K_DEV, CH = 4;
};
template <>
struct KxFmt<GGUF_Q3_K> {
  static constexpr int BS = Q3K_BYTES, DS = Q3K_DEV, CH = 4;
};
template <>
struct KxFmt<GGUF_Q5_K> {
  static constexpr int BS = Q5K_BYTES, DS = Q5K_BYTES, CH = 4;
};

__device__ __forceinline__ uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

__device__ __forceinline__ int q3k_scale(const uint8_t* sc, int s) {
  const int lo = s < 8 ? (sc[s] & 15) : (sc[s - 8] >> 4);
  const int hi = (sc[8 + (s & 3)] >> (2 * (s >> 2))) & 3;
  return (lo | (hi << 4)) - 32;
}

// Element e of one superblock, bit-exact.
template <int QT>
__device__ __forceinline__ float kx_value(const uint8_t* blk, int e) {
  if constexpr (QT == GGUF_Q2_K) {
    const int s = e >> 4;
    const int q = (blk[16 + 32 * (e >> 7) + (e & 31)] >> (2 * ((e >> 5) & 3))) & 3;
    const float d = f16_bits_to_f32(rd16(blk + 80)), dmin = f16_bits_to_f32(rd16(blk + 82));
    const float dl = __fmul_rn(d, (float)(blk[s] & 15));
    const float ml = __fmul_rn(dmin, (float)(blk[s] >> 4));
    return __fsub_rn(__fmul_rn(dl, (float)q), ml);
  } else if constexpr (QT == GGUF_Q3_K) {
    const int lo = (blk[32 + 32 * (e >> 7) + (e & 31)] >> (2 * ((e >> 5) & 3))) & 3;
    const int q = lo - (((blk[e & 31] >> (e >> 5)) & 1) ? 0 : 4);
    const float d = f16_bits_to_f32(rd16(blk + 108));
    return __fmul_rn(__fmul_rn(d, (float)q3k_scale(blk + 96, e >> 4)), (float)q);
  } else {
    const int j = e >> 5, l = e & 31;
    int sc, m;
    q4k_scale_min(blk + 4, j, sc, m);
    const uint8_t byte = blk[48 + 32 * (e >> 6) + l];
    const int q = ((j & 1) ? (byte >> 4) : (byte & 15)) | (((blk[16 + l] >> j) & 1) << 4);
    const float d = f16_bits_to_f32(rd16(blk)), dmin = f16_bits_to_f32(rd16(blk + 2));
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
  }
}

// The eight elements lane + 32i (i = 0..7) of one superblock in shared
// memory, with the same rounding as kx_value.
template <int QT>
__device__ __forceinline__ void kx_decode8(const uint8_t* blk, int lane, float (&w)[8]) {
  if constexpr (QT == GGUF_Q2_K) {
    const float d = f16_bits_to_f32(rd16(blk + 80)), dmin = f16_bits_to_f32(rd16(blk + 82));
    const uint32_t qa = blk[16 + lane], qb = blk[48 + lane];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int sc = blk[2 * i + (lane >> 4)];
      const int q = (((i < 4) ? qa : qb) >> (2 * (i & 3))) & 3;
      w[i] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)(sc & 15)), (float)q), __fmul_rn(dmin, (float)(sc >> 4)));
    }
  } else if constexpr (QT == GGUF_Q3_K) {
    const float d = f16_bits_to_f32(rd16(blk + 108));
    const uint32_t hm = blk[lane], qa = blk[32 + lane], qb = blk[64 + lane];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int lo = (((i < 4) ? qa : qb) >> (2 * (i & 3))) & 3;
      const int q = lo - (((hm >> i) & 1) ? 0 : 4);
      w[i] = __fmul_rn(__fmul_rn(d, (float)q3k_scale(blk + 96, 2 * i + (lane >> 4))), (float)q);
    }
  } else {
    const float d = f16_bits_to_f32(rd16(blk)), dmin = f16_bits_to_f32(rd16(blk + 2));
    const uint32_t hb = blk[16 + lane];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int sc, m;
      q4k_scale_min(blk + 4, i, sc, m);
      const uint32_t byte = blk[48 + 32 * (i >> 1) + lane];
      const int q = (int)(((i & 1) ? (byte >> 4) : (byte & 15)) | (((hb >> i) & 1) << 4));
      w[i] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
    }
  }
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int QT, int MT>
struct KxSmem {
  static constexpr int DS = KxFmt<QT>::DS, CH = KxFmt<QT>::CH;
  static constexpr int XB = MT * CH * 256 * 4;  // activations of one chunk, [MT][CH * 256] f32
  static constexpr int WP = CH * DS;            // one row's bytes of one chunk (a multiple of 16)
  static constexpr int STAGE = XB + KX_RB * WP;
  static constexpr int TOTAL = 2 * STAGE;
  static_assert(WP % 16 == 0, "chunk rows must be whole 16-byte units");
};

template <int QT, int MT>
__global__ void __launch_bounds__(KX_THREADS) kx_gemv_kernel(const uint8_t* __restrict__ q, int64_t row_bytes, int n,
                                                             int sb, const float* __restrict__ x, int m,
                                                             const float* __restrict__ bias, float* __restrict__ y) {
  using L = KxSmem<QT, MT>;
  constexpr int CH = L::CH;
  extern __shared__ __align__(16) uint8_t kx_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * KX_RB;
  const int rows = min(KX_RB, n - row0);
  const int nch = (sb + CH - 1) / CH;
  const int64_t k = (int64_t)sb * 256;

  // chunk c (superblocks [c*CH, c*CH + chv)) into stage buffer `buf`
  auto issue = [&](int c, int buf) {
    uint8_t* st = kx_smem + buf * L::STAGE;
    const int chv = min(CH, sb - c * CH);
    const int xu = chv * 64;  // 16-byte units of one token's activations
    for (int i = threadIdx.x; i < m * xu; i += KX_THREADS) {
      const int t = i / xu, u = i - t * xu;
      cp_async16(st + (size_t)t * CH * 1024 + (size_t)u * 16, x + (int64_t)t * k + (int64_t)c * CH * 256 + u * 4);
    }
    // whole 16-byte units: a partial chunk reads up to 15 bytes past its
    // last superblock, inside the row's padded stride or the allocation's pad
    const int wu = (chv * L::DS + 15) >> 4;
    for (int i = threadIdx.x; i < rows * wu; i += KX_THREADS) {
      const int r = i / wu, u = i - r * wu;
      cp_async16(st + L::XB + r * L::WP + u * 16,
                 q + (int64_t)(row0 + r) * row_bytes + (int64_t)c * CH * L::DS + u * 16);
    }
    cp_async_commit();
  };

  float acc[2][MT];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[r][t] = 0.f;

  issue(0, 0);
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) {
      issue(c + 1, (c + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint8_t* st = kx_smem + (c & 1) * L::STAGE;
    const float* xs = reinterpret_cast<const float*>(st);
    const uint8_t* ws = st + L::XB;
    const int chv = min(CH, sb - c * CH);
    for (int j = 0; j < chv; ++j) {
      float xv[8][MT];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int t = 0; t < MT; ++t) xv[i][t] = t < m ? xs[t * CH * 256 + j * 256 + lane + 32 * i] : 0.f;
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int r = 2 * warp + rr;
        if (r < rows) {
          float w[8];
          kx_decode8<QT>(ws + r * L::WP + j * L::DS, lane, w);
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[rr][t] = fmaf(w[i], xv[i][t], acc[rr][t]);
        }
      }
    }
    __syncthreads();  // the buffer is refilled by the next iteration's issue
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = 2 * warp + rr;
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      float v = acc[rr][t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && r < rows && t < m) y[(int64_t)t * n + row0 + r] = v + (bias ? bias[row0 + r] : 0.f);
    }
  }
}

template <int QT>
__global__ void kx_dequant_kernel(const uint8_t* __restrict__ q, int64_t row_bytes, int64_t k, int64_t row0,
                                  int64_t nrows, float* __restrict__ out) {
  const int64_t total = nrows * k;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / k, i = idx - r * k;
    out[idx] = kx_value<QT>(q + (row0 + r) * row_bytes + (i >> 8) * KxFmt<QT>::DS, (int)(i & 255));
  }
}

template <int QT, int MT>
cudaError_t kx_attr() {
  return cudaFuncSetAttribute(kx_gemv_kernel<QT, MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              KxSmem<QT, MT>::TOTAL);
}

template <int QT>
cudaError_t kx_attrs() {
  cudaError_t e = kx_attr<QT, 1>();
  if (e == cudaSuccess) e = kx_attr<QT, 2>();
  if (e == cudaSuccess) e = kx_attr<QT, 4>();
  if (e == cudaSuccess) e = kx_attr<QT, 8>();
  return e;
}

template <int QT, int MT>
cudaError_t kx_launch(const DevWeight& w, const float* x, int mc, const float* bias, float* y, cudaStream_t s) {
  const unsigned grid = (unsigned)((w.n + KX_RB - 1) / KX_RB);
  kx_gemv_kernel<QT, MT><<<grid, KX_THREADS, KxSmem<QT, MT>::TOTAL, s>>>(w.q, w.row_bytes, (int)w.n, (int)w.sb, x,
                                                                          mc, bias, y);
  return cudaGetLastError();
}

template <int QT>
cudaError_t kx_typed(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y, cudaStream_t s,
                     int* launches) {
  for (int64_t m0 = 0; m0 < m; m0 += 8) {
    const int mc = (int)std::min<int64_t>(8, m - m0);
    const float* xc = x + m0 * w.k;
    float* yc = y + m0 * w.n;
    cudaError_t e;
    if (mc == 1) e = kx_launch<QT, 1>(w, xc, mc, bias, yc, s);
    else if (mc == 2) e = kx_launch<QT, 2>(w, xc, mc, bias, yc, s);
    else if (mc <= 4) e = kx_launch<QT, 4>(w, xc, mc, bias, yc, s);
    else e = kx_launch<QT, 8>(w, xc, mc, bias, yc, s);
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
  }
  return cudaSuccess;
}

}  // namespace

bool kx_type(int type) { return type == GGUF_Q2_K || type == GGUF_Q3_K || type == GGUF_Q5_K; }

int64_t kx_block_bytes(int type) {
  switch (type) {
    case GGUF_Q2_K: return KxFmt<GGUF_Q2_K>::BS;
    case GGUF_Q3_K: return KxFmt<GGUF_Q3_K>::BS;
    case GGUF_Q5_K: return KxFmt<GGUF_Q5_K>::BS;
    default: return 0;
  }
}

int64_t kx_dev_stride(int type) {
  switch (type) {
    case GGUF_Q2_K: return KxFmt<GGUF_Q2_K>::DS;
    case GGUF_Q3_K: return KxFmt<GGUF_Q3_K>::DS;
    case GGUF_Q5_K: return KxFmt<GGUF_Q5_K>::DS;
    default: return 0;
  }
}

cudaError_t kx_init_device() {
  cudaError_t e = kx_attrs<GGUF_Q2_K>();
  if (e == cudaSuccess) e = kx_attrs<GGUF_Q3_K>();
  if (e == cudaSuccess) e = kx_attrs<GGUF_Q5_K>();
  return e;
}

cudaError_t launch_gemv_kx(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y, cudaStream_t s,
                           int* launches, Bracket br) {
  if (m < 1 || w.n < 1) return cudaSuccess;
  if (w.n > (int64_t)1 << 30 || w.sb > (int64_t)1 << 20) return cudaErrorInvalidValue;
  bracket_record(br.start, s);
  cudaError_t e;
  switch (w.type) {
    case GGUF_Q2_K: e = kx_typed<GGUF_Q2_K>(w, x, m, bias, y, s, launches); break;
    case GGUF_Q3_K: e = kx_typed<GGUF_Q3_K>(w, x, m, bias, y, s, launches); break;
    case GGUF_Q5_K: e = kx_typed<GGUF_Q5_K>(w, x, m, bias, y, s, launches); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  bracket_record(br.stop, s);
  return cudaSuccess;
}

cudaError_t launch_dequant_kx(const DevWeight& w, int64_t row0, int64_t nrows, float* out, cudaStream_t s) {
  const int64_t total = nrows * w.k;
  if (total <= 0) return cudaSuccess;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 64);
  switch (w.type) {
    case GGUF_Q2_K: kx_dequant_kernel<GGUF_Q2_K><<<blocks, 256, 0, s>>>(w.q, w.row_bytes, w.k, row0, nrows, out); break;
    case GGUF_Q3_K: kx_dequant_kernel<GGUF_Q3_K><<<blocks, 256, 0, s>>>(w.q, w.row_bytes, w.k, row0, nrows, out); break;
    case GGUF_Q5_K: kx_dequant_kernel<GGUF_Q5_K><<<blocks, 256, 0, s>>>(w.q, w.row_bytes, w.k, row0, nrows, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace kq
