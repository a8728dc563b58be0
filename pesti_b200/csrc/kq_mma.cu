// kq_mma.cu -- K-quant dequant-GEMM on the 5th-generation tensor cores.
//
// y[t][row] = sum_k x[t][k] * W[row][k] for a 128-row weight tile per CTA:
//
//   warps 0-7  dequantize: thread r of warp w owns weight row r = 32*(w%4) +
//              lane of the tile and quarters 2*(w/4), 2*(w/4)+1 of every
//              superblock.  It reads its row's raw superblock from shared
//              memory (TMA-loaded), rebuilds 64 weights at a time as f16 /
//              bf16 pairs and writes them straight into tensor memory
//              (tcgen05.st), where they are the A operand of the MMA.  Warps
//              0-3 also run the epilogue.
//   warp 8     TMA producer of the raw weight tiles (128 rows x one superblock).
//   warp 9     TMA producer of the activation tiles (BN columns x 64 k,
//              128-byte swizzle), in pairs.
//   warp 10    MMA issuer: tcgen05.mma kind::f16, A from TMEM, B from shared
//              memory, accumulator (128 x BN f32) in TMEM; tcgen05.commit
//              frees activation pairs and A superblock slots and signals the
//              epilogue.  Its barrier waits and commits cost about as much
//              issue time as the MMAs, so there is one wait / commit per
//              activation pair and per superblock of A, not per quarter, all
//              from one thread (measured: 838 -> 1111 TFLOP/s on a 14336 x
//              4096 Q4_K weight at 4096 tokens).
//
// The weights' K order inside a superblock is the order in which a thread
// unpacks them cheaply (per 64-weight quarter c and step s: weights e, e+2,
// e+1, e+3 with e = step_elem(s, c)); the activation prep writes x in the same
// order, so the product is unchanged.
//
// f32 activations (kq_linear_f32): each activation is split into f16 hi and
// lo parts (one power-of-two scale per token keeps them in range), the tile's
// BN columns hold BN/2 tokens' hi parts then their lo parts, and A is f16 with
// the superblock scales folded in, so the accumulator runs over the CTA's
// whole K range.  When few row tiles exist K is split over CTAs (grid z):
// partial sums go to a workspace and the last CTA of a row tile adds them in
// a fixed order.  bf16 activations (kq_linear_bf16, prefill): A is bf16.
//
// Every mbarrier wait is bounded (sm100::mbar_wait): a pipeline that stops
// making progress ends the kernel with an error code in *err, never a hang.
#include "kq_common.cuh"
#include "kq_kernels.h"
#include "kq_sm100.cuh"

#include <cuda_bf16.h>

#include <mutex>

namespace kq {
namespace {
using namespace sm100;
// The MMA thread's waits: a completed phase answers a non-blocking test
// (cheaper than the blocking try-wait loop, measured 2-6% on the prefill);
// otherwise the bounded wait.
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* bar, uint32_t parity, int* err, int code) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done ? true : mbar_wait(bar, parity, err, code);
}

constexpr int TM = 128;    // weight rows per CTA = UMMA M
constexpr int KSTEP = 64;  // k per A slot / activation tile (one quarter superblock)
// Warp roles: eight dequant warps (two per TMEM lane quadrant, each doing two
// of the four 64-k quarters of every superblock), one TMA producer for the raw
// weight tiles, one for the activation tiles, one MMA issuer.  The two
// producers run independently, so a raw tile is requested as soon as its ring
// slot is free rather than behind the activation tiles' waits on the MMAs.
struct W {
  static constexpr int DEQ = 8;       // dequant warps
  static constexpr int RAW = DEQ;      // raw-tile producer
  static constexpr int ACT = DEQ + 1;  // activation-tile producer
  static constexpr int MMA = DEQ + 2;
  static constexpr int THREADS = 32 * (DEQ + 3);
};

enum : int { ERR_WAIT_RAW = 1, ERR_WAIT_A = 2, ERR_WAIT_B = 3, ERR_WAIT_ACC = 4, ERR_WAIT_MMA = 5 };

template <int QT>
struct RawTile;
template <>
struct RawTile<GGUF_Q4_K> {
  static constexpr int ROW = Q4K_BYTES;          // bytes per row per superblock
  static constexpr int BODY = TM * Q4K_BYTES;    // 18432
  static constexpr int BYTES = BODY;
};
template <>
struct RawTile<GGUF_Q6_K> {
  static constexpr int ROW = Q6K_BODY;
  static constexpr int BODY = TM * Q6K_BODY;     // 26624
  static constexpr int BYTES = BODY + TM * 16;   // + d of the 128 rows for 8 superblocks
};

template <int QT, int BN>
struct Cfg {
  // The MMA warp's waits and commits cost about as much as its MMAs, so they
  // are made per group: activation tiles come in groups of BG quarters (one
  // full / empty barrier pair per group), the A operand in TMEM per
  // superblock (four 32-column quarters per slot).
  static constexpr int RS = BN <= 64 ? 3 : (QT == GGUF_Q6_K ? 2 : 3);  // raw weight stages
  static constexpr int BG = 2;                            // quarters per activation group
  static constexpr int BGS = BN <= 128 ? 4 : 2;           // activation group slots
  static constexpr int BS = BG * BGS;                     // activation tile slots
  static constexpr int ASB = BN >= 128 ? 2 : 1;           // A superblock slots in TMEM
  static constexpr int AS = 4 * ASB;                      // A quarter slots (32 columns each)
  static constexpr int BTILE = BN * 128;                  // activation tile bytes (64 k x BN x 2 B)
  // Small-N MMAs into one accumulator serialise on their latency, so decode
  // tiles rotate their k16 steps over independent accumulator sets that the
  // epilogue adds up.  Large tiles keep one accumulator.
  static constexpr int ACC_SETS = BN <= 32 ? 4 : BN <= 64 ? 2 : 1;
  static constexpr int ACC_COLS = (ACC_SETS * BN) < 32 ? 32 : ACC_SETS * BN;
  static constexpr int A_COL0 = ACC_COLS;
  static constexpr int TMEM_NEED = ACC_COLS + AS * 32;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                 : TMEM_NEED <= 256 ? 256 : 512;
  static constexpr int OFF_B = 0;                         // 1024-aligned (swizzled tiles)
  static constexpr int OFF_RAW = OFF_B + BS * BTILE;
  static constexpr int OFF_BAR = OFF_RAW + RS * RawTile<QT>::BYTES;
  static constexpr int NBAR = 2 * RS + 2 * BGS + 2 * ASB + 1;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + tmem holder + alignment slack
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

// ---- per-row superblock unpacking (thread = row) ---------------------------
template <bool BF16>
struct H2;
template <>
struct H2<false> {
  using T = __half2;
  static constexpr uint32_t MAGIC = 0x64006400u;  // bits of 1024 + v
  static constexpr uint32_t MAGIC_BYTE = 0x64646464u;
  static constexpr float BIAS = 1024.f;
  __device__ static T from_f(float a) { return __float2half2_rn(a); }
};
template <>
struct H2<true> {
  using T = __nv_bfloat162;
  static constexpr uint32_t MAGIC = 0x43004300u;  // bits of 128 + v (v < 128)
  static constexpr uint32_t MAGIC_BYTE = 0x43434343u;
  static constexpr float BIAS = 128.f;
  __device__ static T from_f(float a) { return __float2bfloat162_rn(a); }
};

template <class T>
__device__ __forceinline__ uint32_t bits_of(T v) {
  return *reinterpret_cast<uint32_t*>(&v);
}
template <class T>
__device__ __forceinline__ T of_bits(uint32_t u) {
  return *reinterpret_cast<T*>(&u);
}
__device__ __forceinline__ uint32_t wof(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t prmt_(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Q4_K quarter c = qs[32c .. 32c+31] (sub-block 2c low nibbles, 2c+1 high).
// A value = (d*sc)*q - dmin*m with the two products rounded to 16 bits.
template <bool BF16>
__device__ __forceinline__ void unpack_q4(const uint4 (&qs)[8], const uint4& hdr, int c,
                                          uint32_t (&out)[32]) {
  using H = H2<BF16>;
  using T = typename H::T;
  const float d = f16_bits_to_f32((uint16_t)(hdr.x & 0xffff));
  const float dmin = f16_bits_to_f32((uint16_t)(hdr.x >> 16));
  int sca, ma, scb, mb;
  q4k_scale_min_w(hdr.y, hdr.z, hdr.w, 2 * c, sca, ma);
  q4k_scale_min_w(hdr.y, hdr.z, hdr.w, 2 * c + 1, scb, mb);
  const T mul_lo = H::from_f(d * (float)sca), add_lo = H::from_f(-(dmin * (float)ma));
  const T mul_hi = H::from_f(d * (float)scb), add_hi = H::from_f(-(dmin * (float)mb));
  const T bias = H::from_f(H::BIAS);
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    const int w = s >> 1, lohi = s & 1;
    const uint32_t W = wof(qs[2 * c + (w >> 2)], w & 3);
    const uint32_t Wn = lohi ? (W >> 4) : W;
    const uint32_t t02 = (Wn & 0x000F000Fu) | H::MAGIC;
    const uint32_t t13 = ((Wn >> 8) & 0x000F000Fu) | H::MAGIC;
    const T mu = lohi ? mul_hi : mul_lo, ad = lohi ? add_hi : add_lo;
    out[2 * s] = bits_of(__hfma2(__hsub2(of_bits<T>(t02), bias), mu, ad));
    out[2 * s + 1] = bits_of(__hfma2(__hsub2(of_bits<T>(t13), bias), mu, ad));
  }
}

// Q6_K quarter c = the 48 device-body bytes of slot c (q6k_body_offset).
// A value = (d*sc)*(q-32), rounded once to 16 bits.
// (d*s, d*s) for the int8 scale byte `b` of word w.  f16: the byte is turned
// into an exact f16 with the 0x64 magic (sign bit flipped first, then 1152
// subtracted) and multiplied by d, which is already an f16 -- the same
// rounding as converting the f32 product.  bf16: via f32.
template <bool BF16>
__device__ __forceinline__ typename H2<BF16>::T group_scale(uint32_t w, int b, float d) {
  if constexpr (BF16) {
    const int sv = (int)(int8_t)((w >> (8 * b)) & 0xff);
    return H2<true>::from_f(d * (float)sv);
  } else {
    const uint32_t sel = (uint32_t)b | 0x0070u | ((uint32_t)b << 8) | 0x7000u;
    const __half2 v = __hsub2(of_bits<__half2>(prmt_(w ^ 0x80808080u, 0x64646464u, sel)),
                              __float2half2_rn(1152.f));
    return __hmul2(v, __float2half2_rn(d));
  }
}

template <bool BF16>
__device__ __forceinline__ void unpack_q6(const uint4& p01, const uint4& p23, const uint4& p45,
                                          const uint4& sc, float d, int c, uint32_t (&out)[32]) {
  using H = H2<BF16>;
  using T = typename H::T;
  const T off = H::from_f(H::BIAS + 32.f);
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    const int p = s >> 2, h = p >> 1, gg = p & 1, w = (s >> 1) & 1, lohi = s & 1;
    const uint32_t W = wof(p < 2 ? p01 : p23, 2 * (p & 1) + w);
    const uint32_t Hq = wof(p45, 2 * h + w);
    const uint32_t hm = (Hq >> (2 * gg)) & 0x33333333u;
    const uint32_t q = lohi ? (((W >> 4) & 0x0F0F0F0Fu) | (hm & 0x30303030u))
                            : ((W & 0x0F0F0F0Fu) | ((hm << 4) & 0x30303030u));
    const int g = gg + 2 * lohi;
    const int si = 8 * h + 2 * g + (c >> 1);
    const T ds = group_scale<BF16>(wof(sc, si >> 2), si & 3, d);
    const uint32_t t02 = prmt_(q, H::MAGIC_BYTE, 0x7250u);  // codes of bytes 0, 2
    const uint32_t t13 = prmt_(q, H::MAGIC_BYTE, 0x7351u);  // codes of bytes 1, 3
    out[2 * s] = bits_of(__hmul2(__hsub2(of_bits<T>(t02), off), ds));
    out[2 * s + 1] = bits_of(__hmul2(__hsub2(of_bits<T>(t13), off), ds));
  }
}

struct Params {
  int n, sb, m;            // rows, superblocks per row, tokens
  int splits;              // K splits (grid z)
  const float* tok_scale;  // f32 path: per-token 2^e (indexed by token), else null
  const float* bias;
  float* y;                // [m][n]
  float* ws;               // [splits][m][n] partial sums (splits > 1)
  unsigned* counters;      // [row tiles x token tiles] arrival counters (splits > 1)
  int* err;
};

// Hand a raw-ring slot back to the TMA producer: this thread's shared-memory
// reads of it (generic proxy) are fenced against the TMA refill (async proxy).
__device__ __forceinline__ void raw_release(uint64_t* empty) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_arrive(empty);
}

template <int QT, int BN, bool BF16>
__global__ void __launch_bounds__(W::THREADS, BN <= 64 ? 2 : 1)
    kq_mma_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap dmap,
                  const __grid_constant__ CUtensorMap xmap, Params P) {
  using C = Cfg<QT, BN>;
  using R = RawTile<QT>;
  constexpr int TPT = BF16 ? BN : BN / 2;  // tokens per tile
  extern __shared__ uint8_t smem_raw[];
  __shared__ int last_cta;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* raw_full = bar;
  uint64_t* raw_empty = raw_full + C::RS;
  uint64_t* b_full = raw_empty + C::RS;  // per activation group slot
  uint64_t* b_empty = b_full + C::BGS;
  uint64_t* a_full = b_empty + C::BGS;   // per A superblock slot
  uint64_t* a_empty = a_full + C::ASB;
  uint64_t* acc_full = a_empty + C::ASB;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * TM;
  const int tok0 = blockIdx.y * TPT;
  const int z = blockIdx.z;
  const int sb_lo = (int)((int64_t)P.sb * z / P.splits), sb_hi = (int)((int64_t)P.sb * (z + 1) / P.splits);
  const int nsb = sb_hi - sb_lo;
  const int nq = 4 * nsb;  // pipeline steps (64-k quarters)

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::RS; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 32 * W::DEQ);
    }
    for (int i = 0; i < C::BGS; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    for (int i = 0; i < C::ASB; ++i) {
      mbar_init(&a_full[i], 32 * W::DEQ);  // every dequant thread, once per superblock
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_holder, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == W::RAW) {
    // ---------------- TMA producer: raw weight tiles, RS superblocks ahead ----------------
    if (lane == 0) {
      tma_prefetch(&wmap);
      if (QT == GGUF_Q6_K) tma_prefetch(&dmap);
      for (int i = 0; i < nsb; ++i) {
        const int rs = i % C::RS;
        if (i >= C::RS && !mbar_wait(&raw_empty[rs], ((i / C::RS) - 1) & 1, P.err, ERR_WAIT_RAW)) break;
        uint8_t* dst = smem + C::OFF_RAW + rs * R::BYTES;
        mbar_expect_tx(&raw_full[rs], R::BYTES);
        const int kb = sb_lo + i;
        tma_load_2d(dst, &wmap, kb * R::ROW, row0, &raw_full[rs]);
        if constexpr (QT == GGUF_Q6_K) tma_load_2d(dst + R::BODY, &dmap, kb & ~7, row0, &raw_full[rs]);
      }
    }
  } else if (warp == W::ACT) {
    // ---------------- TMA producer: activation tiles, BGS groups of BG quarters ahead ----------------
    if (lane == 0) {
      tma_prefetch(&xmap);
      for (int g = 0; g < nq / C::BG; ++g) {
        const int gs = g % C::BGS;
        if (g >= C::BGS && !mbar_wait(&b_empty[gs], ((g / C::BGS) - 1) & 1, P.err, ERR_WAIT_B)) break;
        mbar_expect_tx(&b_full[gs], C::BG * C::BTILE);
#pragma unroll
        for (int j = 0; j < C::BG; ++j)
          tma_load_2d(smem + C::OFF_B + (gs * C::BG + j) * C::BTILE, &xmap, (sb_lo * 4 + g * C::BG + j) * KSTEP,
                      blockIdx.y * BN, &b_full[gs]);
      }
    }
  } else if (warp == W::MMA) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t IDESC = idesc_f16(BF16, TM, BN);
    constexpr int GPS = 4 / C::BG;  // activation groups per superblock
    // one thread waits, issues and commits (no warp votes between the steps)
    if (lane == 0) {
      bool ok = true, issued = false;
      for (int i = 0; i < nsb && ok; ++i) {
        const int as = i % C::ASB;
        ok = mbar_wait_fast(&a_full[as], (i / C::ASB) & 1, P.err, ERR_WAIT_A);
        for (int h = 0; h < GPS && ok; ++h) {
          const int g = GPS * i + h, gs = g % C::BGS;
          ok = mbar_wait_fast(&b_full[gs], (g / C::BGS) & 1, P.err, ERR_WAIT_B);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < C::BG; ++j) {
            const int qq = C::BG * h + j, q = 4 * i + qq;  // quarter within the superblock / overall
            const uint32_t a_addr = tmem + C::A_COL0 + as * 128 + qq * 32;
            // descriptor of the tile's first k16 step; the next steps start 32 bytes
            // further (2 in the address field, which holds addresses / 16 < 2^14)
            const uint64_t b_desc = desc_kmajor_sw128(smem_u32(smem + C::OFF_B + (gs * C::BG + j) * C::BTILE));
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16) {
              const int step = 4 * q + k16;
              const uint32_t d_addr = tmem + (uint32_t)((step % C::ACC_SETS) * BN);
              mma_ts(d_addr, a_addr + 8 * k16, b_desc + (uint64_t)(2 * k16), IDESC, step >= C::ACC_SETS ? 1u : 0u);
            }
          }
          tc_commit(&b_empty[gs]);
          issued = true;
        }
        if (!ok) break;
        tc_commit(&a_empty[as]);
        if (i == nsb - 1) tc_commit(acc_full);
      }
      if (!ok && issued) {
        // stopped early: let the MMAs already issued finish before TMEM is freed
        tc_commit(acc_full);
        mbar_wait(acc_full, 0, P.err, ERR_WAIT_MMA);
      }
    }
    __syncwarp();
  } else {
    // ---------------- dequant (warps 0-7) ----------------
    // Warp w serves TMEM lanes 32*(w%4).. (rows of the tile) and quarters
    // 2*(w/4), 2*(w/4)+1 of every superblock.  The second quarter is unpacked
    // while the first one's TMEM store completes; each thread arrives on the
    // superblock's A slot once both are stored.
    const int r = (warp & 3) * 32 + lane;  // tile row = TMEM lane
    const int c0 = 2 * (warp >> 2);
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    for (int i = 0; i < nsb; ++i) {
      const int rs = i % C::RS, as = i % C::ASB;
      if (!mbar_wait_warp(&raw_full[rs], (i / C::RS) & 1, P.err, ERR_WAIT_RAW)) break;
      const uint8_t* raw = smem + C::OFF_RAW + rs * R::BYTES;
      const uint4* rp = reinterpret_cast<const uint4*>(raw + r * R::ROW);
      const uint32_t a_col = tmem + lane_base + C::A_COL0 + as * 128 + c0 * 32;
      uint32_t a0[32], a1[32];
      if constexpr (QT == GGUF_Q4_K) {
        const uint4 hdr = rp[0];
        uint4 qs[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) qs[2 * c0 + j] = rp[1 + 2 * c0 + j];
        raw_release(&raw_empty[rs]);
        unpack_q4<BF16>(qs, hdr, c0, a0);
        if (i >= C::ASB && !mbar_wait_warp(&a_empty[as], ((i / C::ASB) - 1) & 1, P.err, ERR_WAIT_MMA)) break;
        tmem_st32(a_col, a0);
        unpack_q4<BF16>(qs, hdr, c0 + 1, a1);
      } else {
        const uint4 p0 = rp[3 * c0], p1 = rp[3 * c0 + 1], p2 = rp[3 * c0 + 2];
        const uint4 p3 = rp[3 * c0 + 3], p4 = rp[3 * c0 + 4], p5 = rp[3 * c0 + 5];
        const uint4 sc = rp[12];
        const float d = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(raw + R::BODY)[r * 8 + ((sb_lo + i) & 7)]);
        raw_release(&raw_empty[rs]);
        unpack_q6<BF16>(p0, p1, p2, sc, d, c0, a0);
        if (i >= C::ASB && !mbar_wait_warp(&a_empty[as], ((i / C::ASB) - 1) & 1, P.err, ERR_WAIT_MMA)) break;
        tmem_st32(a_col, a0);
        unpack_q6<BF16>(p3, p4, p5, sc, d, c0 + 1, a1);
      }
      tmem_st32(a_col + 32, a1);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&a_full[as]);
    }
  }
  // epilogue warps: 0-3 for decode tiles, 0-7 for 128/256-token tiles (warps
  // w and w+4 share a TMEM lane quadrant and take one half of the tokens each)
  constexpr int EW = BN >= 128 ? 8 : 4;
  if (warp < EW) {
    // ---------------- epilogue (one tile row per thread) ----------------
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    constexpr int TPW = TPT / (EW / 4);  // tokens per epilogue warp
    const int tb = (warp >> 2) * TPW;    // this warp's first token
    const bool acc_ok = nq > 0 && mbar_wait_warp(acc_full, 0, P.err, ERR_WAIT_ACC);
    tc_fence_after();
    const int row = row0 + r;
    const int mt = min(TPT, P.m - tok0);  // live tokens of this tile
    float* dst;
    int64_t ldd;
    if (P.splits == 1) {
      dst = P.y + (int64_t)tok0 * P.n;
      ldd = P.n;
    } else {
      dst = P.ws + ((int64_t)z * P.m + tok0) * P.n;
      ldd = P.n;
    }
    const float bias = (P.splits == 1 && P.bias && row < P.n) ? P.bias[row] : 0.f;
    constexpr int E = BF16 ? 16 : 8;  // tokens per TMEM round trip
#pragma unroll 1
    for (int t0 = tb; t0 < tb + TPW; t0 += E) {
      float hi[E], lo[E];
#pragma unroll
      for (int j = 0; j < E; ++j) hi[j] = lo[j] = 0.f;
      if (acc_ok) {
#pragma unroll
        for (int set = 0; set < C::ACC_SETS; ++set) {
          uint32_t h[E], l[E];
          if constexpr (BF16) {
            tmem_ld16(tmem + lane_base + set * BN + t0, h);
          } else {
            tmem_ld8(tmem + lane_base + set * BN + t0, h);
            tmem_ld8(tmem + lane_base + set * BN + TPT + t0, l);
          }
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < E; ++j) {
            hi[j] += __uint_as_float(h[j]);
            if constexpr (!BF16) lo[j] += __uint_as_float(l[j]);
          }
        }
      }
      if (row < P.n) {
#pragma unroll
        for (int j = 0; j < E; ++j) {
          const int t = t0 + j;
          if (t < mt) {
            float v = hi[j];
            if constexpr (!BF16) v = (v + lo[j]) * P.tok_scale[tok0 + t];
            dst[(int64_t)t * ldd + row] = v + bias;
          }
        }
      }
    }
    if (P.splits > 1) {
      // the last CTA of this (row tile, token tile) adds the partials in split order
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"r"(32 * EW) : "memory");
      unsigned* ctr = P.counters + (blockIdx.y * gridDim.x + blockIdx.x);
      if (threadIdx.x == 0) last_cta = atomicAdd(ctr, 1u) == (unsigned)(P.splits - 1);
      asm volatile("bar.sync 1, %0;" ::"r"(32 * EW) : "memory");
      if (last_cta) {
        __threadfence();
        if (row < P.n) {
          const float b = P.bias ? P.bias[row] : 0.f;
          for (int t = tb; t < min(tb + TPW, mt); ++t) {
            float s = 0.f;
            for (int zz = 0; zz < P.splits; ++zz)
              s += __ldcg(&P.ws[((int64_t)zz * P.m + tok0 + t) * P.n + row]);
            P.y[(int64_t)(tok0 + t) * P.n + row] = s + b;
          }
        }
        if (threadIdx.x == 0) *ctr = 0u;
      }
    }
  }

  // teardown: every role is done with TMEM
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ---- activation prep ---------------------------------------------------------
// Position p of superblock kb in the MMA's K order holds element
// kb*256 + step_elem(s, c) + {0, 2, 1, 3}[p % 4] with c = (p % 256) / 64,
// s = (p % 64) / 4 -- the order unpack_q4 / unpack_q6 emit weights in.
template <int QT>
__device__ __forceinline__ int perm_elem(int p) {
  const int c = (p >> 6) & 3, s = (p >> 2) & 15, j = p & 3;
  const int e = QT == GGUF_Q4_K ? 64 * c + 32 * (s & 1) + 4 * (s >> 1)
                                : 128 * ((s >> 3) & 1) + 32 * (((s >> 2) & 1) + 2 * (s & 1)) + 8 * c + 4 * ((s >> 1) & 1);
  return (p & ~255) + e + ((j == 1) ? 2 : (j == 2) ? 1 : j);
}

// f32 x [m][k] -> f16 hi rows [tile*BN + j] and lo rows [tile*BN + TPT + j]
// (TPT = BN/2 tokens per tile), permuted, each token divided by 2^e so that
// max|x| / 2^e is in [2^13, 2^14).  One CTA per token slot.
template <int QT>
__global__ void __launch_bounds__(256) prep_f32_kernel(const float* __restrict__ x, int m, int k, int bn,
                                                       __half* __restrict__ xq, float* __restrict__ tok_scale) {
  const int slot = blockIdx.x;  // token slot 0 .. tiles*TPT-1
  const int tpt = bn / 2;
  const int tile = slot / tpt, j = slot % tpt;
  __half* hi = xq + ((int64_t)tile * bn + j) * k;
  __half* lo = xq + ((int64_t)tile * bn + tpt + j) * k;
  __shared__ float red[8];
  const bool live = slot < m;
  const float* xr = x + (int64_t)(live ? slot : 0) * k;
  float amax = 0.f;
  if (live)
    for (int i = threadIdx.x * 4; i < k; i += blockDim.x * 4) {
      const float4 v = *reinterpret_cast<const float4*>(xr + i);
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) amax = fmaxf(amax, red[w]);
  int e = 0;
  if (amax > 0.f && isfinite(amax)) e = ((__float_as_uint(amax) >> 23) & 0xff) - 127 - 13;
  e = max(-120, min(120, e));
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
  if (threadIdx.x == 0) tok_scale[slot] = live ? __uint_as_float((uint32_t)(127 + e) << 23) : 0.f;
  for (int p = threadIdx.x * 4; p < k; p += blockDim.x * 4) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) v = *reinterpret_cast<const float4*>(xr + perm_elem<QT>(p));  // e, e+1, e+2, e+3
    const float a0 = v.x * inv, a2 = v.z * inv, a1 = v.y * inv, a3 = v.w * inv;
    const __half2 h0 = __floats2half2_rn(a0, a2), h1 = __floats2half2_rn(a1, a3);
    const __half2 l0 = __floats2half2_rn(a0 - __low2float(h0), a2 - __high2float(h0));
    const __half2 l1 = __floats2half2_rn(a1 - __low2float(h1), a3 - __high2float(h1));
    *reinterpret_cast<__half2*>(hi + p) = h0;
    *reinterpret_cast<__half2*>(hi + p + 2) = h1;
    *reinterpret_cast<__half2*>(lo + p) = l0;
    *reinterpret_cast<__half2*>(lo + p + 2) = l1;
  }
}

// bf16 x [m][k] -> the same K order, one thread per 4 values.
template <int QT>
__global__ void __launch_bounds__(256) prep_bf16_kernel(const __nv_bfloat16* __restrict__ x, int m, int k,
                                                        __nv_bfloat16* __restrict__ xq) {
  const int64_t quads = (int64_t)m * (k / 4);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < quads; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / (k / 4));
    const int p = (int)(i - (int64_t)t * (k / 4)) * 4;
    const __nv_bfloat16* xr = x + (int64_t)t * k + perm_elem<QT>(p);
    const uint2 v = *reinterpret_cast<const uint2*>(xr);  // elements e .. e+3
    const uint32_t e01 = v.x, e23 = v.y;
    uint2 o;
    o.x = (e01 & 0xffffu) | (e23 << 16);          // e, e+2
    o.y = (e01 >> 16) | (e23 & 0xffff0000u);      // e+1, e+3
    *reinterpret_cast<uint2*>(xq + (int64_t)t * k + p) = o;
  }
}

// ---- host side --------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
    cudaGetLastError();
  });
  return fn;
}

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t inner,
                 uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swz) {
  EncodeTiled fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int QT, int BN, bool BF16>
cudaError_t launch_kernel(const CUtensorMap& wm, const CUtensorMap& dm, const CUtensorMap& xm, const Params& P,
                          dim3 grid, cudaStream_t s) {
  using C = Cfg<QT, BN>;
  kq_mma_kernel<QT, BN, BF16><<<grid, W::THREADS, C::SMEM, s>>>(wm, dm, xm, P);
  return cudaGetLastError();
}

template <int QT, int BN, bool BF16>
cudaError_t set_attr() {
  return cudaFuncSetAttribute(kq_mma_kernel<QT, BN, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Cfg<QT, BN>::SMEM);
}

template <int QT>
cudaError_t set_attrs_q() {
  cudaError_t e = cudaSuccess, r;
  if ((r = set_attr<QT, 16, false>()) != cudaSuccess) e = r;
  if ((r = set_attr<QT, 32, false>()) != cudaSuccess) e = r;
  if ((r = set_attr<QT, 64, false>()) != cudaSuccess) e = r;
  if ((r = set_attr<QT, 128, false>()) != cudaSuccess) e = r;
  if ((r = set_attr<QT, 256, false>()) != cudaSuccess) e = r;
  if ((r = set_attr<QT, 128, true>()) != cudaSuccess) e = r;
  if ((r = set_attr<QT, 256, true>()) != cudaSuccess) e = r;
  return e;
}

template <int QT, bool BF16>
cudaError_t launch_bn(int bn, const CUtensorMap& wm, const CUtensorMap& dm, const CUtensorMap& xm, const Params& P,
                      dim3 grid, cudaStream_t s) {
  switch (bn) {
    case 16: return launch_kernel<QT, 16, BF16>(wm, dm, xm, P, grid, s);
    case 32: return launch_kernel<QT, 32, BF16>(wm, dm, xm, P, grid, s);
    case 64: return launch_kernel<QT, 64, BF16>(wm, dm, xm, P, grid, s);
    case 128: return launch_kernel<QT, 128, BF16>(wm, dm, xm, P, grid, s);
    default: return launch_kernel<QT, 256, BF16>(wm, dm, xm, P, grid, s);
  }
}

int pick_bn_f32(int64_t m) {  // two columns (hi, lo) per token
  return m <= 8 ? 16 : m <= 16 ? 32 : m <= 32 ? 64 : m <= 64 ? 128 : 256;
}

// bf16 (prefill) tile width in tokens: 256, or 128 where 256-token tiles would
// leave SMs without a CTA (a 4096-row weight at 512 tokens: 64 CTAs of 256
// tokens, 128 of 128; each runs alone on its SM).
int pick_bn_bf16(int64_t m, int64_t n, int num_sms) {
  const int64_t rt = (n + TM - 1) / TM;
  return rt * ((m + 255) / 256) < num_sms ? 128 : 256;
}

int64_t splits_for(int64_t m, int64_t n, int64_t k, int num_sms) {
  const int bn = pick_bn_f32(m);
  const int64_t tiles = (m + bn / 2 - 1) / (bn / 2);
  const int64_t rt = (n + TM - 1) / TM;
  if (tiles > 1) return 1;
  // two CTAs fit per SM: fill one wave, never spill into a second one
  return std::max<int64_t>(1, std::min<int64_t>(k / QK, (2 * num_sms) / rt));
}

// scratch layout of the f32 path: xq | tok_scale | partials | counters
struct WsLayout {
  size_t xq, scale, part, ctr, end;
};
WsLayout ws_layout(int64_t m, int64_t n, int64_t k, int num_sms) {
  const int bn = pick_bn_f32(m);
  const int64_t tpt = bn / 2, tiles = (m + tpt - 1) / tpt;
  const int64_t rt = (n + TM - 1) / TM;
  const int64_t splits = splits_for(m, n, k, num_sms);
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  WsLayout L;
  L.xq = 0;
  L.scale = up((size_t)tiles * bn * k * 2);
  L.part = L.scale + up((size_t)tiles * tpt * 4);
  L.ctr = L.part + up((size_t)splits * m * n * 4);
  L.end = L.ctr + up((size_t)rt * tiles * 4);
  return L;
}

}  // namespace

cudaError_t tc_init_device() {
  cudaError_t e = set_attrs_q<GGUF_Q4_K>();
  cudaError_t e2 = set_attrs_q<GGUF_Q6_K>();
  return e != cudaSuccess ? e : e2;
}

void tc_counter_span(int64_t m, int64_t n, int64_t k, int num_sms, size_t* offset, size_t* count) {
  const WsLayout L = ws_layout(m, n, k, num_sms);
  *offset = L.ctr;
  *count = L.end - L.ctr;
}

bool tc_make_weight_maps(DevWeight& w) {
  if (w.type == GGUF_Q4_K || w.type == GGUF_Q5_K || w.type == GGUF_Q3_K || w.type == GGUF_Q2_K) {
    // one box = one superblock of 128 rows (Q5_K / Q3_K / Q2_K rows: sb x 176 / 112 / 96
    // bytes, the integer-MMA kernel's maps)
    const uint32_t bs = w.type == GGUF_Q4_K   ? Q4K_BYTES
                        : w.type == GGUF_Q5_K ? Q5K_BYTES
                        : w.type == GGUF_Q3_K ? Q3K_DEV
                                              : Q2K_DEV;
    const uint64_t rb = (uint64_t)w.sb * bs;
    if (!make_map_2d(&w.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.q, rb, (uint64_t)w.n, rb, bs, TM,
                     CU_TENSOR_MAP_SWIZZLE_NONE))
      return false;
    w.dmap = w.wmap;
    return true;
  }
  if (w.type != GGUF_Q6_K) return false;
  const uint64_t rb = (uint64_t)w.sb * Q6K_BODY;
  if (!make_map_2d(&w.wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.q, rb, (uint64_t)w.n, rb, Q6K_BODY, TM,
                   CU_TENSOR_MAP_SWIZZLE_NONE))
    return false;
  // d [n][d_ld]: one box = the d of 8 superblocks (16 bytes) for 128 rows
  return make_map_2d(&w.dmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w.d, (uint64_t)w.d_ld, (uint64_t)w.n,
                     (uint64_t)w.d_ld * 2, 8, TM, CU_TENSOR_MAP_SWIZZLE_NONE);
}

size_t tc_workspace_bytes(int64_t m, int64_t n, int64_t k, int num_sms) {
  return ws_layout(m, n, k, num_sms).ctr;
}

size_t tc_workspace_bytes_bf16(int64_t m, int64_t k) { return (size_t)m * k * 2 + 256; }

cudaError_t launch_tc_f32(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y, void* ws,
                          int num_sms, int* err, cudaStream_t s, int* launches, Bracket br,
                          unsigned* counters) {
  const int bn = pick_bn_f32(m);
  const int tpt = bn / 2;
  const int64_t tiles = (m + tpt - 1) / tpt;
  const int64_t rt = (w.n + TM - 1) / TM;
  const int64_t splits = splits_for(m, w.n, w.k, num_sms);
  const WsLayout L = ws_layout(m, w.n, w.k, num_sms);
  uint8_t* p = static_cast<uint8_t*>(ws);
  __half* xq = reinterpret_cast<__half*>(p + L.xq);
  float* tok_scale = reinterpret_cast<float*>(p + L.scale);
  float* part = reinterpret_cast<float*>(p + L.part);

  const int sbits = (int)(tiles * tpt);
  if (w.type == GGUF_Q4_K)
    prep_f32_kernel<GGUF_Q4_K><<<sbits, 256, 0, s>>>(x, (int)m, (int)w.k, bn, xq, tok_scale);
  else
    prep_f32_kernel<GGUF_Q6_K><<<sbits, 256, 0, s>>>(x, (int)m, (int)w.k, bn, xq, tok_scale);
  if (launches) ++*launches;
  CUtensorMap xm;
  if (!make_map_2d(&xm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xq, (uint64_t)w.k, (uint64_t)(tiles * bn),
                   (uint64_t)w.k * 2, KSTEP, bn, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  Params P{(int)w.n, (int)w.sb, (int)m, (int)splits, tok_scale, bias, y, part, counters, err};
  dim3 grid((unsigned)rt, (unsigned)tiles, (unsigned)splits);
  bracket_record(br.start, s);
  cudaError_t e = w.type == GGUF_Q4_K ? launch_bn<GGUF_Q4_K, false>(bn, w.wmap, w.dmap, xm, P, grid, s)
                                      : launch_bn<GGUF_Q6_K, false>(bn, w.wmap, w.dmap, xm, P, grid, s);
  bracket_record(br.stop, s);
  if (launches) ++*launches;
  return e;
}

cudaError_t launch_tc_bf16(const DevWeight& w, const void* x, int64_t m, const float* bias, float* y, void* ws,
                           int num_sms, int* err, cudaStream_t s, int* launches, Bracket br) {
  const int bn = pick_bn_bf16(m, w.n, num_sms);
  __nv_bfloat16* xq = static_cast<__nv_bfloat16*>(ws);
  const int64_t quads = m * (w.k / 4);
  const unsigned pg = (unsigned)std::min<int64_t>((quads + 255) / 256, 148 * 32);
  if (w.type == GGUF_Q4_K)
    prep_bf16_kernel<GGUF_Q4_K><<<pg, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), (int)m, (int)w.k, xq);
  else
    prep_bf16_kernel<GGUF_Q6_K><<<pg, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), (int)m, (int)w.k, xq);
  if (launches) ++*launches;
  CUtensorMap xm;
  if (!make_map_2d(&xm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xq, (uint64_t)w.k, (uint64_t)m, (uint64_t)w.k * 2,
                   KSTEP, bn, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  const int64_t rt = (w.n + TM - 1) / TM, tiles = (m + bn - 1) / bn;
  Params P{(int)w.n, (int)w.sb, (int)m, 1, nullptr, bias, y, nullptr, nullptr, err};
  dim3 grid((unsigned)rt, (unsigned)tiles, 1);
  bracket_record(br.start, s);
  cudaError_t e;
  if (bn == 128)
    e = w.type == GGUF_Q4_K ? launch_kernel<GGUF_Q4_K, 128, true>(w.wmap, w.dmap, xm, P, grid, s)
                            : launch_kernel<GGUF_Q6_K, 128, true>(w.wmap, w.dmap, xm, P, grid, s);
  else
    e = w.type == GGUF_Q4_K ? launch_kernel<GGUF_Q4_K, 256, true>(w.wmap, w.dmap, xm, P, grid, s)
                            : launch_kernel<GGUF_Q6_K, 256, true>(w.wmap, w.dmap, xm, P, grid, s);
  bracket_record(br.stop, s);
  if (launches) ++*launches;
  return e;
}

}  // namespace kq
