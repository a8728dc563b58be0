/*
 * kq_oracle.c -- CPU restatements used as the checker (test infrastructure
 * only; see kq_oracle.h).  Built with -O2 -ffp-contract=off so every f32
 * expression is evaluated exactly as written, one rounding per operation.
 */
#include "kq_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

float kqo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      /* subnormal: normalise into an f32 normal (exact) */
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while ((man & 0x400) == 0);
      man &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline uint16_t rd16(const uint8_t *p) {
  return (uint16_t)(p[0] | (p[1] << 8));
}

/* ------------------------------------------------------------------------ */
/* O1: GGUF Q4_K / Q6_K superblocks                                         */
/* ------------------------------------------------------------------------ */

int64_t kqo_gguf_row_bytes(int type, int64_t k) {
  int64_t bs = kqo_gguf_block_bytes(type);
  if (k <= 0 || (k % 256) != 0 || bs < 0) return -1;
  return (k / 256) * bs;
}

int64_t kqo_gguf_block_bytes(int type) {
  switch (type) {
    case KQO_GGUF_Q2_K: return 84;
    case KQO_GGUF_Q3_K: return 110;
    case KQO_GGUF_Q4_K: return 144;
    case KQO_GGUF_Q5_K: return 176;
    case KQO_GGUF_Q6_K: return 210;
    default: return -1;
  }
}

/* Q4_K superblock: d f16 | dmin f16 | 12 bytes of packed 6-bit (scale,min)
 * pairs for 8 sub-blocks of 32 | 128 bytes of nibbles.  Chunk c (0..3) owns
 * qs[32c..32c+31]; its low nibbles are sub-block 2c, high nibbles 2c+1.
 * value = (d*sc)*q - (dmin*m), each product exact in f32. */
static void q4k_scale_min(const uint8_t *s, int j, int *sc, int *m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

int kqo_dequant_q4_k(const uint8_t *blocks, int64_t nblocks, float *out) {
  if (nblocks < 0 || (!blocks && nblocks) || (!out && nblocks)) return KQO_ERR_ARG;
  for (int64_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 144;
    float d = kqo_f16_to_f32(rd16(blk));
    float dmin = kqo_f16_to_f32(rd16(blk + 2));
    const uint8_t *sc = blk + 4;
    const uint8_t *qs = blk + 16;
    float *o = out + b * 256;
    for (int c = 0; c < 4; ++c) {
      int s0, m0, s1, m1;
      q4k_scale_min(sc, 2 * c, &s0, &m0);
      q4k_scale_min(sc, 2 * c + 1, &s1, &m1);
      float d0 = d * (float)s0, dm0 = dmin * (float)m0;
      float d1 = d * (float)s1, dm1 = dmin * (float)m1;
      for (int l = 0; l < 32; ++l) {
        uint8_t byte = qs[32 * c + l];
        o[64 * c + l] = d0 * (float)(byte & 0x0f) - dm0;
        o[64 * c + 32 + l] = d1 * (float)(byte >> 4) - dm1;
      }
    }
  }
  return KQO_OK;
}

/* Q6_K superblock: ql[128] | qh[64] | int8 scales[16] | d f16.  Two halves of
 * 128; in half h, element 32g+l (g 0..3, l 0..31) takes the low (g=0,1) or
 * high (g=2,3) nibble of ql[64h + l + 32*(g&1)] and bits 2g..2g+1 of
 * qh[32h + l] as bits 4..5.  value = (d*scale[e/16]) * (q-32), exact. */
int kqo_dequant_q6_k(const uint8_t *blocks, int64_t nblocks, float *out) {
  if (nblocks < 0 || (!blocks && nblocks) || (!out && nblocks)) return KQO_ERR_ARG;
  for (int64_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 210;
    const uint8_t *ql = blk;
    const uint8_t *qh = blk + 128;
    const int8_t *scales = (const int8_t *)(blk + 192);
    float d = kqo_f16_to_f32(rd16(blk + 208));
    float *o = out + b * 256;
    for (int h = 0; h < 2; ++h) {
      for (int g = 0; g < 4; ++g) {
        for (int l = 0; l < 32; ++l) {
          int e = 128 * h + 32 * g + l;
          uint8_t qlb = ql[64 * h + l + 32 * (g & 1)];
          int lo = (g < 2) ? (qlb & 0x0f) : (qlb >> 4);
          int hi = (qh[32 * h + l] >> (2 * g)) & 3;
          int q = (lo | (hi << 4)) - 32;
          float ds = d * (float)scales[e / 16];
          o[e] = ds * (float)q;
        }
      }
    }
  }
  return KQO_OK;
}

/* Q5_K superblock: d f16 | dmin f16 | the 12 scale/min bytes of Q4_K | qh[32]
 * | qs[128].  Element e: chunk c = e/64 of qs (low nibbles for e%64 < 32,
 * high nibbles above), plus bit e/32 of qh[e%32] as bit 4; sub-block e/32
 * takes (sc, m) as in Q4_K.  value = (d*sc)*q - (dmin*m), q in [0, 31]. */
int kqo_dequant_q5_k(const uint8_t *blocks, int64_t nblocks, float *out) {
  if (nblocks < 0 || (!blocks && nblocks) || (!out && nblocks)) return KQO_ERR_ARG;
  for (int64_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 176;
    float d = kqo_f16_to_f32(rd16(blk));
    float dmin = kqo_f16_to_f32(rd16(blk + 2));
    const uint8_t *sc = blk + 4;
    const uint8_t *qh = blk + 16;
    const uint8_t *qs = blk + 48;
    float *o = out + b * 256;
    for (int e = 0; e < 256; ++e) {
      int j = e / 32, l = e % 32;
      int s, m;
      q4k_scale_min(sc, j, &s, &m);
      uint8_t byte = qs[32 * (e / 64) + l];
      int lo = (j & 1) ? (byte >> 4) : (byte & 0x0f);
      int q = lo | (((qh[l] >> j) & 1) << 4);
      float ds = d * (float)s, dm = dmin * (float)m;
      o[e] = ds * (float)q - dm;
    }
  }
  return KQO_OK;
}

/* Q2_K superblock: scales[16] (low nibble: scale, high nibble: min of each
 * 16-weight sub-block) | qs[64] | d f16 | dmin f16.  Element e: bits
 * 2*((e%128)/32) .. +1 of qs[32*(e/128) + e%32]; sub-block e/16.
 * value = (d*sc)*q - (dmin*m), q in [0, 3]. */
int kqo_dequant_q2_k(const uint8_t *blocks, int64_t nblocks, float *out) {
  if (nblocks < 0 || (!blocks && nblocks) || (!out && nblocks)) return KQO_ERR_ARG;
  for (int64_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 84;
    const uint8_t *sc = blk;
    const uint8_t *qs = blk + 16;
    float d = kqo_f16_to_f32(rd16(blk + 80));
    float dmin = kqo_f16_to_f32(rd16(blk + 82));
    float *o = out + b * 256;
    for (int e = 0; e < 256; ++e) {
      int s = e / 16;
      int q = (qs[32 * (e / 128) + e % 32] >> (2 * ((e % 128) / 32))) & 3;
      float dl = d * (float)(sc[s] & 0x0f);
      float ml = dmin * (float)(sc[s] >> 4);
      o[e] = dl * (float)q - ml;
    }
  }
  return KQO_OK;
}

/* Q3_K sub-block scale s (0..15): a 6-bit value whose low 4 bits are the low
 * (s < 8) or high (s >= 8) nibble of byte s%8, whose high 2 bits are bits
 * 2*(s/4) .. +1 of byte 8 + s%4; the signed scale is that value - 32. */
static int q3k_scale(const uint8_t *sc, int s) {
  int lo = s < 8 ? (sc[s] & 0x0f) : (sc[s - 8] >> 4);
  int hi = (sc[8 + s % 4] >> (2 * (s / 4))) & 3;
  return (lo | (hi << 4)) - 32;
}

/* Q3_K superblock: hmask[32] | qs[64] | scales[12] | d f16.  Element e: two
 * low bits as in Q2_K (qs[32*(e/128) + e%32] at bit 2*((e%128)/32)); the
 * third bit is bit e/32 of hmask[e%32], and a clear bit subtracts 4.
 * value = (d*scale[e/16]) * q, q in [-4, 3]. */
int kqo_dequant_q3_k(const uint8_t *blocks, int64_t nblocks, float *out) {
  if (nblocks < 0 || (!blocks && nblocks) || (!out && nblocks)) return KQO_ERR_ARG;
  for (int64_t b = 0; b < nblocks; ++b) {
    const uint8_t *blk = blocks + b * 110;
    const uint8_t *hm = blk;
    const uint8_t *qs = blk + 32;
    const uint8_t *sc = blk + 96;
    float d = kqo_f16_to_f32(rd16(blk + 108));
    float *o = out + b * 256;
    for (int e = 0; e < 256; ++e) {
      int lo = (qs[32 * (e / 128) + e % 32] >> (2 * ((e % 128) / 32))) & 3;
      int hb = (hm[e % 32] >> (e / 32)) & 1;
      int q = lo - (hb ? 0 : 4);
      float ds = d * (float)q3k_scale(sc, e / 16);
      o[e] = ds * (float)q;
    }
  }
  return KQO_OK;
}

int kqo_dequant_blocks(int type, const uint8_t *blocks, int64_t nblocks, float *out) {
  switch (type) {
    case KQO_GGUF_Q2_K: return kqo_dequant_q2_k(blocks, nblocks, out);
    case KQO_GGUF_Q3_K: return kqo_dequant_q3_k(blocks, nblocks, out);
    case KQO_GGUF_Q4_K: return kqo_dequant_q4_k(blocks, nblocks, out);
    case KQO_GGUF_Q5_K: return kqo_dequant_q5_k(blocks, nblocks, out);
    case KQO_GGUF_Q6_K: return kqo_dequant_q6_k(blocks, nblocks, out);
    default: return KQO_ERR_UNSUPPORTED;
  }
}

int kqo_gguf_dequant_rows(int type, const uint8_t *w, int64_t n, int64_t k,
                          int64_t row0, int64_t nrows, float *out) {
  int64_t rb = kqo_gguf_row_bytes(type, k);
  if (rb < 0) return KQO_ERR_UNSUPPORTED;
  if (row0 < 0 || nrows < 0 || row0 + nrows > n) return KQO_ERR_ARG;
  for (int64_t r = 0; r < nrows; ++r) {
    const uint8_t *row = w + (row0 + r) * rb;
    float *o = out + r * k;
    kqo_dequant_blocks(type, row, k / 256, o);
  }
  return KQO_OK;
}

typedef struct {
  int type;
  const uint8_t *w;
  int64_t n, k, m;
  const float *x, *bias;
  float *y;
  int64_t r0, r1;
  int rc;
} gguf_job;

static void *gguf_linear_worker(void *arg) {
  gguf_job *j = (gguf_job *)arg;
  float *row = (float *)malloc(sizeof(float) * (size_t)j->k);
  if (!row) {
    j->rc = KQO_ERR_ARG;
    return NULL;
  }
  for (int64_t o = j->r0; o < j->r1; ++o) {
    kqo_gguf_dequant_rows(j->type, j->w, j->n, j->k, o, 1, row);
    for (int64_t b = 0; b < j->m; ++b) {
      const float *xr = j->x + b * j->k;
      float acc = 0.0f;
      for (int64_t i = 0; i < j->k; ++i) acc += xr[i] * row[i];
      if (j->bias) acc += j->bias[o];
      j->y[b * j->n + o] = acc;
    }
  }
  free(row);
  j->rc = KQO_OK;
  return NULL;
}

int kqo_gguf_linear(int type, const uint8_t *w, int64_t n, int64_t k,
                    const float *x, int64_t m, const float *bias, float *y,
                    int nthreads) {
  if (kqo_gguf_row_bytes(type, k) < 0) return KQO_ERR_UNSUPPORTED;
  if (n < 0 || m < 0 || !w || !x || !y) return KQO_ERR_ARG;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  if (nthreads > n) nthreads = n > 0 ? (int)n : 1;
  pthread_t th[256];
  gguf_job jobs[256];
  for (int t = 0; t < nthreads; ++t) {
    gguf_job j = {type, w, n, k, m, x, bias, y,
                  n * t / nthreads, n * (t + 1) / nthreads, 0};
    jobs[t] = j;
  }
  for (int t = 1; t < nthreads; ++t)
    pthread_create(&th[t], NULL, gguf_linear_worker, &jobs[t]);
  gguf_linear_worker(&jobs[0]);
  int rc = jobs[0].rc;
  for (int t = 1; t < nthreads; ++t) {
    pthread_join(th[t], NULL);
    if (jobs[t].rc) rc = jobs[t].rc;
  }
  return rc;
}

/* ------------------------------------------------------------------------ */
/* O2: pesti-legacy blocks (the reference's own CPU decode)                 */
/* ------------------------------------------------------------------------ */

/* quantized_linear.rs:86-95 */
int64_t kqo_legacy_row_bytes(int type, int64_t in_features) {
  if (in_features < 0) return -1;
  if (type == KQO_PESTI_Q4_K_LEGACY) return ((in_features + 15) / 16) * 28;
  if (type == KQO_PESTI_Q5_K_LEGACY) return ((in_features + 15) / 16) * 36;
  if (type == KQO_PESTI_Q6_K_LEGACY) return ((in_features + 15) / 16) * 42;
  return -1;
}

/* tile_dequant.rs:223-293.  Full block (28 B): d f16 | delta f16 | qs_low u32 |
 * qs_high u32 | h0 f16 | h1 f16 | 12 unused.  Element i<8 uses nibble i of
 * qs_low with h0, i>=8 nibble i-8 of qs_high with h1:
 *   value = ((delta*h) * (q - 4.0)) + d      (evaluated left to right)
 * A trailing partial block (<16 elements) is 4 bytes (d, delta); its elements
 * all equal d. */
int kqo_legacy_dequant_q4_k_tile(const uint8_t *data, int64_t len,
                                 int64_t tile_size, float *out) {
  if (tile_size < 0 || len < 0) return KQO_ERR_ARG;
  int64_t nfull = tile_size / 16, rem = tile_size % 16;
  int64_t expected = nfull * 28 + (rem > 0 ? 4 : 0);
  if (len < expected) return KQO_ERR_SHORT;
  int64_t w = 0;
  for (int64_t b = 0; b < nfull; ++b) {
    const uint8_t *p = data + b * 28;
    float d = kqo_f16_to_f32(rd16(p));
    float delta = kqo_f16_to_f32(rd16(p + 2));
    uint32_t lo = (uint32_t)p[4] | ((uint32_t)p[5] << 8) |
                  ((uint32_t)p[6] << 16) | ((uint32_t)p[7] << 24);
    uint32_t hi = (uint32_t)p[8] | ((uint32_t)p[9] << 8) |
                  ((uint32_t)p[10] << 16) | ((uint32_t)p[11] << 24);
    float h0 = kqo_f16_to_f32(rd16(p + 12));
    float h1 = kqo_f16_to_f32(rd16(p + 14));
    for (int i = 0; i < 8; ++i) {
      float q = (float)((lo >> (4 * i)) & 0x0f);
      float t = delta * h0;
      t = t * (q - 4.0f);
      out[w++] = t + d;
    }
    for (int i = 0; i < 8; ++i) {
      float q = (float)((hi >> (4 * i)) & 0x0f);
      float t = delta * h1;
      t = t * (q - 4.0f);
      out[w++] = t + d;
    }
  }
  if (rem > 0) {
    float d = kqo_f16_to_f32(rd16(data + nfull * 28));
    for (int64_t i = 0; i < rem; ++i) out[w++] = d;
  }
  return KQO_OK;
}

/* tile_dequant.rs:141-180, 333-379.  Block (42 B): d f16 | 4 x f16 scales |
 * qs_low 8 B at +10 | flags 4 B at +18 | 20 pad.  Element i: q_low = 2 bits of
 * byte i/4 at +10 (bit 2*(i%4)), flag = 2 bits of byte i/4 at +18,
 * q = q_low + 4*(flag ? flag-1 : 0), value = (d * (q - 32.0)) * scale[i/4].
 * Blocks are always whole (ceil(tile/16) of them); output is truncated. */
int kqo_legacy_dequant_q6_k_tile(const uint8_t *data, int64_t len,
                                 int64_t tile_size, float *out) {
  if (tile_size < 0 || len < 0) return KQO_ERR_ARG;
  int64_t nb = (tile_size + 15) / 16;
  if (len < nb * 42) return KQO_ERR_SHORT;
  int64_t w = 0;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t *p = data + b * 42;
    float d = kqo_f16_to_f32(rd16(p));
    float sc[4];
    for (int s = 0; s < 4; ++s) sc[s] = kqo_f16_to_f32(rd16(p + 2 + 2 * s));
    for (int i = 0; i < 16 && w < tile_size; ++i) {
      int qlow = (p[10 + i / 4] >> ((i % 4) * 2)) & 3;
      int flag = (p[18 + i / 4] >> ((i % 4) * 2)) & 3;
      int qhigh = flag == 0 ? 0 : flag - 1;
      int q = qlow + 4 * qhigh;
      float t = d * ((float)q - 32.0f);
      out[w++] = t * sc[i / 4];
    }
  }
  return KQO_OK;
}

/* QuantizedLinear's Q5_K rows are 36 bytes per 16 weights
 * (quantized_linear.rs:91) but are decoded by the Q4_K tile routine
 * (quantized_linear.rs:170-173): the 28-byte Q4_K blocks are read from the
 * start of each 36-byte-per-16 row. */
static int legacy_tile(int type, const uint8_t *p, int64_t len, int64_t k,
                       float *out) {
  if (type == KQO_PESTI_Q4_K_LEGACY || type == KQO_PESTI_Q5_K_LEGACY)
    return kqo_legacy_dequant_q4_k_tile(p, len, k, out);
  return kqo_legacy_dequant_q6_k_tile(p, len, k, out);
}

int kqo_legacy_dequant_rows(int type, const uint8_t *data, int64_t len,
                            int64_t in_features, int64_t row0, int64_t nrows,
                            float *out) {
  int64_t rb = kqo_legacy_row_bytes(type, in_features);
  if (rb < 0) return KQO_ERR_UNSUPPORTED;
  if (row0 < 0 || nrows < 0) return KQO_ERR_ARG;
  for (int64_t r = 0; r < nrows; ++r) {
    int64_t off = (row0 + r) * rb;
    if (off >= len) return KQO_ERR_SHORT;
    int64_t end = off + rb < len ? off + rb : len;
    int rc = legacy_tile(type, data + off, end - off, in_features,
                         out + r * in_features);
    if (rc) return rc;
  }
  return KQO_OK;
}

typedef struct {
  const float *w;
  const float *x;
  float *y;
  int64_t k, n;
  int64_t b0, b1; /* batch rows */
  int64_t o0, o1; /* output rows */
} fwd_job;

typedef struct {
  int type;
  const uint8_t *data;
  int64_t len, k, o0, o1;
  float *w;
  int rc;
} deq_job;

static void *legacy_deq_worker(void *arg) {
  deq_job *j = (deq_job *)arg;
  j->rc = j->o1 > j->o0 ? kqo_legacy_dequant_rows(j->type, j->data, j->len, j->k, j->o0, j->o1 - j->o0,
                                                  j->w + j->o0 * j->k)
                        : KQO_OK;
  return NULL;
}

static void *legacy_fwd_worker(void *arg) {
  fwd_job *j = (fwd_job *)arg;
  for (int64_t b = j->b0; b < j->b1; ++b) {
    const float *xr = j->x + b * j->k;
    for (int64_t o = j->o0; o < j->o1; ++o) {
      const float *wr = j->w + o * j->k;
      float acc = 0.0f;
      for (int64_t i = 0; i < j->k; ++i) acc += xr[i] * wr[i];
      j->y[b * j->n + o] = acc;
    }
  }
  return NULL;
}

int kqo_legacy_forward(int type, const uint8_t *data, int64_t len,
                       int64_t in_features, int64_t out_features,
                       const float *x, int64_t batch, const float *bias,
                       float *y, int nthreads, int threads_over_batch) {
  int64_t k = in_features, n = out_features, m = batch;
  if (kqo_legacy_row_bytes(type, k) < 0) return KQO_ERR_UNSUPPORTED;
  if (k < 0 || n < 0 || m < 0 || !x || !y) return KQO_ERR_ARG;
  memset(y, 0, sizeof(float) * (size_t)(m * n));
  /* dequantize the full weight first, as quantized_linear.rs:108 does */
  float *w = (float *)malloc(sizeof(float) * (size_t)(n * k > 0 ? n * k : 1));
  if (!w) return KQO_ERR_ARG;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  int rc;
  if (threads_over_batch) {
    rc = kqo_legacy_dequant_rows(type, data, len, k, 0, n, w);
  } else {
    /* the all-cores variant also spreads the dequantization over the threads,
     * each taking the block of output rows it later multiplies */
    int nd = n < nthreads ? (int)(n > 0 ? n : 1) : nthreads;
    deq_job dj[256];
    for (int t = 0; t < nd; ++t) {
      deq_job j = {type, data, len, k, n * t / nd, n * (t + 1) / nd, w, 0};
      dj[t] = j;
    }
    for (int t = 1; t < nd; ++t) pthread_create(&th[t], NULL, legacy_deq_worker, &dj[t]);
    legacy_deq_worker(&dj[0]);
    rc = dj[0].rc;
    for (int t = 1; t < nd; ++t) {
      pthread_join(th[t], NULL);
      if (dj[t].rc && !rc) rc = dj[t].rc;
    }
  }
  if (rc) {
    free(w);
    return rc; /* the reference prints and returns the zeroed output */
  }
  fwd_job jobs[256];
  int nt;
  if (threads_over_batch) {
    nt = m < nthreads ? (int)(m > 0 ? m : 1) : nthreads;
    for (int t = 0; t < nt; ++t) {
      fwd_job j = {w, x, y, k, n, m * t / nt, m * (t + 1) / nt, 0, n};
      jobs[t] = j;
    }
  } else {
    nt = n < nthreads ? (int)(n > 0 ? n : 1) : nthreads;
    for (int t = 0; t < nt; ++t) {
      fwd_job j = {w, x, y, k, n, 0, m, n * t / nt, n * (t + 1) / nt};
      jobs[t] = j;
    }
  }
  for (int t = 1; t < nt; ++t)
    pthread_create(&th[t], NULL, legacy_fwd_worker, &jobs[t]);
  legacy_fwd_worker(&jobs[0]);
  for (int t = 1; t < nt; ++t) pthread_join(th[t], NULL);
  /* bias is added after the product (quantized_linear.rs:133-140) */
  if (bias)
    for (int64_t b = 0; b < m; ++b)
      for (int64_t o = 0; o < n; ++o) y[b * n + o] += bias[o];
  free(w);
  return KQO_OK;
}
