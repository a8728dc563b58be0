/* pesti_decoder.h -- decoder-step kernels around the quantized linears of
 * include/pesti_kq.h: the device form of pesti-runner's CPU decoder step
 * (transformer/layer.rs, rms_norm.rs, rope.rs, kv_cache.rs).  All pointers
 * are device pointers, work is queued on the context's stream, activations
 * are f32 batch-major [batch][dim], KV caches are f16
 * [batch][kv_heads][max_seq][head_dim].  Status codes as in pesti_kq.h. */
#ifndef PESTI_DECODER_H
#define PESTI_DECODER_H

#include <stddef.h>
#include <stdint.h>

#include "pesti_kq.h"

#ifdef __cplusplus
extern "C" {
#endif

/* out = x / sqrt(mean(x^2) + eps) * w per row (RmsNorm::forward, rms_norm.rs:24-43);
 * rows of x and out are x_ld / out_ld floats apart. */
int kq_dec_rmsnorm(kq_ctx *ctx, const float *x, int64_t x_ld, const float *w, float *out, int64_t out_ld,
                   int64_t rows, int64_t dim, float eps);
/* Token b's row qkv + b*ld holds q (heads x head_dim), k and v (kv_heads x
 * head_dim each).  Rotary embedding of q in place and of k at position `pos`
 * (pairs i, i + head_dim/2, angle pos * theta^(-i/(head_dim/2));
 * RopeConfig::apply_single, rope.rs:56-77), then the rotated k and v appended
 * to the caches at `pos` (LayerKvCache::append, kv_cache.rs:57-80), rounded
 * to f16. */
int kq_dec_rope_append(kq_ctx *ctx, float *qkv, int64_t ld, void *k_cache, void *v_cache, int64_t batch, int heads,
                       int kv_heads, int head_dim, int64_t pos, int64_t max_seq, float theta);
/* Scratch bytes kq_dec_attention needs for these sizes (0 if unsupported). */
size_t kq_dec_attention_scratch(kq_ctx *ctx, int64_t batch, int heads, int kv_heads, int head_dim, int64_t len);
/* Softmax(q . k^T / sqrt(head_dim)) . v over cache positions [0, len) with
 * grouped query heads (Attention::forward_with_cache, layer.rs:169-244); q
 * rows q_ld floats apart, out rows out_ld apart.  head_dim 64 or 128, heads /
 * kv_heads in {1, 2, 4, 7, 8}. */
int kq_dec_attention(kq_ctx *ctx, const float *q, int64_t q_ld, const void *k_cache, const void *v_cache,
                     float *out, int64_t out_ld, int64_t batch, int heads, int kv_heads, int head_dim, int64_t len,
                     int64_t max_seq, void *scratch, size_t scratch_bytes);
/* out[b][i] from gate_up[b] = [gate(ffn) | up(ffn)].  mode 0: pesti's
 * swiglu (layer.rs:16-29), whose negative-gate branch uses g / (1 + e^g) as
 * the sigmoid; mode 1: SiLU(gate) * up. */
int kq_dec_swiglu(kq_ctx *ctx, const float *gate_up, float *out, int64_t batch, int64_t ffn, int mode);
/* h[r][c] += y[r][c] for c < cols (the residual connections, layer.rs:346-368). */
int kq_dec_add(kq_ctx *ctx, float *h, int64_t h_ld, const float *y, int64_t y_ld, int64_t rows, int64_t cols);
/* out[b] = table[tokens[b]] (Model::embed, model.rs:966-984); table f32 [vocab][dim]. */
int kq_dec_embed(kq_ctx *ctx, const float *table, const int32_t *tokens, float *out, int64_t out_ld,
                 int64_t batch, int64_t dim);

#ifdef __cplusplus
}
#endif
#endif /* PESTI_DECODER_H */
