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
/* Scratch bytes kq_dec_attention / kq_dec_rope_attention need for these sizes
 * (len: the longest sequence the scratch will serve).  The scratch must be
 * zero-filled before its first use (it holds arrival counters that every
 * call leaves at zero). */
size_t kq_dec_attention_scratch(kq_ctx *ctx, int64_t batch, int heads, int kv_heads, int head_dim, int64_t len);
/* Softmax(q . k^T / sqrt(head_dim)) . v over cache positions [0, len) with
 * grouped query heads (Attention::forward_with_cache, layer.rs:169-244); q
 * rows q_ld floats apart, out rows out_ld apart.  head_dim 64 or 128, heads /
 * kv_heads in {1, 2, 4, 7, 8}. */
int kq_dec_attention(kq_ctx *ctx, const float *q, int64_t q_ld, const void *k_cache, const void *v_cache,
                     float *out, int64_t out_ld, int64_t batch, int heads, int kv_heads, int head_dim, int64_t len,
                     int64_t max_seq, void *scratch, size_t scratch_bytes);
/* kq_dec_rope_append followed by kq_dec_attention over [0, pos], in one
 * kernel: qkv rows as in kq_dec_rope_append; the query heads are rotated in
 * registers (qkv is not modified), the rotated k and v of position pos are
 * appended to the caches, and the attention output goes to out. */
int kq_dec_rope_attention(kq_ctx *ctx, const float *qkv, int64_t ld, void *k_cache, void *v_cache, float *out,
                          int64_t out_ld, int64_t batch, int heads, int kv_heads, int head_dim, int64_t pos,
                          int64_t max_seq, float theta, void *scratch, size_t scratch_bytes);
/* out[b][i] from gate_up[b] = [gate(ffn) | up(ffn)].  mode 0: pesti's
 * swiglu (layer.rs:16-29), whose negative-gate branch uses g / (1 + e^g) as
 * the sigmoid; mode 1: SiLU(gate) * up. */
int kq_dec_swiglu(kq_ctx *ctx, const float *gate_up, float *out, int64_t batch, int64_t ffn, int mode);
/* h[r][c] += y[r][c] for c < cols (the residual connections, layer.rs:346-368). */
int kq_dec_add(kq_ctx *ctx, float *h, int64_t h_ld, const float *y, int64_t y_ld, int64_t rows, int64_t cols);
/* Fused single-token linears (batch 1, GGUF Q4_K / Q6_K, in_features <= 30720):
 * the activation transform runs inside the GEMV's activation staging.
 * bias may alias y, which makes the call the residual update y += W . act(x).
 * KQ_ERR_UNSUPPORTED when the single-token kernel does not apply (the caller
 * then queues kq_dec_rmsnorm / kq_dec_swiglu and kq_linear_f32).
 *   norm_linear:   y = rmsnorm(x[0:dim]; norm_w, eps) . W^T + bias, the
 *                  normalised vector zero past dim (dim <= in_features, a
 *                  multiple of 4).  act -1: y has out_features values;
 *                  act 0 / 1 (SwiGLU mode as in kq_dec_swiglu): W's rows are
 *                  (gate, up) pairs and y[j] = swiglu(row 2j, row 2j+1), so
 *                  the FFN's gate and up projections and the SwiGLU are one
 *                  call (out_features / 2 values);
 *   swiglu_linear: y = swiglu(gate_up; mode) . W^T + bias with gate_up =
 *                  [gate (in_features) | up (in_features)], mode as in kq_dec_swiglu;
 *   residual_linear: h += x . W^T.
 * flags: KQ_SYNC or 0 (pointers are device pointers). */
int kq_dec_norm_linear(kq_ctx *ctx, const kq_weight *w, const float *x, const float *norm_w, int64_t dim, float eps,
                       int act, const float *bias, float *y, int flags);
int kq_dec_swiglu_linear(kq_ctx *ctx, const kq_weight *w, const float *gate_up, int mode, const float *bias, float *y,
                         int flags);
/* h[0:out_features] += x . W^T (the residual connection fused into the linear). */
int kq_dec_residual_linear(kq_ctx *ctx, const kq_weight *w, const float *x, float *h, int flags);
/* Batched forms (m tokens; GGUF Q4_K / Q5_K / Q6_K where the AUTO choice for
 * this weight and m is the integer tensor-core kernel: Q4_K / Q5_K 2 <= m <=
 * 64, Q6_K 3 <= m <= 8; KQ_ERR_UNSUPPORTED otherwise, with nothing queued,
 * and the caller queues kq_dec_rmsnorm / kq_linear_f32 / kq_dec_add).
 * No reference counterpart: the reference runs these steps one after the
 * other on the host (layer.rs:169-244).
 *   norm_linear_batch:     y[m][out_features] = rmsnorm(x[t][0:dim]; norm_w,
 *                          eps) . W^T, the normalised rows zero past dim
 *                          (dim a multiple of 4 <= in_features; x rows x_ld
 *                          floats apart, x_ld >= in_features and a multiple
 *                          of 4; x and norm_w 16-byte aligned);
 *   residual_linear_batch: h[m][out_features] += x[m][in_features] . W^T.
 * flags: KQ_SYNC or 0 (pointers are device pointers). */
int kq_dec_norm_linear_batch(kq_ctx *ctx, const kq_weight *w, const float *x, int64_t x_ld, int64_t m,
                             const float *norm_w, int64_t dim, float eps, float *y, int flags);
int kq_dec_residual_linear_batch(kq_ctx *ctx, const kq_weight *w, const float *x, int64_t m, float *h, int flags);
/* Tensor-parallel single-token linears (batch 1) for the column-split
 * layout: a projection whose input is split across the ranks (the output
 * projection over this rank's heads, the down projection over its FFN block)
 * holds W[:, this rank's columns] and produces a partial of the full output;
 * kq_dec_tp_partial_linear sends that partial to every rank (stores into
 * their exchange buffers over NVLink, inside the GEMV) and publishes the
 * exchange.  The next kq_dec_tp_reduce_linear on every rank waits for all
 * partials, forms h_out = h_in + sum over ranks (rank order: identical on
 * every rank), then y = [rmsnorm](h_out[0:dim]) . W^T with its own
 * (row-split or replicated) weight.  Two exchanges per transformer layer.
 *   partial: act -1 = x as is (in_features floats), 0 / 1 = SwiGLU mode of
 *            x = [gate | up] (as kq_dec_swiglu_linear); out_features =
 *            the partial's length.
 *   reduce:  norm_w NULL = no norm; dim = the partials' length; h_in and
 *            h_out distinct; act as in kq_dec_norm_linear (with a norm).
 *            Status codes as kq_dec_norm_linear. */
int kq_dec_tp_partial_linear(kq_tp *tp, const kq_weight *w, const float *x, int act, int flags);
int kq_dec_tp_reduce_linear(kq_tp *tp, const kq_weight *w, const float *h_in, float *h_out, const float *norm_w,
                            int64_t dim, float eps, int act, float *y, int flags);
/* ---- the batch-1 decode step as one persistent kernel ----------------------
 * A step program lists the step's linears and attention in order; one
 * cooperative launch of one CTA per SM runs them all (kq_step_run), a
 * producer warp per SM streaming every stage's weight rows and KV tile ahead
 * of the compute warps, grid barriers where a stage reads a vector other CTAs
 * wrote, and exchange words for the residual updates.  It replaces the
 * layer's separate kernels (the forward pass of transformer/layer.rs:344-372
 * per layer, model.rs:1025-1061 over the layers) with one launch per token.
 * Weights: GGUF Q4_K / Q6_K (in_features <= 30720).  Pointers are device
 * pointers; vectors are batch 1.
 *   in_mode:  PLAIN     x[0:in_features] as is;
 *             NORM      rmsnorm(x[0:dim]; norm_w, eps), zero past dim (dim a
 *                       multiple of 8);
 *             RESIDUAL  the new residual h' = h + u of the preceding PARTIAL
 *                       stage's update (the sum, in rank order, of the parts
 *                       every rank sent), also written to h; x is not read;
 *                       dim = the update's length;
 *             RESIDUAL_NORM  the same, then RMSNorm.
 *   out_mode: STORE     y[0:out_features];
 *             SWIGLU    W's rows are (gate, up) pairs, y[j] = swiglu(row 2j,
 *                       row 2j + 1; act) (act as kq_dec_swiglu's mode);
 *             PARTIAL   this rank's part of the update u of out_features
 *                       values (a column-split weight, or the whole weight on
 *                       one GPU) to the residual h (h NULL: a bare sum of the
 *                       parts); consumed by the next RESIDUAL stage; y unused.
 * kq_step_attention adds RoPE + KV append + attention of the new token
 * (heads / kv_heads heads of head_dim 64 or 128, group <= 8) over this rank's
 * caches [kv_heads][max_seq][head_dim] f16; qkv = q | k | v of this rank's
 * heads.  With a tensor-parallel group every rank builds the same sequence of
 * stages over its own shards.  kq_step_run(pos) queues one launch on the
 * context's stream; its first call sizes and allocates the step's scratch
 * (make it before any stream capture). */
typedef struct kq_step kq_step;
#define KQ_STEP_IN_PLAIN 0
#define KQ_STEP_IN_NORM 1
#define KQ_STEP_IN_RESIDUAL 2
#define KQ_STEP_IN_RESIDUAL_NORM 3
#define KQ_STEP_OUT_STORE 0
#define KQ_STEP_OUT_SWIGLU 1
#define KQ_STEP_OUT_PARTIAL 2
int kq_step_create(kq_ctx *ctx, kq_tp *tp, kq_step **out);
int kq_step_linear(kq_step *step, const kq_weight *w, int in_mode, const float *x, const float *norm_w, int64_t dim,
                   float eps, float *h, int out_mode, float *y, int act);
int kq_step_attention(kq_step *step, const float *qkv, void *k_cache, void *v_cache, float *out, int heads,
                      int kv_heads, int head_dim, int64_t max_seq, float theta);
int kq_step_run(kq_step *step, int64_t pos, int flags);
/* Profiling hook: while `trace` (device memory, words >= SMs x stages x 6) is
 * set, every run stores, per CTA and stage, six global-timer stamps (ns):
 * before the stage's grid barrier, after it, after the input staging (GEMV) or
 * the query rotation (attention), after the weight loop (attention: once the
 * first KV tile has landed), after the outputs (attention: after the KV loop),
 * and at the stage's end.  NULL stops it.  No reference counterpart. */
int kq_step_trace(kq_step *step, uint64_t *trace, size_t words);
int kq_step_destroy(kq_step *step);

/* out[b] = table[tokens[b]] (Model::embed, model.rs:966-984); table f32 [vocab][dim]. */
int kq_dec_embed(kq_ctx *ctx, const float *table, const int32_t *tokens, float *out, int64_t out_ld,
                 int64_t batch, int64_t dim);

#ifdef __cplusplus
}
#endif
#endif /* PESTI_DECODER_H */
