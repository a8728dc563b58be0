/*
 * pesti_kq.h -- C ABI of libpesti_kq.so, the B200 (sm_100a) K-quant linear
 * library.  This is the layer the reference's `cuda-oxide` crate stands for
 * (cuda-oxide/src/kernels.rs:4-36 and pesti-runner/src/dequantize_cuda.rs:12-55
 * are stubs that return "not yet implemented"); the Rust QuantizedLinear
 * (pesti-runner/src/quantized_linear.rs:12-183) binds to it as a drop-in.
 *
 * Conventions
 *  - Every entry returns an int status: KQ_OK (0) or a KQ_ERR_* code.  No entry
 *    aborts, traps or falls back to the CPU; kq_last_error() describes the
 *    most recent failure on a context.
 *  - A context owns one CUDA device and one stream (its own, or one the caller
 *    installs with kq_ctx_set_stream).  A context is not thread-safe: callers
 *    serialise use of one context (the Rust side wraps it in a Mutex).
 *  - Weights are immutable once uploaded and may be used from any context on
 *    the same device.
 *  - Pointer arguments of the compute entries are host pointers unless
 *    KQ_DEVICE_PTRS is set, in which case they are device pointers on the
 *    context's device and the call is stream-ordered (asynchronous unless
 *    KQ_SYNC is also set).  Host-pointer calls are synchronous, unless
 *    KQ_ASYNC queues them (the copies through the context's staging buffers
 *    are ordered on its stream, so queued calls may follow one another).
 */
#ifndef PESTI_KQ_H
#define PESTI_KQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KQ_ABI_VERSION 1

/* status codes */
#define KQ_OK 0
#define KQ_ERR_INVALID_ARG 1  /* null pointer, bad size, bad flag        */
#define KQ_ERR_UNSUPPORTED 2  /* unknown kq_type / shape not supported  */
#define KQ_ERR_CUDA 3         /* a CUDA runtime call failed             */
#define KQ_ERR_SHORT_BUFFER 4 /* weight bytes too short for the shape   */
#define KQ_ERR_NCCL 5         /* a collective failed                    */
#define KQ_ERR_STATE 6        /* call out of order (e.g. no TP group)   */
#define KQ_ERR_NOMEM 7        /* device allocation failed               */
#define KQ_ERR_FORMAT 8       /* file unreadable or not well-formed GGUF */

/* weight encodings (values follow GGML's type ids for the GGUF layouts) */
enum kq_type {
  KQ_GGUF_Q2_K = 10,          /* 84 B per 256 weights (CUDA-core kernels) */
  KQ_GGUF_Q3_K = 11,          /* 110 B per 256 weights (CUDA-core)        */
  KQ_GGUF_Q4_K = 12,          /* 144 B per 256 weights                    */
  KQ_GGUF_Q5_K = 13,          /* 176 B per 256 weights (CUDA-core)        */
  KQ_GGUF_Q6_K = 14,          /* 210 B per 256 weights                    */
  KQ_PESTI_Q4_K_LEGACY = 112, /* tile_dequant.rs 28 B per 16 weights      */
  KQ_PESTI_Q5_K_LEGACY = 113, /* QuantizedLinear Q5_K rows: 36 B per 16   */
                              /* weights read as 28 B Q4_K tiles          */
                              /* (quantized_linear.rs:91,170-173)         */
  KQ_PESTI_Q6_K_LEGACY = 114, /* tile_dequant.rs 42 B per 16 weights      */
};

/* flags of the compute entries */
#define KQ_HOST_PTRS 0   /* x / bias / y are host pointers (synchronous)  */
#define KQ_DEVICE_PTRS 1 /* x / bias / y are device pointers (async)      */
#define KQ_SYNC 2        /* synchronise the context stream before return  */
#define KQ_ACCUMULATE 4  /* kq_tp_allgather_f32 / _allreduce_f32: add into y  */
#define KQ_ASYNC 8       /* kq_linear_f32 / kq_linear_bf16 with host pointers:  */
                         /* queue the copies and kernels without waiting; the   */
                         /* caller keeps x, bias and y alive (pinned memory     */
                         /* lets the copies overlap) until kq_ctx_synchronize   */

/* kernel families for GGUF weights with f32 activations (kq_ctx_set_path) */
#define KQ_PATH_AUTO 0    /* default: DP4A m = 1; Q4_K IMMA m <= 64; Q6_K    */
                          /* DP4A m = 2, IMMA m <= 8, MMA m <= 64; TCGEN05   */
#define KQ_PATH_TCGEN05 1 /* tcgen05.mma, dequantized A written to TMEM      */
#define KQ_PATH_MMA 2     /* warp-level mma.sync tiles (cp.async staging)     */
#define KQ_PATH_DP4A 3    /* CUDA-core integer dot products, m <= 4 only;    */
                          /* larger m falls back to the AUTO choice          */
#define KQ_PATH_IMMA 4    /* integer mma.sync on the raw 4/6-bit codes        */
                          /* (TMA-fed 128-row tiles, split-K)                */
/* Q2_K / Q3_K / Q5_K: m = 1 under AUTO and DP4A runs the single-token dp4a  */
/* kernel (in_features <= 30720), 2 <= m <= 64 under AUTO and IMMA the      */
/* integer MMA kernel; every other case the CUDA-core f32 kernel.            */
/* KQ_PESTI_Q4_K_LEGACY / _Q6_K_LEGACY: m <= 4 with in_features a multiple  */
/* of 256 (<= 30720) under AUTO and DP4A runs the single-token dp4a kernel   */
/* once per token; every other case the block kernel.                        */

typedef struct kq_ctx kq_ctx;
typedef struct kq_weight kq_weight;
typedef struct kq_tp kq_tp;

/* ---- context ------------------------------------------------------------ */
/* New context on `device` with its own non-blocking stream.
 * Replaces cuda-oxide's device/stream placeholders (cuda-oxide/src/stream.rs:6-15). */
int kq_ctx_create(int device, kq_ctx **out);
int kq_ctx_destroy(kq_ctx *ctx);
/* Install an external cudaStream_t (NULL restores the context's own). */
int kq_ctx_set_stream(kq_ctx *ctx, void *cuda_stream);
/* Wait for the context stream; also reports a device-side pipeline error of
 * an earlier asynchronous call (KQ_ERR_CUDA with a message). */
int kq_ctx_synchronize(kq_ctx *ctx);
/* Select the kernel family for GGUF weights (KQ_PATH_*). */
int kq_ctx_set_path(kq_ctx *ctx, int path);
/* Reserve scratch for calls on weight `w` with up to `m` activation rows, so
 * that later calls allocate nothing (e.g. before CUDA-graph capture). */
int kq_ctx_reserve(kq_ctx *ctx, const kq_weight *w, int64_t m);
/* Hint: the compute call queued after the next one will read weight `next`.
 * The next linear call on this context (kq_linear_f32 and the fused decoder
 * linears, single-token GGUF kernel) prefetches `next` into L2 while it
 * streams its own weight, so the following call starts on cached data; the
 * hint is consumed by that call whatever path it takes.  NULL clears it.
 * No reference counterpart (pesti-runner's forward is synchronous). */
int kq_ctx_prefetch_next(kq_ctx *ctx, const kq_weight *next);
/* Number of kernels this context has launched so far. */
int64_t kq_ctx_launch_count(const kq_ctx *ctx);
/* Bracket the main kernel of each of the next `max_calls` compute calls with a
 * pair of CUDA events on the context stream (event nodes when the stream is
 * being captured into a CUDA graph).  kq_ctx_profile_end synchronises the
 * stream and returns the summed elapsed time of the recorded pairs (for a
 * replayed graph: of its most recent replay) and their count.  This is the
 * benchmark's timing hook; the reference has none (it times with Instant,
 * pesti-runner/examples/quant_bench.rs:89-101). */
int kq_ctx_profile_begin(kq_ctx *ctx, int max_calls);
int kq_ctx_profile_end(kq_ctx *ctx, double *total_ms, int64_t *count);
/* Same sums without ending the session: after each replay of a graph that
 * holds the brackets, this reads that replay's kernel times. */
int kq_ctx_profile_read(kq_ctx *ctx, double *total_ms, int64_t *count);
const char *kq_last_error(const kq_ctx *ctx);
const char *kq_status_string(int status);
int kq_abi_version(void);

/* ---- weights ------------------------------------------------------------ */
/* Bytes of one row of `in_features` weights in the given encoding (GGUF types:
 * in_features must be a multiple of 256).  Replaces QuantizedLinear::row_bytes
 * (quantized_linear.rs:86-95) for the legacy types, which it reproduces. */
int kq_row_bytes(int kq_type, int64_t in_features, int64_t *out);
/* Upload a row-major [out_features][row bytes] weight and keep it resident on
 * the context's device (QuantizedLinear::new / from_quantized,
 * quantized_linear.rs:27-67, with the bytes moved to HBM once).  `nbytes` must
 * cover every row (legacy: the last row only needs the bytes its tile reads).
 * `bytes` may be host memory or device memory of any GPU CUDA can address. */
int kq_weight_upload(kq_ctx *ctx, int kq_type, const void *bytes, size_t nbytes,
                     int64_t out_features, int64_t in_features, kq_weight **out);
int kq_weight_free(kq_weight *w);
int kq_weight_info(const kq_weight *w, int *kq_type, int64_t *out_features,
                   int64_t *in_features, int64_t *device_bytes);

/* ---- compute ------------------------------------------------------------ */
/* y[m][out] = x[m][in] . W[out][in] (+ bias[out]), f32 in and out.
 * QuantizedLinear::forward (quantized_linear.rs:101-143) / Linear::forward
 * (transformer/linear.rs:108-150).  bias may be NULL.  Every kq_type is
 * served; GGUF Q2_K / Q3_K / Q5_K run on one CUDA-core kernel family whatever
 * kq_ctx_set_path selects. */
int kq_linear_f32(kq_ctx *ctx, const kq_weight *w, const float *x, int64_t m,
                  const float *bias, float *y, int flags);
/* Prefill form: x is bf16 [m][in] (raw 16-bit values), y f32 [m][out].  The
 * weights are dequantized to bf16 tiles on the tensor cores (tcgen05); GGUF
 * weights only.  No reference counterpart: the reference has no prefill
 * dequant-GEMM. */
int kq_linear_bf16(kq_ctx *ctx, const kq_weight *w, const void *x_bf16, int64_t m,
                   const float *bias, float *y, int flags);
/* Same product for callers that must not allocate device memory during the
 * call.  No counterpart in the reference (its CPU path has no device memory).
 * GGUF weights, 1 <= m <= 4, device pointers only (flags must hold
 * KQ_DEVICE_PTRS).  Scratch comes from one fixed 256 KiB device array per
 * device (enough for in_features <= 16384); larger shapes are rejected with
 * KQ_ERR_UNSUPPORTED.  The array's address is looked up (host side) on every
 * call; the first lookup on a device may load the library's device code, so
 * make the first call on each device before any stream capture.  Calls on
 * one device that are not ordered with each other race on the shared scratch. */
int kq_linear_f32_static(kq_ctx *ctx, const kq_weight *w, const float *x, int64_t m,
                         const float *bias, float *y, int flags);
/* Dequantize rows [row0, row0+nrows) to f32 [nrows][in_features], bit-exact
 * with the CPU decode of the same encoding (QuantizedLinear::
 * dequantize_full_row_range, quantized_linear.rs:146-183, for legacy types). */
int kq_dequant_f32(kq_ctx *ctx, const kq_weight *w, int64_t row0, int64_t nrows,
                   float *out, int flags);

/* ---- tensor parallel (one process per GPU of one node) ------------------- */
/* Row-sharded linears whose output slices are all-gathered over NVLink: each
 * rank stores its rows straight into every rank's exchange buffer (CUDA IPC
 * peer memory) as 8-byte words {value, epoch of the call}; each rank reads
 * its full image once every word carries the call's epoch (no fences or
 * flags), and copies it out.  Replaces the survey's NCCL all-gather
 * policy (kq_tp_init with an NCCL id); no counterpart in the reference, which
 * is single-process CPU code.  Setup: kq_tp_create on every rank, exchange
 * the kq_tp_handle blobs (any host channel), kq_tp_open with all of them in
 * rank order.  max_out_elems bounds m * out_features of any call. */
int kq_tp_create(kq_ctx *ctx, int world, int rank, int64_t max_out_elems, kq_tp **out);
/* This rank's handle blob; with out == NULL only writes its size. */
int kq_tp_handle(const kq_tp *tp, void *out, size_t *size);
int kq_tp_open(kq_tp *tp, const void *handles, size_t nbytes);
/* y[m][n_total] = x[m][in] . W^T for a weight whose rows [row0, row0 +
 * out_features(shard)) this rank holds as `shard`; every rank of the group
 * must make the same sequence of calls.  Device pointers only (flags must hold
 * KQ_DEVICE_PTRS); bias is the shard's slice. */
int kq_tp_linear_f32(kq_tp *tp, const kq_weight *shard, int64_t row0, int64_t n_total,
                     const float *x, int64_t m, const float *bias, float *y, int flags);
/* The all-gather alone: y_local holds columns [row0, row0 + rows) of
 * y[m][n_total]; y's rows are y_ld floats apart (>= n_total).  With
 * KQ_ACCUMULATE in flags the gathered values are added to y (a residual). */
int kq_tp_allgather_f32(kq_tp *tp, const float *y_local, int64_t m, int64_t row0, int64_t rows,
                        int64_t n_total, float *y, int64_t y_ld, int flags);
/* All-reduce of per-rank partials (no reference counterpart: the reference
 * runs on one device): partial[m][n] is this rank's contribution; y[m][n]
 * (rows y_ld floats apart) receives the sum over the ranks, taken in rank
 * order so every rank holds the same bits, or with KQ_ACCUMULATE has it
 * added.  Needs world x m x n <= the group's max_out_elems.  Device pointers
 * only; every rank makes the same sequence of calls. */
int kq_tp_allreduce_f32(kq_tp *tp, const float *partial, int64_t m, int64_t n, float *y, int64_t y_ld, int flags);
int kq_tp_destroy(kq_tp *tp);

/* ---- GGUF files ----------------------------------------------------------- */
/* A GGUF (version 2 or 3) file's metadata and tensor directory, read once on
 * open; tensor bytes are read on demand.  Stands in for the external
 * pesti-gguf reader the reference calls to get raw tensor bytes
 * (extract_tensor_bytes_from_path, pesti-runner/src/gguf_weight_loader.rs:
 * 79-81; GgufDtype / stored_size, :20-21).  Host code: no context or GPU is
 * needed except for kq_gguf_upload.  A malformed file gives KQ_ERR_FORMAT and
 * a message in err (err_len bytes, may be 0). */
typedef struct kq_gguf kq_gguf;
int kq_gguf_open(const char *path, kq_gguf **out, char *err, size_t err_len);
void kq_gguf_close(kq_gguf *f);
/* Tensors: index 0 .. count-1 in file order; -1 when not found. */
int64_t kq_gguf_tensor_count(const kq_gguf *f);
int64_t kq_gguf_find_tensor(const kq_gguf *f, const char *name);
/* ggml_type: the file's type code (12 Q4_K, 14 Q6_K, 0 F32, ...); dims[4]:
 * ne[0] (innermost, the row length) first, unused dims 1; file_offset:
 * absolute; nbytes: 0 for a type the reader does not size.  name stays valid
 * until kq_gguf_close. */
int kq_gguf_tensor_info(const kq_gguf *f, int64_t i, const char **name, int *ggml_type, int *n_dims,
                        int64_t *dims, uint64_t *file_offset, uint64_t *nbytes);
/* The tensor's bytes as stored into dst (dst_bytes >= nbytes). */
int kq_gguf_read_tensor(const kq_gguf *f, int64_t i, void *dst, uint64_t dst_bytes);
/* A 2-D Q2_K / Q3_K / Q4_K / Q5_K / Q6_K tensor [ne1 rows][ne0] as a
 * device-resident weight (out_features = ne[1], in_features = ne[0]),
 * through kq_weight_upload. */
int kq_gguf_upload(kq_ctx *ctx, const kq_gguf *f, int64_t i, kq_weight **out);
/* Metadata: value_type / elem_type are GGUF's codes (0 u8 .. 12 f64, 8
 * string, 9 array; elem_type -1 unless an array); count: 1 for a scalar or a
 * string, the element count of an array.  Nested arrays are listed with their
 * count only.  kq_gguf_meta_int takes any integer or bool scalar,
 * kq_gguf_meta_float any number; kq_gguf_meta_string a string (j = 0) or
 * element j of a string array; kq_gguf_meta_array the packed little-endian
 * elements of a numeric array.  Pointers stay valid until kq_gguf_close. */
int64_t kq_gguf_meta_count(const kq_gguf *f);
int64_t kq_gguf_find_meta(const kq_gguf *f, const char *key);
int kq_gguf_meta_info(const kq_gguf *f, int64_t i, const char **key, int *value_type, int *elem_type,
                      uint64_t *count);
int kq_gguf_meta_int(const kq_gguf *f, int64_t i, int64_t *v);
int kq_gguf_meta_float(const kq_gguf *f, int64_t i, double *v);
int kq_gguf_meta_string(const kq_gguf *f, int64_t i, uint64_t j, const char **s, uint64_t *len);
int kq_gguf_meta_array(const kq_gguf *f, int64_t i, const void **data, uint64_t *elem_bytes);

#ifdef __cplusplus
}
#endif
#endif /* PESTI_KQ_H */
