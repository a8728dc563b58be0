// kq_kernels.h -- internal launch interface between the C-ABI layer
// (kq_api.cu) and the kernels.  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kq {

constexpr int QK = 256;         // weights per K-quant superblock
constexpr int Q4K_BYTES = 144;  // GGUF Q4_K superblock
constexpr int Q6K_BYTES = 210;  // GGUF Q6_K superblock
constexpr int Q6K_BODY = 208;   // device Q6_K body: ql(128) | qh(64) | scales(16)
constexpr int Q2K_BYTES = 84;   // GGUF Q2_K superblock
constexpr int Q2K_DEV = 96;     // device Q2_K superblock: the 84 bytes + 12 zero bytes (16-byte aligned)
constexpr int Q3K_BYTES = 110;  // GGUF Q3_K superblock
constexpr int Q3K_DEV = 112;    // device Q3_K superblock: the 110 bytes + 2 zero bytes (16-byte aligned)
constexpr int Q5K_BYTES = 176;  // GGUF Q5_K superblock (stored as is)

enum QType : int {
  GGUF_Q2_K = 10,
  GGUF_Q3_K = 11,
  GGUF_Q4_K = 12,
  GGUF_Q5_K = 13,
  GGUF_Q6_K = 14,
  LEGACY_Q4_K = 112,
  LEGACY_Q5_K = 113,  // QuantizedLinear's Q5_K: 36 B per 16 weights, decoded as Q4_K tiles
  LEGACY_Q6_K = 114,
};

// Device-resident weight.  For GGUF types the row count is n, the row length k
// (a multiple of 256) and sb = k/256 superblocks per row.
//  GGUF_Q4_K: q = raw GGUF superblocks [n][sb][144]; d unused.
//  GGUF_Q6_K: q = bodies [n][sb][208] (ql|qh|scales), d = f16 [n][d_ld]
//             (row-major, d_ld = sb rounded up to 8 so every row's d is a
//             whole number of 16-byte units and a block of rows is one run).
//  GGUF_Q5_K: q = raw superblocks, rows row_bytes = 176 sb apart.
//  GGUF_Q3_K / Q2_K: q = superblocks at a 112 / 96-byte stride (each padded
//             with zero bytes, so every superblock starts on a 16-byte
//             boundary and is one TMA box column), rows row_bytes = 112 / 96 sb
//             apart.
//  LEGACY_*:  q = raw bytes as uploaded (row stride = legacy row bytes), len.
// wmap / dmap: TMA descriptors of q (128 rows x one superblock per box) and d.
struct DevWeight {
  int type;
  int64_t n, k, sb;
  const uint8_t* q;
  const uint16_t* d;
  int64_t d_ld;
  int64_t len;        // uploaded byte count (legacy) / device bytes
  int64_t row_bytes;  // row stride: legacy types and GGUF Q2_K / Q3_K / Q5_K
  CUtensorMap wmap, dmap;
};

__host__ __device__ inline int64_t q6k_d_ld(int64_t sb) { return (sb + 7) & ~int64_t(7); }

// One-time per-device kernel set-up (shared-memory carve-outs); call with the
// device current, outside any stream capture.
cudaError_t gemv_init_device();

// Scratch needed by launch_gemv_gguf for an m x k activation (bytes): the
// permuted activations and per-run activation sums.
size_t gemv_gguf_workspace_bytes(int64_t m, int64_t k);

// Optional timing bracket: when both events are set they are recorded on the
// stream immediately before and after the main (weight-streaming) kernels.
struct Bracket {
  cudaEvent_t start = nullptr, stop = nullptr;
};

// Launch with programmatic dependent launch allowed: the kernel may start
// while its predecessor on the stream finishes; it must execute
// griddepcontrol.wait before reading anything the predecessor writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// Record a timing event; under stream capture it becomes an event-record node
// of the graph (cudaEventRecordExternal), so graph replays keep timing it.
inline void bracket_record(cudaEvent_t e, cudaStream_t s) {
  if (e) cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
}

// y[m][n] = x[m][k] . W[n][k] (+ bias[n]) for GGUF Q4_K / Q6_K weights; x, y,
// bias are device pointers.  `ws` must hold gemv_gguf_workspace_bytes(m, k)
// bytes, 16-byte aligned.  `launches` (nullable) is incremented per kernel.
cudaError_t launch_gemv_gguf(const DevWeight& w, const float* x, int64_t m, const float* bias,
                             float* y, void* ws, cudaStream_t s, int* launches,
                             Bracket br = Bracket());

// Same product for pesti-legacy weights (no workspace).
cudaError_t launch_gemv_legacy(const DevWeight& w, const float* x, int64_t m, const float* bias,
                               float* y, cudaStream_t s, int* launches, Bracket br = Bracket());

// Bit-exact dequantization of rows [row0, row0+nrows) to f32 [nrows][k].
cudaError_t launch_dequant_f32(const DevWeight& w, int64_t row0, int64_t nrows, float* out,
                               cudaStream_t s);

// Re-lay GGUF Q6_K superblocks [n][sb][210] into bodies [n][sb][208] and
// d [n][d_ld] (padding entries are left as they are).
cudaError_t launch_q6k_relayout(const uint8_t* raw, int64_t n, int64_t sb, uint8_t* body, uint16_t* d,
                                cudaStream_t s);

// ---- GGUF Q2_K / Q3_K / Q5_K: kq_kx.cu ----
bool kx_type(int type);
int64_t kx_block_bytes(int type);  // bytes of one 256-weight superblock (0: not one of these types)
int64_t kx_dev_stride(int type);   // device bytes between superblocks of a row
cudaError_t kx_init_device();
// y = x . W^T (+bias), f32 x and y, any m (tiles of up to 8 tokens per launch).
cudaError_t launch_gemv_kx(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y, cudaStream_t s,
                           int* launches, Bracket br = Bracket());
// Bit-exact dequantization of rows [row0, row0 + nrows) to f32 [nrows][k].
cudaError_t launch_dequant_kx(const DevWeight& w, int64_t row0, int64_t nrows, float* out, cudaStream_t s);

// ---- integer tensor-core batched decode, GGUF Q4_K / Q5_K / Q6_K: kq_imma.cu ----
cudaError_t imma_init_device();
// Scratch (bytes) for m tokens of an n x k weight, and the zeroed counters.
size_t imma_workspace_bytes(int64_t m, int64_t n, int64_t k, int num_sms);
size_t imma_counter_bytes(int64_t n);
// Options of the batched decoder forms: x rows x_ld floats apart (0: k);
// nw != nullptr: the activations are RMSNorm(x[0:dim]; nw, eps), zero past dim
// (dim a multiple of 4, x rows 16-byte aligned); accumulate: y += the product.
struct ImOpts {
  int64_t x_ld = 0;
  const float* nw = nullptr;
  int dim = 0;
  float eps = 0.f;
  bool accumulate = false;
};
// y = x . W^T (+bias) for GGUF Q4_K / Q5_K / Q6_K (cudaErrorNotSupported
// otherwise); any m, in chunks of 32 tokens; *err receives 27 / 28 if a
// pipeline wait gave up.
cudaError_t launch_gemv_imma(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y, void* ws,
                             unsigned* ctr, int num_sms, int* err, cudaStream_t s, int* launches,
                             Bracket br = Bracket(), const ImOpts& op = ImOpts());

// ---- CUDA-core integer decode path: kq_dp4a.cu ----
constexpr int DP4A_MAX_M = 4;
// Per-device set-up of the dp4a kernels (shared-memory carve-outs).
cudaError_t dp4a_init_device();
// Scratch for launch_gemv_dp4a (prepared activations for m tokens).
size_t dp4a_workspace_bytes(int type, int64_t m, int64_t sb);
// y = x . W^T (+bias) for GGUF Q4_K / Q6_K, 1 <= m <= DP4A_MAX_M, f32 x.
// The batched dp4a kernels (prepare + GEMV) with caller-provided scratch of
// dp4a_workspace_bytes(type, m, sb) bytes; 1 <= m <= DP4A_MAX_M.
cudaError_t launch_gemv_dp4a_batched(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y,
                                     void* ws, int num_sms, cudaStream_t s, int* launches);
// Fixed scratch of DP4A_STATIC_SCRATCH bytes in device memory (a file-scope
// __device__ array): its address on the current device, looked up once per
// device.  Used by the no-allocation entry point.
constexpr size_t DP4A_STATIC_SCRATCH = 256 * 1024;
cudaError_t dp4a_static_scratch(void** ptr);
// Up to two byte ranges (a weight's quants and, for Q6_K, its d array) the
// single-token kernel prefetches into L2 while it runs: the weight the next
// kernel on the stream will read.
struct Prefetch {
  const void* p[2] = {nullptr, nullptr};
  int64_t bytes[2] = {0, 0};
};
// *err (device int) receives a nonzero code if a pipeline wait gave up.
cudaError_t launch_gemv_dp4a(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y,
                             void* ws, int num_sms, int* err, cudaStream_t s, int* launches,
                             Bracket br = Bracket(), const Prefetch* pf = nullptr);
// Activation source of the single-token kernel.  The REDUCE forms are the
// tensor-parallel consumers: x = h_in + the partial vectors every rank sent
// in the last exchange (summed in rank order, so every rank gets the same
// bits), written to h_out, then (REDUCE_NORM) RMS-normalised.
enum : int { XS_X_PLAIN = 0, XS_X_NORM = 1, XS_X_SWIGLU = 2, XS_X_REDUCE = 3, XS_X_REDUCE_NORM = 4 };
// Destination of y: this rank's buffer, or (XS_Y_PEERS) slot rows
// [rank * n, rank * n + n) of every rank's exchange image, then the
// exchange's epoch is published in every rank's flags.
// XS_Y_SWIGLU: the weight's rows are (gate, up) pairs and y[j] =
// swiglu_gate(row 2j, act) * row 2j+1 (n / 2 outputs).
enum : int { XS_Y_LOCAL = 0, XS_Y_PEERS = 1, XS_Y_SWIGLU = 2 };
constexpr int TP_MAX_WORLD = 8;
// Exchange buffers (as in TpArgs): two slots of slot_elems 8-byte words.
// A word is {f32 value bits, epoch}: a reader takes a value once its word
// carries the epoch of the exchange it waits for, so no fences or flags are
// needed (each 64-bit word is stored and loaded as one single-copy-atomic
// access).  Slot = epoch % 2.
struct XsTp {
  unsigned long long* exch[TP_MAX_WORLD] = {};  // every rank's buffer, mapped here
  int64_t slot_elems = 0;
  int world = 1, rank = 0;
  unsigned* ctr = nullptr;          // CTA arrival counter (zero between calls)
  unsigned* epoch = nullptr;        // last published exchange epoch
  const float* h_in = nullptr;      // REDUCE: residual stream in / out
  float* h_out = nullptr;
};
struct XsInput {
  int mode = XS_X_PLAIN;
  int ymode = XS_Y_LOCAL;
  XsTp tp;                    // REDUCE modes and XS_Y_PEERS
  const float* x = nullptr;   // [k] (XS_X_SWIGLU: the gate)
  const float* x2 = nullptr;  // XS_X_SWIGLU: the up projection [k]
  const float* nw = nullptr;  // XS_X_NORM: norm weights [dim]
  int dim = 0;                // XS_X_NORM: elements normalised (x and the result are zero past dim)
  float eps = 0.f;
  int act = 0;                // XS_X_SWIGLU / XS_Y_SWIGLU: gate activation (swiglu_gate)
};
// Single-token GEMV y = act(x) . W^T (+bias; bias may alias y) for GGUF
// Q4_K / Q6_K; cudaErrorNotSupported when the kernel does not apply to the
// shape (more than 120 superblocks per row).
cudaError_t launch_gemv_xs(const DevWeight& w, const XsInput& in, const float* bias, float* y, int num_sms, int* err,
                           const Prefetch* pf, cudaStream_t s, int* launches, Bracket br = Bracket());

// ---- persistent batch-1 decode step: kq_step.cu ----
constexpr int STEP_COMPUTE_WARPS = 15;
constexpr int STEP_THREADS = 32 * (STEP_COMPUTE_WARPS + 1);
constexpr int STEP_MAX_SMEM = 227 * 1024 - 1024;  // dynamic shared memory (static use stays below 1 KB)
constexpr int STEP_ATTN_MAX_GROUP = 8;            // query heads per KV head
constexpr int STEP_TRACE_POINTS = 6;              // global-timer stamps per CTA and stage
// sync words (zero between launches): barrier arrivals, exits, then one
// arrival counter per KV head of the attention stages
enum : int { STEP_SYNC_BAR = 0, STEP_SYNC_EXIT = 1, STEP_SYNC_ATTN = 2 };
enum : int { STEP_GEMV = 0, STEP_ATTN = 1 };
// GEMV input: x as is; RMSNorm of x[0:dim]; x = the sum of the pending
// exchange's parts (the new residual, written to h_out), optionally RMS-normalised
enum : int { SX_PLAIN = 0, SX_NORM = 1, SX_REDUCE = 2, SX_REDUCE_NORM = 3 };
// GEMV output: y; SwiGLU of (gate, up) row pairs into y; this rank's part of
// a residual update, sent to every rank as exchange words (rank 0 adds h_in,
// the residual being updated)
enum : int { SY_STORE = 0, SY_SWIGLU = 1, SY_PARTIAL = 2 };
struct StepStage {
  int kind = STEP_GEMV;
  int barrier = 0;  // grid barrier before the stage (its input was produced by other CTAs)
  // GEMV (GGUF Q4_K / Q6_K)
  int qt = 0, n = 0, sb = 0, nk = 0, G = 0;
  int64_t row_bytes = 0;
  int d_row_bytes = 0;
  const uint8_t* q = nullptr;
  const uint16_t* d = nullptr;
  int xmode = SX_PLAIN, ymode = SY_STORE;
  const float* x = nullptr;   // PLAIN / NORM input
  const float* nw = nullptr;  // NORM weights
  int dim = 0;                // NORM / REDUCE: vector length
  float eps = 0.f;
  int act = 0;                // SWIGLU gate activation
  float* y = nullptr;
  int exch = 0;               // REDUCE: exchange read; PARTIAL: exchange written (index within the step)
  const float* h_in = nullptr;  // PARTIAL: the residual the update applies to (rank 0 adds it), or NULL
  float* h_out = nullptr;       // REDUCE: receives the new residual
  // ATTN (batch 1): qkv row = q (hq heads) | k (hkv) | v (hkv), caches [hkv][max_seq][hd] f16
  const float* qkv = nullptr;
  void* kc = nullptr;
  void* vc = nullptr;
  float* out = nullptr;       // [hq][hd]
  int hq = 0, hkv = 0, hd = 0, splits = 0, tile = 0;
  int64_t max_seq = 0;
  float theta = 0.f;
};
struct StepArgs {
  const StepStage* stages = nullptr;
  int nstages = 0;
  int64_t pos = 0;                 // the new token's position
  unsigned* sync = nullptr;        // STEP_SYNC_* words
  float* attn_part = nullptr;      // [hkv][splits][G][hd + 4] partials of the attention splits
  int* err = nullptr;
  unsigned long long* exch[TP_MAX_WORLD] = {};  // every rank's exchange buffer (two slots)
  int64_t slot_elems = 0;
  int world = 1, rank = 0;
  unsigned* epoch = nullptr;       // last published exchange epoch of this rank
  int nexch = 0;                   // exchanges per step
  int S = 0, slot_bytes = 0, nk_max = 0, rows_max = 0, xr_floats = 0, nw_floats = 0, attn_bytes = 0;
  unsigned long long* trace = nullptr;  // optional [CTAs][stages][STEP_TRACE_POINTS] global-timer stamps
};
// Dynamic shared memory of the step kernel: ring | staged x | sums | 2^e per
// superblock | row partials | reduction | reduced x (REDUCE) | barriers; the
// attention scratch reuses the staging area.
struct StepSmem {
  size_t ring, xw, sums, xsf, part, red, xr, nw, attn, bar, end;
  __host__ __device__ StepSmem(int S, int slot_bytes, int nk_max, int rows_max, int xr_floats, int nw_floats,
                               int attn_bytes) {
    const size_t units = (size_t)8 * nk_max * 4;
    ring = 0;
    xw = (size_t)S * (size_t)slot_bytes;
    sums = xw + units * 128;
    xsf = sums + units * 64;
    part = xsf + units;
    red = (part + (size_t)rows_max * nk_max * 4 + 15) & ~size_t(15);
    xr = red + 32 * 4;
    nw = xr + (size_t)xr_floats * 4;
    attn = xw;
    const size_t gemv_end = nw + (size_t)nw_floats * 4, attn_end = attn + (size_t)attn_bytes;
    bar = ((gemv_end > attn_end ? gemv_end : attn_end) + 15) & ~size_t(15);
    end = bar + (size_t)2 * S * 8;
  }
};
cudaError_t step_init_device();
// One cooperative launch of `grid` CTAs (the SM count: one per SM).
cudaError_t launch_step(const StepArgs& a, int grid, cudaStream_t s);

// ---- tensor parallel: all-gather of row-sharded outputs over peer memory (kq_tp.cu) ----
struct TpArgs {
  const float* y_local;                  // [m][r1 - r0] this rank's block
  float* y_out;                          // [m][y_ld] the gathered result (first n columns)
  int64_t y_ld;
  int accumulate;                        // nonzero: y_out += gathered
  int64_t m, n, r0, r1;                  // tokens, total columns, this rank's columns
  unsigned long long* exch[TP_MAX_WORLD];  // every rank's exchange buffer: 2 slots of max_elems words
  int64_t max_elems;
  int world, rank;
  unsigned* epoch;                       // local device counter: the last completed call's epoch
  unsigned* ctr;                         // zero between calls (last-CTA detection)
  int* err;                              // set to a nonzero code if a wait gave up
};
// One launch per call; `blocks` must fit the GPU at once (<= SM count).
cudaError_t launch_tp_allgather(const TpArgs& a, int blocks, cudaStream_t s);
// All-reduce: y_local [m][n] is this rank's partial (r0 / r1 unused); y_out
// receives (or, accumulate, adds) the rank-ordered sum; needs world * m * n
// <= max_elems.
cudaError_t launch_tp_allreduce(const TpArgs& a, int blocks, cudaStream_t s);

// ---- decoder step kernels: kq_decoder.cu ----
cudaError_t dec_rmsnorm(const float* x, int64_t x_ld, const float* w, float* out, int64_t out_ld, int64_t rows,
                        int64_t dim, float eps, cudaStream_t s);
cudaError_t dec_rope_append(float* qkv, int64_t ld, void* kc, void* vc, int64_t batch, int hq, int hkv, int hd,
                            int64_t pos, int64_t max_seq, float theta, cudaStream_t s);
// Per-device set-up of the decoder kernels (shared-memory sizes).
cudaError_t dec_init_device();
int dec_attention_splits(int64_t batch, int hkv, int64_t len, int num_sms);
size_t dec_attention_scratch_bytes(int64_t batch, int hq, int hkv, int hd, int splits);
// Attention of token b's query heads (q + b * q_ld) over cache positions
// [0, len), one kernel.  rope: q is the fused qkv row; the query heads are
// rotated in registers and the rotated k and v of position len - 1 are
// appended to the caches first.  scratch: dec_attention_scratch_bytes,
// zero-filled before its first use.  *err receives 24 if a tile copy wait
// gave up (the output is then invalid and the scratch must be re-zeroed).
cudaError_t dec_attention(const float* q, int64_t q_ld, void* kc, void* vc, float* out, int64_t out_ld,
                          int64_t batch, int hq, int hkv, int hd, int64_t len, int64_t max_seq, void* scratch,
                          int splits, bool rope, float theta, int* err, cudaStream_t s);
cudaError_t dec_swiglu(const float* gu, float* out, int64_t batch, int64_t ffn, int mode, cudaStream_t s);
cudaError_t dec_add(float* h, int64_t h_ld, const float* y, int64_t y_ld, int64_t rows, int64_t cols,
                    cudaStream_t s);
cudaError_t dec_embed(const float* table, const int* tokens, float* out, int64_t out_ld, int64_t batch, int64_t dim,
                      cudaStream_t s);

// ---- tensor-core (tcgen05) path: kq_mma.cu ----
// Build the TMA descriptors of a GGUF weight (after its device arrays exist).
bool tc_make_weight_maps(DevWeight& w);
// Per-device set-up of the tcgen05 kernels (shared-memory carve-outs).
cudaError_t tc_init_device();
// Scratch for launch_tc_f32 / launch_tc_bf16.
size_t tc_workspace_bytes(int64_t m, int64_t n, int64_t k, int num_sms);
size_t tc_workspace_bytes_bf16(int64_t m, int64_t k);
// Bytes of split-K arrival counters launch_tc_f32 needs (reported as a span;
// `offset` is kept for callers that place them after the scratch).  They must
// be zero before the first call; the kernel leaves them zero.
void tc_counter_span(int64_t m, int64_t n, int64_t k, int num_sms, size_t* offset, size_t* count);
// y = x . W^T (+bias) with f32 x (split into f16 hi/lo) on tcgen05 tensor cores.
// *err (device int) receives a nonzero code if a pipeline wait gave up.
cudaError_t launch_tc_f32(const DevWeight& w, const float* x, int64_t m, const float* bias, float* y,
                          void* ws, int num_sms, int* err, cudaStream_t s, int* launches, Bracket br,
                          unsigned* counters);
// Same with bf16 x (prefill); A is dequantized to bf16.  Tiles of 256 tokens,
// or 128 where 256-token tiles would leave SMs idle (num_sms).
cudaError_t launch_tc_bf16(const DevWeight& w, const void* x, int64_t m, const float* bias, float* y,
                           void* ws, int num_sms, int* err, cudaStream_t s, int* launches,
                           Bracket br = Bracket());

}  // namespace kq
