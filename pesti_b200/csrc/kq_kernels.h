// kq_kernels.h -- internal launch interface between the C-ABI layer
// (kq_api.cu) and the kernels.  Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kq {

constexpr int QK = 256;         // weights per K-quant superblock
constexpr int Q4K_BYTES = 144;  // GGUF Q4_K superblock
constexpr int Q6K_BYTES = 210;  // GGUF Q6_K superblock
constexpr int Q6K_BODY = 208;   // device Q6_K body: ql(128) | qh(64) | scales(16)

enum QType : int {
  GGUF_Q4_K = 12,
  GGUF_Q6_K = 14,
  LEGACY_Q4_K = 112,
  LEGACY_Q6_K = 114,
};

// Device-resident weight.  For GGUF types the row count is n, the row length k
// (a multiple of 256) and sb = k/256 superblocks per row.
//  GGUF_Q4_K: q = raw GGUF superblocks [n][sb][144]; d unused.
//  GGUF_Q6_K: q = bodies [n][sb][208] (ql|qh|scales), d = f16 [n][sb].
//  LEGACY_*:  q = raw bytes as uploaded (row stride = legacy row bytes), len.
struct DevWeight {
  int type;
  int64_t n, k, sb;
  const uint8_t* q;
  const uint16_t* d;
  int64_t len;        // uploaded byte count (legacy) / device bytes
  int64_t row_bytes;  // legacy row stride
};

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

// Re-lay GGUF Q6_K superblocks [nsb][210] into bodies [nsb][208] + d [nsb].
cudaError_t launch_q6k_relayout(const uint8_t* raw, int64_t nsb, uint8_t* body, uint16_t* d,
                                cudaStream_t s);

}  // namespace kq
