// kq_api.cu -- the C ABI (include/pesti_kq.h): contexts, device-resident
// weights, argument validation, host<->device staging and kernel dispatch.
// Every failure is reported as a status code plus a message on the context;
// nothing here aborts, traps, or computes on the CPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/pesti_decoder.h"
#include "../../include/pesti_kq.h"
#include "kq_kernels.h"

struct kq_ctx {
  int device = 0;
  int num_sms = 148;
  int path = KQ_PATH_AUTO;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  void* ws = nullptr;  // kernel scratch (prepared activations, partial sums)
  size_t ws_bytes = 0;
  void* ctr = nullptr;  // split-K arrival counters: zero between calls
  size_t ctr_bytes = 0;
  int* dev_err = nullptr;   // set by a tensor-core kernel whose pipeline wait gave up
  int* host_err = nullptr;  // pinned mirror of dev_err, read after synchronising
  void* xbuf = nullptr;     // device staging of host inputs
  size_t xbuf_bytes = 0;
  void* ybuf = nullptr;  // device staging of host outputs
  size_t ybuf_bytes = 0;
  void* bbuf = nullptr;  // device staging of a host bias
  size_t bbuf_bytes = 0;
  int64_t launches = 0;
  std::string err;
  // one-shot L2 prefetch hint for the next linear call (kq_ctx_prefetch_next)
  kq::Prefetch pf;
  bool pf_set = false;
  const kq::Prefetch* take_prefetch() {
    if (!pf_set) return nullptr;
    pf_set = false;
    return &pf;
  }
  // timing brackets of the main kernel (kq_ctx_profile_begin/end)
  std::vector<cudaEvent_t> prof_ev;  // 2 per slot
  int prof_cap = 0, prof_next = 0;
  bool prof_on = false;

  kq::Bracket next_bracket() {
    kq::Bracket b;
    if (prof_on && prof_next < prof_cap) {
      b.start = prof_ev[2 * prof_next];
      b.stop = prof_ev[2 * prof_next + 1];
      ++prof_next;
    }
    return b;
  }
};

// A tensor-parallel group member: this rank's exchange buffer (two slots of
// max_elems 8-byte words {f32 bits, epoch}), its block buffer, and the
// peers' exchange buffers mapped over CUDA IPC.
struct kq_tp {
  kq_ctx* ctx = nullptr;
  int world = 0, rank = 0;
  int64_t max_elems = 0;
  void* exch = nullptr;
  float* ylocal = nullptr;
  unsigned* ctr = nullptr;
  void* peer_base[kq::TP_MAX_WORLD] = {};
  bool opened = false;
};

struct kq_weight {
  int device = 0;
  kq::DevWeight dw{};
  void* q_alloc = nullptr;
  void* d_alloc = nullptr;
  int64_t device_bytes = 0;
};

// A decode-step program (kq_step_*): its stages on the host, and once built,
// their device copy and the scratch the persistent kernel needs.
struct kq_step {
  kq_ctx* ctx = nullptr;
  kq_tp* tp = nullptr;  // NULL: one GPU, with a local exchange buffer
  std::vector<kq::StepStage> stages;
  int nexch = 0;             // PARTIAL stages so far
  int64_t pending_len = -1;  // length of the exchange a RESIDUAL stage may consume (-1: none)
  bool built = false;
  kq::StepArgs args{};
  void* d_stages = nullptr;
  void* sync = nullptr;      // sync words, zero between launches
  void* attn_part = nullptr;
  void* exch = nullptr;      // one GPU: two slots of exchange words
  void* epoch = nullptr;     // one GPU: the exchange epoch
  unsigned long long* trace = nullptr;  // kq_step_trace buffer (caller's), or NULL
};

namespace {

const char* kNoCtx = "no context";

int fail(kq_ctx* ctx, int status, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return status;
}

int cuda_fail(kq_ctx* ctx, cudaError_t e, const char* what) {
  cudaGetLastError();  // clear a non-sticky error so the context stays usable
  return fail(ctx, KQ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// Makes `dev` current for the scope and restores the caller's device.
struct DeviceGuard {
  int prev = -1;
  cudaError_t status = cudaSuccess;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) status = cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// Grow-only device buffer; `zero` clears a newly allocated buffer.
int ensure(kq_ctx* ctx, void** buf, size_t* have, size_t need, const char* what, bool zero = false) {
  if (need <= *have) return KQ_OK;
  if (*buf) {
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "synchronize before growing scratch");
    cudaFree(*buf);
    *buf = nullptr;
    *have = 0;
  }
  size_t sz = (need + 255) & ~size_t(255);
  cudaError_t e = cudaMalloc(buf, sz);
  if (e != cudaSuccess) {
    *buf = nullptr;
    cudaGetLastError();
    return fail(ctx, KQ_ERR_NOMEM, "cudaMalloc(%zu) for %s failed: %s", sz, what,
                cudaGetErrorString(e));
  }
  if (zero) {
    e = cudaMemset(*buf, 0, sz);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "clear scratch");
  }
  *have = sz;
  return KQ_OK;
}

// GGUF Q4_K / Q6_K: the types every kernel family serves
bool is_gguf(int t) { return t == kq::GGUF_Q4_K || t == kq::GGUF_Q6_K; }
// GGUF Q2_K / Q3_K / Q5_K: the CUDA-core kernels of kq_kx.cu
bool is_kx(int t) { return kq::kx_type(t); }
bool is_legacy(int t) { return t == kq::LEGACY_Q4_K || t == kq::LEGACY_Q5_K || t == kq::LEGACY_Q6_K; }

int64_t legacy_row_bytes(int t, int64_t k) {
  if (t == kq::LEGACY_Q4_K) return ((k + 15) / 16) * 28;
  if (t == kq::LEGACY_Q5_K) return ((k + 15) / 16) * 36;  // quantized_linear.rs:91
  return ((k + 15) / 16) * 42;
}

// Bytes the legacy tile decoder reads from the last row (tile_dequant.rs:224-227, 334-335).
int64_t legacy_tile_bytes(int t, int64_t k) {
  if (t == kq::LEGACY_Q4_K || t == kq::LEGACY_Q5_K) return (k / 16) * 28 + ((k % 16) ? 4 : 0);
  return ((k + 15) / 16) * 42;
}

int check_ctx(kq_ctx* ctx) { return ctx ? KQ_OK : KQ_ERR_INVALID_ARG; }

// After the stream is synchronised: report (and clear) a device-side wait
// that gave up.  The split-K counters may then be stale, so they are cleared too.
int check_device_error(kq_ctx* ctx) {
  const int code = *reinterpret_cast<volatile int*>(ctx->host_err);
  if (code == 0) return KQ_OK;
  *ctx->host_err = 0;
  cudaMemset(ctx->dev_err, 0, sizeof(int));
  if (ctx->ctr) cudaMemset(ctx->ctr, 0, ctx->ctr_bytes);
  cudaDeviceSynchronize();
  cudaGetLastError();
  return fail(ctx, KQ_ERR_CUDA,
              "a device-side wait gave up (code %d: 1-5 tcgen05 pipeline, 21-23 decode weight ring, "
              "27-28 batched integer-MMA ring, 31-32 tensor-parallel peer flag, 41-45 decode-step ring, "
              "barrier or exchange); the call's output is invalid",
              code);
}

// Stream-ordered copy of the device error word into the pinned mirror.
cudaError_t stage_error_word(kq_ctx* ctx) {
  return cudaMemcpyAsync(ctx->host_err, ctx->dev_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
}

int finish_sync(kq_ctx* ctx, const char* what) {
  cudaError_t e = stage_error_word(ctx);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  return check_device_error(ctx);
}

// The CUDA-core f32 kernel of Q2_K / Q3_K / Q5_K (kq_kx.cu): internal
// family code, never a KQ_PATH_* value.
constexpr int FAM_KX = -1;

// Kernel family for a GGUF f32 call of m tokens.  AUTO follows the measured
// decode throughput of each family: integer dot products for one token (and
// two Q6_K tokens), integer tensor-core tiles for Q4_K up to 64 tokens and
// Q6_K up to 8, mma.sync bf16 tiles for Q6_K up to 64, tcgen05 above.
// Q2_K / Q3_K / Q5_K: the single-token kernel at one token (AUTO, DP4A),
// on integer tensor-core tiles up to 64 tokens (AUTO, IMMA), otherwise
// the CUDA-core f32 kernel.
int f32_family(const kq_ctx* ctx, const kq::DevWeight& w, int64_t m) {
  if (is_kx(w.type)) {
    const bool auto_ = ctx->path == KQ_PATH_AUTO;
    if (m == 1 && (auto_ || ctx->path == KQ_PATH_DP4A)) return KQ_PATH_DP4A;
    if (m <= 64 && (auto_ || ctx->path == KQ_PATH_IMMA)) return KQ_PATH_IMMA;
    return FAM_KX;
  }
  const bool q4 = w.type == kq::GGUF_Q4_K;
  if (ctx->path == KQ_PATH_IMMA || ctx->path == KQ_PATH_MMA || ctx->path == KQ_PATH_TCGEN05) return ctx->path;
  if (m == 1 || (ctx->path == KQ_PATH_DP4A && m <= kq::DP4A_MAX_M)) return KQ_PATH_DP4A;
  if (q4) return m <= 64 ? KQ_PATH_IMMA : KQ_PATH_TCGEN05;
  if (m == 2) return KQ_PATH_DP4A;
  if (m <= 8) return KQ_PATH_IMMA;
  return m <= 64 ? KQ_PATH_MMA : KQ_PATH_TCGEN05;
}

// Scratch bytes and zeroed counter bytes a GGUF f32 call of m tokens needs
// (the single-token kernel and the Q2_K / Q3_K / Q5_K f32 kernel need none).
void f32_needs(const kq_ctx* ctx, const kq::DevWeight& w, int64_t m, size_t* ws, size_t* ctr) {
  *ws = 0;
  *ctr = 0;
  const int fam = f32_family(ctx, w, m);
  if (fam == KQ_PATH_DP4A) {
    *ws = kq::dp4a_workspace_bytes(w.type, m, w.sb);
  } else if (fam == KQ_PATH_IMMA) {
    *ws = kq::imma_workspace_bytes(m, w.n, w.k, ctx->num_sms);
    *ctr = kq::imma_counter_bytes(w.n);
  } else if (fam == KQ_PATH_TCGEN05) {
    *ws = kq::tc_workspace_bytes(m, w.n, w.k, ctx->num_sms);
    size_t off = 0;
    kq::tc_counter_span(m, w.n, w.k, ctx->num_sms, &off, ctr);
  } else if (fam != FAM_KX) {
    *ws = kq::gemv_gguf_workspace_bytes(m, w.k);
  }
}

int prepare_f32(kq_ctx* ctx, const kq::DevWeight& w, int64_t m) {
  size_t ws = 0, ctr = 0;
  f32_needs(ctx, w, m, &ws, &ctr);
  int rc = ensure(ctx, &ctx->ws, &ctx->ws_bytes, ws, "workspace");
  if (rc == KQ_OK && ctr) rc = ensure(ctx, &ctx->ctr, &ctx->ctr_bytes, ctr, "counters", true);
  return rc;
}

}  // namespace

namespace kq {
// kq_last_error text for entry points defined in other files (the GGUF reader)
int api_fail(kq_ctx* ctx, int status, const char* msg) { return fail(ctx, status, "%s", msg); }
}  // namespace kq

extern "C" {

int kq_abi_version(void) { return KQ_ABI_VERSION; }

const char* kq_status_string(int status) {
  switch (status) {
    case KQ_OK: return "ok";
    case KQ_ERR_INVALID_ARG: return "invalid argument";
    case KQ_ERR_UNSUPPORTED: return "unsupported";
    case KQ_ERR_CUDA: return "CUDA error";
    case KQ_ERR_SHORT_BUFFER: return "buffer too short";
    case KQ_ERR_NCCL: return "collective error";
    case KQ_ERR_STATE: return "invalid state";
    case KQ_ERR_NOMEM: return "out of device memory";
    case KQ_ERR_FORMAT: return "malformed or unreadable file";
    default: return "unknown status";
  }
}

const char* kq_last_error(const kq_ctx* ctx) { return ctx ? ctx->err.c_str() : kNoCtx; }

int kq_ctx_create(int device, kq_ctx** out) {
  if (!out) return KQ_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return KQ_ERR_CUDA;
  }
  if (device < 0 || device >= n) return KQ_ERR_INVALID_ARG;
  DeviceGuard g(device);
  if (g.status != cudaSuccess) return KQ_ERR_CUDA;
  e = kq::gemv_init_device();
  if (e == cudaSuccess) e = kq::tc_init_device();
  if (e == cudaSuccess) e = kq::dp4a_init_device();
  if (e == cudaSuccess) e = kq::imma_init_device();
  if (e == cudaSuccess) e = kq::dec_init_device();
  if (e == cudaSuccess) e = kq::kx_init_device();
  if (e == cudaSuccess) e = kq::step_init_device();
  if (e != cudaSuccess) {
    cudaGetLastError();
    return KQ_ERR_CUDA;
  }
  kq_ctx* ctx = new kq_ctx();
  ctx->device = device;
  cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
  e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->dev_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->dev_err, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaHostAlloc(&ctx->host_err, sizeof(int), cudaHostAllocDefault);
  if (e != cudaSuccess) {
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    delete ctx;
    cudaGetLastError();
    return KQ_ERR_CUDA;
  }
  *ctx->host_err = 0;
  ctx->stream = ctx->own_stream;
  *out = ctx;
  return KQ_OK;
}

int kq_ctx_destroy(kq_ctx* ctx) {
  if (!ctx) return KQ_ERR_INVALID_ARG;
  {
    DeviceGuard g(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->ctr) cudaFree(ctx->ctr);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->host_err) cudaFreeHost(ctx->host_err);
    if (ctx->xbuf) cudaFree(ctx->xbuf);
    if (ctx->ybuf) cudaFree(ctx->ybuf);
    if (ctx->bbuf) cudaFree(ctx->bbuf);
    for (cudaEvent_t ev : ctx->prof_ev) cudaEventDestroy(ev);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    cudaGetLastError();
  }
  delete ctx;
  return KQ_OK;
}

int kq_ctx_set_stream(kq_ctx* ctx, void* stream) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
  return KQ_OK;
}

int kq_ctx_set_path(kq_ctx* ctx, int path) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (path != KQ_PATH_AUTO && path != KQ_PATH_TCGEN05 && path != KQ_PATH_MMA && path != KQ_PATH_DP4A &&
      path != KQ_PATH_IMMA)
    return fail(ctx, KQ_ERR_INVALID_ARG, "unknown path %d", path);
  ctx->path = path;
  return KQ_OK;
}

int kq_ctx_prefetch_next(kq_ctx* ctx, const kq_weight* next) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  ctx->pf = kq::Prefetch();
  ctx->pf_set = false;
  if (!next) return KQ_OK;
  if (next->device != ctx->device)
    return fail(ctx, KQ_ERR_INVALID_ARG, "weight lives on device %d, context on %d", next->device, ctx->device);
  const kq::DevWeight& w = next->dw;
  if (w.type == kq::GGUF_Q4_K) {
    ctx->pf.p[0] = w.q;
    ctx->pf.bytes[0] = w.n * w.sb * kq::Q4K_BYTES;
  } else if (w.type == kq::GGUF_Q6_K) {
    ctx->pf.p[0] = w.q;
    ctx->pf.bytes[0] = w.n * w.sb * kq::Q6K_BODY;
    ctx->pf.p[1] = w.d;
    ctx->pf.bytes[1] = w.n * w.d_ld * 2;
  } else {
    return KQ_OK;  // legacy blocks: no hint
  }
  for (int r = 0; r < 2; ++r)  // bulk prefetches start on 16-byte boundaries
    if (reinterpret_cast<uintptr_t>(ctx->pf.p[r]) & 15) ctx->pf.p[r] = nullptr;
  ctx->pf_set = true;
  return KQ_OK;
}

int kq_ctx_synchronize(kq_ctx* ctx) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  return finish_sync(ctx, "cudaStreamSynchronize");
}

int kq_ctx_reserve(kq_ctx* ctx, const kq_weight* w, int64_t m) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!w || m < 0) return fail(ctx, KQ_ERR_INVALID_ARG, "bad reserve arguments");
  if ((!is_gguf(w->dw.type) && !is_kx(w->dw.type)) || m == 0 || w->dw.k == 0)
    return KQ_OK;  // the other types need no scratch
  DeviceGuard g(ctx->device);
  // every call with 1..m rows may pick a different kernel family: cover them all
  size_t ws = is_gguf(w->dw.type) ? kq::tc_workspace_bytes_bf16(m, w->dw.k) : 0, ctr = 0;
  for (int64_t i = 1; i <= m; ++i) {
    size_t a = 0, b = 0;
    f32_needs(ctx, w->dw, i, &a, &b);
    ws = a > ws ? a : ws;
    ctr = b > ctr ? b : ctr;
  }
  int rc = ensure(ctx, &ctx->ws, &ctx->ws_bytes, ws, "workspace");
  if (rc == KQ_OK && ctr) rc = ensure(ctx, &ctx->ctr, &ctx->ctr_bytes, ctr, "counters", true);
  return rc;
}

int64_t kq_ctx_launch_count(const kq_ctx* ctx) { return ctx ? ctx->launches : -1; }

int kq_ctx_profile_begin(kq_ctx* ctx, int max_calls) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (max_calls < 0 || max_calls > (1 << 20)) return fail(ctx, KQ_ERR_INVALID_ARG, "max_calls %d", max_calls);
  DeviceGuard g(ctx->device);
  while ((int)ctx->prof_ev.size() < 2 * max_calls) {
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreate(&ev);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaEventCreate");
    ctx->prof_ev.push_back(ev);
  }
  ctx->prof_cap = max_calls;
  ctx->prof_next = 0;
  ctx->prof_on = true;
  return KQ_OK;
}

static int profile_sums(kq_ctx* ctx, double* total_ms, int64_t* count);

int kq_ctx_profile_end(kq_ctx* ctx, double* total_ms, int64_t* count) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!ctx->prof_on) return fail(ctx, KQ_ERR_STATE, "profiling was not started");
  ctx->prof_on = false;
  return profile_sums(ctx, total_ms, count);
}

int kq_ctx_profile_read(kq_ctx* ctx, double* total_ms, int64_t* count) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!ctx->prof_on) return fail(ctx, KQ_ERR_STATE, "profiling was not started");
  return profile_sums(ctx, total_ms, count);
}

static int profile_sums(kq_ctx* ctx, double* total_ms, int64_t* count) {
  DeviceGuard g(ctx->device);
  int rc = finish_sync(ctx, "cudaStreamSynchronize");
  if (rc) return rc;
  double sum = 0.0;
  for (int i = 0; i < ctx->prof_next; ++i) {
    float ms = 0.f;
    cudaError_t e = cudaEventElapsedTime(&ms, ctx->prof_ev[2 * i], ctx->prof_ev[2 * i + 1]);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaEventElapsedTime");
    sum += ms;
  }
  if (total_ms) *total_ms = sum;
  if (count) *count = ctx->prof_next;
  return KQ_OK;
}

int kq_row_bytes(int type, int64_t in_features, int64_t* out) {
  if (!out || in_features < 0) return KQ_ERR_INVALID_ARG;
  if (is_gguf(type)) {
    if (in_features % kq::QK) return KQ_ERR_UNSUPPORTED;
    *out = (in_features / kq::QK) * (type == kq::GGUF_Q4_K ? kq::Q4K_BYTES : kq::Q6K_BYTES);
    return KQ_OK;
  }
  if (is_kx(type)) {
    if (in_features % kq::QK) return KQ_ERR_UNSUPPORTED;
    *out = (in_features / kq::QK) * kq::kx_block_bytes(type);
    return KQ_OK;
  }
  if (is_legacy(type)) {
    *out = legacy_row_bytes(type, in_features);
    return KQ_OK;
  }
  return KQ_ERR_UNSUPPORTED;
}

int kq_weight_upload(kq_ctx* ctx, int type, const void* bytes, size_t nbytes, int64_t n, int64_t k,
                     kq_weight** out) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!out) return fail(ctx, KQ_ERR_INVALID_ARG, "out is null");
  *out = nullptr;
  if (n < 0 || k < 0) return fail(ctx, KQ_ERR_INVALID_ARG, "negative shape %lld x %lld", (long long)n, (long long)k);
  if (!is_gguf(type) && !is_kx(type) && !is_legacy(type))
    return fail(ctx, KQ_ERR_UNSUPPORTED, "unsupported kq_type %d", type);
  if ((is_gguf(type) || is_kx(type)) && k % kq::QK)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "GGUF K-quant rows hold whole 256-weight superblocks; in_features=%lld",
                (long long)k);
  if (n > (int64_t)1 << 31 || k > (int64_t)1 << 28)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "shape %lld x %lld too large", (long long)n, (long long)k);
  int64_t need;
  if (is_gguf(type)) {
    need = n * (k / kq::QK) * (type == kq::GGUF_Q4_K ? kq::Q4K_BYTES : kq::Q6K_BYTES);
  } else if (is_kx(type)) {
    need = n * (k / kq::QK) * kq::kx_block_bytes(type);
  } else {
    need = (n == 0 || k == 0) ? 0 : (n - 1) * legacy_row_bytes(type, k) + legacy_tile_bytes(type, k);
  }
  if ((int64_t)nbytes < need)
    return fail(ctx, KQ_ERR_SHORT_BUFFER, "weight has %zu bytes, shape %lld x %lld needs %lld", nbytes, (long long)n,
                (long long)k, (long long)need);
  if (need > 0 && !bytes) return fail(ctx, KQ_ERR_INVALID_ARG, "bytes is null");

  DeviceGuard g(ctx->device);
  if (g.status != cudaSuccess) return cuda_fail(ctx, g.status, "cudaSetDevice");
  kq_weight* w = new kq_weight();
  w->device = ctx->device;
  w->dw.type = type;
  w->dw.n = n;
  w->dw.k = k;
  w->dw.sb = (is_gguf(type) || is_kx(type)) ? k / kq::QK : 0;
  w->dw.row_bytes = is_legacy(type) ? legacy_row_bytes(type, k) : 0;
  cudaError_t e = cudaSuccess;
  const size_t pad = 64;  // vector loads never read past the allocation
  if (type == kq::GGUF_Q6_K) {
    const int64_t nsb = n * w->dw.sb;
    const int64_t dld = kq::q6k_d_ld(w->dw.sb);
    w->dw.d_ld = dld;
    void* raw = nullptr;
    e = cudaMalloc(&raw, (size_t)nsb * kq::Q6K_BYTES + pad);
    if (e == cudaSuccess) e = cudaMalloc(&w->q_alloc, (size_t)nsb * kq::Q6K_BODY + pad);
    if (e == cudaSuccess) e = cudaMalloc(&w->d_alloc, (size_t)n * dld * 2 + pad);
    if (e == cudaSuccess) e = cudaMemsetAsync(w->d_alloc, 0, (size_t)n * dld * 2 + pad, ctx->stream);
    if (e == cudaSuccess && nsb)
      e = cudaMemcpyAsync(raw, bytes, (size_t)nsb * kq::Q6K_BYTES, cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess)
      e = kq::launch_q6k_relayout(static_cast<const uint8_t*>(raw), n, w->dw.sb, static_cast<uint8_t*>(w->q_alloc),
                                  static_cast<uint16_t*>(w->d_alloc), ctx->stream);
    if (e == cudaSuccess) {
      ++ctx->launches;
      e = cudaStreamSynchronize(ctx->stream);
    }
    if (raw) cudaFree(raw);
    w->device_bytes = nsb * (kq::Q6K_BODY + 2);
    w->dw.len = w->device_bytes;
  } else if (is_kx(type)) {
    // rows at a 16-byte stride (the row's bytes rounded up), one 2-D copy;
    // Q3_K: superblocks at their device stride (each padded to 112 bytes)
    const int64_t bs = kq::kx_block_bytes(type), ds = kq::kx_dev_stride(type);
    const int64_t src_rb = w->dw.sb * bs;
    const int64_t dst_rb = (w->dw.sb * ds + 15) & ~int64_t(15);
    w->dw.row_bytes = dst_rb;
    e = cudaMalloc(&w->q_alloc, (size_t)(n * dst_rb) + pad);
    if (e == cudaSuccess) e = cudaMemsetAsync(w->q_alloc, 0, (size_t)(n * dst_rb) + pad, ctx->stream);
    if (e == cudaSuccess && need) {
      if (ds == bs)
        e = cudaMemcpy2DAsync(w->q_alloc, (size_t)dst_rb, bytes, (size_t)src_rb, (size_t)src_rb, (size_t)n,
                              cudaMemcpyDefault, ctx->stream);
      else  // dst_rb == sb * ds: the superblocks of all rows are one run of n * sb
        e = cudaMemcpy2DAsync(w->q_alloc, (size_t)ds, bytes, (size_t)bs, (size_t)bs, (size_t)(n * w->dw.sb),
                              cudaMemcpyDefault, ctx->stream);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    w->device_bytes = n * dst_rb;
    w->dw.len = w->device_bytes;
  } else {
    e = cudaMalloc(&w->q_alloc, (size_t)need + pad);
    if (e == cudaSuccess) e = cudaMemsetAsync(w->q_alloc, 0, (size_t)need + pad, ctx->stream);
    if (e == cudaSuccess && need)
      e = cudaMemcpyAsync(w->q_alloc, bytes, (size_t)need, cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    w->device_bytes = need;
    w->dw.len = need;
  }
  if (e != cudaSuccess) {
    int rc = cuda_fail(ctx, e, "weight upload");
    if (w->q_alloc) cudaFree(w->q_alloc);
    if (w->d_alloc) cudaFree(w->d_alloc);
    delete w;
    return rc;
  }
  w->dw.q = static_cast<const uint8_t*>(w->q_alloc);
  w->dw.d = static_cast<const uint16_t*>(w->d_alloc);
  // TMA descriptors: Q4_K / Q6_K (every tensor-core path), the other K-quants (integer MMA)
  if ((is_gguf(type) || is_kx(type)) && n > 0 && k > 0 &&
      !kq::tc_make_weight_maps(w->dw)) {
    cudaFree(w->q_alloc);
    if (w->d_alloc) cudaFree(w->d_alloc);
    delete w;
    return fail(ctx, KQ_ERR_CUDA, "could not build the weight's TMA descriptors");
  }
  *out = w;
  return KQ_OK;
}

int kq_weight_free(kq_weight* w) {
  if (!w) return KQ_ERR_INVALID_ARG;
  DeviceGuard g(w->device);
  if (w->q_alloc) cudaFree(w->q_alloc);
  if (w->d_alloc) cudaFree(w->d_alloc);
  cudaGetLastError();
  delete w;
  return KQ_OK;
}

int kq_weight_info(const kq_weight* w, int* type, int64_t* n, int64_t* k, int64_t* bytes) {
  if (!w) return KQ_ERR_INVALID_ARG;
  if (type) *type = w->dw.type;
  if (n) *n = w->dw.n;
  if (k) *k = w->dw.k;
  if (bytes) *bytes = w->device_bytes;
  return KQ_OK;
}

// Shared body of kq_linear_f32 / kq_linear_bf16.
static int linear_impl(kq_ctx* ctx, const kq_weight* w, const void* x, size_t xelem, int64_t m, const float* bias,
                       float* y, int flags, bool bf16) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!w) return fail(ctx, KQ_ERR_INVALID_ARG, "weight is null");
  if (flags & ~(KQ_DEVICE_PTRS | KQ_SYNC | KQ_ASYNC)) return fail(ctx, KQ_ERR_INVALID_ARG, "bad flags 0x%x", flags);
  if ((flags & KQ_ASYNC) && (flags & (KQ_DEVICE_PTRS | KQ_SYNC)))
    return fail(ctx, KQ_ERR_INVALID_ARG, "KQ_ASYNC applies to host pointers without KQ_SYNC (flags 0x%x)", flags);
  if (w->device != ctx->device)
    return fail(ctx, KQ_ERR_INVALID_ARG, "weight lives on device %d, context on %d", w->device, ctx->device);
  if (m < 0) return fail(ctx, KQ_ERR_INVALID_ARG, "negative m");
  if (m > (int64_t)1 << 24) return fail(ctx, KQ_ERR_UNSUPPORTED, "m = %lld is too large", (long long)m);
  if (bf16 && !is_gguf(w->dw.type))
    return fail(ctx, KQ_ERR_UNSUPPORTED, "bf16 activations need a GGUF Q4_K / Q6_K weight (type %d)", w->dw.type);
  const int64_t n = w->dw.n, k = w->dw.k;
  if (m == 0 || n == 0) return KQ_OK;
  if (!y || (k > 0 && !x)) return fail(ctx, KQ_ERR_INVALID_ARG, "x or y is null");
  const bool dev = flags & KQ_DEVICE_PTRS;
  // the kernels read activations in 16-byte vectors and write y in 4-byte words
  if (dev && k > 0 && (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(ctx, KQ_ERR_INVALID_ARG, "device x must be 16-byte aligned");
  if (dev && ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(bias)) & 3))
    return fail(ctx, KQ_ERR_INVALID_ARG, "device y and bias must be 4-byte aligned");
  DeviceGuard g(ctx->device);
  if (g.status != cudaSuccess) return cuda_fail(ctx, g.status, "cudaSetDevice");
  cudaStream_t s = ctx->stream;
  cudaError_t e = cudaSuccess;
  int rc;
  const kq::Prefetch* pf = ctx->take_prefetch();

  const void* xd = x;
  const float* bd = bias;
  float* yd = y;
  if (!dev) {
    if ((rc = ensure(ctx, &ctx->xbuf, &ctx->xbuf_bytes, (size_t)(m * k) * xelem, "input staging"))) return rc;
    if ((rc = ensure(ctx, &ctx->ybuf, &ctx->ybuf_bytes, (size_t)(m * n * 4), "output staging"))) return rc;
    if (k > 0) {
      e = cudaMemcpyAsync(ctx->xbuf, x, (size_t)(m * k) * xelem, cudaMemcpyHostToDevice, s);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "copy x to device");
    }
    if (bias) {
      if ((rc = ensure(ctx, &ctx->bbuf, &ctx->bbuf_bytes, (size_t)(n * 4), "bias staging"))) return rc;
      e = cudaMemcpyAsync(ctx->bbuf, bias, (size_t)(n * 4), cudaMemcpyHostToDevice, s);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "copy bias to device");
      bd = static_cast<const float*>(ctx->bbuf);
    }
    xd = ctx->xbuf;
    yd = static_cast<float*>(ctx->ybuf);
  }

  int launches = 0;
  if (k == 0) {
    // no inputs: the product is empty, y = bias (quantized_linear.rs:147-150)
    if (bd) {
      for (int64_t i = 0; i < m && e == cudaSuccess; ++i)
        e = cudaMemcpyAsync(yd + i * n, bd, (size_t)n * 4, cudaMemcpyDeviceToDevice, s);
    } else {
      e = cudaMemsetAsync(yd, 0, (size_t)(m * n * 4), s);
    }
  } else if (bf16) {
    if ((rc = ensure(ctx, &ctx->ws, &ctx->ws_bytes, kq::tc_workspace_bytes_bf16(m, k), "workspace"))) return rc;
    e = kq::launch_tc_bf16(w->dw, xd, m, bd, yd, ctx->ws, ctx->num_sms, ctx->dev_err, s, &launches, ctx->next_bracket());
  } else if (is_kx(w->dw.type) && f32_family(ctx, w->dw, m) != KQ_PATH_IMMA) {
    // one token: the single-token dp4a kernel (AUTO / DP4A; widths it cannot
    // stage fall through); otherwise the CUDA-core f32 kernel
    const kq::Bracket br = ctx->next_bracket();
    e = cudaErrorNotSupported;
    if (f32_family(ctx, w->dw, m) == KQ_PATH_DP4A) {
      kq::XsInput in;
      in.x = static_cast<const float*>(xd);
      e = kq::launch_gemv_xs(w->dw, in, bd, yd, ctx->num_sms, ctx->dev_err, pf, s, &launches, br);
    }
    if (e == cudaErrorNotSupported)
      e = kq::launch_gemv_kx(w->dw, static_cast<const float*>(xd), m, bd, yd, s, &launches, br);
  } else if (is_gguf(w->dw.type) || is_kx(w->dw.type)) {
    if ((rc = prepare_f32(ctx, w->dw, m))) return rc;
    const int fam = f32_family(ctx, w->dw, m);
    if (fam == KQ_PATH_IMMA) {
      e = kq::launch_gemv_imma(w->dw, static_cast<const float*>(xd), m, bd, yd, ctx->ws,
                               static_cast<unsigned*>(ctx->ctr), ctx->num_sms, ctx->dev_err, s, &launches,
                               ctx->next_bracket());
    } else if (fam == KQ_PATH_DP4A) {
      e = kq::launch_gemv_dp4a(w->dw, static_cast<const float*>(xd), m, bd, yd, ctx->ws, ctx->num_sms,
                               ctx->dev_err, s, &launches, ctx->next_bracket(), pf);
    } else if (fam == KQ_PATH_TCGEN05) {
      // counters live in their own zeroed buffer; the scratch layout's counter span is unused
      e = kq::launch_tc_f32(w->dw, static_cast<const float*>(xd), m, bd, yd, ctx->ws, ctx->num_sms, ctx->dev_err,
                            s, &launches, ctx->next_bracket(), static_cast<unsigned*>(ctx->ctr));
    } else {
      e = kq::launch_gemv_gguf(w->dw, static_cast<const float*>(xd), m, bd, yd, ctx->ws, s, &launches,
                               ctx->next_bracket());
    }
  } else {
    // the reference's blocks over whole 256-weight spans (Q4_K / Q6_K tiles), up
    // to 4 tokens, under AUTO / DP4A: one pass of the single-token kernel per
    // token (each pass streams the weight again, and still beats the block
    // kernel's 4-token pass, measured); otherwise the block kernel
    const kq::Bracket br = ctx->next_bracket();
    e = cudaErrorNotSupported;
    if (m <= kq::DP4A_MAX_M && (ctx->path == KQ_PATH_AUTO || ctx->path == KQ_PATH_DP4A) && k % kq::QK == 0 &&
        (w->dw.type == kq::LEGACY_Q4_K || w->dw.type == kq::LEGACY_Q6_K)) {
      kq::DevWeight lw = w->dw;
      lw.sb = k / kq::QK;
      for (int64_t t = 0; t < m; ++t) {
        kq::XsInput in;
        in.x = static_cast<const float*>(xd) + t * k;
        e = kq::launch_gemv_xs(lw, in, bd, yd + t * n, ctx->num_sms, ctx->dev_err, t == 0 ? pf : nullptr, s,
                               &launches, t == 0 ? br : kq::Bracket());
        if (e != cudaSuccess) break;  // not supported: the first pass, before anything ran
      }
    }
    if (e == cudaErrorNotSupported)
      e = kq::launch_gemv_legacy(w->dw, static_cast<const float*>(xd), m, bd, yd, s, &launches, br);
  }
  ctx->launches += launches;
  if (e != cudaSuccess) return cuda_fail(ctx, e, "kernel launch");
  if (!dev) {
    e = cudaMemcpyAsync(y, ctx->ybuf, (size_t)(m * n * 4), cudaMemcpyDeviceToHost, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "copy y to host");
  }
  if ((!dev && !(flags & KQ_ASYNC)) || (flags & KQ_SYNC)) return finish_sync(ctx, "linear");
  return KQ_OK;
}

int kq_linear_f32(kq_ctx* ctx, const kq_weight* w, const float* x, int64_t m, const float* bias, float* y,
                  int flags) {
  return linear_impl(ctx, w, x, 4, m, bias, y, flags, false);
}

int kq_linear_bf16(kq_ctx* ctx, const kq_weight* w, const void* x_bf16, int64_t m, const float* bias, float* y,
                   int flags) {
  return linear_impl(ctx, w, x_bf16, 2, m, bias, y, flags, true);
}

int kq_linear_f32_static(kq_ctx* ctx, const kq_weight* w, const float* x, int64_t m, const float* bias, float* y,
                         int flags) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!w) return fail(ctx, KQ_ERR_INVALID_ARG, "weight is null");
  if (flags & ~(KQ_DEVICE_PTRS | KQ_SYNC)) return fail(ctx, KQ_ERR_INVALID_ARG, "bad flags 0x%x", flags);
  if (!(flags & KQ_DEVICE_PTRS))
    return fail(ctx, KQ_ERR_INVALID_ARG, "kq_linear_f32_static takes device pointers only (KQ_DEVICE_PTRS)");
  if (w->device != ctx->device)
    return fail(ctx, KQ_ERR_INVALID_ARG, "weight lives on device %d, context on %d", w->device, ctx->device);
  if (!is_gguf(w->dw.type)) return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_linear_f32_static needs a GGUF Q4_K / Q6_K weight");
  if (m < 1 || m > kq::DP4A_MAX_M)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_linear_f32_static serves 1..%d rows, got m = %lld", kq::DP4A_MAX_M,
                (long long)m);
  const size_t need = kq::dp4a_workspace_bytes(w->dw.type, m, w->dw.sb);
  if (need > kq::DP4A_STATIC_SCRATCH)
    return fail(ctx, KQ_ERR_UNSUPPORTED,
                "m = %lld x in_features = %lld needs %zu bytes of scratch; the fixed scratch holds %zu "
                "(enough for m <= 4 with in_features <= 16384)",
                (long long)m, (long long)w->dw.k, need, kq::DP4A_STATIC_SCRATCH);
  if (w->dw.n == 0) return KQ_OK;
  if (!y || !x) return fail(ctx, KQ_ERR_INVALID_ARG, "x or y is null");
  if ((reinterpret_cast<uintptr_t>(x) & 15) ||
      ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(bias)) & 3))
    return fail(ctx, KQ_ERR_INVALID_ARG, "x must be 16-byte aligned, y and bias 4-byte aligned");
  DeviceGuard g(ctx->device);
  if (g.status != cudaSuccess) return cuda_fail(ctx, g.status, "cudaSetDevice");
  void* scratch = nullptr;
  cudaError_t e = kq::dp4a_static_scratch(&scratch);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaGetSymbolAddress of the fixed scratch");
  int launches = 0;
  e = kq::launch_gemv_dp4a_batched(w->dw, x, m, bias, y, scratch, ctx->num_sms, ctx->stream, &launches);
  ctx->launches += launches;
  if (e != cudaSuccess) return cuda_fail(ctx, e, "kernel launch");
  if (flags & KQ_SYNC) return finish_sync(ctx, "linear");
  return KQ_OK;
}

// ---- tensor parallel --------------------------------------------------------------

// Exchange buffer: two slots of max_elems 8-byte words {f32 bits, epoch}.
static size_t tp_exchange_bytes(int64_t max_elems) { return (size_t)2 * (size_t)max_elems * 8; }

int kq_tp_create(kq_ctx* ctx, int world, int rank, int64_t max_out_elems, kq_tp** out) {
  if (check_ctx(ctx) || !out) return KQ_ERR_INVALID_ARG;
  *out = nullptr;
  if (world < 1 || world > kq::TP_MAX_WORLD || rank < 0 || rank >= world)
    return fail(ctx, KQ_ERR_INVALID_ARG, "world %d / rank %d (world must be 1..%d)", world, rank, kq::TP_MAX_WORLD);
  if (max_out_elems < 1 || max_out_elems > ((int64_t)1 << 31))
    return fail(ctx, KQ_ERR_INVALID_ARG, "max_out_elems %lld", (long long)max_out_elems);
  DeviceGuard g(ctx->device);
  if (g.status != cudaSuccess) return cuda_fail(ctx, g.status, "cudaSetDevice");
  kq_tp* tp = new kq_tp;
  tp->ctx = ctx;
  tp->world = world;
  tp->rank = rank;
  tp->max_elems = max_out_elems;
  const size_t xbytes = tp_exchange_bytes(max_out_elems);
  cudaError_t e = cudaMalloc(&tp->exch, xbytes);
  if (e == cudaSuccess) e = cudaMemset(tp->exch, 0, xbytes);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&tp->ylocal), (size_t)max_out_elems * 4);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&tp->ctr), 256);  // [0] CTA counter, [1] epoch
  if (e == cudaSuccess) e = cudaMemset(tp->ctr, 0, 256);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    kq_tp_destroy(tp);
    return cuda_fail(ctx, e, "allocate the tensor-parallel exchange buffer");
  }
  tp->peer_base[rank] = tp->exch;
  *out = tp;
  return KQ_OK;
}

int kq_tp_handle(const kq_tp* tp, void* out, size_t* size) {
  if (!tp || !size) return KQ_ERR_INVALID_ARG;
  const size_t need = sizeof(cudaIpcMemHandle_t);
  if (!out) {
    *size = need;
    return KQ_OK;
  }
  if (*size < need) return fail(tp->ctx, KQ_ERR_SHORT_BUFFER, "handle needs %zu bytes", need);
  DeviceGuard g(tp->ctx->device);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, tp->exch);
  if (e != cudaSuccess) return cuda_fail(tp->ctx, e, "cudaIpcGetMemHandle");
  std::memcpy(out, &h, need);
  *size = need;
  return KQ_OK;
}

int kq_tp_open(kq_tp* tp, const void* handles, size_t nbytes) {
  if (!tp || !handles) return KQ_ERR_INVALID_ARG;
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  if (nbytes < hb * (size_t)tp->world)
    return fail(tp->ctx, KQ_ERR_SHORT_BUFFER, "need %d handles of %zu bytes", tp->world, hb);
  if (tp->opened) return fail(tp->ctx, KQ_ERR_STATE, "peers are already open");
  DeviceGuard g(tp->ctx->device);
  for (int r = 0; r < tp->world; ++r) {
    if (r == tp->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + hb * r, hb);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(tp->ctx, e, "cudaIpcOpenMemHandle (is the peer on another GPU of this node?)");
    tp->peer_base[r] = p;
  }
  tp->opened = true;
  return KQ_OK;
}

int kq_tp_allgather_f32(kq_tp* tp, const float* y_local, int64_t m, int64_t row0, int64_t rows, int64_t n_total,
                        float* y, int64_t y_ld, int flags) {
  if (!tp) return KQ_ERR_INVALID_ARG;
  kq_ctx* ctx = tp->ctx;
  if (!tp->opened) return fail(ctx, KQ_ERR_STATE, "kq_tp_open has not been called");
  if (!(flags & KQ_DEVICE_PTRS)) return fail(ctx, KQ_ERR_INVALID_ARG, "tensor-parallel calls take device pointers");
  if (flags & ~(KQ_DEVICE_PTRS | KQ_SYNC | KQ_ACCUMULATE))
    return fail(ctx, KQ_ERR_INVALID_ARG, "bad flags 0x%x", flags);
  if (m < 1 || rows < 0 || row0 < 0 || row0 + rows > n_total || n_total < 1 || !y || (rows > 0 && !y_local) ||
      y_ld < n_total)
    return fail(ctx, KQ_ERR_INVALID_ARG, "bad all-gather shape");
  if (m * n_total > tp->max_elems)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "m x n = %lld exceeds the exchange buffer (%lld floats)",
                (long long)(m * n_total), (long long)tp->max_elems);
  DeviceGuard g(ctx->device);
  kq::TpArgs a{};
  a.y_local = y_local;
  a.y_out = y;
  a.y_ld = y_ld;
  a.accumulate = (flags & KQ_ACCUMULATE) ? 1 : 0;
  a.m = m;
  a.n = n_total;
  a.r0 = row0;
  a.r1 = row0 + rows;
  a.world = tp->world;
  a.rank = tp->rank;
  for (int p = 0; p < tp->world; ++p) a.exch[p] = static_cast<unsigned long long*>(tp->peer_base[p]);
  a.max_elems = tp->max_elems;
  a.ctr = tp->ctr;
  a.epoch = tp->ctr + 1;
  a.err = ctx->dev_err;
  // about 8 gathered elements per thread (one batch of reads), at most one CTA per SM
  const int64_t work = m * n_total;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ctx->num_sms, (work + 4095) / 4096));
  cudaError_t e = kq::launch_tp_allgather(a, blocks, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "all-gather launch");
  ctx->launches += 1;
  if (flags & KQ_SYNC) return finish_sync(ctx, "all-gather");
  return KQ_OK;
}

int kq_tp_allreduce_f32(kq_tp* tp, const float* partial, int64_t m, int64_t n, float* y, int64_t y_ld, int flags) {
  if (!tp) return KQ_ERR_INVALID_ARG;
  kq_ctx* ctx = tp->ctx;
  if (!tp->opened) return fail(ctx, KQ_ERR_STATE, "kq_tp_open has not been called");
  if (!(flags & KQ_DEVICE_PTRS)) return fail(ctx, KQ_ERR_INVALID_ARG, "tensor-parallel calls take device pointers");
  if (flags & ~(KQ_DEVICE_PTRS | KQ_SYNC | KQ_ACCUMULATE))
    return fail(ctx, KQ_ERR_INVALID_ARG, "bad flags 0x%x", flags);
  if (m < 1 || n < 1 || !partial || !y || y_ld < n) return fail(ctx, KQ_ERR_INVALID_ARG, "bad all-reduce shape");
  if ((int64_t)tp->world * m * n > tp->max_elems)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "world x m x n = %lld exceeds the exchange buffer (%lld words)",
                (long long)(tp->world * m * n), (long long)tp->max_elems);
  DeviceGuard g(ctx->device);
  kq::TpArgs a{};
  a.y_local = partial;
  a.y_out = y;
  a.y_ld = y_ld;
  a.accumulate = (flags & KQ_ACCUMULATE) ? 1 : 0;
  a.m = m;
  a.n = n;
  a.r0 = 0;
  a.r1 = n;
  a.world = tp->world;
  a.rank = tp->rank;
  for (int p = 0; p < tp->world; ++p) a.exch[p] = static_cast<unsigned long long*>(tp->peer_base[p]);
  a.max_elems = tp->max_elems;
  a.ctr = tp->ctr;
  a.epoch = tp->ctr + 1;
  a.err = ctx->dev_err;
  // about 4 summed elements per thread, at most one CTA per SM
  const int64_t work = m * n;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(ctx->num_sms, (work + 2047) / 2048));
  cudaError_t e = kq::launch_tp_allreduce(a, blocks, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "all-reduce launch");
  ctx->launches += 1;
  if (flags & KQ_SYNC) return finish_sync(ctx, "all-reduce");
  return KQ_OK;
}

int kq_tp_linear_f32(kq_tp* tp, const kq_weight* shard, int64_t row0, int64_t n_total, const float* x, int64_t m,
                     const float* bias, float* y, int flags) {
  if (!tp || !shard) return KQ_ERR_INVALID_ARG;
  kq_ctx* ctx = tp->ctx;
  if (!(flags & KQ_DEVICE_PTRS)) return fail(ctx, KQ_ERR_INVALID_ARG, "tensor-parallel calls take device pointers");
  if (flags & KQ_ACCUMULATE) return fail(ctx, KQ_ERR_INVALID_ARG, "KQ_ACCUMULATE applies to kq_tp_allgather_f32");
  if (row0 < 0 || row0 + shard->dw.n > n_total)
    return fail(ctx, KQ_ERR_INVALID_ARG, "shard rows [%lld, %lld) outside the %lld-row weight", (long long)row0,
                (long long)(row0 + shard->dw.n), (long long)n_total);
  if (m < 1 || m * n_total > tp->max_elems)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "m x n = %lld exceeds the exchange buffer (%lld floats)",
                (long long)(m * n_total), (long long)tp->max_elems);
  int rc = kq_linear_f32(ctx, shard, x, m, bias, tp->ylocal, KQ_DEVICE_PTRS);
  if (rc) return rc;
  return kq_tp_allgather_f32(tp, tp->ylocal, m, row0, shard->dw.n, n_total, y, n_total, flags);
}

int kq_tp_destroy(kq_tp* tp) {
  if (!tp) return KQ_ERR_INVALID_ARG;
  DeviceGuard g(tp->ctx->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < tp->world; ++r)
    if (r != tp->rank && tp->peer_base[r]) cudaIpcCloseMemHandle(tp->peer_base[r]);
  if (tp->exch) cudaFree(tp->exch);
  if (tp->ylocal) cudaFree(tp->ylocal);
  if (tp->ctr) cudaFree(tp->ctr);
  cudaGetLastError();
  delete tp;
  return KQ_OK;
}

// ---- decoder step kernels ----------------------------------------------------------

static int dec_status(kq_ctx* ctx, cudaError_t e, const char* what) {
  return e == cudaSuccess ? KQ_OK : cuda_fail(ctx, e, what);
}

int kq_dec_rmsnorm(kq_ctx* ctx, const float* x, int64_t x_ld, const float* w, float* out, int64_t out_ld,
                   int64_t rows, int64_t dim, float eps) {
  if (check_ctx(ctx) || !x || !w || !out || rows < 0 || dim < 0 || x_ld < dim || out_ld < dim)
    return KQ_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  ctx->launches += rows > 0 && dim > 0;
  return dec_status(ctx, kq::dec_rmsnorm(x, x_ld, w, out, out_ld, rows, dim, eps, ctx->stream), "rmsnorm");
}

int kq_dec_rope_append(kq_ctx* ctx, float* qkv, int64_t ld, void* k_cache, void* v_cache, int64_t batch, int heads,
                       int kv_heads, int head_dim, int64_t pos, int64_t max_seq, float theta) {
  if (check_ctx(ctx) || !qkv || !k_cache || !v_cache) return KQ_ERR_INVALID_ARG;
  if (batch < 1 || heads < 1 || kv_heads < 1 || head_dim < 2 || head_dim % 2 || pos < 0 || pos >= max_seq ||
      ld < (int64_t)(heads + 2 * kv_heads) * head_dim)
    return fail(ctx, KQ_ERR_INVALID_ARG, "rope: bad shape or position %lld of %lld", (long long)pos,
                (long long)max_seq);
  DeviceGuard g(ctx->device);
  ctx->launches += 1;
  return dec_status(
      ctx, kq::dec_rope_append(qkv, ld, k_cache, v_cache, batch, heads, kv_heads, head_dim, pos, max_seq, theta,
                               ctx->stream),
      "rope");
}

size_t kq_dec_attention_scratch(kq_ctx* ctx, int64_t batch, int heads, int kv_heads, int head_dim, int64_t len) {
  if (!ctx || batch < 1 || heads < 1 || kv_heads < 1 || len < 1 || head_dim < 1) return 0;
  const int sp = kq::dec_attention_splits(batch, kv_heads, len, ctx->num_sms);
  return kq::dec_attention_scratch_bytes(batch, heads, kv_heads, head_dim, sp);
}

static int attention_impl(kq_ctx* ctx, const float* q, int64_t q_ld, void* k_cache, void* v_cache, float* out,
                          int64_t out_ld, int64_t batch, int heads, int kv_heads, int head_dim, int64_t len,
                          int64_t max_seq, void* scratch, size_t scratch_bytes, bool rope, float theta) {
  if (check_ctx(ctx) || !q || !k_cache || !v_cache || !out || !scratch) return KQ_ERR_INVALID_ARG;
  if (len < 1 || len > max_seq || batch < 1)
    return fail(ctx, KQ_ERR_INVALID_ARG, "attention over %lld of %lld positions", (long long)len, (long long)max_seq);
  if (kv_heads < 1 || heads < 1)
    return fail(ctx, KQ_ERR_INVALID_ARG, "attention: %d heads / %d kv heads", heads, kv_heads);
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
    return fail(ctx, KQ_ERR_INVALID_ARG, "attention: the caches must be 16-byte aligned");
  const int sp = kq::dec_attention_splits(batch, kv_heads, len, ctx->num_sms);
  if (scratch_bytes < kq::dec_attention_scratch_bytes(batch, heads, kv_heads, head_dim, sp))
    return fail(ctx, KQ_ERR_SHORT_BUFFER, "attention scratch too small");
  DeviceGuard g(ctx->device);
  cudaError_t e = kq::dec_attention(q, q_ld, k_cache, v_cache, out, out_ld, batch, heads, kv_heads, head_dim, len,
                                    max_seq, scratch, sp, rope, theta, ctx->dev_err, ctx->stream);
  if (e == cudaErrorInvalidValue) {
    cudaGetLastError();
    return fail(ctx, KQ_ERR_UNSUPPORTED, "attention: head_dim %d / group %d unsupported", head_dim,
                heads / kv_heads);
  }
  ctx->launches += 1;
  return dec_status(ctx, e, "attention");
}

int kq_dec_attention(kq_ctx* ctx, const float* q, int64_t q_ld, const void* k_cache, const void* v_cache, float* out,
                     int64_t out_ld, int64_t batch, int heads, int kv_heads, int head_dim, int64_t len,
                     int64_t max_seq, void* scratch, size_t scratch_bytes) {
  // the caches are only read without rope
  return attention_impl(ctx, q, q_ld, const_cast<void*>(k_cache), const_cast<void*>(v_cache), out, out_ld, batch,
                        heads, kv_heads, head_dim, len, max_seq, scratch, scratch_bytes, false, 0.f);
}

int kq_dec_rope_attention(kq_ctx* ctx, const float* qkv, int64_t ld, void* k_cache, void* v_cache, float* out,
                          int64_t out_ld, int64_t batch, int heads, int kv_heads, int head_dim, int64_t pos,
                          int64_t max_seq, float theta, void* scratch, size_t scratch_bytes) {
  if (pos < 0) return fail(ctx, KQ_ERR_INVALID_ARG, "rope_attention: negative position");
  return attention_impl(ctx, qkv, ld, k_cache, v_cache, out, out_ld, batch, heads, kv_heads, head_dim, pos + 1,
                        max_seq, scratch, scratch_bytes, true, theta);
}

int kq_dec_swiglu(kq_ctx* ctx, const float* gate_up, float* out, int64_t batch, int64_t ffn, int mode) {
  if (check_ctx(ctx) || !gate_up || !out || batch < 0 || ffn < 0 || (mode != 0 && mode != 1))
    return KQ_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  ctx->launches += batch * ffn > 0;
  return dec_status(ctx, kq::dec_swiglu(gate_up, out, batch, ffn, mode, ctx->stream), "swiglu");
}

int kq_dec_add(kq_ctx* ctx, float* h, int64_t h_ld, const float* y, int64_t y_ld, int64_t rows, int64_t cols) {
  if (check_ctx(ctx) || !h || !y || rows < 0 || cols < 0 || h_ld < cols || y_ld < cols) return KQ_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  ctx->launches += rows * cols > 0;
  return dec_status(ctx, kq::dec_add(h, h_ld, y, y_ld, rows, cols, ctx->stream), "add");
}

// Shared checks of the fused single-token linears.
static int fused_linear(kq_ctx* ctx, const kq_weight* w, const kq::XsInput& in, const float* bias, float* y,
                        int flags, const char* what) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!w || !in.x || (!y && in.ymode == kq::XS_Y_LOCAL))
    return fail(ctx, KQ_ERR_INVALID_ARG, "%s: null weight, input or output", what);
  if (flags & ~(KQ_SYNC | KQ_DEVICE_PTRS)) return fail(ctx, KQ_ERR_INVALID_ARG, "%s: bad flags 0x%x", what, flags);
  if (w->device != ctx->device)
    return fail(ctx, KQ_ERR_INVALID_ARG, "weight lives on device %d, context on %d", w->device, ctx->device);
  if (!is_gguf(w->dw.type)) return fail(ctx, KQ_ERR_UNSUPPORTED, "%s needs a GGUF Q4_K / Q6_K weight", what);
  const uintptr_t x16 = reinterpret_cast<uintptr_t>(in.x) | reinterpret_cast<uintptr_t>(in.x2) |
                        reinterpret_cast<uintptr_t>(in.nw);
  if ((x16 & 15) || ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(bias)) & 3))
    return fail(ctx, KQ_ERR_INVALID_ARG, "%s: inputs must be 16-byte aligned, y and bias 4-byte aligned", what);
  DeviceGuard g(ctx->device);
  if (g.status != cudaSuccess) return cuda_fail(ctx, g.status, "cudaSetDevice");
  const kq::Prefetch* pf = ctx->take_prefetch();
  int launches = 0;
  const cudaError_t e = kq::launch_gemv_xs(w->dw, in, bias, y, ctx->num_sms, ctx->dev_err, pf, ctx->stream,
                                           &launches, ctx->next_bracket());
  ctx->launches += launches;
  if (e == cudaErrorNotSupported)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "%s: in_features %lld is beyond the single-token kernel", what,
                (long long)w->dw.k);
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  if (flags & KQ_SYNC) return finish_sync(ctx, what);
  return KQ_OK;
}

// Shared checks of the batched decoder forms (m tokens on the integer
// tensor-core kernel; KQ_ERR_UNSUPPORTED, with nothing queued, where AUTO
// would pick another kernel family for this weight and m).
static int batched_linear(kq_ctx* ctx, const kq_weight* w, const float* x, int64_t m, float* y,
                          const kq::ImOpts& op, int flags, const char* what) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!w || !x || !y || m < 1) return fail(ctx, KQ_ERR_INVALID_ARG, "%s: null weight, input or output, or m < 1", what);
  if (flags & ~(KQ_SYNC | KQ_DEVICE_PTRS)) return fail(ctx, KQ_ERR_INVALID_ARG, "%s: bad flags 0x%x", what, flags);
  if (w->device != ctx->device)
    return fail(ctx, KQ_ERR_INVALID_ARG, "weight lives on device %d, context on %d", w->device, ctx->device);
  if (w->dw.k == 0 || w->dw.n == 0) return fail(ctx, KQ_ERR_UNSUPPORTED, "%s: empty weight", what);
  if ((!is_gguf(w->dw.type) && !is_kx(w->dw.type)) || f32_family(ctx, w->dw, m) != KQ_PATH_IMMA)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "%s: the integer tensor-core kernel does not serve type %d at m = %lld",
                what, w->dw.type, (long long)m);
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(op.nw)) & 15) ||
      (reinterpret_cast<uintptr_t>(y) & 3))
    return fail(ctx, KQ_ERR_INVALID_ARG, "%s: x and the norm weights must be 16-byte aligned, y 4-byte", what);
  DeviceGuard g(ctx->device);
  if (g.status != cudaSuccess) return cuda_fail(ctx, g.status, "cudaSetDevice");
  if (int rc = prepare_f32(ctx, w->dw, m)) return rc;
  int launches = 0;
  const cudaError_t e =
      kq::launch_gemv_imma(w->dw, x, m, nullptr, y, ctx->ws, static_cast<unsigned*>(ctx->ctr), ctx->num_sms,
                           ctx->dev_err, ctx->stream, &launches, ctx->next_bracket(), op);
  ctx->launches += launches;
  if (e != cudaSuccess) return cuda_fail(ctx, e, what);
  if (flags & KQ_SYNC) return finish_sync(ctx, what);
  return KQ_OK;
}

int kq_dec_norm_linear_batch(kq_ctx* ctx, const kq_weight* w, const float* x, int64_t x_ld, int64_t m,
                             const float* norm_w, int64_t dim, float eps, float* y, int flags) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!norm_w) return fail(ctx, KQ_ERR_INVALID_ARG, "norm_linear_batch: null norm weights");
  if (!w || dim < 4 || (dim & 3) || dim > w->dw.k || x_ld < w->dw.k || (x_ld & 3))
    return fail(ctx, KQ_ERR_INVALID_ARG,
                "norm_linear_batch: dim %lld must be a positive multiple of 4 <= in_features, x_ld %lld a "
                "multiple of 4 >= in_features", (long long)dim, (long long)x_ld);
  kq::ImOpts op;
  op.x_ld = x_ld;
  op.nw = norm_w;
  op.dim = (int)dim;
  op.eps = eps;
  return batched_linear(ctx, w, x, m, y, op, flags, "norm_linear_batch");
}

int kq_dec_residual_linear_batch(kq_ctx* ctx, const kq_weight* w, const float* x, int64_t m, float* h, int flags) {
  kq::ImOpts op;
  op.accumulate = true;
  return batched_linear(ctx, w, x, m, h, op, flags, "residual_linear_batch");
}

// act -1: plain rows; 0 / 1: (gate, up) row pairs through the SwiGLU gate.
static int set_pairs(kq_ctx* ctx, const kq_weight* w, int act, kq::XsInput& in, const char* what) {
  if (act < -1 || act > 1) return fail(ctx, KQ_ERR_INVALID_ARG, "%s: activation %d", what, act);
  if (act >= 0) {
    if (!w || (w->dw.n & 1))
      return fail(ctx, KQ_ERR_INVALID_ARG, "%s: a SwiGLU output needs (gate, up) row pairs", what);
    in.ymode = kq::XS_Y_SWIGLU;
    in.act = act;
  }
  return KQ_OK;
}

int kq_dec_norm_linear(kq_ctx* ctx, const kq_weight* w, const float* x, const float* norm_w, int64_t dim, float eps,
                       int act, const float* bias, float* y, int flags) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!norm_w) return fail(ctx, KQ_ERR_INVALID_ARG, "norm_linear: null norm weights");
  if (!w || dim < 4 || (dim & 3) || dim > w->dw.k)
    return fail(ctx, KQ_ERR_INVALID_ARG, "norm_linear: dim %lld must be a positive multiple of 4 <= in_features",
                (long long)dim);
  kq::XsInput in;
  in.mode = kq::XS_X_NORM;
  in.x = x;
  in.nw = norm_w;
  in.dim = (int)dim;
  in.eps = eps;
  if (int rc = set_pairs(ctx, w, act, in, "norm_linear")) return rc;
  return fused_linear(ctx, w, in, bias, y, flags, "norm_linear");
}

int kq_dec_swiglu_linear(kq_ctx* ctx, const kq_weight* w, const float* gate_up, int mode, const float* bias,
                         float* y, int flags) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (mode != 0 && mode != 1) return fail(ctx, KQ_ERR_INVALID_ARG, "swiglu_linear: mode %d", mode);
  if (!w || !gate_up) return fail(ctx, KQ_ERR_INVALID_ARG, "swiglu_linear: null weight or input");
  kq::XsInput in;
  in.mode = kq::XS_X_SWIGLU;
  in.x = gate_up;
  in.x2 = gate_up + w->dw.k;
  in.act = mode;
  return fused_linear(ctx, w, in, bias, y, flags, "swiglu_linear");
}

int kq_dec_residual_linear(kq_ctx* ctx, const kq_weight* w, const float* x, float* h, int flags) {
  kq::XsInput in;
  in.x = x;
  return fused_linear(ctx, w, in, h, h, flags, "residual_linear");
}

// Exchange-buffer view of a tensor-parallel group for the fused linears.
static kq::XsTp xs_tp(const kq_tp* tp) {
  kq::XsTp t;
  for (int p = 0; p < tp->world; ++p) t.exch[p] = static_cast<unsigned long long*>(tp->peer_base[p]);
  t.slot_elems = tp->max_elems;
  t.world = tp->world;
  t.rank = tp->rank;
  t.ctr = tp->ctr;
  t.epoch = tp->ctr + 1;
  return t;
}

int kq_dec_tp_reduce_linear(kq_tp* tp, const kq_weight* w, const float* h_in, float* h_out, const float* norm_w,
                            int64_t dim, float eps, int act, float* y, int flags) {
  if (!tp) return KQ_ERR_INVALID_ARG;
  kq_ctx* ctx = tp->ctx;
  if (!tp->opened) return fail(ctx, KQ_ERR_STATE, "kq_tp_open has not been called");
  if (!w || !h_in || !h_out || h_in == h_out)
    return fail(ctx, KQ_ERR_INVALID_ARG, "tp_reduce_linear: h_in and h_out must be distinct device buffers");
  if (dim < 4 || (dim & 3) || dim > w->dw.k)
    return fail(ctx, KQ_ERR_INVALID_ARG, "tp_reduce_linear: dim %lld must be a positive multiple of 4 <= in_features",
                (long long)dim);
  if (dim * tp->world > tp->max_elems)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "tp_reduce_linear: %d partials of %lld exceed the exchange slot",
                tp->world, (long long)dim);
  if ((reinterpret_cast<uintptr_t>(h_in) | reinterpret_cast<uintptr_t>(h_out)) & 15)
    return fail(ctx, KQ_ERR_INVALID_ARG, "tp_reduce_linear: h_in and h_out must be 16-byte aligned");
  kq::XsInput in;
  in.mode = norm_w ? kq::XS_X_REDUCE_NORM : kq::XS_X_REDUCE;
  in.x = h_in;
  in.nw = norm_w;
  in.dim = (int)dim;
  in.eps = eps;
  in.tp = xs_tp(tp);
  in.tp.h_in = h_in;
  in.tp.h_out = h_out;
  if (act >= 0 && !norm_w) return fail(ctx, KQ_ERR_UNSUPPORTED, "tp_reduce_linear: a SwiGLU output needs the norm");
  if (int rc = set_pairs(ctx, w, act, in, "tp_reduce_linear")) return rc;
  return fused_linear(ctx, w, in, nullptr, y, flags, "tp_reduce_linear");
}

int kq_dec_tp_partial_linear(kq_tp* tp, const kq_weight* w, const float* x, int act, int flags) {
  if (!tp) return KQ_ERR_INVALID_ARG;
  kq_ctx* ctx = tp->ctx;
  if (!tp->opened) return fail(ctx, KQ_ERR_STATE, "kq_tp_open has not been called");
  if (!w || !x) return fail(ctx, KQ_ERR_INVALID_ARG, "tp_partial_linear: null weight or input");
  if (act < -1 || act > 1) return fail(ctx, KQ_ERR_INVALID_ARG, "tp_partial_linear: activation %d", act);
  if (w->dw.n * tp->world > tp->max_elems)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "tp_partial_linear: %d partials of %lld exceed the exchange slot",
                tp->world, (long long)w->dw.n);
  kq::XsInput in;
  in.mode = act < 0 ? kq::XS_X_PLAIN : kq::XS_X_SWIGLU;
  in.x = x;
  in.x2 = act < 0 ? nullptr : x + w->dw.k;
  in.act = act < 0 ? 0 : act;
  in.ymode = kq::XS_Y_PEERS;
  in.tp = xs_tp(tp);
  return fused_linear(ctx, w, in, nullptr, nullptr, flags, "tp_partial_linear");
}

int kq_dec_embed(kq_ctx* ctx, const float* table, const int32_t* tokens, float* out, int64_t out_ld, int64_t batch,
                 int64_t dim) {
  if (check_ctx(ctx) || !table || !tokens || !out || batch < 1 || dim < 1 || out_ld < dim) return KQ_ERR_INVALID_ARG;
  DeviceGuard g(ctx->device);
  ctx->launches += 1;
  return dec_status(ctx, kq::dec_embed(table, tokens, out, out_ld, batch, dim, ctx->stream), "embed");
}

// ---- persistent decode step ------------------------------------------------------

int kq_step_create(kq_ctx* ctx, kq_tp* tp, kq_step** out) {
  if (check_ctx(ctx) || !out) return KQ_ERR_INVALID_ARG;
  *out = nullptr;
  if (tp && (tp->ctx != ctx || !tp->opened))
    return fail(ctx, KQ_ERR_STATE, "kq_step_create: the tensor-parallel group must be open and on this context");
  kq_step* st = new kq_step;
  st->ctx = ctx;
  st->tp = tp;
  *out = st;
  return KQ_OK;
}

static void step_release(kq_step* st) {
  for (void* p : {st->d_stages, st->sync, st->attn_part, st->exch, st->epoch})
    if (p) cudaFree(p);
  st->d_stages = st->sync = st->attn_part = st->exch = st->epoch = nullptr;
  st->built = false;
}

int kq_step_destroy(kq_step* st) {
  if (!st) return KQ_ERR_INVALID_ARG;
  {
    DeviceGuard g(st->ctx->device);
    cudaStreamSynchronize(st->ctx->stream);
    step_release(st);
    cudaGetLastError();
  }
  delete st;
  return KQ_OK;
}

int kq_step_linear(kq_step* st, const kq_weight* w, int in_mode, const float* x, const float* norm_w, int64_t dim,
                   float eps, float* h, int out_mode, float* y, int act) {
  if (!st) return KQ_ERR_INVALID_ARG;
  kq_ctx* ctx = st->ctx;
  if (!w || w->device != ctx->device) return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_linear: no weight on this device");
  if (!is_gguf(w->dw.type))
    return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_step_linear: the step kernel serves GGUF Q4_K / Q6_K weights");
  const int nk = (int)((w->dw.sb + 7) / 8);
  if (w->dw.n < 1 || nk < 1 || nk > kq::STEP_COMPUTE_WARPS || w->dw.n > (int64_t)1 << 30)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_step_linear: %lld x %lld is outside the step kernel's shapes",
                (long long)w->dw.n, (long long)w->dw.k);
  if (in_mode < KQ_STEP_IN_PLAIN || in_mode > KQ_STEP_IN_RESIDUAL_NORM || out_mode < KQ_STEP_OUT_STORE ||
      out_mode > KQ_STEP_OUT_PARTIAL || act < 0 || act > 1)
    return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_linear: bad mode (in %d, out %d, act %d)", in_mode, out_mode, act);
  const bool residual = in_mode == KQ_STEP_IN_RESIDUAL || in_mode == KQ_STEP_IN_RESIDUAL_NORM;
  const bool norm = in_mode == KQ_STEP_IN_NORM || in_mode == KQ_STEP_IN_RESIDUAL_NORM;
  if ((!residual && !x) || (norm && !norm_w) || (residual && !h) || (out_mode != KQ_STEP_OUT_PARTIAL && !y))
    return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_linear: missing x, norm weights, h or y");
  if (residual && out_mode == KQ_STEP_OUT_PARTIAL)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_step_linear: a residual input cannot feed a partial output");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(norm_w)) & 15)
    return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_linear: x, h and norm weights must be 16-byte aligned");
  if ((norm || residual) && (dim < 8 || (dim & 7) || dim > w->dw.k))
    return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_linear: dim %lld must be a positive multiple of 8 <= in_features",
                (long long)dim);
  if (residual && st->pending_len != dim)
    return fail(ctx, KQ_ERR_STATE, "kq_step_linear: a residual input needs a preceding partial output of length %lld",
                (long long)dim);
  if (out_mode == KQ_STEP_OUT_PARTIAL) {
    if (st->pending_len >= 0)
      return fail(ctx, KQ_ERR_STATE, "kq_step_linear: the previous partial output has not been consumed");
    if (w->dw.n & 7) return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_step_linear: a partial output needs rows % 8 == 0");
    if (st->tp && w->dw.n * st->tp->world > st->tp->max_elems)
      return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_step_linear: %d partials of %lld exceed the exchange slot",
                  st->tp->world, (long long)w->dw.n);
  }
  if (out_mode == KQ_STEP_OUT_SWIGLU && (w->dw.n & 1))
    return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_linear: SwiGLU rows come in (gate, up) pairs");
  kq::StepStage S;
  S.kind = kq::STEP_GEMV;
  S.barrier = !residual && !st->stages.empty();
  S.qt = w->dw.type;
  S.n = (int)w->dw.n;
  S.sb = (int)w->dw.sb;
  S.nk = nk;
  S.G = kq::STEP_COMPUTE_WARPS / nk;
  S.row_bytes = w->dw.sb * (w->dw.type == kq::GGUF_Q4_K ? kq::Q4K_BYTES : kq::Q6K_BODY);
  S.d_row_bytes = w->dw.type == kq::GGUF_Q6_K ? (int)(w->dw.d_ld * 2) : 0;
  S.q = w->dw.q;
  S.d = w->dw.d;
  S.xmode = in_mode == KQ_STEP_IN_PLAIN ? kq::SX_PLAIN
            : in_mode == KQ_STEP_IN_NORM ? kq::SX_NORM
            : in_mode == KQ_STEP_IN_RESIDUAL ? kq::SX_REDUCE : kq::SX_REDUCE_NORM;
  S.ymode = out_mode == KQ_STEP_OUT_STORE ? kq::SY_STORE : out_mode == KQ_STEP_OUT_SWIGLU ? kq::SY_SWIGLU
                                                                                          : kq::SY_PARTIAL;
  S.x = residual ? nullptr : x;
  S.nw = norm_w;
  S.dim = (int)((norm || residual) ? dim : 0);
  S.eps = eps;
  S.act = act;
  S.y = y;
  S.h_in = out_mode == KQ_STEP_OUT_PARTIAL ? h : nullptr;
  S.h_out = residual ? h : nullptr;
  if (residual) {
    S.exch = st->nexch - 1;
    st->pending_len = -1;
  }
  if (out_mode == KQ_STEP_OUT_PARTIAL) {
    S.exch = st->nexch++;
    st->pending_len = w->dw.n;
  }
  st->stages.push_back(S);
  st->built = false;
  return KQ_OK;
}

int kq_step_attention(kq_step* st, const float* qkv, void* k_cache, void* v_cache, float* out, int heads,
                      int kv_heads, int head_dim, int64_t max_seq, float theta) {
  if (!st) return KQ_ERR_INVALID_ARG;
  kq_ctx* ctx = st->ctx;
  if (!qkv || !k_cache || !v_cache || !out)
    return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_attention: null qkv, cache or output");
  if ((head_dim != 64 && head_dim != 128) || kv_heads < 1 || heads < kv_heads || heads % kv_heads ||
      heads / kv_heads > kq::STEP_ATTN_MAX_GROUP || (heads / kv_heads) * head_dim / 2 > 32 * kq::STEP_COMPUTE_WARPS ||
      max_seq < 1)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_step_attention: %d / %d heads of %d (head_dim 64 or 128, group <= %d)",
                heads, kv_heads, head_dim, kq::STEP_ATTN_MAX_GROUP);
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
    return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_attention: the caches must be 16-byte aligned");
  kq::StepStage S;
  S.kind = kq::STEP_ATTN;
  S.barrier = !st->stages.empty();
  S.qkv = qkv;
  S.kc = k_cache;
  S.vc = v_cache;
  S.out = out;
  S.hq = heads;
  S.hkv = kv_heads;
  S.hd = head_dim;
  S.max_seq = max_seq;
  S.theta = theta;
  S.splits = std::max(1, ctx->num_sms / kv_heads);
  st->stages.push_back(S);
  st->built = false;
  return KQ_OK;
}

// Size the kernel's shared memory and scratch for the stages, and copy them
// to the device (synchronous: call outside any stream capture).
static int step_build(kq_step* st) {
  kq_ctx* ctx = st->ctx;
  if (st->stages.empty()) return fail(ctx, KQ_ERR_STATE, "kq_step_run: the program has no stages");
  if (st->pending_len >= 0 && !st->tp)
    return fail(ctx, KQ_ERR_STATE, "kq_step_run: the last partial output is never consumed");
  step_release(st);
  const int C = ctx->num_sms;
  kq::StepArgs& a = st->args;
  a = kq::StepArgs();
  int64_t slot = 0, xr = 0, nwf = 0, partial = 0;
  int nk_max = 1, rows_max = 1, max_hkv = 0;
  for (auto& S : st->stages) {
    if (S.kind != kq::STEP_GEMV) continue;
    slot = std::max<int64_t>(slot, 2 * S.G * (S.row_bytes + S.d_row_bytes));
    nk_max = std::max(nk_max, S.nk);
    for (int b = 0; b < C; ++b) {  // the kernel's row split (sp_rows)
      int64_t r0, r1;
      if (S.ymode == kq::SY_SWIGLU) {
        r0 = 2 * ((int64_t)(S.n / 2) * b / C);
        r1 = 2 * ((int64_t)(S.n / 2) * (b + 1) / C);
      } else if (S.ymode == kq::SY_PARTIAL) {
        r0 = 4 * ((int64_t)(S.n / 4) * b / C);
        r1 = b == C - 1 ? S.n : 4 * ((int64_t)(S.n / 4) * (b + 1) / C);
        partial = std::max<int64_t>(partial, S.n);
      } else {
        r0 = (int64_t)S.n * b / C;
        r1 = (int64_t)S.n * (b + 1) / C;
      }
      rows_max = std::max(rows_max, (int)(r1 - r0));
    }
    if (S.xmode == kq::SX_REDUCE || S.xmode == kq::SX_REDUCE_NORM) xr = std::max<int64_t>(xr, S.dim);
    if (S.xmode == kq::SX_NORM || S.xmode == kq::SX_REDUCE_NORM) nwf = std::max<int64_t>(nwf, S.dim);
  }
  int attn_bytes = 0;
  int64_t part_floats = 0;
  for (auto& S : st->stages) {
    if (S.kind != kq::STEP_ATTN) continue;
    slot = std::max<int64_t>(slot, (int64_t)S.hd * 2 * 64);  // at least 64 positions per KV tile
  }
  slot = (slot + 127) & ~int64_t(127);
  for (auto& S : st->stages) {
    if (S.kind != kq::STEP_ATTN) continue;
    S.tile = (int)std::min<int64_t>(slot / (S.hd * 2), 1024);
    const int G = S.hq / S.hkv;
    attn_bytes = std::max(attn_bytes, G * S.hd * 4 + G * (S.tile + 4) * 4 + 3 * kq::STEP_ATTN_MAX_GROUP * 4 +
                                          G * S.splits * 4 + 2 * S.hd * 2 + 16);
    part_floats = std::max<int64_t>(part_floats, (int64_t)S.hkv * S.splits * G * (S.hd + 4));
    max_hkv = std::max(max_hkv, S.hkv);
  }
  const size_t fixed =
      kq::StepSmem(0, (int)slot, nk_max, rows_max, (int)((xr + 3) & ~3), (int)((nwf + 3) & ~3), attn_bytes).end;
  if (slot > (1 << 20) || fixed + 2 * (size_t)slot > (size_t)kq::STEP_MAX_SMEM)
    return fail(ctx, KQ_ERR_UNSUPPORTED, "kq_step_run: a stage needs %lld-byte ring slots; two do not fit",
                (long long)slot);
  const int fit = (int)((kq::STEP_MAX_SMEM - fixed - 64) / (size_t)slot);
  a.S = std::max(2, std::min(fit, std::max(2, (int)((176 * 1024) / slot))));
  a.slot_bytes = (int)slot;
  a.nk_max = nk_max;
  a.rows_max = rows_max;
  a.xr_floats = (int)((xr + 3) & ~3);
  a.nw_floats = (int)((nwf + 3) & ~3);
  a.attn_bytes = attn_bytes;
  a.nexch = st->nexch;
  DeviceGuard g(ctx->device);
  const size_t sync_bytes = (size_t)(kq::STEP_SYNC_ATTN + max_hkv + 2) * sizeof(unsigned);
  cudaError_t e = cudaMalloc(&st->sync, sync_bytes);
  if (e == cudaSuccess) e = cudaMemset(st->sync, 0, sync_bytes);
  if (e == cudaSuccess && part_floats) e = cudaMalloc(&st->attn_part, (size_t)part_floats * 4);
  if (e == cudaSuccess) e = cudaMalloc(&st->d_stages, st->stages.size() * sizeof(kq::StepStage));
  if (e == cudaSuccess)
    e = cudaMemcpy(st->d_stages, st->stages.data(), st->stages.size() * sizeof(kq::StepStage), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && st->tp) {
    for (int p = 0; p < st->tp->world; ++p) a.exch[p] = static_cast<unsigned long long*>(st->tp->peer_base[p]);
    a.slot_elems = st->tp->max_elems;
    a.world = st->tp->world;
    a.rank = st->tp->rank;
    a.epoch = st->tp->ctr + 1;
  } else if (e == cudaSuccess) {
    const int64_t elems = std::max<int64_t>(partial, 4);
    e = cudaMalloc(&st->exch, (size_t)2 * elems * 8);
    if (e == cudaSuccess) e = cudaMemset(st->exch, 0, (size_t)2 * elems * 8);
    if (e == cudaSuccess) e = cudaMalloc(&st->epoch, 16);
    if (e == cudaSuccess) e = cudaMemset(st->epoch, 0, 16);
    a.exch[0] = static_cast<unsigned long long*>(st->exch);
    a.slot_elems = elems;
    a.world = 1;
    a.rank = 0;
    a.epoch = static_cast<unsigned*>(st->epoch);
  }
  if (e != cudaSuccess) {
    step_release(st);
    return cuda_fail(ctx, e, "kq_step_run: allocate the step's scratch");
  }
  a.stages = static_cast<const kq::StepStage*>(st->d_stages);
  a.nstages = (int)st->stages.size();
  a.sync = static_cast<unsigned*>(st->sync);
  a.attn_part = static_cast<float*>(st->attn_part);
  a.err = ctx->dev_err;
  st->built = true;
  return KQ_OK;
}

int kq_step_trace(kq_step* st, uint64_t* trace, size_t words) {
  if (!st) return KQ_ERR_INVALID_ARG;
  const size_t need = (size_t)st->ctx->num_sms * st->stages.size() * kq::STEP_TRACE_POINTS;
  if (trace && words < need)
    return fail(st->ctx, KQ_ERR_SHORT_BUFFER, "kq_step_trace: %zu words; the program needs %zu", words, need);
  st->trace = reinterpret_cast<unsigned long long*>(trace);
  return KQ_OK;
}

int kq_step_run(kq_step* st, int64_t pos, int flags) {
  if (!st) return KQ_ERR_INVALID_ARG;
  kq_ctx* ctx = st->ctx;
  if (flags & ~KQ_SYNC) return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_run: bad flags 0x%x", flags);
  for (const auto& S : st->stages)
    if (S.kind == kq::STEP_ATTN && (pos < 0 || pos >= S.max_seq))
      return fail(ctx, KQ_ERR_INVALID_ARG, "kq_step_run: position %lld outside the cache (%lld)", (long long)pos,
                  (long long)S.max_seq);
  DeviceGuard g(ctx->device);
  if (g.status != cudaSuccess) return cuda_fail(ctx, g.status, "cudaSetDevice");
  if (!st->built) {
    const int rc = step_build(st);
    if (rc) return rc;
  }
  kq::StepArgs a = st->args;
  a.pos = pos;
  a.trace = st->trace;
  kq::Bracket br = ctx->next_bracket();
  kq::bracket_record(br.start, ctx->stream);
  cudaError_t e = kq::launch_step(a, ctx->num_sms, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "kq_step_run: launch");
  kq::bracket_record(br.stop, ctx->stream);
  ctx->launches += 1;
  if (flags & KQ_SYNC) {
    const int rc = finish_sync(ctx, "kq_step_run");
    if (rc != KQ_OK && st->sync) {  // a wait gave up: counters may be left mid-count
      st->built = false;  // the next run rebuilds (and re-zeroes) every scratch word
    }
    return rc;
  }
  return KQ_OK;
}

int kq_dequant_f32(kq_ctx* ctx, const kq_weight* w, int64_t row0, int64_t nrows, float* out, int flags) {
  if (check_ctx(ctx)) return KQ_ERR_INVALID_ARG;
  if (!w) return fail(ctx, KQ_ERR_INVALID_ARG, "weight is null");
  if (flags & ~(KQ_DEVICE_PTRS | KQ_SYNC)) return fail(ctx, KQ_ERR_INVALID_ARG, "bad flags 0x%x", flags);
  if (w->device != ctx->device) return fail(ctx, KQ_ERR_INVALID_ARG, "weight on another device");
  if (row0 < 0 || nrows < 0 || row0 + nrows > w->dw.n)
    return fail(ctx, KQ_ERR_INVALID_ARG, "rows [%lld, %lld) outside [0, %lld)", (long long)row0,
                (long long)(row0 + nrows), (long long)w->dw.n);
  const int64_t count = nrows * w->dw.k;
  if (count == 0) return KQ_OK;
  if (!out) return fail(ctx, KQ_ERR_INVALID_ARG, "out is null");
  const bool dev = flags & KQ_DEVICE_PTRS;
  DeviceGuard g(ctx->device);
  if (g.status != cudaSuccess) return cuda_fail(ctx, g.status, "cudaSetDevice");
  int rc;
  float* od = out;
  if (!dev) {
    if ((rc = ensure(ctx, &ctx->ybuf, &ctx->ybuf_bytes, (size_t)count * 4, "output staging"))) return rc;
    od = static_cast<float*>(ctx->ybuf);
  }
  cudaError_t e = is_kx(w->dw.type) ? kq::launch_dequant_kx(w->dw, row0, nrows, od, ctx->stream)
                                    : kq::launch_dequant_f32(w->dw, row0, nrows, od, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "dequant launch");
  ++ctx->launches;
  if (!dev) {
    e = cudaMemcpyAsync(out, od, (size_t)count * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "copy to host");
  }
  if (!dev || (flags & KQ_SYNC)) return finish_sync(ctx, "kq_dequant_f32");
  return KQ_OK;
}

}  // extern "C"
