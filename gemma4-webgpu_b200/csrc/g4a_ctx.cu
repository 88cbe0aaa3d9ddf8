// Context, memory, errors and synchronisation entry points of libg4attn.
//
// The reference's equivalents are the WebGPU device plumbing in src/engine.ts: initWebGPU
// (:402-437), buffer creation (:1347-1426), queue.onSubmittedWorkDone (:2474) and the
// `deviceLost` flag checked by every public entry point (:432-435, :2214, :2509).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <chrono>
#include <thread>

#include "g4a_internal.cuh"

static thread_local std::string t_last_error;

void g4a_set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

g4a_status g4a_fail(g4a_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return st;
}

g4a_status g4a_cuda_fail(cudaError_t e, const char* what) {
  g4a_set_error("%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
  return e == cudaErrorMemoryAllocation ? G4A_ENOMEM : G4A_ECUDA;
}

g4a_status g4a_check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return g4a_cuda_fail(e, what);
  return G4A_OK;
}

g4a_status g4a_ensure_workspace(g4a_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->workspace_bytes) return G4A_OK;
  // Growing must not free memory that queued kernels still read.
  G4A_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (ctx->workspace) {
    cudaFree(ctx->workspace);
    ctx->workspace = nullptr;
    ctx->workspace_bytes = 0;
  }
  size_t want = bytes < (size_t)(1u << 20) ? (size_t)(1u << 20) : bytes;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, want);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaMalloc(workspace)");
  ctx->workspace = p;
  ctx->workspace_bytes = want;
  return G4A_OK;
}

const char* const g4a_prof_names[G4A_PROF_NUM_LABELS] = {
    "norm_rope", "rms_norm_no_weight", "kv_store", "decode_prep", "decode_splitkv",
    "decode_merge", "decode_generic", "lse_merge", "prefill_prep", "prefill_attn", "matmul"};

static cudaEvent_t prof_event(g4a_ctx* ctx) {
  if (!ctx->prof_free.empty()) {
    cudaEvent_t e = ctx->prof_free.back();
    ctx->prof_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

g4a_prof_scope::g4a_prof_scope(g4a_ctx* c, int l) : ctx(c), label(l) {
  if (!ctx || !ctx->prof_enabled) return;
  cudaEvent_t b = prof_event(ctx);
  end = prof_event(ctx);
  if (!b || !end) {
    end = nullptr;
    return;
  }
  cudaEventRecord(b, ctx->stream);
  ctx->prof_pending.push_back({label, b, end});
}

g4a_prof_scope::~g4a_prof_scope() {
  if (end) cudaEventRecord(end, ctx->stream);
}

// Fold completed event pairs into the per-label totals (waits for the stream).
static g4a_status prof_collect(g4a_ctx* ctx) {
  if (ctx->prof_pending.empty()) return G4A_OK;
  G4A_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  for (auto& r : ctx->prof_pending) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, r.begin, r.end) == cudaSuccess) {
      ctx->prof_ms[r.label] += ms;
      ctx->prof_count[r.label] += 1;
    }
    ctx->prof_free.push_back(r.begin);
    ctx->prof_free.push_back(r.end);
  }
  ctx->prof_pending.clear();
  return G4A_OK;
}

extern "C" {

g4a_status g4a_profile_enable(g4a_ctx* ctx, int enable) {
  G4A_CHECK_CTX(ctx);
  ctx->prof_enabled = enable != 0;
  return G4A_OK;
}

g4a_status g4a_profile_reset(g4a_ctx* ctx) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = prof_collect(ctx)) return s;
  for (int i = 0; i < G4A_PROF_NUM_LABELS; i++) {
    ctx->prof_ms[i] = 0.0;
    ctx->prof_count[i] = 0;
  }
  return G4A_OK;
}

g4a_status g4a_profile_read(g4a_ctx* ctx, const char* label, double* total_ms, uint64_t* count) {
  G4A_CHECK_CTX(ctx);
  if (!label || !total_ms || !count) return g4a_fail(G4A_EINVAL, "g4a_profile_read: null argument");
  if (g4a_status s = prof_collect(ctx)) return s;
  for (int i = 0; i < G4A_PROF_NUM_LABELS; i++) {
    if (strcmp(label, g4a_prof_names[i]) == 0) {
      *total_ms = ctx->prof_ms[i];
      *count = ctx->prof_count[i];
      return G4A_OK;
    }
  }
  return g4a_fail(G4A_EINVAL, "g4a_profile_read: unknown label '%s'", label);
}

const char* g4a_last_error(void) { return t_last_error.c_str(); }

const char* g4a_version(void) { return "g4attn 0.1.0 sm_100a"; }

g4a_status g4a_create(int device, g4a_ctx** out_ctx) {
  if (out_ctx == nullptr) return g4a_fail(G4A_EINVAL, "g4a_create: out_ctx is null");
  *out_ctx = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n)
    return g4a_fail(G4A_EINVAL, "g4a_create: device %d out of range [0,%d)", device, n);
  G4A_CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  G4A_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return g4a_fail(G4A_EUNSUPPORTED, "g4a_create: device %d is sm_%d%d; this build targets sm_100a (B200)", device,
                    prop.major, prop.minor);
  g4a_ctx* ctx = new g4a_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->smem_optin = prop.sharedMemPerBlockOptin;
  e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete ctx;
    return g4a_cuda_fail(e, "cudaStreamCreate");
  }
  ctx->stream = ctx->own_stream;
  int* hp = nullptr;
  e = cudaHostAlloc((void**)&hp, sizeof(int), cudaHostAllocMapped);
  if (e != cudaSuccess) {
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return g4a_cuda_fail(e, "cudaHostAlloc(dev_err)");
  }
  *hp = 0;
  ctx->dev_err_host = hp;
  e = cudaHostGetDevicePointer((void**)&ctx->dev_err_dev, hp, 0);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->sync_event, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    cudaFreeHost(hp);
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return g4a_cuda_fail(e, "g4a_create");
  }
  *out_ctx = ctx;
  return G4A_OK;
}

g4a_status g4a_destroy(g4a_ctx* ctx) {
  if (ctx == nullptr) return G4A_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  g4a_dist_release(ctx);
  for (auto& r : ctx->prof_pending) {
    cudaEventDestroy(r.begin);
    cudaEventDestroy(r.end);
  }
  for (auto e : ctx->prof_free) cudaEventDestroy(e);
  if (ctx->workspace) cudaFree(ctx->workspace);
  if (ctx->seq_lens) cudaFree(ctx->seq_lens);
  if (ctx->sync_event) cudaEventDestroy(ctx->sync_event);
  if (ctx->dev_err_host) cudaFreeHost((void*)ctx->dev_err_host);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return G4A_OK;
}

g4a_status g4a_set_stream(g4a_ctx* ctx, void* cuda_stream) {
  G4A_CHECK_CTX(ctx);
  ctx->stream = (cudaStream_t)cuda_stream;  // 0 is the legacy default stream
  return G4A_OK;
}

g4a_status g4a_use_own_stream(g4a_ctx* ctx) {
  G4A_CHECK_CTX(ctx);
  ctx->stream = ctx->own_stream;
  return G4A_OK;
}

void* g4a_get_stream(g4a_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

g4a_status g4a_sync(g4a_ctx* ctx, uint32_t timeout_ms) {
  G4A_CHECK_CTX(ctx);
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  G4A_CUDA_TRY(cudaEventRecord(ctx->sync_event, ctx->stream));
  auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  while (true) {
    cudaError_t e = cudaEventQuery(ctx->sync_event);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return g4a_cuda_fail(e, "g4a_sync");
    const bool late = std::chrono::steady_clock::now() >= deadline;
    // a pending collective that failed or outlived the deadline: abort the communicator (its
    // kernels stop) and report, as the reference turns a lost device into an error
    if (ctx->nccl_comm != nullptr)
      if (g4a_status s = g4a_dist_check(ctx, late, timeout_ms)) return s;
    if (late) return g4a_fail(G4A_ETIMEOUT, "g4a_sync: work still running after %u ms", timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  int derr = *ctx->dev_err_host;
  if (derr != 0) {
    *ctx->dev_err_host = 0;
    return g4a_fail(G4A_ETIMEOUT, "g4a_sync: a kernel reported device error code %d (%s)", derr,
                    derr == G4A_DEVERR_PAGE        ? "page id out of range, row skipped"
                    : derr == G4A_DEVERR_KVLEN     ? "kv_len beyond page-table capacity, capped"
                    : derr == G4A_DEVERR_WAIT_PEER ? "a peer's split-KV partial did not arrive, output zeroed"
                                                   : "bounded wait gave up");
  }
  return G4A_OK;
}

g4a_status g4a_alloc(g4a_ctx* ctx, size_t bytes, void** out_dptr) {
  G4A_CHECK_CTX(ctx);
  if (out_dptr == nullptr) return g4a_fail(G4A_EINVAL, "g4a_alloc: out pointer is null");
  *out_dptr = nullptr;
  if (bytes == 0) return G4A_OK;
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  cudaError_t e = cudaMalloc(out_dptr, bytes);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaMalloc");
  return G4A_OK;
}

g4a_status g4a_free(g4a_ctx* ctx, void* dptr) {
  G4A_CHECK_CTX(ctx);
  if (dptr == nullptr) return G4A_OK;
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  G4A_CUDA_TRY(cudaFree(dptr));
  return G4A_OK;
}

g4a_status g4a_memcpy_h2d(g4a_ctx* ctx, void* dst, const void* src, size_t bytes) {
  G4A_CHECK_CTX(ctx);
  if (bytes == 0) return G4A_OK;
  if (!dst || !src) return g4a_fail(G4A_EINVAL, "g4a_memcpy_h2d: null pointer");
  G4A_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return G4A_OK;
}

g4a_status g4a_memcpy_d2h(g4a_ctx* ctx, void* dst, const void* src, size_t bytes) {
  G4A_CHECK_CTX(ctx);
  if (bytes == 0) return G4A_OK;
  if (!dst || !src) return g4a_fail(G4A_EINVAL, "g4a_memcpy_d2h: null pointer");
  G4A_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return G4A_OK;
}

g4a_status g4a_memset(g4a_ctx* ctx, void* dst, int value, size_t bytes) {
  G4A_CHECK_CTX(ctx);
  if (bytes == 0) return G4A_OK;
  if (!dst) return g4a_fail(G4A_EINVAL, "g4a_memset: null pointer");
  G4A_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, ctx->stream));
  return G4A_OK;
}

}  // extern "C"
