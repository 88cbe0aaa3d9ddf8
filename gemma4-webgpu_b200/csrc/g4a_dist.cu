// Multi-GPU split-KV decode through the C ABI: one NCCL communicator per context.
//
// A single long context is split along the KV length over ranks (one process per GPU, one
// context per process).  Each rank computes the (m, l, o) partial of its slice
// (g4a_decode_attn_partial), the ranks all-gather the partials (8,256 bytes per rank at
// head_dim 256) with ncclAllGather over NVLink, and every rank merges them (g4a_lse_merge).
// The reference decodes one sequence on one WebGPU device and has no collective; its failure
// semantics are the deviceLost checks that turn a lost device into an error at the next call
// (src/engine.ts:432-435, 2214, 2509).  Here a collective that cannot complete is the analogue:
// the communicator is created non-blocking (ncclConfig_t.blocking = 0), every NCCL call is
// polled with ncclCommGetAsyncError under a caller-given deadline, and a deadline that passes --
// or an asynchronous error such as a peer that went away -- aborts the communicator
// (ncclCommAbort, which also stops its kernels) and surfaces as G4A_ETIMEOUT / G4A_ENCCL.  The
// same check runs inside g4a_sync, so a collective stuck behind a missing rank ends the wait with
// an error instead of blocking it.
//
// libnccl.so.2 is loaded at run time (dlopen) rather than linked: a process that already holds
// an NCCL (the PyTorch test harness) keeps using that one, and a host without NCCL can still load
// this library for single-GPU work.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "g4a_internal.cuh"

namespace {

struct NcclApi {
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*getErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*getVersion)(int*) = nullptr;
};

std::once_flag g_nccl_once;
NcclApi g_nccl;
std::string g_nccl_load_error;

void load_nccl() {
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
  if (!h) {
    const char* e = dlerror();
    g_nccl_load_error = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
    return;
  }
  NcclApi a;
  auto sym = [&](const char* name) { return dlsym(h, name); };
  a.getUniqueId = reinterpret_cast<decltype(a.getUniqueId)>(sym("ncclGetUniqueId"));
  a.commInitRankConfig = reinterpret_cast<decltype(a.commInitRankConfig)>(sym("ncclCommInitRankConfig"));
  a.commGetAsyncError = reinterpret_cast<decltype(a.commGetAsyncError)>(sym("ncclCommGetAsyncError"));
  a.commAbort = reinterpret_cast<decltype(a.commAbort)>(sym("ncclCommAbort"));
  a.commDestroy = reinterpret_cast<decltype(a.commDestroy)>(sym("ncclCommDestroy"));
  a.allGather = reinterpret_cast<decltype(a.allGather)>(sym("ncclAllGather"));
  a.getErrorString = reinterpret_cast<decltype(a.getErrorString)>(sym("ncclGetErrorString"));
  a.getVersion = reinterpret_cast<decltype(a.getVersion)>(sym("ncclGetVersion"));
  if (!a.getUniqueId || !a.commInitRankConfig || !a.commGetAsyncError || !a.commAbort || !a.commDestroy ||
      !a.allGather || !a.getErrorString || !a.getVersion) {
    g_nccl_load_error = "libnccl.so.2 lacks the non-blocking communicator API (NCCL >= 2.14 needed)";
    return;
  }
  g_nccl = a;
}

g4a_status nccl_api(const NcclApi** out) {
  std::call_once(g_nccl_once, load_nccl);
  if (!g_nccl.getUniqueId) return g4a_fail(G4A_EUNSUPPORTED, "%s", g_nccl_load_error.c_str());
  *out = &g_nccl;
  return G4A_OK;
}

const char* nccl_str(const NcclApi& api, ncclResult_t r) {
  return api.getErrorString ? api.getErrorString(r) : "NCCL error";
}

// Wait until an operation issued on a non-blocking communicator leaves ncclInProgress.  `first`
// is the value the issuing call returned.  On an error, or when `timeout_ms` passes first, the
// communicator is aborted (*aborted set) and G4A_ENCCL / G4A_ETIMEOUT returned.
g4a_status nccl_wait(const NcclApi& api, ncclComm_t comm, ncclResult_t first, uint32_t timeout_ms, const char* what,
                     bool* aborted) {
  *aborted = false;
  ncclResult_t st = first;
  const auto t0 = std::chrono::steady_clock::now();
  const auto deadline = t0 + std::chrono::milliseconds(timeout_ms);
  while (true) {
    if (st == ncclSuccess) return G4A_OK;
    if (st != ncclInProgress) {
      api.commAbort(comm);
      *aborted = true;
      return g4a_fail(G4A_ENCCL, "%s: %s (%d); the communicator was aborted", what, nccl_str(api, st), (int)st);
    }
    if (std::chrono::steady_clock::now() >= deadline) {
      api.commAbort(comm);
      *aborted = true;
      return g4a_fail(G4A_ETIMEOUT, "%s: not complete after %u ms (a rank did not join); the communicator was aborted",
                      what, timeout_ms);
    }
    // an enqueue normally completes within microseconds: spin for the first 2 ms, then back off
    if (std::chrono::steady_clock::now() - t0 < std::chrono::milliseconds(2))
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(100));
    const ncclResult_t q = api.commGetAsyncError(comm, &st);
    if (q != ncclSuccess && q != ncclInProgress) st = q;
  }
}

g4a_status require_comm(g4a_ctx* ctx, const char* fn) {
  if (ctx->nccl_comm == nullptr)
    return g4a_fail(G4A_EINVAL, "%s: no communicator on this context (call g4a_dist_init%s)", fn,
                    ctx->dist_aborted ? " again: the previous one was aborted" : "");
  return G4A_OK;
}

void drop_comm(g4a_ctx* ctx, bool aborted) {
  ctx->nccl_comm = nullptr;
  ctx->dist_rank = -1;
  ctx->dist_nranks = 0;
  ctx->dist_aborted = aborted;
}

// Fake NCCL for g4a_dist_poll_selftest: commGetAsyncError follows a scripted scenario.
int g_fake_scenario = 0, g_fake_polls = 0, g_fake_aborts = 0;
ncclResult_t fake_async_error(ncclComm_t, ncclResult_t* st) {
  g_fake_polls++;
  switch (g_fake_scenario) {
    case 0: *st = g_fake_polls >= 3 ? ncclSuccess : ncclInProgress; break;     // completes on the 3rd poll
    case 1: *st = ncclInProgress; break;                                      // a rank never joins
    default: *st = g_fake_polls >= 2 ? ncclRemoteError : ncclInProgress; break;  // a peer fails
  }
  return ncclSuccess;
}
ncclResult_t fake_abort(ncclComm_t) {
  g_fake_aborts++;
  return ncclSuccess;
}
const char* fake_error_string(ncclResult_t) { return "fake NCCL error"; }

}  // namespace

// Called by g4a_sync while it waits (see g4a_internal.cuh).
g4a_status g4a_dist_check(g4a_ctx* ctx, bool deadline_passed, uint32_t timeout_ms) {
  if (ctx->nccl_comm == nullptr) return G4A_OK;
  const NcclApi* api = nullptr;
  if (nccl_api(&api) != G4A_OK) return G4A_OK;
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
  ncclResult_t st = ncclSuccess;
  const ncclResult_t q = api->commGetAsyncError(comm, &st);
  if (q != ncclSuccess && q != ncclInProgress) st = q;
  if (st != ncclSuccess && st != ncclInProgress) {
    api->commAbort(comm);
    drop_comm(ctx, true);
    return g4a_fail(G4A_ENCCL, "g4a_sync: a collective failed: %s (%d); the communicator was aborted",
                    nccl_str(*api, st), (int)st);
  }
  if (deadline_passed) {
    api->commAbort(comm);
    drop_comm(ctx, true);
    return g4a_fail(G4A_ETIMEOUT,
                    "g4a_sync: work still running after %u ms with a collective pending (a rank did not join); "
                    "the communicator was aborted",
                    timeout_ms);
  }
  return G4A_OK;
}

void g4a_dist_release(g4a_ctx* ctx) {
  if (ctx->nccl_comm == nullptr) return;
  const NcclApi* api = nullptr;
  if (nccl_api(&api) == G4A_OK) api->commDestroy(static_cast<ncclComm_t>(ctx->nccl_comm));
  drop_comm(ctx, false);
}

extern "C" {

g4a_status g4a_dist_unique_id(void* id_out) {
  if (id_out == nullptr) return g4a_fail(G4A_EINVAL, "g4a_dist_unique_id: null output");
  const NcclApi* api = nullptr;
  if (g4a_status s = nccl_api(&api)) return s;
  ncclUniqueId id;
  const ncclResult_t r = api->getUniqueId(&id);
  if (r != ncclSuccess) return g4a_fail(G4A_ENCCL, "ncclGetUniqueId: %s", nccl_str(*api, r));
  static_assert(sizeof(id) == G4A_DIST_ID_BYTES, "unique id size");
  memcpy(id_out, &id, sizeof(id));
  return G4A_OK;
}

g4a_status g4a_dist_init(g4a_ctx* ctx, int rank, int nranks, const void* id, uint32_t timeout_ms) {
  G4A_CHECK_CTX(ctx);
  if (id == nullptr) return g4a_fail(G4A_EINVAL, "g4a_dist_init: null unique id");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return g4a_fail(G4A_EINVAL, "g4a_dist_init: rank %d of %d is out of range", rank, nranks);
  if (ctx->nccl_comm != nullptr) return g4a_fail(G4A_EINVAL, "g4a_dist_init: the context already has a communicator");
  const NcclApi* api = nullptr;
  if (g4a_status s = nccl_api(&api)) return s;
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  const ncclResult_t r = api->commInitRankConfig(&comm, nranks, uid, rank, &cfg);
  if (comm == nullptr)
    return g4a_fail(G4A_ENCCL, "ncclCommInitRankConfig: %s (%d)", nccl_str(*api, r), (int)r);
  bool aborted = false;
  if (g4a_status s = nccl_wait(*api, comm, r, timeout_ms, "g4a_dist_init (ncclCommInitRankConfig)", &aborted)) {
    drop_comm(ctx, aborted);
    return s;
  }
  ctx->nccl_comm = comm;
  ctx->dist_rank = rank;
  ctx->dist_nranks = nranks;
  ctx->dist_aborted = false;
  return G4A_OK;
}

g4a_status g4a_dist_destroy(g4a_ctx* ctx) {
  G4A_CHECK_CTX(ctx);
  g4a_dist_release(ctx);
  ctx->dist_aborted = false;
  return G4A_OK;
}

g4a_status g4a_dist_info(g4a_ctx* ctx, int* rank, int* nranks) {
  G4A_CHECK_CTX(ctx);
  if (!rank || !nranks) return g4a_fail(G4A_EINVAL, "g4a_dist_info: null output");
  *rank = ctx->dist_rank;
  *nranks = ctx->dist_nranks;
  return G4A_OK;
}

g4a_status g4a_allgather_partials(g4a_ctx* ctx, const float* part, float* parts_all, size_t floats_per_rank,
                                  uint32_t timeout_ms) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = require_comm(ctx, __func__)) return s;
  if (!part || !parts_all || floats_per_rank == 0)
    return g4a_fail(G4A_EINVAL, "g4a_allgather_partials: null buffer or zero size");
  const NcclApi* api = nullptr;
  if (g4a_status s = nccl_api(&api)) return s;
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
  const ncclResult_t r = api->allGather(part, parts_all, floats_per_rank, ncclFloat32, comm, ctx->stream);
  bool aborted = false;
  g4a_status s = nccl_wait(*api, comm, r, timeout_ms, "g4a_allgather_partials (ncclAllGather)", &aborted);
  if (aborted) drop_comm(ctx, true);
  return s;
}

g4a_status g4a_dist_allgather_host(g4a_ctx* ctx, const void* send, void* recv, size_t bytes, uint32_t timeout_ms) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = require_comm(ctx, __func__)) return s;
  if (!send || !recv || bytes == 0) return g4a_fail(G4A_EINVAL, "g4a_dist_allgather_host: null buffer or zero size");
  const NcclApi* api = nullptr;
  if (g4a_status s = nccl_api(&api)) return s;
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  const size_t n = (size_t)ctx->dist_nranks;
  void* dev = nullptr;
  cudaError_t e = cudaMalloc(&dev, bytes * (n + 1));
  if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaMalloc(g4a_dist_allgather_host)");
  char* d_send = static_cast<char*>(dev) + bytes * n;
  g4a_status s = G4A_OK;
  e = cudaMemcpyAsync(d_send, send, bytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) s = g4a_cuda_fail(e, "cudaMemcpyAsync(g4a_dist_allgather_host)");
  if (s == G4A_OK) {
    ncclComm_t comm = static_cast<ncclComm_t>(ctx->nccl_comm);
    const ncclResult_t r = api->allGather(d_send, dev, bytes, ncclUint8, comm, ctx->stream);
    bool aborted = false;
    s = nccl_wait(*api, comm, r, timeout_ms, "g4a_dist_allgather_host (ncclAllGather)", &aborted);
    if (aborted) drop_comm(ctx, true);
  }
  if (s == G4A_OK) {
    e = cudaMemcpyAsync(recv, dev, bytes * n, cudaMemcpyDeviceToHost, ctx->stream);
    s = (e != cudaSuccess) ? g4a_cuda_fail(e, "cudaMemcpyAsync(g4a_dist_allgather_host)") : g4a_sync(ctx, timeout_ms);
  }
  cudaStreamSynchronize(ctx->stream);  // the buffer is freed below; after an abort the stream has drained
  cudaFree(dev);
  return s;
}

g4a_status g4a_decode_attn_splitkv(g4a_ctx* ctx, const float* q, const uint16_t* k_slice, const uint16_t* v_slice,
                                   uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim, uint32_t kv_begin,
                                   uint32_t kv_end, uint32_t kv_len_total, float scale, uint32_t sliding_window,
                                   float* parts_all, float* out, uint32_t timeout_ms) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = require_comm(ctx, __func__)) return s;
  if (!parts_all || !out) return g4a_fail(G4A_EINVAL, "g4a_decode_attn_splitkv: null parts_all or out");
  if (num_kv_heads != 1)
    return g4a_fail(G4A_EINVAL, "g4a_decode_attn_splitkv: one kv head per call (got %u)", num_kv_heads);
  const size_t per_rank = (size_t)num_q_heads * (head_dim + 2);
  float* mine = parts_all + per_rank * (size_t)ctx->dist_rank;
  if (g4a_status s = g4a_decode_attn_partial(ctx, q, k_slice, v_slice, num_q_heads, num_kv_heads, head_dim, kv_begin,
                                             kv_end, kv_len_total, scale, sliding_window, mine))
    return s;
  // in place: rank r's partial already sits at parts_all + r * per_rank
  if (g4a_status s = g4a_allgather_partials(ctx, mine, parts_all, per_rank, timeout_ms)) return s;
  return g4a_lse_merge(ctx, parts_all, (uint32_t)ctx->dist_nranks, num_q_heads, head_dim, out);
}

g4a_status g4a_dist_poll_selftest(int scenario, uint32_t timeout_ms, int* aborted) {
  if (aborted == nullptr) return g4a_fail(G4A_EINVAL, "g4a_dist_poll_selftest: null output");
  NcclApi fake;
  fake.commGetAsyncError = fake_async_error;
  fake.commAbort = fake_abort;
  fake.getErrorString = fake_error_string;
  g_fake_scenario = scenario;
  g_fake_polls = 0;
  g_fake_aborts = 0;
  bool ab = false;
  g4a_status s = nccl_wait(fake, nullptr, ncclInProgress, timeout_ms, "g4a_dist_poll_selftest", &ab);
  *aborted = (ab && g_fake_aborts == 1) ? 1 : (ab ? -1 : 0);
  return s;
}

}  // extern "C"
