// Internal header of libg4attn: context, error plumbing and sm_100a PTX helpers.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "g4attn.h"

// Kernel labels of the per-kernel profiler (CUDA events around each launch, aggregated per
// label), the counterpart of the reference's per-pass timestamp queries
// (src/engine.ts:3208-3285).
enum g4a_prof_label : int {
  G4A_PROF_NORM_ROPE = 0,
  G4A_PROF_RMS_NORM,
  G4A_PROF_KV_STORE,
  G4A_PROF_DECODE_PREP,
  G4A_PROF_DECODE_SPLITKV,
  G4A_PROF_DECODE_MERGE,
  G4A_PROF_DECODE_GENERIC,
  G4A_PROF_LSE_MERGE,
  G4A_PROF_PREFILL_PREP,
  G4A_PROF_PREFILL_ATTN,
  G4A_PROF_MATMUL,
  G4A_PROF_NUM_LABELS
};
extern const char* const g4a_prof_names[G4A_PROF_NUM_LABELS];

struct g4a_prof_rec {
  int label;
  cudaEvent_t begin, end;
};

// ----------------------------------------------------------------------------- host side

struct g4a_ctx {
  int device = 0;
  int num_sms = 148;
  size_t smem_optin = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  // Split-KV partials: [segments] x (m[8] | l[8] | o[8][hd]) f32, plus per-problem segment
  // ranges.  Grown on demand by the decode entry points (or once by g4a_reserve_workspace).
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  // Per-token kv lengths of a prefill that runs through the decode kernels (grown on demand).
  int* seq_lens = nullptr;
  size_t seq_lens_cap = 0;
  // Device-written error word in mapped pinned host memory: kernels whose bounded waits give
  // up (or that skip an invalid page id) store a nonzero code here; g4a_sync reports and
  // clears it.
  volatile int* dev_err_host = nullptr;
  int* dev_err_dev = nullptr;
  cudaEvent_t sync_event = nullptr;
  // Tensor-map encoder from the driver (for the prefill kernel), resolved on first use.
  void* encode_tiled = nullptr;
  // NCCL communicator of g4a_dist_init (an ncclComm_t), its rank and size; dist_aborted is set
  // when a deadline or an asynchronous error aborted it.
  void* nccl_comm = nullptr;
  int dist_rank = -1;
  int dist_nranks = 0;
  bool dist_aborted = false;
  // Profiler state: pending event pairs, free events, per-label totals.
  bool prof_enabled = false;
  std::vector<g4a_prof_rec> prof_pending;
  std::vector<cudaEvent_t> prof_free;
  double prof_ms[G4A_PROF_NUM_LABELS] = {};
  uint64_t prof_count[G4A_PROF_NUM_LABELS] = {};
};

// Record a begin/end event pair around a launch when profiling is on (no-op otherwise).
struct g4a_prof_scope {
  g4a_ctx* ctx;
  int label;
  cudaEvent_t end = nullptr;
  g4a_prof_scope(g4a_ctx* c, int l);
  ~g4a_prof_scope();
};

// Per-thread last-error message (set by every failing entry point).
void g4a_set_error(const char* fmt, ...);
g4a_status g4a_fail(g4a_status st, const char* fmt, ...);
g4a_status g4a_cuda_fail(cudaError_t e, const char* what);
g4a_status g4a_check_launch(const char* what);
g4a_status g4a_ensure_workspace(g4a_ctx* ctx, size_t bytes);
// Communicator checks of g4a_sync (g4a_dist.cu): an asynchronous NCCL error, or the deadline
// passing while a communicator exists, aborts the communicator and returns the error.
g4a_status g4a_dist_check(g4a_ctx* ctx, bool deadline_passed, uint32_t timeout_ms);
void g4a_dist_release(g4a_ctx* ctx);
// Prefill through the decode kernels (shapes the tensor-core prefill kernel does not cover).
g4a_status prefill_via_decode(g4a_ctx* ctx, const uint16_t* q16, const uint16_t* k, const uint16_t* v, float* out,
                              uint32_t T, uint32_t start_pos, uint32_t nqh, uint32_t nkh, uint32_t hd, float scale,
                              uint32_t window);

#define G4A_CHECK_CTX(ctx)                                                           \
  do {                                                                               \
    if ((ctx) == nullptr) return g4a_fail(G4A_EINVAL, "%s: null context", __func__); \
  } while (0)

#define G4A_CUDA_TRY(expr)                                  \
  do {                                                      \
    cudaError_t _e = (expr);                                \
    if (_e != cudaSuccess) return g4a_cuda_fail(_e, #expr); \
  } while (0)

// Device error codes written to g4a_ctx::dev_err_*.
enum : int {
  G4A_DEVERR_NONE = 0,
  G4A_DEVERR_WAIT_FULL = 1,   // consumer gave up waiting for a TMA stage
  G4A_DEVERR_WAIT_EMPTY = 2,  // producer gave up waiting for a free stage
  G4A_DEVERR_WAIT_MMA = 3,    // tensor-core completion wait gave up
  G4A_DEVERR_TMEM = 4,        // TMEM allocation failed / inconsistent
  G4A_DEVERR_WAIT_PEER = 5,   // a peer's exchange flag did not arrive in time
  G4A_DEVERR_KVLEN = 16,      // kv_lens[b] exceeded the page table's capacity (capped)
  G4A_DEVERR_PAGE = 17,       // page id out of [0, num_pages) (row skipped)
};

// ----------------------------------------------------------------------------- device side

#ifdef __CUDACC__

namespace g4a {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// mbarrier primitives (shared::cta).
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: spins on try_wait (which itself suspends for a hardware-defined window) and
// gives up after `limit_ns` of wall time, recording `code` in the device error word.  Returns
// true when the phase completed.  Every wait in this library goes through here so that no
// kernel can spin forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err, int code,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0u) {
      if (globaltimer_ns() - t0 > limit_ns) {
        if (err) atomicExch(err, code);
        return false;
      }
    }
  }
}

// Plain (non-multicast) bulk copy global -> shared memory completing on an mbarrier, with an
// L2 eviction-priority hint.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Named barrier among `count` threads (multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Programmatic dependent launch controls (no-ops when the launch has no PDL attribute).
__device__ __forceinline__ void pdl_wait_primary() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t packed) {
  __half2 h = *reinterpret_cast<__half2*>(&packed);
  return __half22float2(h);
}

// 2^x on the MUFU unit (relative error ~2 ulp); flushes subnormal results to zero.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace g4a

// Launch helper shared by the entry points: optional programmatic-dependent-launch attribute.
template <typename Kernel, typename... Args>
static inline cudaError_t g4a_launch(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                     bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

#endif  // __CUDACC__
