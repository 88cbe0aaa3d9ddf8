// Multi-GPU split-KV exchange over NVLink peer memory (no counterpart in the reference, which
// runs on one WebGPU device).
//
// A long sequence is split along its KV length over `world` GPUs; each rank computes the
// partial (m | l | o) of its slice (g4a_decode_attn_partial).  Instead of an all-gather followed
// by a merge, one kernel per step does both: it stores this rank's partial straight into slot
// `rank` of every rank's exchange buffer through NVLink (plain P2P stores to a peer's memory
// opened with CUDA IPC), then raises that slot's flag in every buffer with a release store of
// the step number, waits (bounded) until all `world` flags of its own buffer carry the step
// number, and merges the `world` partials of its own buffer into the output.
//
// Exchange buffer of a rank (allocated by the caller, zeroed once):
//   [2 parities][world slots][ps] f32 partials (ps = nqh * (hd + 2) rounded up to a multiple of 4),
//   then [2 parities][world] u32 flags.
// Step s uses parity s & 1.  A rank can be at most one step ahead of another (it cannot finish
// step s without every rank's step-s flag), so by the time it writes parity (s+1) & 1 again,
// every rank has finished merging step s-1 from it.
#include <string.h>

#include "g4a_internal.cuh"

namespace {

constexpr int kMaxWorld = 8;

struct PeerBufs {
  float* buf[kMaxWorld];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid = num_q_heads CTAs of 256 threads.  CTA b pushes this rank's partial to ranks b, b + nqh,
// ...; every CTA then waits for all flags and merges head b.
// (`peers` stays in parameter space: __grid_constant__ lets peers.buf[dst] index it directly.)
__global__ void __launch_bounds__(256) exchange_merge_kernel(const float* part, const __grid_constant__ PeerBufs peers,
                                                             int world, int rank, uint32_t seq, int nqh, int hd,
                                                             float* out, int* err) {
  const int tid = threadIdx.x;
  const int pf = nqh * (hd + 2);  // floats per partial
  const int ps = (pf + 3) & ~3;   // slot stride (16-byte aligned slots)
  const int par = (int)(seq & 1u);
  const size_t slots_floats = (size_t)2 * world * ps;
  g4a::pdl_wait_primary();  // the partial is written by the preceding kernel
  // ---- push: slot `rank` of parity `par` in every destination's buffer
  for (int dst = blockIdx.x; dst < world; dst += gridDim.x) {
    float* slot = peers.buf[dst] + ((size_t)par * world + rank) * ps;
    for (int i = tid; i < pf / 4; i += blockDim.x)
      reinterpret_cast<float4*>(slot)[i] = __ldcg(reinterpret_cast<const float4*>(part) + i);
    for (int i = (pf & ~3) + tid; i < pf; i += blockDim.x) slot[i] = __ldcg(part + i);
    // The CTA barrier orders every thread's stores before thread 0's system-scope fence, which
    // makes them visible to the destination GPU before the release store of the flag.
    __syncthreads();
    if (tid == 0) {
      uint32_t* flags = reinterpret_cast<uint32_t*>(peers.buf[dst] + slots_floats);
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      st_release_sys(flags + par * world + rank, seq);
    }
  }
  // ---- wait for every rank's slot in this rank's own buffer (bounded).  Lane j of warp 0 polls
  // the flag of rank j, so the world acquire loads are in flight together rather than one after
  // another (each is a system-scope round trip); the CTA barrier then orders every lane's
  // acquire before the other threads' reads of the slots.
  __shared__ int ok;
  if (tid < 32) {
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(peers.buf[rank] + slots_floats) + par * world;
    bool good = true;
    if (tid < world) {
      const uint64_t t0 = g4a::globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_sys(flags + tid) != seq) {
        if ((++spins & 1023u) == 0u && g4a::globaltimer_ns() - t0 > 2000000000ull) {
          good = false;
          if (err) atomicExch(err, G4A_DEVERR_WAIT_PEER);
          break;
        }
      }
    }
    const bool all_good = __all_sync(0xffffffffu, good);
    if (tid == 0) ok = all_good ? 1 : 0;
    __threadfence();
  }
  __syncthreads();
  // ---- merge head h = blockIdx.x of the world partials (read through L2: peers wrote them)
  const int h = blockIdx.x;
  if (h >= nqh) return;
  const float* base = peers.buf[rank] + (size_t)par * world * ps;
  if (!ok) {
    for (int d = tid; d < hd; d += blockDim.x) out[(size_t)h * hd + d] = 0.f;
    return;
  }
  // every rank's (m, l) of head h loaded before any is used: one round trip, not one per rank
  float mv[kMaxWorld], lv[kMaxWorld];
#pragma unroll
  for (int r = 0; r < kMaxWorld; r++) {
    mv[r] = (r < world) ? __ldcg(base + (size_t)r * ps + h) : -INFINITY;
    lv[r] = (r < world) ? __ldcg(base + (size_t)r * ps + nqh + h) : 0.f;
  }
  float M = -INFINITY;
#pragma unroll
  for (int r = 0; r < kMaxWorld; r++) M = fmaxf(M, mv[r]);
  float L = 0.f;
  float w[kMaxWorld];
#pragma unroll
  for (int r = 0; r < kMaxWorld; r++) {
    w[r] = (r < world && mv[r] != -INFINITY) ? exp2f(mv[r] - M) : 0.f;
    L += w[r] * lv[r];
  }
  const float inv = (L > 0.f) ? 1.0f / L : 0.f;
  for (int d = tid; d < hd; d += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxWorld; r++)
      if (r < world && w[r] != 0.f) acc += w[r] * __ldcg(base + (size_t)r * ps + 2 * nqh + (size_t)h * hd + d);
    out[(size_t)h * hd + d] = acc * inv;
  }
}

}  // namespace

extern "C" {

g4a_status g4a_ipc_get_handle(g4a_ctx* ctx, void* dptr, uint8_t* out_handle) {
  G4A_CHECK_CTX(ctx);
  if (!dptr || !out_handle) return g4a_fail(G4A_EINVAL, "g4a_ipc_get_handle: null pointer");
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  G4A_CUDA_TRY(cudaIpcGetMemHandle(&h, dptr));
  static_assert(sizeof(h) == G4A_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(out_handle, &h, sizeof(h));
  return G4A_OK;
}

g4a_status g4a_ipc_open_handle(g4a_ctx* ctx, const uint8_t* handle, void** out_dptr) {
  G4A_CHECK_CTX(ctx);
  if (!handle || !out_dptr) return g4a_fail(G4A_EINVAL, "g4a_ipc_open_handle: null pointer");
  *out_dptr = nullptr;
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  G4A_CUDA_TRY(cudaIpcOpenMemHandle(out_dptr, h, cudaIpcMemLazyEnablePeerAccess));
  return G4A_OK;
}

g4a_status g4a_ipc_close_handle(g4a_ctx* ctx, void* dptr) {
  G4A_CHECK_CTX(ctx);
  if (!dptr) return G4A_OK;
  G4A_CUDA_TRY(cudaSetDevice(ctx->device));
  G4A_CUDA_TRY(cudaIpcCloseMemHandle(dptr));
  return G4A_OK;
}

size_t g4a_exchange_buffer_bytes(uint32_t world, uint32_t num_q_heads, uint32_t head_dim) {
  const size_t ps = ((size_t)num_q_heads * (head_dim + 2) + 3) & ~size_t(3);
  return 2 * (size_t)world * ps * sizeof(float) + 2 * (size_t)world * sizeof(uint32_t);
}

g4a_status g4a_splitkv_exchange_merge(g4a_ctx* ctx, const float* part, void* const* rank_buffers, uint32_t world,
                                      uint32_t rank, uint32_t seq, uint32_t num_q_heads, uint32_t head_dim,
                                      float* out) {
  G4A_CHECK_CTX(ctx);
  if (!part || !rank_buffers || !out) return g4a_fail(G4A_EINVAL, "g4a_splitkv_exchange_merge: null pointer");
  if (world < 1 || world > (uint32_t)kMaxWorld || rank >= world)
    return g4a_fail(G4A_EINVAL, "g4a_splitkv_exchange_merge: world %u / rank %u (1 <= world <= %d)", world, rank,
                    kMaxWorld);
  if (seq == 0) return g4a_fail(G4A_EINVAL, "g4a_splitkv_exchange_merge: seq must be >= 1 (flags start at 0)");
  if (num_q_heads == 0 || head_dim == 0 || (head_dim % 8) != 0)
    return g4a_fail(G4A_EINVAL, "g4a_splitkv_exchange_merge: num_q_heads > 0 and head_dim a multiple of 8");
  if (((uintptr_t)part & 15u) != 0) return g4a_fail(G4A_EINVAL, "g4a_splitkv_exchange_merge: part not 16-byte aligned");
  PeerBufs pb = {};
  for (uint32_t r = 0; r < world; r++) {
    if (!rank_buffers[r] || ((uintptr_t)rank_buffers[r] & 15u) != 0)
      return g4a_fail(G4A_EINVAL, "g4a_splitkv_exchange_merge: buffer of rank %u null or not 16-byte aligned", r);
    pb.buf[r] = static_cast<float*>(rank_buffers[r]);
  }
  g4a_prof_scope ps(ctx, G4A_PROF_LSE_MERGE);
  cudaError_t e = g4a_launch(exchange_merge_kernel, dim3(num_q_heads), dim3(256), 0, ctx->stream, true, part, pb,
                             (int)world, (int)rank, seq, (int)num_q_heads, (int)head_dim, out, ctx->dev_err_dev);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "launch exchange_merge_kernel");
  return G4A_OK;
}

}  // extern "C"
