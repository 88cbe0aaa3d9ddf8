/*
 * g4attn.h -- C ABI of libg4attn.so, the B200 (sm_100a) attention hot path of gemma4-webgpu.
 *
 * Drop-in boundary.  The reference issues six WebGPU dispatches per transformer layer for
 * attention (src/engine.ts:2061-2094): v_norm, q/k norm+RoPE, KV-cache store, attention score,
 * softmax and attention output.  Each is a WGSL compute shader whose "operator API" is its
 * bind-group layout plus a `Params` uniform struct.  Every entry point below names the
 * dispatch and the Params struct it replaces; argument names and meanings follow those
 * structs one for one, so a TypeScript backend can forward the same uniforms it writes today
 * (src/engine.ts:548-590 and the per-token writes at :1971-1987).
 *
 * Conventions.
 *   - Every function returns g4a_status and never throws or aborts.  A failing call stores a
 *     message readable with g4a_last_error() (thread-local, valid until the next failing call
 *     on the same thread).  This replaces the reference's "throw if deviceLost"
 *     (src/engine.ts:2214, 2509, 2754).
 *   - Device pointers are plain CUDA device addresses (from g4a_alloc or any allocator on the
 *     same device).  f16 data is passed as uint16_t (IEEE binary16 bit patterns).
 *   - Kernel calls are asynchronous on the context's stream and return once enqueued.  Device
 *     faults surface at g4a_sync or at the next call.  g4a_sync never blocks forever.
 *   - Calls on one context must be serialised by the caller (like one GPUQueue).
 *
 * Data layout in device memory.
 *   q, k, v work buffers : f32, [num_heads, head_dim] per token (src/engine.ts:1369-1372).
 *   KV cache (contiguous): f16, [max_seq_len, num_kv_heads, head_dim]; row `slot` holds one
 *                          token (reference: f32, src/engine.ts:1415-1425).
 *   KV cache (paged)     : f16 page pool [num_pages, page_size, num_kv_heads, head_dim] plus an
 *                          int32 page table [batch, max_pages_per_seq].
 *   attention output     : f32, [num_q_heads, head_dim] (src/engine.ts:1372 `attnOut`).
 */
#ifndef G4ATTN_H_
#define G4ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; every declaration below is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef enum {
  G4A_OK = 0,
  G4A_EINVAL = 1,       /* bad argument (null pointer, unsupported shape, size out of range) */
  G4A_ECUDA = 2,        /* CUDA runtime / launch / device error */
  G4A_ENOMEM = 3,       /* device allocation failed */
  G4A_ETIMEOUT = 4,     /* g4a_sync deadline passed, or a kernel's bounded wait gave up */
  G4A_ENCCL = 5,        /* a collective failed (NCCL error; the communicator was aborted) */
  G4A_EUNSUPPORTED = 6  /* valid request that this build does not implement */
} g4a_status;

typedef struct g4a_ctx g4a_ctx;

/* ------------------------------------------------------------------ context, memory, sync */

/* Create a context on CUDA device `device` with its own non-blocking stream.
 * Replaces initWebGPU/createPipelines (src/engine.ts:402-457). */
g4a_status g4a_create(int device, g4a_ctx** out_ctx);
g4a_status g4a_destroy(g4a_ctx* ctx);

/* Message of the last failing call on this thread ("" if none). */
const char* g4a_last_error(void);

/* Library version string, e.g. "g4attn 0.1.0 sm_100a". */
const char* g4a_version(void);

/* Run subsequent calls on a caller-owned cudaStream_t (0 = the legacy default stream), or
 * back on the context's own non-blocking stream. */
g4a_status g4a_set_stream(g4a_ctx* ctx, void* cuda_stream);
g4a_status g4a_use_own_stream(g4a_ctx* ctx);
void* g4a_get_stream(g4a_ctx* ctx);

/* Wait for all work on the context's stream, at most timeout_ms milliseconds (0 = poll once).
 * Returns G4A_ETIMEOUT if the work is still running at the deadline (the work is not
 * cancelled), G4A_ECUDA on an asynchronous device error, and G4A_ETIMEOUT also when a kernel
 * reported that one of its bounded waits gave up or it skipped an invalid page id.  Mirrors
 * queue.onSubmittedWorkDone (src/engine.ts:2474) with a deadline. */
g4a_status g4a_sync(g4a_ctx* ctx, uint32_t timeout_ms);

/* Device memory owned by the caller (the TS side holds no GPUBuffer any more). */
g4a_status g4a_alloc(g4a_ctx* ctx, size_t bytes, void** out_dptr);
g4a_status g4a_free(g4a_ctx* ctx, void* dptr);
/* Asynchronous copies on the context's stream (host memory should be pinned for overlap). */
g4a_status g4a_memcpy_h2d(g4a_ctx* ctx, void* dst_device, const void* src_host, size_t bytes);
g4a_status g4a_memcpy_d2h(g4a_ctx* ctx, void* dst_host, const void* src_device, size_t bytes);
g4a_status g4a_memset(g4a_ctx* ctx, void* dst_device, int value, size_t bytes);

/* Pre-size the split-KV partials workspace for up to `max_batch` sequences, so that later
 * decode calls allocate nothing (needed before capturing them into a CUDA graph). */
g4a_status g4a_reserve_workspace(g4a_ctx* ctx, uint32_t max_batch, uint32_t head_dim,
                                 uint32_t num_q_heads);

/* Per-kernel profiler: when enabled, every kernel launch is bracketed by CUDA events and its
 * device time is summed per label ("norm_rope", "rms_norm_no_weight", "kv_store",
 * "decode_prep", "decode_splitkv", "decode_merge", "decode_generic", "lse_merge",
 * "prefill_prep", "prefill_attn", "matmul").  Counterpart of the reference's per-pass timestamp
 * queries (src/engine.ts:3208-3285, src/diagnostics/profile.ts:48-132).  Reading waits for
 * the context's stream.  Leave it off for timing whole steps: the events serialise launches. */
g4a_status g4a_profile_enable(g4a_ctx* ctx, int enable);
g4a_status g4a_profile_reset(g4a_ctx* ctx);
g4a_status g4a_profile_read(g4a_ctx* ctx, const char* label, double* total_ms, uint64_t* count);

/* ------------------------------------------------------------------ producers */

/* Per-head RMSNorm with an f16 weight, then NeoX half-split RoPE, in place on x
 * [num_heads, head_dim] f32.  Replaces shaders/fused_per_head_norm_rope.wgsl dispatched at
 * src/engine.ts:2078-2084 with Params {num_heads, head_dim, eps, position, theta,
 * apply_divisor} (src/engine.ts:583-588).  rope_freqs is the f16 divisor table read only when
 * apply_divisor != 0 (global Gemma layers, src/engine.ts:571-576); it may be NULL otherwise.
 * head_dim must be even and <= 1024.  Bit-exact against the reference arithmetic. */
g4a_status g4a_norm_rope(g4a_ctx* ctx, float* x, const uint16_t* weight, const uint16_t* rope_freqs,
                         uint32_t num_heads, uint32_t head_dim, float eps, uint32_t position,
                         float theta, uint32_t apply_divisor);

/* Weightless per-head RMSNorm in place (Gemma v_norm).  Replaces
 * shaders/per_head_rms_norm_no_weight.wgsl dispatched at src/engine.ts:2061-2066 with Params
 * {num_heads, head_dim, eps, pad}. */
g4a_status g4a_rms_norm_no_weight(g4a_ctx* ctx, float* x, uint32_t num_heads, uint32_t head_dim,
                                  float eps);

/* KV-cache store of one token into the f16 cache at row `slot`, with the weightless v_norm
 * fused in when fuse_v_norm != 0 (v is then also normalised in place, as the reference's
 * separate v_norm dispatch leaves it).  Replaces shaders/kv_cache_store.wgsl dispatched at
 * src/engine.ts:2089-2091 with Params {num_kv_heads, head_dim, position(=slot), max_seq_len}
 * (src/engine.ts:548-550, slot written at :1979) plus the v_norm dispatch above.
 * slot must be < max_seq_len. */
g4a_status g4a_kv_store(g4a_ctx* ctx, const float* k, float* v, uint16_t* k_cache,
                        uint16_t* v_cache, uint32_t num_kv_heads, uint32_t head_dim,
                        uint32_t slot, uint32_t max_seq_len, float eps, uint32_t fuse_v_norm);

/* ------------------------------------------------------------------ decode attention */

/* Decode attention of one token over a contiguous f16 cache: the attn_score -> softmax ->
 * attn_output chain (shaders/attn_score.wgsl, softmax.wgsl, attn_output.wgsl dispatched at
 * src/engine.ts:2092-2094, Params {num_q_heads, num_kv_heads, head_dim, seq_len, scale,
 * sliding_window} at :562-566 with seq_len = kv_len written at :1980) as one split-KV
 * flash-decode kernel plus a log-sum-exp merge.  Keys [max(0, kv_len - sliding_window),
 * kv_len) are attended (sliding_window 0 = all); kv head of q head h is
 * h*num_kv_heads/num_q_heads.  out is f32 [num_q_heads, head_dim]; kv_len 0 gives zeros.
 * head_dim must be a multiple of 8 and <= 512. */
g4a_status g4a_decode_attn(g4a_ctx* ctx, const float* q, const uint16_t* k_cache,
                           const uint16_t* v_cache, float* out, uint32_t num_q_heads,
                           uint32_t num_kv_heads, uint32_t head_dim, uint32_t kv_len, float scale,
                           uint32_t sliding_window);

/* g4a_decode_attn without any memory allocation (no counterpart in the reference).  For
 * callers that cannot call cudaMalloc while decoding: an engine that sizes every device buffer
 * once at load time and owns all device memory from then on (the reference engine creates all
 * of its work buffers when the model loads), or a process held to a fixed device-memory budget
 * where an allocation in the middle of generation may fail or stall the device.  Same arguments,
 * semantics and results as g4a_decode_attn; its split-KV scratch is a fixed 4 MiB
 * statically allocated device area instead of the context's workspace, which g4a_decode_attn
 * grows with cudaMalloc.  The area fits every shape with num_kv_heads <= 64 and head_dim <= 512
 * on a 148-SM B200; a shape that needs more is rejected with G4A_EINVAL and a message giving
 * the bytes needed, and nothing is launched.  Nothing in the area has to start at zero.  The
 * first call on each device looks up the area's address (cudaGetSymbolAddress): make that
 * first call before any stream capture.  Calls that overlap in time on the same device (other
 * streams, other contexts, other host threads) share the one area and race: serialise them.
 * Fails with G4A_EINVAL while the context's profiler is enabled (it creates events). */
g4a_status g4a_decode_attn_noalloc(g4a_ctx* ctx, const float* q, const uint16_t* k_cache,
                                   const uint16_t* v_cache, float* out, uint32_t num_q_heads,
                                   uint32_t num_kv_heads, uint32_t head_dim, uint32_t kv_len,
                                   float scale, uint32_t sliding_window);

/* Batched decode over a paged f16 cache (no reference counterpart: the reference decodes
 * one sequence, src/types.ts:636-639).  q is [batch, num_q_heads, head_dim] f32; sequence b
 * has kv_lens[b] tokens whose rows live at page page_table[b*max_pages_per_seq + t/page_size],
 * row t%page_size.  out is [batch, num_q_heads, head_dim] f32.  kv_lens and page_table are
 * device arrays; host_kv_lens (may be NULL) is an optional host copy used only to size the
 * launch; with NULL the launch is sized from batch*max_pages_per_seq*page_size.  Page ids
 * outside [0, num_pages) are not read: the row is skipped and g4a_sync reports the error.
 * kv_lens[b] is capped at max_pages_per_seq*page_size the same way. */
g4a_status g4a_decode_attn_paged(g4a_ctx* ctx, const float* q, const uint16_t* k_pages,
                                 const uint16_t* v_pages, const int32_t* page_table,
                                 const int32_t* kv_lens, const int32_t* host_kv_lens,
                                 uint32_t batch, uint32_t page_size, uint32_t max_pages_per_seq,
                                 uint32_t num_pages, uint32_t num_q_heads, uint32_t num_kv_heads,
                                 uint32_t head_dim, float scale, uint32_t sliding_window,
                                 float* out);

/* Split-KV partial for multi-GPU long-context decode (no reference counterpart).  The caller's
 * k_cache/v_cache hold positions [kv_begin, kv_end) of a kv_len_total-long sequence (row 0 of
 * the buffers is position kv_begin).  The sliding window is measured from kv_len_total.
 * `part` receives num_q_heads*(head_dim+2) floats laid out as
 *   m[num_q_heads] | l[num_q_heads] | o[num_q_heads, head_dim]
 * with m the running max of score*scale*log2(e) (base-2 domain), l = sum 2^(s - m) and o the
 * un-normalised sum 2^(s - m) * v.  A part with no visible key has m = -inf, l = 0, o = 0. */
g4a_status g4a_decode_attn_partial(g4a_ctx* ctx, const float* q, const uint16_t* k_cache,
                                   const uint16_t* v_cache, uint32_t num_q_heads,
                                   uint32_t num_kv_heads, uint32_t head_dim, uint32_t kv_begin,
                                   uint32_t kv_end, uint32_t kv_len_total, float scale,
                                   uint32_t sliding_window, float* part);

/* Log-sum-exp merge of n_parts partials laid out back to back as produced by
 * g4a_decode_attn_partial (e.g. after an all-gather): out[h,d] = sum_r 2^(m_r - M) o_r[h,d] /
 * sum_r 2^(m_r - M) l_r with M = max_r m_r.  All parts empty gives zeros. */
g4a_status g4a_lse_merge(g4a_ctx* ctx, const float* parts, uint32_t n_parts,
                         uint32_t num_q_heads, uint32_t head_dim, float* out);

/* One producer (or consumer) layer's whole decode attention block: q norm+RoPE, k norm+RoPE +
 * v_norm + store at `slot` (only when is_producer != 0) in one launch, then attention over
 * kv_len keys.  Same semantics as the individual calls above chained in the reference's order
 * (src/engine.ts:2061-2094).  q/k/v are modified in place like the reference's work buffers. */
g4a_status g4a_attn_decode_layer(g4a_ctx* ctx, float* q, float* k, float* v,
                                 const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                 const uint16_t* rope_freqs, uint16_t* k_cache,
                                 uint16_t* v_cache, float* out, uint32_t num_q_heads,
                                 uint32_t num_kv_heads, uint32_t head_dim, float eps,
                                 uint32_t position, uint32_t slot, uint32_t kv_len,
                                 uint32_t max_seq_len, float theta, uint32_t apply_divisor,
                                 float scale, uint32_t sliding_window, uint32_t is_producer);

/* g4a_attn_decode_layer with its token's inputs and its output in host memory, for a caller
 * whose q / k / v come from the host (no counterpart in the reference, where they are produced
 * on the GPU): in one call, copies q | k | v (packed f32: num_q_heads*head_dim, then
 * num_kv_heads*head_dim twice; only q for a consumer layer) from qkv_host to the device work
 * buffer qkv_dev, runs the layer on it (q, k and v are then modified in place in qkv_dev), and
 * copies the output [num_q_heads, head_dim] from out_dev back to out_host.  Everything is
 * enqueued on the context's stream; out_host holds the result after g4a_sync, and qkv_host must
 * keep its contents until then.  When both host buffers are pinned (page-locked) memory the
 * device can address, 16-byte aligned, there are no copies: the producer kernel reads q | k | v
 * from host memory and the attention writes the output into host memory (out_dev is then not
 * used).  Otherwise the two copies are ordinary asynchronous copies (synchronous for pageable
 * memory). */
g4a_status g4a_attn_decode_layer_io(g4a_ctx* ctx, const float* qkv_host, float* qkv_dev, float* out_dev,
                                    float* out_host, const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                    const uint16_t* rope_freqs, uint16_t* k_cache, uint16_t* v_cache,
                                    uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim, float eps,
                                    uint32_t position, uint32_t slot, uint32_t kv_len, uint32_t max_seq_len,
                                    float theta, uint32_t apply_divisor, float scale, uint32_t sliding_window,
                                    uint32_t is_producer);

/* ------------------------------------------------------------------ prefill */

/* Prefill input stage for T tokens at positions start_pos..start_pos+T-1 (the reference runs
 * T single-token forwards, src/engine.ts:2460-2479, each doing the producers above).  In one
 * launch: q rows get norm+RoPE and are written as f16 to q16_out [T, num_q_heads, head_dim];
 * k rows get norm+RoPE, v rows the weightless v_norm, and both are stored as f16 into the
 * cache rows start_pos+i (cache slot = position).  q, k, v are f32 [T, heads, head_dim] and are
 * left unmodified.  start_pos + T must be <= max_seq_len; head_dim a multiple of 64, <= 512. */
g4a_status g4a_prefill_qkv_prep(g4a_ctx* ctx, const float* q, const float* k, const float* v,
                                const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                const uint16_t* rope_freqs, uint16_t* q16_out,
                                uint16_t* k_cache, uint16_t* v_cache, uint32_t T,
                                uint32_t start_pos, uint32_t max_seq_len, uint32_t num_q_heads,
                                uint32_t num_kv_heads, uint32_t head_dim, float eps, float theta,
                                uint32_t apply_divisor);

/* Causal (sliding_window 0) or sliding-window prefill attention on the tensor cores
 * (tcgen05.mma, TMEM accumulators, TMA tile loads).  q16 is f16 [T, num_q_heads, head_dim];
 * the cache already holds rows 0 .. start_pos+T-1.  Row i attends to cache positions
 * [max(0, start_pos+i+1-W), start_pos+i] -- exactly decode at kv_len = start_pos+i+1, which is
 * what the reference's token-by-token prefill computes.  out is f32 [T, num_q_heads,
 * head_dim].  num_q_heads/num_kv_heads = 8 at head_dim 128, 256 or 512 runs on the tcgen05
 * tensor cores (at head_dim 512, Gemma's global layers, each tile on a 2-CTA cluster that splits
 * the head dims); every other shape (head_dim a multiple of 8 up to 512, any num_kv_heads <= num_q_heads)
 * runs through the decode kernels, one decode problem per prompt token, with the same results
 * and several times the run time.  All pointers 16-byte aligned. */
g4a_status g4a_prefill_attn(g4a_ctx* ctx, const uint16_t* q16, const uint16_t* k_cache,
                            const uint16_t* v_cache, float* out, uint32_t T, uint32_t start_pos,
                            uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim,
                            float scale, uint32_t sliding_window);

/* ------------------------------------------------------------------ multi-GPU exchange */

/* Split-KV decode over several GPUs with the partial exchange done over NVLink peer memory
 * instead of a collective library call (no reference counterpart: the reference runs on one
 * WebGPU device).  One process per GPU.  Each rank allocates one exchange buffer of
 * g4a_exchange_buffer_bytes(world, num_q_heads, head_dim) bytes with g4a_alloc, zeroes it once
 * with g4a_memset, exports it with g4a_ipc_get_handle, sends the handle to every other rank
 * (g4a_dist_allgather_host below, or any other channel), and opens the others' handles with
 * g4a_ipc_open_handle.
 * Every step, every rank calls g4a_splitkv_exchange_merge with the same `seq` (1, 2, 3, ...):
 * it stores this rank's partial (the m | l | o layout of g4a_decode_attn_partial) into slot
 * `rank` of every rank's buffer, raises its flag there, waits until every rank's partial of
 * this step is in its own buffer (2 s bound; then the output is zeroed and g4a_sync reports
 * the error), and writes the merged attention output [num_q_heads, head_dim] to `out`.
 * rank_buffers is a host array of `world` device pointers: this rank's own buffer at index
 * `rank`, the opened peer buffers elsewhere.  1 <= world <= 8.  Before freeing a buffer, make
 * sure no rank will write to it again (e.g. a barrier after the last step). */
#define G4A_IPC_HANDLE_BYTES 64
size_t g4a_exchange_buffer_bytes(uint32_t world, uint32_t num_q_heads, uint32_t head_dim);
g4a_status g4a_ipc_get_handle(g4a_ctx* ctx, void* dptr, uint8_t* out_handle);
g4a_status g4a_ipc_open_handle(g4a_ctx* ctx, const uint8_t* handle, void** out_dptr);
g4a_status g4a_ipc_close_handle(g4a_ctx* ctx, void* dptr);
g4a_status g4a_splitkv_exchange_merge(g4a_ctx* ctx, const float* part, void* const* rank_buffers,
                                      uint32_t world, uint32_t rank, uint32_t seq,
                                      uint32_t num_q_heads, uint32_t head_dim, float* out);

/* ------------------------------------------------------------------ multi-GPU over NCCL */

/* Split-KV decode of one long context over N GPUs through this ABI alone (no PyTorch): one
 * process and one context per GPU, an NCCL communicator per context.  The reference decodes one
 * sequence on one WebGPU device and has no collective; its failure handling -- a lost device
 * turns into an error at the next call (src/engine.ts:432-435, 2214, 2509) -- is what the
 * deadlines below mirror.  NCCL (libnccl.so.2) is loaded when first needed; without it these
 * calls return G4A_EUNSUPPORTED.
 *
 * g4a_dist_unique_id: rank 0 creates the 128-byte id and sends it to every rank out of band.
 * g4a_dist_init: creates the context's communicator (ncclCommInitRankConfig, non-blocking) and
 *   waits for all ranks to join; if they have not after timeout_ms, or NCCL reports an error,
 *   the communicator is aborted and G4A_ETIMEOUT / G4A_ENCCL returned.
 * g4a_allgather_partials: enqueues ncclAllGather of floats_per_rank floats from `part` into
 *   parts_all [nranks * floats_per_rank] on the context's stream (part may be the rank's own
 *   slot of parts_all).  Completion is observed by g4a_sync, which also watches the communicator:
 *   an asynchronous NCCL error, or the sync deadline passing with the collective still pending
 *   (a rank that never joined), aborts the communicator -- its kernels stop -- and returns
 *   G4A_ENCCL / G4A_ETIMEOUT.  After an abort, dist calls fail until g4a_dist_init is called again.
 * g4a_decode_attn_splitkv: the whole step on this rank -- g4a_decode_attn_partial over its slice
 *   (k_slice / v_slice hold positions [kv_begin, kv_end) of a kv_len_total-long cache), the
 *   all-gather into parts_all (device, nranks * num_q_heads * (head_dim + 2) floats) and
 *   g4a_lse_merge into out [num_q_heads, head_dim].  One kv head per call.
 * g4a_dist_allgather_host: a synchronous all-gather of `bytes` host bytes from every rank into
 *   recv [nranks * bytes] (bootstrap of the peer-exchange IPC handles without another channel).
 * g4a_dist_destroy: releases the communicator (also done by g4a_destroy).
 * g4a_dist_poll_selftest: runs the deadline logic of these calls against a built-in fake of NCCL
 *   -- scenario 0: the operation completes on the third poll, 1: a rank never joins, 2: a peer
 *   fails -- without a GPU or NCCL; *aborted = 1 when the fake communicator was aborted once. */
#define G4A_DIST_ID_BYTES 128
g4a_status g4a_dist_unique_id(void* id_out);
g4a_status g4a_dist_init(g4a_ctx* ctx, int rank, int nranks, const void* id, uint32_t timeout_ms);
g4a_status g4a_dist_destroy(g4a_ctx* ctx);
g4a_status g4a_dist_info(g4a_ctx* ctx, int* rank, int* nranks);
g4a_status g4a_allgather_partials(g4a_ctx* ctx, const float* part, float* parts_all, size_t floats_per_rank,
                                  uint32_t timeout_ms);
g4a_status g4a_decode_attn_splitkv(g4a_ctx* ctx, const float* q, const uint16_t* k_slice, const uint16_t* v_slice,
                                   uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim, uint32_t kv_begin,
                                   uint32_t kv_end, uint32_t kv_len_total, float scale, uint32_t sliding_window,
                                   float* parts_all, float* out, uint32_t timeout_ms);
g4a_status g4a_dist_allgather_host(g4a_ctx* ctx, const void* send, void* recv, size_t bytes, uint32_t timeout_ms);
g4a_status g4a_dist_poll_selftest(int scenario, uint32_t timeout_ms, int* aborted);

/* ------------------------------------------------------------------ projections (GEMV) */

/* The matrix-vector products on either side of attention: the Q/K/V projections of the
 * normed hidden state (src/engine.ts:2043-2053, pass 'attn.linearQKV') and the output
 * projection of the attention output (src/engine.ts:2096, pass 'attn.linearOut').
 * out[m] = sum_k W[m, k] * input[k] for an [M, N] weight in one of the reference's three
 * storage modes (`weightQuant`, src/engine.ts:107):
 *   G4A_WEIGHT_F16 : weight = f16 [M, N] row-major.  Replaces shaders/matmul_quant.wgsl and
 *                    matmul_quant_mr4.wgsl (bindings input, weight, output, Params {M, N}).
 *   G4A_WEIGHT_Q8  : weight = int8 [M, N] packed 4 per uint32 (element k of row m is byte
 *                    (m*N + k) % 4 of word (m*N + k) / 4), scales = f16 [M, N/32], one per
 *                    32-element block; value = int8 * scale.  N % 32 == 0.  Replaces
 *                    shaders/matmul_q8.wgsl / matmul_q8_mr.wgsl (bindings input, qweight,
 *                    qscale, output, Params {M, N}); layout made by createQ8Buffers
 *                    (src/engine.ts:638-674).
 *   G4A_WEIGHT_Q4K : weight = 4-bit [M, N] packed 8 per uint32 (nibble (m*N + k) % 8 of word
 *                    (m*N + k) / 8), scales = the f16 meta [M, N/256, 16]: for each
 *                    256-element super-block 8 sub-block scales then 8 sub-block mins (32
 *                    elements per sub-block); value = scale * nibble + min.  N % 256 == 0.
 *                    Replaces shaders/matmul_q4k.wgsl / matmul_q4k_mr.wgsl; layout made by
 *                    createQ4KBuffers (src/engine.ts:699-739).
 * Every output is bit-identical to the shaders' arithmetic without contraction: the
 * 256-thread partial sums over k = t, t + 256, ... in order, then the stride-halving tree.
 * input and out are f32 device arrays; the weight pointer must be 16-byte aligned for Q8 and
 * Q4K (F16 takes any 2-byte aligned pointer and any N). */
#define G4A_WEIGHT_F16 0u
#define G4A_WEIGHT_Q8 1u
#define G4A_WEIGHT_Q4K 2u
g4a_status g4a_matmul(g4a_ctx* ctx, uint32_t weight_format, const float* input, const void* weight,
                      const uint16_t* scales, float* out, uint32_t M, uint32_t N);

/* Several matrices over the same input in one launch, as the reference's 'attn.linearQKV'
 * pass dispatches the Q, K and V matmuls from one bind of the normed hidden state
 * (src/engine.ts:2045-2052).  1 <= num_jobs <= G4A_MATMUL_MAX_JOBS; all jobs share
 * weight_format and N; scales may be NULL for G4A_WEIGHT_F16. */
#define G4A_MATMUL_MAX_JOBS 4
typedef struct {
  const void* weight;
  const uint16_t* scales;
  float* out;
  uint32_t M;
} g4a_matmul_job;
g4a_status g4a_matmul_group(g4a_ctx* ctx, uint32_t weight_format, const float* input, uint32_t N,
                            const g4a_matmul_job* jobs, uint32_t num_jobs);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* G4ATTN_H_ */
