// Prefill attention for head_dim 512 (the global layers of Gemma 4: src/config/gemma4-e2b.ts:
// 33-34) with 8 q heads per kv head, as one flash-attention pass on the warp-level tensor-core
// MMA (mma.sync m16n8k16, f16 in, f32 accumulate).
//
// Semantics are those of the reference's token-by-token prefill (prefillBatched,
// src/engine.ts:2460-2479): row (token i, head h) is decode attention over the keys
// [max(0, hi - W), hi) with hi = start_pos + i + 1 (W = 0: all), the score scale applied to the
// dot product (attn_score.wgsl:39) and kv head h / 8 (attn_score.wgsl:31).
//
// Why not the tcgen05 kernel: at head_dim 512 a 128-row accumulator of O alone fills the 512
// TMEM columns and a 128-row f16 Q tile is 128 KB of shared memory, so the TMEM/TMA design of
// g4a_prefill.cu has no room for its score buffers and rings.  Here O lives in registers:
//
// Tile: 8 tokens x the 8 q heads of one kv head = 64 query rows, one CTA of 8 warps.  Warp
// (g, half), g = 0..3, half = 0..1, owns rows 16g .. 16g+15 (tokens 2g and 2g+1) and output
// dims [256 half, 256 half + 256): 128 f32 accumulators per lane.  Per block of 32 keys:
//   S  : each warp multiplies its half of the head dim (Q from shared memory, K^T from the
//        block), the two warps of a row group add their partial scores through shared memory
//        (named barrier of 64 threads), so both hold the full scores;
//   softmax in base 2, masked per (token, key), running max with the O rescale skipped when no
//        row's max moved (warp vote), P rounded to f16 and its rounded values summed for l;
//   PV : P (registers, the accumulator layout re-packed as A fragments) times V of the warp's
//        256 dims (ldmatrix.trans).
// Shared memory: Q 64 KB, K and V blocks double-buffered (cp.async, 2 x 2 x 32 KB), the score
// exchange 16 KB; rows of 1 KB use an XOR swizzle of the 16-byte chunks (chunk ^ (row & 7)) so
// the ldmatrix phases hit eight distinct bank groups.  Rows outside the cache (past the tile's
// last key) and query rows past T are zero-filled, never read from memory.  There are no
// spin-waits: cp.async groups and CTA / named barriers only.
#include <cuda_fp16.h>

#include "g4a_internal.cuh"

namespace {

constexpr int kWideHD = 512;
constexpr int kWideTok = 8;                 // tokens per tile
constexpr int kWideRows = kWideTok * 8;     // 64 query rows (8 q heads per kv head)
constexpr int kWideKeys = 32;               // keys per block
constexpr int kWideThreads = 256;
constexpr int kRowBytes = kWideHD * 2;      // 1 KB per f16 row
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kWideRows * kRowBytes;          // 2 buffers
constexpr int kOffV = kOffK + 2 * kWideKeys * kRowBytes;      // 2 buffers
constexpr int kOffX = kOffV + 2 * kWideKeys * kRowBytes;      // score exchange [4][2][16][32] f32
constexpr int kWideSmem = kOffX + 4 * 2 * 16 * 32 * 4;        // 212,992 B
constexpr float kLog2eW = 1.4426950408889634f;

// Byte offset of 16-byte chunk c of row r in a swizzled 1 KB-row buffer.
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) { return r * kRowBytes + ((c ^ (r & 7u)) << 4); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const uint32_t n = valid ? 16u : 0u;  // 0: no bytes read, the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct WideParams {
  const __half* q16;  // [T, nqh, 512]
  const __half* k;    // [rows, nkh, 512]
  const __half* v;
  float* out;         // [T, nqh, 512]
  uint32_t T, start_pos, nqh, nkh, window, ntiles;
  float scale_log2;
};

__global__ void __launch_bounds__(kWideThreads, 1) prefill_wide_kernel(const __grid_constant__ WideParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const uint32_t sbase = g4a::smem_u32(smem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = warp & 3, half = warp >> 2;
  const uint32_t kvh = blockIdx.x % p.nkh;
  const uint32_t tile = p.ntiles - 1u - blockIdx.x / p.nkh;  // latest (heaviest) tiles first
  const uint32_t t0 = tile * kWideTok;
  const uint32_t nt = min((uint32_t)kWideTok, p.T - t0);
  // Key positions fit in 32 bits: the host checks start_pos + T < 2^32.
  const uint32_t hi_max = p.start_pos + t0 + nt;  // keys [.., hi_max) exist in the cache
  const uint32_t hi_min = p.start_pos + t0 + 1;   // the tile's first token sees keys below this
  const uint32_t lo_min = (p.window && hi_min > p.window) ? hi_min - p.window : 0u;
  const uint32_t lo_max = (p.window && hi_max > p.window) ? hi_max - p.window : 0u;  // last token's window start
  const uint32_t j0 = lo_min / kWideKeys, j1 = (uint32_t)(((uint64_t)hi_max + kWideKeys - 1) / kWideKeys);
  const size_t kv_stride = (size_t)p.nkh * kWideHD;  // elements between consecutive cache rows
  // 256 threads: thread `tid` copies chunk c = tid % 64 of rows tid / 64 + 4 i.
  const uint32_t cc = (uint32_t)tid & 63u, n0 = (uint32_t)tid >> 6;

  g4a::pdl_wait_primary();  // q16 and the cache rows are written by the preceding kernels

  // Q tile: row r = token * 8 + head (the 8 heads of a token are contiguous in q16).
#pragma unroll
  for (int i = 0; i < kWideRows / 4; i++) {
    const uint32_t r = n0 + 4u * i, tok = r >> 3, head = r & 7u;
    const bool ok = tok < nt;
    const __half* src = ok ? p.q16 + ((size_t)(t0 + tok) * p.nqh + kvh * 8u + head) * kWideHD + cc * 8u : p.q16;
    cp_async16(sbase + kOffQ + swz(r, cc), src, ok);
  }
  const size_t lane_off = (size_t)kvh * kWideHD + cc * 8u;
  auto load_block = [&](uint32_t j, int buf) {
    const uint32_t kb = j * kWideKeys;
    const size_t row0 = ((size_t)kb + n0) * kv_stride + lane_off;
    const uint32_t dk = sbase + kOffK + buf * (kWideKeys * kRowBytes), dv = dk + (kOffV - kOffK);
#pragma unroll
    for (int i = 0; i < kWideKeys / 4; i++) {
      const uint32_t n = n0 + 4u * i;
      const bool ok = (uint64_t)kb + n < hi_max;
      const size_t off = ok ? row0 + (size_t)(4 * i) * kv_stride : 0;
      cp_async16(dk + swz(n, cc), p.k + off, ok);
      cp_async16(dv + swz(n, cc), p.v + off, ok);
    }
  };
  load_block(j0, 0);
  cp_async_commit();  // group: Q + first block

  // Rows of this lane: A = (token 2g, head lane/4) in c0/c1, B = (token 2g+1, same head) in c2/c3.
  // Rows past T are computed like the others (their q rows are zero) and never written.
  const uint32_t tokA = t0 + 2u * g, tokB = tokA + 1u;
  const uint32_t hiA = p.start_pos + tokA + 1, hiB = hiA + 1;
  const uint32_t loA = (p.window && hiA > p.window) ? hiA - p.window : 0u;
  const uint32_t loB = (p.window && hiB > p.window) ? hiB - p.window : 0u;
  const bool rowA = tokA < p.T, rowB = tokB < p.T;

  float o[32][4];
#pragma unroll
  for (int t = 0; t < 32; t++) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  float* xbuf = reinterpret_cast<float*>(smem + kOffX);
  float* xmine = xbuf + ((g * 2 + half) * 16) * 32 + lane;
  const float* xpeer = xbuf + ((g * 2 + (1 - half)) * 16) * 32 + lane;

  for (uint32_t j = j0; j < j1; j++) {
    const int buf = (int)((j - j0) & 1u);
    if (j + 1 < j1) {
      load_block(j + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kbase = sbase + kOffK + buf * (kWideKeys * kRowBytes);
    const uint32_t vbase = sbase + kOffV + buf * (kWideKeys * kRowBytes);

    // ---- partial scores over this warp's 256 dims: s[n-tile][4]
    float s[4][4];
#pragma unroll
    for (int t = 0; t < 4; t++) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
#pragma unroll 4
    for (int ks = 0; ks < 16; ks++) {
      const uint32_t cq = (uint32_t)(half * 32 + ks * 2);
      uint32_t a[4];
      ldsm_x4(sbase + kOffQ + swz((uint32_t)(16 * g + (lane & 15)), cq + (uint32_t)(lane >> 4)), a);
#pragma unroll
      for (int np = 0; np < 2; np++) {
        const int mi = lane >> 3;
        uint32_t b[4];
        ldsm_x4(kbase + swz((uint32_t)(np * 16 + (mi >> 1) * 8 + (lane & 7)), cq + (uint32_t)(mi & 1)), b);
        mma16816(s[2 * np], a, b[0], b[1]);
        mma16816(s[2 * np + 1], a, b[2], b[3]);
      }
    }
    // ---- the two halves of the row group add their partial scores
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
      for (int e = 0; e < 4; e++) xmine[(t * 4 + e) * 32] = s[t][e];
    g4a::named_bar_sync(1u + (uint32_t)g, 64);
#pragma unroll
    for (int t = 0; t < 4; t++)
#pragma unroll
      for (int e = 0; e < 4; e++) s[t][e] = __fadd_rn(s[t][e], xpeer[(t * 4 + e) * 32]);

    // ---- mask (only blocks that cross some row's window edge or diagonal), running max, P
    float bmA = -INFINITY, bmB = -INFINITY;
    const uint32_t kb = j * kWideKeys;
    if (kb >= lo_max && (uint64_t)kb + kWideKeys <= hi_min) {  // every key visible to every row of the tile
#pragma unroll
      for (int t = 0; t < 4; t++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          s[t][e] *= p.scale_log2;
          s[t][2 + e] *= p.scale_log2;
          bmA = fmaxf(bmA, s[t][e]);
          bmB = fmaxf(bmB, s[t][2 + e]);
        }
    } else {
#pragma unroll
      for (int t = 0; t < 4; t++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const uint32_t key = kb + (uint32_t)(t * 8 + 2 * (lane & 3) + e);
          const bool okA = key >= loA && key < hiA, okB = key >= loB && key < hiB;
          s[t][e] = okA ? s[t][e] * p.scale_log2 : -INFINITY;
          s[t][2 + e] = okB ? s[t][2 + e] * p.scale_log2 : -INFINITY;
          bmA = fmaxf(bmA, s[t][e]);
          bmB = fmaxf(bmB, s[t][2 + e]);
        }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      bmA = fmaxf(bmA, __shfl_xor_sync(0xffffffffu, bmA, off));
      bmB = fmaxf(bmB, __shfl_xor_sync(0xffffffffu, bmB, off));
    }
    const float nA = fmaxf(mA, bmA), nB = fmaxf(mB, bmB);
    if (__any_sync(0xffffffffu, nA > mA || nB > mB)) {
      const float alA = (nA > mA) ? g4a::fast_exp2(mA - nA) : 1.f;  // mA = -inf gives 0 (O, l are 0)
      const float alB = (nB > mB) ? g4a::fast_exp2(mB - nB) : 1.f;
#pragma unroll
      for (int t = 0; t < 32; t++) {
        o[t][0] *= alA;
        o[t][1] *= alA;
        o[t][2] *= alB;
        o[t][3] *= alB;
      }
      lA *= alA;
      lB *= alB;
      mA = nA;
      mB = nB;
    }
    const float uA = (mA == -INFINITY) ? 0.f : mA, uB = (mB == -INFINITY) ? 0.f : mB;
    uint32_t pa[4][2];  // P as f16 pairs: [n-tile][row A / row B]
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const __half2 hA = __floats2half2_rn(g4a::fast_exp2(s[t][0] - uA), g4a::fast_exp2(s[t][1] - uA));
      const __half2 hB = __floats2half2_rn(g4a::fast_exp2(s[t][2] - uB), g4a::fast_exp2(s[t][3] - uB));
      const float2 fA = __half22float2(hA), fB = __half22float2(hB);
      lA += fA.x + fA.y;
      lB += fB.x + fB.y;
      pa[t][0] = *reinterpret_cast<const uint32_t*>(&hA);
      pa[t][1] = *reinterpret_cast<const uint32_t*>(&hB);
    }

    // ---- O += P V over this warp's 256 dims
#pragma unroll
    for (int s2 = 0; s2 < 2; s2++) {
      const uint32_t a[4] = {pa[2 * s2][0], pa[2 * s2][1], pa[2 * s2 + 1][0], pa[2 * s2 + 1][1]};
      const int mi = lane >> 3;
      const uint32_t vrow = (uint32_t)(s2 * 16 + (mi & 1) * 8 + (lane & 7));
#pragma unroll
      for (int dp = 0; dp < 16; dp++) {
        uint32_t b[4];
        ldsm_x4_t(vbase + swz(vrow, (uint32_t)(half * 32 + dp * 2 + (mi >> 1))), b);
        mma16816(o[2 * dp], a, b[0], b[1]);
        mma16816(o[2 * dp + 1], a, b[2], b[3]);
      }
    }
    __syncthreads();  // every warp is done with this buffer and with the score exchange
  }
  g4a::pdl_launch_dependents();

  // ---- epilogue: the row sums over the quad, then O / l
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, off);
    lB += __shfl_xor_sync(0xffffffffu, lB, off);
  }
  const float iA = lA > 0.f ? 1.f / lA : 0.f, iB = lB > 0.f ? 1.f / lB : 0.f;
  const uint32_t head = kvh * 8u + (uint32_t)(lane >> 2);
  const uint32_t col = (uint32_t)(half * 256 + 2 * (lane & 3));
  if (rowA) {
    float* dst = p.out + ((size_t)tokA * p.nqh + head) * kWideHD + col;
#pragma unroll
    for (int t = 0; t < 32; t++) *reinterpret_cast<float2*>(dst + t * 8) = make_float2(o[t][0] * iA, o[t][1] * iA);
  }
  if (rowB) {
    float* dst = p.out + ((size_t)tokB * p.nqh + head) * kWideHD + col;
#pragma unroll
    for (int t = 0; t < 32; t++) *reinterpret_cast<float2*>(dst + t * 8) = make_float2(o[t][2] * iB, o[t][3] * iB);
  }
}

}  // namespace

// Host entry used by g4a_prefill_attn for head_dim 512 with num_q_heads = 8 * num_kv_heads.
g4a_status prefill_wide(g4a_ctx* ctx, const uint16_t* q16, const uint16_t* k, const uint16_t* v, float* out,
                        uint32_t T, uint32_t start_pos, uint32_t nqh, uint32_t nkh, float scale, uint32_t window) {
  WideParams p;
  p.q16 = reinterpret_cast<const __half*>(q16);
  p.k = reinterpret_cast<const __half*>(k);
  p.v = reinterpret_cast<const __half*>(v);
  p.out = out;
  p.T = T;
  p.start_pos = start_pos;
  p.nqh = nqh;
  p.nkh = nkh;
  p.window = window;
  p.ntiles = (T + kWideTok - 1) / kWideTok;
  p.scale_log2 = scale * kLog2eW;
  const uint64_t ctas = (uint64_t)p.ntiles * nkh;
  if (ctas > 0x7fffffffull) return g4a_fail(G4A_EINVAL, "g4a_prefill_attn: T %u x %u kv heads is too large", T, nkh);
  const cudaError_t a =
      cudaFuncSetAttribute(prefill_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWideSmem);
  if (a != cudaSuccess) return g4a_cuda_fail(a, "cudaFuncSetAttribute(prefill_wide_kernel)");
  g4a_prof_scope ps(ctx, G4A_PROF_PREFILL_ATTN);
  const cudaError_t e = g4a_launch(prefill_wide_kernel, dim3((unsigned)ctas), dim3(kWideThreads), (size_t)kWideSmem,
                                   ctx->stream, true, p);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "launch prefill_wide_kernel");
  return G4A_OK;
}
