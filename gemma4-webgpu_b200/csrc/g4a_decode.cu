// Decode attention: the reference's attn_score -> softmax -> attn_output chain
// (shaders/attn_score.wgsl:15-40, softmax.wgsl:7-46, attn_output.wgsl:7-23, dispatched at
// src/engine.ts:2092-2094) as one split-KV flash-decode kernel plus a log-sum-exp merge.
//
// Semantics kept from the reference:
//   - keys [max(0, L - W), L) are attended, L = kv_len, W = sliding_window (0 = all)
//     (attn_score.wgsl:23-30).  Masked keys are never read, which is exactly the reference's
//     -1e30 score: exp(-1e30 - max) is 0 in f32.
//   - kv head of q head h is h * NKH / NQH (attn_score.wgsl:31); scale multiplies the dot
//     (attn_score.wgsl:39); output f32 [NQH, HD] (attn_output.wgsl:22); L = 0 gives zeros.
//
// Fast path (NQH = 8 * NKH, HD in {128, 256, 512}): persistent CTAs, one per SM, 8 warps.  A
// call whose stages would not fill the SMs (short contexts) uses half-size stages instead.
// The flattened list of "stages" (64 keys for HD 256) of every (sequence, kv head) problem is
// split evenly over the grid, so a CTA may cover the end of one problem and the start of the
// next.  Warp 0 is also the producer: it TMA-bulk-copies every K and V row of a stage (no
// multicast) from HBM into a 3-deep ring of padded shared-memory rows guarded by mbarriers.
// The two contractions run on the tensor cores (mma.sync m16n8k16, f32 accumulate): q is split
// into f16 hi + lo halves stacked as the 16 rows of the A operand, and so are the softmax
// probabilities, which keeps ~22 significant bits through f16 operands.  Decode has only 8 query
// rows per kv head (16 with the split), below the 64-row minimum of tcgen05.mma, and is HBM-bound;
// on the CUDA cores the 8 FLOP per KV byte would need ~70% of the FP32 pipe at the HBM roofline
// (measured: the CUDA-core version of this kernel reached 23% of HBM with the FMA pipe as the
// ceiling).  Online softmax in base 2 with lazy rescaling (the running max is only raised when a
// score exceeds it by more than 2^8).  At the end of each segment (a problem's stages inside one
// CTA) the key groups merge through shared memory and write either the final row (segment =
// whole problem) or an un-normalised partial (m, l, o) that the merge kernel combines.
#include <math.h>

#include <algorithm>
#include <atomic>

#include <cudaTypedefs.h>

#include "g4a_internal.cuh"

namespace {

constexpr int kGroup = 8;  // q heads per kv head on the fast path
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;  // 2 warps per SM sub-partition: up to 255 registers each
constexpr float kLazyRescale = 8.0f;   // log2 units
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kBalancedMaxStages = 8;  // single-sequence calls up to this many stages per SM get a balanced grid
constexpr int kScanRegs = 4;           // problems per lane held in registers by the work-partition scans

enum : int { F_SEG_FIRST = 1, F_SEG_LAST = 2, F_PROB_FIRST = 4, F_PROB_LAST = 8 };

struct StageMeta {
  int problem;
  int key0;    // first position of the stage (a multiple of the stage size)
  int kfirst;  // valid rows of the stage are [kfirst, kend)
  int kend;
  int flags;
  int seg;
};

struct DecodeParams {
  const float* q;         // [P * 8 (fast) | B * nqh, hd] f32
  const __half* q16;      // the same queries in f16 (prefill through the decode kernels), or null
  const __half* k;        // cache or page pool base
  const __half* v;
  const int* page_table;  // [B, max_pages] or null (contiguous)
  const int* kv_lens;     // [B] device, or null: every sequence has kv_len_scalar
  uint32_t kv_len_scalar;
  int B, nqh, nkh, hd;
  int page_size, max_pages, num_pages;
  float scale_log2;   // scale * log2(e)
  uint32_t window;
  uint32_t row_base;  // position of buffer row 0 (split-KV partial buffers)
  uint32_t kv_end;    // keys at positions >= kv_end are not in the buffer (partial mode)
  float* part;        // [segments, 8 * (hd + 2)] partial workspace
  int2* seg_range;    // [P] first/last segment id of each problem
  float* out;         // [P * 8, hd]; null in partial mode
  int* err;
  int kps;            // keys per stage of the launched main kernel
  int main_grid;      // grid of the launched main kernel
};

__device__ __forceinline__ uint32_t seq_len_of(const DecodeParams& p, int seq) {
  return p.kv_lens ? (uint32_t)max(p.kv_lens[seq], 0) : p.kv_len_scalar;
}

// Visible key range [lo, hi) of a sequence of length L (window measured from the full length).
__device__ __forceinline__ void key_range_of_len(const DecodeParams& p, uint32_t L, uint32_t& lo, uint32_t& hi) {
  if (p.page_table) {
    uint32_t cap = (uint32_t)p.max_pages * (uint32_t)p.page_size;
    if (L > cap) {
      if (p.err) atomicExch(p.err, G4A_DEVERR_KVLEN);
      L = cap;
    }
  }
  uint32_t ws = 0;
  if (p.window != 0u && L > p.window) ws = L - p.window;
  lo = max(ws, p.row_base);
  hi = min(L, p.kv_end);
  if (hi < lo) hi = lo;
}
__device__ __forceinline__ void key_range(const DecodeParams& p, int seq, uint32_t& lo, uint32_t& hi) {
  key_range_of_len(p, seq_len_of(p, seq), lo, hi);
}

// Address of the row of position t for (seq, kvh); null if its page id is out of range.
__device__ __forceinline__ const __half* row_ptr(const DecodeParams& p, const __half* base, int seq, int kvh,
                                                 uint32_t t) {
  uint32_t r = t - p.row_base;
  size_t abs_row;
  if (p.page_table) {
    int page = p.page_table[(size_t)seq * p.max_pages + r / (uint32_t)p.page_size];
    if (page < 0 || page >= p.num_pages) return nullptr;
    abs_row = (size_t)page * p.page_size + r % (uint32_t)p.page_size;
  } else {
    abs_row = r;
  }
  return base + (abs_row * p.nkh + kvh) * p.hd;
}

// Tile shape of the tensor-core decode kernel for one head_dim.  The 8 warps of a CTA form NKG
// key groups of 16 keys x NDQ slices.  Warp (kg, dq) contracts the scores of key group kg over
// the dq-th slice of HD/NDQ dims; the NDQ partial scores are summed through shared memory (in a
// fixed order, so every warp of the group holds identical scores), and the warp then
// accumulates p*V for its DPW output dims.  A stage holds KPS keys of
// K and of V as HD/64 column boxes of [KPS rows x 128 B] each, written by TMA with the 128-byte
// swizzle (16-byte chunk c of row r stored at chunk c ^ (r & 7)), so ldmatrix reads of 8 rows
// hit 8 different bank groups without padding.
// SHORT halves the stage (twice the k-slices per key group): for calls whose stages of the
// regular shape would not fill the SMs, more and smaller stages start the CTAs sooner.
template <int HD, bool SHORT = false>
struct Cfg {
  static constexpr int NDQ = (SHORT ? 2 : 1) * (HD / 128);  // score k-slices = output-dim slices
  static constexpr int DPW = HD / NDQ;                 // output dims per warp
  static constexpr int NT = DPW / 8;                   // n-tiles of the p*V MMA per warp
  static constexpr int NKG = kWarps / NDQ;             // key groups of 16 keys
  static constexpr int KPS = 16 * NKG;                 // keys per stage (64 KB of K+V)
  static constexpr int KSTEPS = HD / 16;               // k-steps of the score MMA
  static constexpr int KPW = KSTEPS / NDQ;             // k-steps of the score MMA per warp
  static constexpr int NCB = HD / 64;                  // 64-dim column boxes per row
  static constexpr int CB_BYTES = KPS * 128;           // one column box of a stage
  static constexpr int STAGE_BYTES = 2 * NCB * CB_BYTES;  // K boxes then V boxes
  static constexpr int STAGES = 196608 / STAGE_BYTES;  // depth of the shared-memory ring (192 KB)
  static constexpr int OSTRIDE = DPW + 4;              // floats per head row of a merge slot
  static constexpr int OSLOT = kGroup * OSTRIDE + 2 * kGroup;  // o[8][DPW+4] | m[8] | l[8]
  static constexpr int NSLOT = (NKG / 2) * NDQ;
  static constexpr int SX_FLOATS = 2 * kWarps * 32 * 4;  // double-buffered partial-score exchange
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + (size_t)NSLOT * OSLOT * 4 +
                                 (size_t)SX_FLOATS * 4 + STAGES * sizeof(StageMeta) + 2 * STAGES * 8 + 64;
  static_assert(NKG >= 2 && NKG * NDQ == kWarps && NT % 2 == 0 && KPW % 4 == 0, "tile shape");
  static_assert(CB_BYTES % 1024 == 0 && STAGES >= 3, "swizzle atoms / ring depth");
  static_assert(SMEM <= 232448, "shared memory");
};

// Stages of a problem: KPS-aligned blocks of positions covering [lo, hi).
template <int KPS>
__device__ __forceinline__ int stages_of(const DecodeParams& p, int prob) {
  uint32_t lo, hi;
  key_range(p, prob / p.nkh, lo, hi);
  return hi > lo ? (int)((hi + KPS - 1) / KPS - lo / KPS) : 0;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D += A(16x16, f16, row) * B(16x8, f16, col), f32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Pack two floats as f16 (low half = a) and return the residuals x - f32(f16(x)).
__device__ __forceinline__ uint32_t pack_hi(float a, float b, float& ra, float& rb) {
  const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
  ra = a - __half2float(ha);
  rb = b - __half2float(hb);
  return (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
}
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  return (uint32_t)__half_as_ushort(__float2half_rn(a)) | ((uint32_t)__half_as_ushort(__float2half_rn(b)) << 16);
}
// Tiled TMA loads (no multicast) completing on an mbarrier, with an L2 cache hint.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(g4a::smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            int c4, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(g4a::smem_u32(bar)),
      "l"(pol)
      : "memory");
}

// Split-KV flash-decode on the tensor cores.
//
// The q block of one kv head (8 heads x HD, f32) is split as q = hi + lo with hi = f16(q) and
// lo = f16(q - hi) and stacked into the 16 rows of the MMA's A operand (rows 0-7 hi, 8-15 lo),
// so one m16n8k16 MMA per k-step yields both halves of every score and their sum carries ~22
// mantissa bits of q; K and V are exact f16.  The probabilities are split the same way for the
// p*V MMA.  Thread (g = lane/4, c = lane%4) of a warp owns head g: it holds the scores of keys
// {2c, 2c+1, 8+2c, 9+2c} of its 16-key group (the accumulator rows g and g+8 are the hi and lo
// halves of the same head), so the online softmax, the hi/lo split of p into the A fragment of
// the p*V MMA, the masking of out-of-range keys (their scores become -inf and their V halves in
// the B fragments become 0) and the rescaling of its output accumulators are all thread-local;
// only the row max and the final row sum need two shuffles.
template <int HD, bool SHORT>
__global__ void __launch_bounds__(kThreads, 1)
    decode_splitkv_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv) {
  using C = Cfg<HD, SHORT>;
  constexpr int NDQ = C::NDQ, KPS = C::KPS, KPW = C::KPW, NCB = C::NCB, CBB = C::CB_BYTES;
  constexpr int NKG = C::NKG, NT = C::NT, DPW = C::DPW, kStages = C::STAGES;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~uintptr_t(1023));
  unsigned char* stage_base = smem;
  float* oslot = reinterpret_cast<float*>(smem + (size_t)kStages * C::STAGE_BYTES);
  float* sx = oslot + C::NSLOT * C::OSLOT;  // [2][warp][lane][4] partial scores
  StageMeta* meta = reinterpret_cast<StageMeta*>(sx + C::SX_FLOATS);
  uint64_t* full = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(meta + kStages) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int P = p.B * p.nkh;
  // Uniform mode (no per-sequence kv_lens): every problem has the same visible key range and
  // stage count, so the work partition and the position of every stage follow from the launch
  // parameters alone.  They are computed before the PDL wait, in closed form, and the stages
  // need no metadata in shared memory.
  const bool uniform = (p.kv_lens == nullptr);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      g4a::mbar_init(&full[s], 1);
      g4a::mbar_init(&empty[s], kWarps);
    }
    g4a::fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
  }
  __syncwarp();  // warp 0 was diverged by the initialisation above
  __syncthreads();
  g4a::pdl_launch_dependents();

  // ---- stage range [s0, s1) of this CTA over the flattened stage list (every warp computes it)
  long long S = 0;
  // Non-uniform mode with at most 32 * kScanRegs problems: each lane keeps the stage counts of
  // problems lane, lane + 32, ... in registers, so both scans below cost one round trip of
  // kv_lens loads (issued together) instead of one per 32 problems and per scan.
  const bool scan_regs = !uniform && P <= 32 * kScanRegs;
  int cnt[kScanRegs];
  int nstg = 0;                // uniform mode: stages per problem
  uint32_t ulo = 0, uhi = 0;   // uniform mode: visible key range of every problem
  if (uniform) {
    key_range(p, 0, ulo, uhi);
    nstg = uhi > ulo ? (int)((uhi + KPS - 1) / KPS - ulo / KPS) : 0;
    S = (long long)P * nstg;
  } else {
    // kv_lens, like q and the cache rows, may be written by the preceding kernel: with a
    // programmatic (PDL) launch, wait for it before reading any of them.
    g4a::pdl_wait_primary();
    if (scan_regs) {
      // all the loads first (a clamped index keeps them unconditional), then the counts
      uint32_t len[kScanRegs];
#pragma unroll
      for (int k = 0; k < kScanRegs; k++) len[k] = seq_len_of(p, min(32 * k + lane, P - 1) / p.nkh);
#pragma unroll
      for (int k = 0; k < kScanRegs; k++) {
        uint32_t lo, hi;
        key_range_of_len(p, len[k], lo, hi);
        cnt[k] = (32 * k + lane < P && hi > lo) ? (int)((hi + KPS - 1) / KPS - lo / KPS) : 0;
      }
#pragma unroll
      for (int k = 0; k < kScanRegs; k++) {
        int n = cnt[k];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
        S += n;
      }
    } else {
      for (int base = 0; base < P; base += 32) {
        const int pr = base + lane;
        int n = (pr < P) ? stages_of<KPS>(p, pr) : 0;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
        S += n;
      }
    }
  }
  // Only the first min(grid, S) CTAs take part, so every active CTA owns at least one stage and
  // the segment ids blockIdx.x + problem of one problem form a gap-free range.
  const long long G = (long long)gridDim.x < S ? (long long)gridDim.x : S;
  if ((long long)blockIdx.x >= G) return;  // uniform across the CTA
  // The CTAs with the lowest indices take the one extra stage: the last CTAs of the grid are
  // the ones that start late (they wait for the SMs the previous kernel still occupies).
  const long long q_st = S / G, r_st = S % G, b_st = (long long)blockIdx.x;
  const long long s0 = b_st * q_st + (b_st < r_st ? b_st : r_st);
  const long long s1 = s0 + q_st + (b_st < r_st ? 1 : 0);
  const int my_stages = (int)(s1 - s0);

  // ---- cursor (problem, stage within the problem) of this CTA's first stage, in every warp
  int prob0 = 0, j0 = 0;
  if (uniform) {
    prob0 = (int)(s0 / nstg);
    j0 = (int)(s0 - (long long)prob0 * nstg);
    // While the preceding kernel finishes, pull this CTA's first stage (its K and V boxes, the
    // same coordinates as the loads below) into L2.  A prefetch only moves lines into L2, which
    // the preceding kernel's writes update as well, so the loads after the wait see current data.
    // One stage measured best (32k: 13.4 -> 12.2 us per layer-call); prefetching two or six
    // stages slowed the calls that follow the producer kernel, whose wait is short.
    if (p.page_table == nullptr && warp == 1 && lane < 2) {
      const uint32_t key0 = (ulo / KPS + (uint32_t)j0) * KPS;
      asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                       reinterpret_cast<uint64_t>(lane ? &tmv : &tmk)),
                   "r"(0), "r"(prob0 % p.nkh), "r"((int)key0 - (int)p.row_base), "r"(0)
                   : "memory");
    }
    g4a::pdl_wait_primary();
  } else {
    long long acc = 0;
    bool found = false;
    for (int base = 0; base < P && !found; base += 32) {
      const int pr = base + lane;
      int n = 0;
      if (scan_regs) {
#pragma unroll
        for (int k = 0; k < kScanRegs; k++)
          if (32 * k == base) n = cnt[k];
      } else {
        n = (pr < P) ? stages_of<KPS>(p, pr) : 0;
      }
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const long long lane_start = acc + incl - n;
      const bool hit = (pr < P) && n > 0 && (s0 >= lane_start) && (s0 < lane_start + n);
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (m) {
        const int src = __ffs(m) - 1;
        prob0 = __shfl_sync(0xffffffffu, pr, src);
        j0 = (int)(s0 - __shfl_sync(0xffffffffu, lane_start, src));
        found = true;
      }
      acc += __shfl_sync(0xffffffffu, incl, 31);
    }
  }

  // ---- consumer geometry, and the q block (8 heads x HD f32) of the first segment: coalesced
  // loads issued before the KV stream so that they do not queue behind it, staged through the
  // merge area of shared memory (rows padded by 8 floats: the fragment reads are conflict-free).
  const int kg = warp / NDQ;  // key group: keys [16 kg, 16 kg + 16) of every stage
  const int dq = warp % NDQ;  // output dims [DPW dq, DPW dq + DPW)
  const int g = lane >> 2;    // head owned by this thread
  const int c = lane & 3;
  constexpr int QV = kGroup * HD / 4 / kThreads;  // float4 of the q block per thread
  constexpr int QROW = HD + 8;                     // staged row stride (floats)
  static_assert(kGroup * QROW * 4 <= C::NSLOT * C::OSLOT * 4, "q staging fits the merge area");
  float4 qv[QV];
  auto load_q = [&](int problem) {
    if (p.q16 != nullptr) {  // f16 queries: 4 per 8-byte load, exact in f32 (the lo half is 0)
      const uint2* src = reinterpret_cast<const uint2*>(p.q16 + (size_t)problem * kGroup * HD);
#pragma unroll
      for (int i = 0; i < QV; i++) {
        const uint2 u = src[threadIdx.x + i * kThreads];
        const float2 a = g4a::h2_to_f2(u.x), b = g4a::h2_to_f2(u.y);
        qv[i] = make_float4(a.x, a.y, b.x, b.y);
      }
    } else {
      const float4* src = reinterpret_cast<const float4*>(p.q + (size_t)problem * kGroup * HD);
#pragma unroll
      for (int i = 0; i < QV; i++) qv[i] = src[threadIdx.x + i * kThreads];
    }
  };
  // Stores the loaded block, waits for every warp, and builds this thread's A fragments
  // [q_hi; q_lo] of its KPW k-steps.
  uint32_t qa[KPW][4];
  auto stage_q = [&]() {
#pragma unroll
    for (int i = 0; i < QV; i++) {
      const int e = (threadIdx.x + i * kThreads) * 4;
      *reinterpret_cast<float4*>(oslot + (e / HD) * QROW + (e % HD)) = qv[i];
    }
    g4a::named_bar_sync(1, kThreads);
    const float* qs = oslot + g * QROW + dq * KPW * 16 + 2 * c;
#pragma unroll
    for (int ks = 0; ks < KPW; ks++) {
      const float2 x0 = *reinterpret_cast<const float2*>(qs + ks * 16);
      const float2 x1 = *reinterpret_cast<const float2*>(qs + ks * 16 + 8);
      float r0, r1, r2, r3;
      qa[ks][0] = pack_hi(x0.x, x0.y, r0, r1);
      qa[ks][1] = pack_f16(r0, r1);
      qa[ks][2] = pack_hi(x1.x, x1.y, r2, r3);
      qa[ks][3] = pack_f16(r2, r3);
    }
  };
  load_q(prob0);

  // =========================== producer role (warp 0 issues the TMA copies)
  // Stage n of this CTA goes to slot n % kStages.  Warp 0 keeps the cursor (problem, stage
  // within problem) and, before consuming stage it, issues stage it + kStages - 1 once all
  // eight warps have released that slot.  A stage is the KPS-aligned block of positions
  // [key0, key0 + KPS); its valid rows are [kfirst, kend).  Rows outside come from the fill of
  // out-of-range boxes or from neighbouring cache rows and are masked by the consumers.
  int prob = prob0, j = j0, nprob = 0;
  uint32_t lo = 0, hi = 0;
  uint64_t pol = 0;
  if (warp == 0) {
    if (uniform) {
      nprob = nstg;
      lo = ulo;
      hi = uhi;
    } else {
      nprob = stages_of<KPS>(p, prob);
      key_range(p, prob / p.nkh, lo, hi);
    }
    pol = g4a::l2_policy_evict_first();
  }
  auto issue = [&](int n) {
    const int slot = n % kStages;
    const uint32_t par = ((n / kStages) & 1) ^ 1;
    if (lane == 0) g4a::mbar_wait_bounded(&empty[slot], par, p.err, G4A_DEVERR_WAIT_EMPTY);
    __syncwarp();
    const int seq = prob / p.nkh, kvh = prob % p.nkh;
    const uint32_t key0 = (lo / KPS + (uint32_t)j) * KPS;
    const uint32_t sK = g4a::smem_u32(stage_base + (size_t)slot * C::STAGE_BYTES);
    const uint32_t sV = sK + NCB * CBB;
    if (p.page_table == nullptr) {
      // one op per tensor fills the KPS rows of all HD/64 column boxes
      if (lane == 0) {
        if (!uniform) {
          StageMeta& mt = meta[slot];
          mt.problem = prob;
          mt.key0 = (int)key0;
          mt.kfirst = (int)(max(lo, key0) - key0);
          mt.kend = (int)(min(hi, key0 + KPS) - key0);
          int fl = 0;
          if (n == 0 || j == 0) fl |= F_SEG_FIRST;
          if (n == my_stages - 1 || j == nprob - 1) fl |= F_SEG_LAST;
          if (j == 0) fl |= F_PROB_FIRST;
          if (j == nprob - 1) fl |= F_PROB_LAST;
          mt.flags = fl;
          mt.seg = (int)blockIdx.x + prob;
        }
        g4a::mbar_arrive_expect_tx(&full[slot], (uint32_t)(KPS * 128 * NCB * 2));
      }
      __syncwarp();
      if (lane < 2)
        tma_load_4d(lane ? sV : sK, lane ? &tmv : &tmk, 0, kvh, (int)key0 - (int)p.row_base, 0, &full[slot], pol);
    } else {
      const int kfirst = (int)(max(lo, key0) - key0);
      const int kend = (int)(min(hi, key0 + KPS) - key0);
      // Sub-boxes of BR rows (BR = KPS, or the page size when pages are smaller than a stage).
      const int BR = min(p.page_size, KPS);
      const int nsub = KPS / BR;
      // Sub-box s is loaded if it holds a valid row and its page id is in range.
      bool need = false;
      if (lane < nsub) {
        const int r0 = lane * BR;
        need = (r0 < kend) && (r0 + BR > kfirst);
        if (need) {
          const uint32_t pos = key0 + (uint32_t)r0;
          const uint32_t pidx = pos / (uint32_t)p.page_size;
          const int my_page =
              (pidx < (uint32_t)p.max_pages) ? p.page_table[(size_t)seq * p.max_pages + pidx] : -1;
          if (my_page < 0 || my_page >= p.num_pages) {
            if (p.err) atomicExch(p.err, G4A_DEVERR_PAGE);
            need = false;
          }
        }
      }
      const unsigned need_mask = __ballot_sync(0xffffffffu, need);
      if (lane == 0) {
        if (!uniform) {
          StageMeta& mt = meta[slot];
          mt.problem = prob;
          mt.key0 = (int)key0;
          mt.kfirst = kfirst;
          mt.kend = kend;
          int fl = 0;
          if (n == 0 || j == 0) fl |= F_SEG_FIRST;
          if (n == my_stages - 1 || j == nprob - 1) fl |= F_SEG_LAST;
          if (j == 0) fl |= F_PROB_FIRST;
          if (j == nprob - 1) fl |= F_PROB_LAST;
          mt.flags = fl;
          mt.seg = (int)blockIdx.x + prob;
        }
        g4a::mbar_arrive_expect_tx(&full[slot], (uint32_t)__popc(need_mask) * (uint32_t)(BR * 128 * NCB * 2));
      }
      __syncwarp();
      // One op per (sub-box, tensor): each op fills the sub-box rows of all HD/64 column boxes.
      if (lane < 2 * nsub) {
        const int s = lane >> 1;
        const bool is_v = lane & 1;
        if ((need_mask >> s) & 1u) {
          const uint32_t dst = (is_v ? sV : sK) + s * NCB * BR * 128;  // sub-box s: [chunk][BR][128 B]
          const CUtensorMap* map = is_v ? &tmv : &tmk;
          // page id of sub-box s (lane s validated it above; the table line is in L1)
          const uint32_t pos = key0 + (uint32_t)(s * BR);
          const int page = p.page_table[(size_t)seq * p.max_pages + pos / (uint32_t)p.page_size];
          tma_load_5d(dst, map, 0, kvh, (int)(pos % (uint32_t)p.page_size), page, 0, &full[slot], pol);
        }
      }
    }
    if (++j == nprob) {  // advance the cursor to the next problem with stages
      j = 0;
      if (n + 1 < my_stages) {
        if (uniform) {
          prob++;
        } else {
          do {
            prob++;
            nprob = stages_of<KPS>(p, prob);
          } while (nprob == 0 && prob < P - 1);
          key_range(p, prob / p.nkh, lo, hi);
        }
      }
    }
  };
  if (warp == 0) {
    const int n0 = min(kStages - 1, my_stages);
    if (uniform && p.page_table == nullptr) {
      // The first slots are free: lanes 2n and 2n + 1 load K and V of stage n in one go.
      if (lane < 2 * n0) {
        const int n = lane >> 1;
        int pr = prob, jj = j + n;
        while (jj >= nstg) {
          jj -= nstg;
          pr++;
        }
        const uint32_t key0 = (lo / KPS + (uint32_t)jj) * KPS;
        const uint32_t sK = g4a::smem_u32(stage_base + (size_t)n * C::STAGE_BYTES);
        if ((lane & 1) == 0) g4a::mbar_arrive_expect_tx(&full[n], (uint32_t)(KPS * 128 * NCB * 2));
        tma_load_4d((lane & 1) ? sK + NCB * CBB : sK, (lane & 1) ? &tmv : &tmk, 0, pr % p.nkh,
                    (int)key0 - (int)p.row_base, 0, &full[n], pol);
      }
      j += n0;
      while (j >= nprob) {
        j -= nprob;
        prob++;
      }
    } else {
      // The first stage only: its page-table lookup is a dependent load, and every warp waits
      // for warp 0 in stage_q; the second stage is issued right after.
      if (n0 > 0) issue(0);
    }
  }
  stage_q();
  if (warp == 0 && !(uniform && p.page_table == nullptr)) {
    const int n0 = min(kStages - 1, my_stages);
    for (int n = 1; n < n0; n++) issue(n);
  }

  // =========================== consumer role (all warps)
  float o[NT][4];             // NT n-tiles of 8 output dims: rows g (hi part) and g+8 (lo part)
  float m_run = -INFINITY;    // running max of head g (base 2)
  float l_part = 0.f;         // this thread's share of the running sum of head g
  bool seg_whole_start = false;
  bool q_ready = false;       // qv holds the q block of the next segment (loaded during a merge)
  int cprob = prob0, cj = j0; // uniform mode: consumer cursor
  // ldmatrix lanes: matrix mi = lane/8, row r8 = lane%8.  A stage tensor is a sequence of
  // sub-boxes of BR rows (BR = KPS, or the page size when pages are smaller), each holding its
  // rows of every 64-dim column chunk as [chunk][BR rows][128 B] with the 128-byte swizzle
  // (16-byte chunk ch of row r stored at ch ^ (r & 7)); every row below is 8-aligned plus r8.
  const int mi = lane >> 3, r8 = lane & 7;
  const int BRc = p.page_table ? min(p.page_size, KPS) : KPS;
  const uint32_t cstride = (uint32_t)BRc * 128;  // bytes between column chunks of a sub-box
  auto row_off = [&](int row) -> uint32_t {
    return (uint32_t)(row / BRc) * (NCB * cstride) + (uint32_t)(row % BRc) * 128;
  };
  // K (non-trans): matrices (keys 0-7 | 8-15) x (dims +0 | +8) of a 16-dim k-step.
  const uint32_t k_row = row_off(kg * 16 + r8 + 8 * (mi >> 1));
  const int k_chunk = (mi & 1) ^ r8;  // chunk of k-step 0; k-step ks adds 2*(ks&3) by XOR
  // V (trans): matrices (keys 0-7 | 8-15) x (dims +0 | +8) of a 16-dim pair of n-tiles.
  const uint32_t v_row = row_off(kg * 16 + r8 + 8 * (mi & 1));
  const int v_chunk = (mi >> 1) ^ r8;

  for (int it = 0; it < my_stages; it++) {
    if (warp == 0 && it + kStages - 1 < my_stages) issue(it + kStages - 1);
    const int slot = it % kStages;
    const uint32_t par = (it / kStages) & 1;
    StageMeta mt;
    if (uniform) {
      const uint32_t key0 = (ulo / KPS + (uint32_t)cj) * KPS;
      mt.problem = cprob;
      mt.key0 = (int)key0;
      mt.kfirst = (int)(max(ulo, key0) - key0);
      mt.kend = (int)(min(uhi, key0 + KPS) - key0);
      int fl = 0;
      if (it == 0 || cj == 0) fl |= F_SEG_FIRST;
      if (it == my_stages - 1 || cj == nstg - 1) fl |= F_SEG_LAST;
      if (cj == 0) fl |= F_PROB_FIRST;
      if (cj == nstg - 1) fl |= F_PROB_LAST;
      mt.flags = fl;
      mt.seg = (int)blockIdx.x + cprob;
      if (++cj == nstg) {
        cj = 0;
        cprob++;
      }
    }
    g4a::mbar_wait_bounded(&full[slot], par, p.err, G4A_DEVERR_WAIT_FULL);
    if (!uniform) mt = meta[slot];

    if (mt.flags & F_SEG_FIRST) {
      if (it > 0) {  // a later segment: its q block (the merge area is free again)
        if (!q_ready) load_q(mt.problem);
        q_ready = false;
        stage_q();
      }
#pragma unroll
      for (int n = 0; n < NT; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      m_run = -INFINITY;
      l_part = 0.f;
      seg_whole_start = (mt.flags & F_PROB_FIRST) != 0;
    }

    const int kb = kg * 16;
    if (kb < mt.kend && kb + 16 > mt.kfirst) {  // warp-uniform: the key group has a valid key
      const uint32_t sK = g4a::smem_u32(stage_base + (size_t)slot * C::STAGE_BYTES);
      const uint32_t sV = sK + NCB * CBB;
      // ---- partial scores of 16 keys over this warp's KPW k-steps (two n-tiles; even and odd
      // k-steps in separate accumulators to halve the MMA dependency chain)
      float sa0[4] = {0.f, 0.f, 0.f, 0.f}, sa1[4] = {0.f, 0.f, 0.f, 0.f};
      float sb0[4] = {0.f, 0.f, 0.f, 0.f}, sb1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < KPW; j += 2) {
        uint32_t b00, b01, b10, b11, c00, c01, c10, c11;
        const uint32_t box = sK + (dq * (KPW / 4) + (j >> 2)) * cstride + k_row;
        ldsm_x4(box + ((k_chunk ^ (2 * (j & 3))) << 4), b00, b01, b10, b11);
        ldsm_x4(box + ((k_chunk ^ (2 * ((j + 1) & 3))) << 4), c00, c01, c10, c11);
        mma_16816(sa0, qa[j][0], qa[j][1], qa[j][2], qa[j][3], b00, b01);
        mma_16816(sa1, qa[j][0], qa[j][1], qa[j][2], qa[j][3], b10, b11);
        mma_16816(sb0, qa[j + 1][0], qa[j + 1][1], qa[j + 1][2], qa[j + 1][3], c00, c01);
        mma_16816(sb1, qa[j + 1][0], qa[j + 1][1], qa[j + 1][2], qa[j + 1][3], c10, c11);
      }
      // keys 2c, 2c+1 (tile 0) and 8+2c, 9+2c (tile 1) of head g: hi row + lo row
      float4 mine = make_float4(sa0[0] + sa0[2] + sb0[0] + sb0[2], sa0[1] + sa0[3] + sb0[1] + sb0[3],
                                sa1[0] + sa1[2] + sb1[0] + sb1[2], sa1[1] + sa1[3] + sb1[1] + sb1[3]);
      // ---- sum the NDQ partials of this key group (fixed order: identical in every warp)
      float t[4] = {mine.x, mine.y, mine.z, mine.w};
      if (NDQ > 1) {
        float4* sxb = reinterpret_cast<float4*>(sx) + (size_t)(it & 1) * kWarps * 32;
        sxb[warp * 32 + lane] = mine;
        g4a::named_bar_sync(2 + kg, NDQ * 32);
        t[0] = t[1] = t[2] = t[3] = 0.f;
#pragma unroll
        for (int d2 = 0; d2 < NDQ; d2++) {
          const float4 x = sxb[(kg * NDQ + d2) * 32 + lane];
          t[0] += x.x;
          t[1] += x.y;
          t[2] += x.z;
          t[3] += x.w;
        }
      }
      const int kl[4] = {kb + 2 * c, kb + 2 * c + 1, kb + 8 + 2 * c, kb + 9 + 2 * c};
      bool ok[4];
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        ok[i] = kl[i] >= mt.kfirst && kl[i] < mt.kend;
        t[i] = ok[i] ? t[i] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, t[i]);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const bool need = mx > m_run + kLazyRescale;
      if (__any_sync(0xffffffffu, need)) {
        const float alpha = need ? ((m_run == -INFINITY) ? 0.f : g4a::fast_exp2(m_run - mx)) : 1.f;
        if (need) m_run = mx;
        l_part *= alpha;
#pragma unroll
        for (int n = 0; n < NT; n++) {
          o[n][0] *= alpha;
          o[n][1] *= alpha;
          o[n][2] *= alpha;
          o[n][3] *= alpha;
        }
      }
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        pr[i] = ok[i] ? g4a::fast_exp2(t[i] - m_run) : 0.f;
        l_part += pr[i];
      }
      float e0, e1, e2, e3;
      const uint32_t pa0 = pack_hi(pr[0], pr[1], e0, e1);
      const uint32_t pa1 = pack_f16(e0, e1);
      const uint32_t pa2 = pack_hi(pr[2], pr[3], e2, e3);
      const uint32_t pa3 = pack_f16(e2, e3);
      // ---- o += p * V over this warp's DPW output dims (NT/2 pairs of n-tiles).  The B
      // fragment halves of this thread belong to its own keys {2c, 2c+1} (b*0) and {8+2c, 9+2c}
      // (b*1); halves of keys outside the stage's valid range are zeroed.
      const uint32_t mlo = (ok[0] ? 0x0000ffffu : 0u) | (ok[1] ? 0xffff0000u : 0u);
      const uint32_t mhi = (ok[2] ? 0x0000ffffu : 0u) | (ok[3] ? 0xffff0000u : 0u);
#pragma unroll
      for (int np = 0; np < NT / 2; np++) {
        const int dim = dq * DPW + np * 16;  // first dim of the pair of n-tiles
        const uint32_t box = sV + (dim >> 6) * cstride + v_row;
        uint32_t b00, b01, b10, b11;
        ldsm_x4_trans(box + ((v_chunk ^ ((dim & 63) >> 3)) << 4), b00, b01, b10, b11);
        mma_16816(o[2 * np], pa0, pa1, pa2, pa3, b00 & mlo, b01 & mhi);
        mma_16816(o[2 * np + 1], pa0, pa1, pa2, pa3, b10 & mlo, b11 & mhi);
      }
    }
    __syncwarp();
    if (lane == 0) g4a::mbar_arrive(&empty[slot]);

    if (mt.flags & F_SEG_LAST) {
      // ---- merge the NKG key groups of each output slice (tree over shared memory).  The
      // first barrier orders the q reads of the merge area before the tree's writes.
      g4a::named_bar_sync(1, kThreads);
      // When another segment follows in this CTA, its q block is loaded now, so that the loads
      // are in flight during the merge instead of stalling every warp at the next segment's
      // start.  Its problem: the consumer cursor (uniform mode), or the metadata of stage it + 1,
      // which warp 0 wrote before the barrier above (it issues two stages ahead).
      if (it + 1 < my_stages) {
        load_q(uniform ? cprob : meta[(it + 1) % kStages].problem);
        q_ready = true;
      }
      float l_head = l_part;
      l_head += __shfl_xor_sync(0xffffffffu, l_head, 1);
      l_head += __shfl_xor_sync(0xffffffffu, l_head, 2);
      float ov[NT][2];
#pragma unroll
      for (int n = 0; n < NT; n++) {
        ov[n][0] = o[n][0] + o[n][2];
        ov[n][1] = o[n][1] + o[n][3];
      }
      float m_h = m_run;
#pragma unroll
      for (int stride = NKG / 2; stride >= 1; stride >>= 1) {
        if (kg >= stride && kg < 2 * stride) {
          float* sl = oslot + ((kg - stride) * NDQ + dq) * C::OSLOT;
#pragma unroll
          for (int n = 0; n < NT; n++)
            *reinterpret_cast<float2*>(sl + g * C::OSTRIDE + n * 8 + 2 * c) = make_float2(ov[n][0], ov[n][1]);
          if (c == 0) {
            sl[kGroup * C::OSTRIDE + g] = m_h;
            sl[kGroup * C::OSTRIDE + kGroup + g] = l_head;
          }
        }
        g4a::named_bar_sync(1, kThreads);
        if (kg < stride) {
          const float* sl = oslot + (kg * NDQ + dq) * C::OSLOT;
          const float mb = sl[kGroup * C::OSTRIDE + g];
          const float lb = sl[kGroup * C::OSTRIDE + kGroup + g];
          const float M = fmaxf(m_h, mb);
          const float wa = (m_h == -INFINITY) ? 0.f : g4a::fast_exp2(m_h - M);
          const float wb = (mb == -INFINITY) ? 0.f : g4a::fast_exp2(mb - M);
#pragma unroll
          for (int n = 0; n < NT; n++) {
            const float2 x = *reinterpret_cast<const float2*>(sl + g * C::OSTRIDE + n * 8 + 2 * c);
            ov[n][0] = ov[n][0] * wa + x.x * wb;
            ov[n][1] = ov[n][1] * wa + x.y * wb;
          }
          l_head = l_head * wa + lb * wb;
          m_h = M;
        }
        g4a::named_bar_sync(1, kThreads);
      }
      if (kg == 0) {
        const bool whole = seg_whole_start && (mt.flags & F_PROB_LAST);
        if (whole && p.out != nullptr) {
          const float inv = 1.0f / l_head;
          float* op = p.out + ((size_t)mt.problem * kGroup + g) * HD + dq * DPW + 2 * c;
#pragma unroll
          for (int n = 0; n < NT; n++)
            *reinterpret_cast<float2*>(op + n * 8) = make_float2(ov[n][0] * inv, ov[n][1] * inv);
        } else {
          float* part_row = p.part + (size_t)mt.seg * (kGroup * (HD + 2));
          float* op = part_row + 2 * kGroup + g * HD + dq * DPW + 2 * c;
#pragma unroll
          for (int n = 0; n < NT; n++) *reinterpret_cast<float2*>(op + n * 8) = make_float2(ov[n][0], ov[n][1]);
          if (dq == 0 && c == 0) {
            part_row[g] = m_h;
            part_row[kGroup + g] = l_head;
          }
        }
        if (warp == 0 && lane == 0) {
          if (seg_whole_start) p.seg_range[mt.problem].x = mt.seg;
          if (mt.flags & F_PROB_LAST) p.seg_range[mt.problem].y = mt.seg;
        }
      }
    }
  }
}

// Merge the segments of each problem: one CTA per (problem, head, 64 output dims), NW warps =
// 2 NW segment lanes x 16 float4 chunks.  Every thread issues the loads of up to kMergeBatch
// segments (m, l and a float4 of o) before using any of them, so up to 10 NW segments cost one
// memory round trip, and merges them with a log-sum-exp; the two segment lanes of a warp
// combine by shuffle, the NW warps through shared memory.  The grid is small (HD/64 x 8 CTAs per
// problem) and lets its dependents launch at once: the next call's decode CTAs take the SMs it
// leaves free and warm L2 with their first stages while this merge runs (they read nothing this
// kernel writes before their own PDL wait).  mode 0: normalised output rows (problems with a
// single segment were written by the main kernel); mode 1: one merged partial per problem.
constexpr int kMergeBatch = 5;

// 16-byte store, or four scalar stores when the destination is not 16-byte aligned.
__device__ __forceinline__ void store_f4(float* dst, float4 v) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    *reinterpret_cast<float4*>(dst) = v;
  } else {
    dst[0] = v.x;
    dst[1] = v.y;
    dst[2] = v.z;
    dst[3] = v.w;
  }
}

// NW warps: 16 for one problem (its segments are every active CTA), 2 for many problems (each
// split over a few CTAs), so a batch launches small CTAs that all fit in one wave.
template <int NW>
__global__ void __launch_bounds__(NW * 32) merge_segments_kernel(const DecodeParams p, int mode, float* part_out) {
  g4a::pdl_launch_dependents();
  // Everything up to the PDL wait depends on launch parameters only.
  const int prob = blockIdx.x, h = blockIdx.y;
  const int hd = p.hd;
  const int ch = threadIdx.x & 15;  // float4 chunk: output dims d .. d + 3
  const int sl = threadIdx.x >> 4;  // segment lane
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = blockIdx.z * 64 + ch * 4;
  const size_t prow = (size_t)kGroup * (hd + 2);
  float* po = (mode == 0) ? nullptr : part_out + (size_t)prob * prow;
  float* dst = (mode == 0) ? p.out + ((size_t)prob * kGroup + h) * hd + d : po + 2 * kGroup + (size_t)h * hd + d;
  const bool single = (p.B * p.nkh == 1);
  uint32_t lo = 0, hi = 0;
  int2 r = make_int2(0, 0);
  if (single) {  // one problem: its segments are the active CTAs 0 .. G-1
    key_range(p, 0, lo, hi);
    const uint32_t S = hi > lo ? (hi + p.kps - 1) / p.kps - lo / p.kps : 0;
    r = make_int2(0, (int)min((uint32_t)p.main_grid, S) - 1);
  }
  g4a::pdl_wait_primary();
  if (!single) key_range(p, prob / p.nkh, lo, hi);  // kv_lens may come from the preceding kernel
  if (hi <= lo) {  // no visible key: zeros (the reference's seq_len 0 output)
    if (sl == 0) {
      store_f4(dst, make_float4(0.f, 0.f, 0.f, 0.f));
      if (mode == 1 && ch == 0 && blockIdx.z == 0) {
        po[h] = -INFINITY;
        po[kGroup + h] = 0.f;
      }
    }
    return;
  }
  if (!single) r = p.seg_range[prob];
  if (mode == 0 && r.x == r.y) return;  // single segment: the main kernel wrote the row
  // The segment weights use the hardware exp2 (as the main kernel's softmax does): the merge is a
  // serial tail behind the main kernel, and exp2f's extra instructions cost 0.2 us of it at 32k.
  float M = -INFINITY, L = 0.f;
  float4 A = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int base = r.x + sl; base <= r.y; base += 2 * NW * kMergeBatch) {
    float mv[kMergeBatch], lv[kMergeBatch];
    float4 ov[kMergeBatch];
#pragma unroll
    for (int i = 0; i < kMergeBatch; i++) {
      const int s = base + 2 * NW * i;
      const float* row = p.part + (size_t)(s <= r.y ? s : r.x) * prow;
      mv[i] = __ldcg(row + h);
      lv[i] = __ldcg(row + kGroup + h);
      ov[i] = __ldcg(reinterpret_cast<const float4*>(row + 2 * kGroup + (size_t)h * hd + d));
      if (s > r.y) mv[i] = -INFINITY;
    }
    float Mn = M;
#pragma unroll
    for (int i = 0; i < kMergeBatch; i++) Mn = fmaxf(Mn, mv[i]);
    const float wa = (M == -INFINITY) ? 0.f : g4a::fast_exp2(M - Mn);
    A.x *= wa;
    A.y *= wa;
    A.z *= wa;
    A.w *= wa;
    L *= wa;
#pragma unroll
    for (int i = 0; i < kMergeBatch; i++) {
      const float w = (mv[i] == -INFINITY) ? 0.f : g4a::fast_exp2(mv[i] - Mn);
      A.x += w * ov[i].x;
      A.y += w * ov[i].y;
      A.z += w * ov[i].z;
      A.w += w * ov[i].w;
      L += w * lv[i];
    }
    M = Mn;
  }
  // the two segment lanes of this warp (lanes l and l ^ 16 hold the same chunk)
  {
    const float Mo = __shfl_xor_sync(0xffffffffu, M, 16);
    const float Lo = __shfl_xor_sync(0xffffffffu, L, 16);
    float4 Ao;
    Ao.x = __shfl_xor_sync(0xffffffffu, A.x, 16);
    Ao.y = __shfl_xor_sync(0xffffffffu, A.y, 16);
    Ao.z = __shfl_xor_sync(0xffffffffu, A.z, 16);
    Ao.w = __shfl_xor_sync(0xffffffffu, A.w, 16);
    const float Mn = fmaxf(M, Mo);
    const float wa = (M == -INFINITY) ? 0.f : g4a::fast_exp2(M - Mn);
    const float wb = (Mo == -INFINITY) ? 0.f : g4a::fast_exp2(Mo - Mn);
    A.x = A.x * wa + Ao.x * wb;
    A.y = A.y * wa + Ao.y * wb;
    A.z = A.z * wa + Ao.z * wb;
    A.w = A.w * wa + Ao.w * wb;
    L = L * wa + Lo * wb;
    M = Mn;
  }
  __shared__ float sM[NW][16], sL[NW][16];
  __shared__ float4 sA[NW][16];
  if (lane < 16) {
    sM[warp][lane] = M;
    sL[warp][lane] = L;
    sA[warp][lane] = A;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const int t = threadIdx.x;
    float Mt = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; w++) Mt = fmaxf(Mt, sM[w][t]);
    float Lt = 0.f;
    float4 At = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < NW; w++) {
      const float mw = sM[w][t];
      const float wt = (mw == -INFINITY) ? 0.f : g4a::fast_exp2(mw - Mt);
      const float4 a = sA[w][t];
      At.x += wt * a.x;
      At.y += wt * a.y;
      At.z += wt * a.z;
      At.w += wt * a.w;
      Lt += wt * sL[w][t];
    }
    if (mode == 0) {
      const float inv = 1.0f / Lt;
      store_f4(dst, make_float4(At.x * inv, At.y * inv, At.z * inv, At.w * inv));
    } else {
      store_f4(dst, At);
      if (t == 0 && blockIdx.z == 0) {
        po[h] = Mt;
        po[kGroup + h] = Lt;
      }
    }
  }
}

// ----------------------------------------------------------------------------- generic path
// Any NQH/NKH and head_dim (multiple of 8, <= 512): one CTA per (sequence, q head), 8 warps
// stride over keys with a warp-wide dot and an online softmax, then a shared-memory merge.
// Correct for every shape the reference's Params allow; the fast path above covers Gemma.
__global__ void __launch_bounds__(256) decode_generic_kernel(const DecodeParams p, int mode, float* part_out) {
  const int seq = blockIdx.x / p.nqh;
  const int h = blockIdx.x % p.nqh;
  const int kvh = h * p.nkh / p.nqh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int MAXD = 16;  // dims per lane (head_dim <= 512)
  uint32_t lo, hi;
  key_range(p, seq, lo, hi);
  const size_t qrow = ((size_t)seq * p.nqh + h) * p.hd;
  float qv[MAXD], o[MAXD];
#pragma unroll
  for (int i = 0; i < MAXD; i++) {
    const int d = lane + 32 * i;
    qv[i] = d < p.hd ? (p.q16 ? __half2float(p.q16[qrow + d]) : p.q[qrow + d]) : 0.f;
    o[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (uint32_t t = lo + warp; t < hi; t += 8) {
    const __half* kr = row_ptr(p, p.k, seq, kvh, t);
    if (!kr) {
      if (lane == 0 && p.err) atomicExch(p.err, G4A_DEVERR_PAGE);
      continue;
    }
    const __half* vr = p.v + (kr - p.k);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < MAXD; i++) {
      const int d = lane + 32 * i;
      if (d < p.hd) dot += qv[i] * __half2float(kr[d]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const float s = dot * p.scale_log2;
    const float mn = fmaxf(m, s);
    const float a = (m == -INFINITY) ? 0.f : exp2f(m - mn);
    const float e = exp2f(s - mn);
    l = l * a + e;
#pragma unroll
    for (int i = 0; i < MAXD; i++) {
      const int d = lane + 32 * i;
      o[i] = o[i] * a + (d < p.hd ? e * __half2float(vr[d]) : 0.f);
    }
    m = mn;
  }
  __shared__ float sm[8], sl[8];
  __shared__ float so[8][512];
  if (lane == 0) {
    sm[warp] = m;
    sl[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < MAXD; i++) {
    const int d = lane + 32 * i;
    if (d < p.hd) so[warp][d] = o[i];
  }
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < 8; w++) M = fmaxf(M, sm[w]);
  float L = 0.f;
  for (int w = 0; w < 8; w++) L += (sm[w] == -INFINITY) ? 0.f : exp2f(sm[w] - M) * sl[w];
  for (int d = threadIdx.x; d < p.hd; d += 256) {
    float acc = 0.f;
    for (int w = 0; w < 8; w++) acc += (sm[w] == -INFINITY) ? 0.f : exp2f(sm[w] - M) * so[w][d];
    if (mode == 0) {
      p.out[((size_t)seq * p.nqh + h) * p.hd + d] = (L > 0.f) ? acc / L : 0.f;
    } else {
      // partial layout with nqh heads: m[nqh] | l[nqh] | o[nqh, hd]
      float* po = part_out + (size_t)seq * p.nqh * (p.hd + 2);
      po[2 * p.nqh + (size_t)h * p.hd + d] = acc;
      if (d == 0) {
        po[h] = M;
        po[p.nqh + h] = L;
      }
    }
  }
}

// LSE merge of n parts of nqh*(hd+2) floats: grid (nqh), block 256.
__global__ void __launch_bounds__(256) lse_merge_kernel(const float* parts, int n, int nqh, int hd, float* out) {
  const int h = blockIdx.x;
  const size_t prow = (size_t)nqh * (hd + 2);
  float M = -INFINITY;
  for (int r = 0; r < n; r++) M = fmaxf(M, parts[r * prow + h]);
  float L = 0.f;
  for (int r = 0; r < n; r++) {
    const float mr = parts[r * prow + h];
    if (mr != -INFINITY) L += exp2f(mr - M) * parts[r * prow + nqh + h];
  }
  for (int d = threadIdx.x; d < hd; d += 256) {
    float acc = 0.f;
    for (int r = 0; r < n; r++) {
      const float mr = parts[r * prow + h];
      if (mr != -INFINITY) acc += exp2f(mr - M) * parts[r * prow + 2 * nqh + (size_t)h * hd + d];
    }
    out[(size_t)h * hd + d] = (L > 0.f) ? acc / L : 0.f;
  }
}

// ----------------------------------------------------------------------------- host side

bool fast_path_ok(uint32_t nqh, uint32_t nkh, uint32_t hd) {
  return nkh > 0 && nqh == kGroup * nkh && (hd == 128 || hd == 256 || hd == 512);
}

int kps_of(uint32_t hd);

// The paged fast path loads page-aligned boxes: pages must tile stages (or stages pages).
bool paged_fast_ok(uint32_t page_size, uint32_t hd) {
  const uint32_t kps = (uint32_t)kps_of(hd);
  return page_size >= 8 && page_size <= 256 * 1024 && (page_size % kps == 0 || kps % page_size == 0);
}

template <int HD, bool SHORT>
g4a_status configure_kernel(g4a_ctx* ctx) {
  // Per-device flags, atomic because several host threads may make their first call at once
  // (setting the attribute twice is harmless).
  static std::atomic<bool> done[64];
  if (ctx->device < 64 && done[ctx->device].load(std::memory_order_acquire)) return G4A_OK;
  cudaError_t e = cudaFuncSetAttribute(decode_splitkv_kernel<HD, SHORT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)Cfg<HD, SHORT>::SMEM);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaFuncSetAttribute(decode_splitkv_kernel)");
  if (ctx->device < 64) done[ctx->device].store(true, std::memory_order_release);
  return G4A_OK;
}

// Resolve cuTensorMapEncodeTiled from the driver once per context (no link-time libcuda).
g4a_status get_encoder(g4a_ctx* ctx, PFN_cuTensorMapEncodeTiled_v12000* out) {
  if (!ctx->encode_tiled) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return g4a_fail(G4A_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    ctx->encode_tiled = fn;
  }
  *out = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ctx->encode_tiled);
  return G4A_OK;
}

// Tensor maps of the K and V caches.  The 64-element column chunk of a row is the innermost
// dimension and the chunk index the outermost one (stride 128 B), so one box of {64, rows, HD/64
// chunks} lands in shared memory as HD/64 column boxes of [rows x 128 B] -- the layout the
// consumers read -- with the 128-byte swizzle, and a stage costs one TMA op per tensor.
// Contiguous: {64, nkh, rows, chunks}; paged: {64, nkh, page_size, num_pages, chunks}.
// Elements outside the tensor are zero-filled.
g4a_status encode_kv_maps(g4a_ctx* ctx, const DecodeParams& p, int kps, uint64_t rows, CUtensorMap* mk,
                          CUtensorMap* mv) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (g4a_status s = get_encoder(ctx, &enc)) return s;
  const cuuint64_t hd = (cuuint64_t)p.hd, nkh = (cuuint64_t)p.nkh, ncb = hd / 64;
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5], estr[5] = {1, 1, 1, 1, 1};
  cuuint32_t rank;
  if (p.page_table) {
    rank = 5;
    dims[0] = 64; dims[1] = nkh; dims[2] = (cuuint64_t)p.page_size; dims[3] = (cuuint64_t)p.num_pages; dims[4] = ncb;
    strides[0] = hd * 2; strides[1] = nkh * hd * 2; strides[2] = (cuuint64_t)p.page_size * nkh * hd * 2; strides[3] = 128;
    box[0] = 64; box[1] = 1; box[2] = (cuuint32_t)std::min(p.page_size, kps); box[3] = 1; box[4] = (cuuint32_t)ncb;
  } else {
    rank = 4;
    dims[0] = 64; dims[1] = nkh; dims[2] = rows; dims[3] = ncb;
    strides[0] = hd * 2; strides[1] = nkh * hd * 2; strides[2] = 128;
    box[0] = 64; box[1] = 1; box[2] = (cuuint32_t)kps; box[3] = (cuuint32_t)ncb;
  }
  for (int t = 0; t < 2; t++) {
    CUresult r = enc(t ? mv : mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<__half*>(t ? p.v : p.k), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return g4a_fail(G4A_ECUDA, "cuTensorMapEncodeTiled failed (%d) for the %s cache", (int)r, t ? "V" : "K");
  }
  return G4A_OK;
}

// A scratch area of fixed size supplied by the caller instead of the context's growable
// workspace (used by g4a_decode_attn_noalloc).
struct FixedScratch {
  void* ptr;
  size_t bytes;
  const char* who;  // entry-point name for error messages
};

template <int HD, bool SHORT>
g4a_status launch_fast(g4a_ctx* ctx, DecodeParams& p, long long stages_upper, int mode, float* part_out, bool pdl,
                       const FixedScratch* fixed, bool balance) {
  using C = Cfg<HD, SHORT>;
  if (g4a_status s = configure_kernel<HD, SHORT>(ctx)) return s;
  const int P = p.B * p.nkh;
  int grid = (int)std::min<long long>(stages_upper + P, (long long)ctx->num_sms);
  if (grid < 1) grid = 1;
  // One sequence of up to kBalancedMaxStages stages per SM: launch ceil(S / k) CTAs for
  // k = ceil(S / SMs), so that every CTA gets k or k - 1 whole stages instead of a few CTAs
  // running one more stage after the rest are done, and the SMs left over take the merge kernel's
  // CTAs as soon as it launches.  Measured per layer-call (graph replay): 32k 11.8 -> 10.9 us,
  // 8k 8.0 -> 7.3, 24k 10.7 -> 9.9, 48k 14.5 -> 13.5; from ~10 stages per SM on it no longer
  // pays (96k: 21.1 -> 21.2 us), so longer calls keep one CTA per SM.  Right behind the layer
  // entries' producer kernel the same grid measured slower (end to end at 32k 19.9 -> 20.7 us),
  // so those calls do not ask for it.
  if (balance && P == 1 && stages_upper > grid) {
    const long long k = (stages_upper + grid - 1) / grid;
    if (k <= kBalancedMaxStages) grid = (int)((stages_upper + k - 1) / k);
  }
  const size_t prow = (size_t)kGroup * (HD + 2) * sizeof(float);
  const size_t segs = (size_t)grid + (size_t)P + 1;
  const size_t part_bytes = (segs * prow + 255) & ~size_t(255);
  const size_t need = part_bytes + (size_t)P * sizeof(int2) + 256;
  char* ws;
  if (fixed) {  // caller-provided scratch of fixed size: never grown
    if (need > fixed->bytes)
      return g4a_fail(G4A_EINVAL,
                      "%s: this call needs %zu bytes of split-KV scratch (num_kv_heads %d, head_dim %d, %d CTAs) "
                      "but the fixed scratch area holds %zu bytes",
                      fixed->who, need, p.nkh, HD, grid, fixed->bytes);
    ws = static_cast<char*>(fixed->ptr);
  } else {
    if (g4a_status s = g4a_ensure_workspace(ctx, need)) return s;
    ws = static_cast<char*>(ctx->workspace);
  }
  p.part = reinterpret_cast<float*>(ws);
  p.seg_range = reinterpret_cast<int2*>(ws + part_bytes);
  p.err = ctx->dev_err_dev;
  p.kps = C::KPS;
  p.main_grid = grid;
  if (stages_upper > 0) {
    // rows held by a contiguous buffer: positions [row_base, min(kv_end, kv_len))
    const uint64_t end = std::min<uint64_t>(p.kv_end, p.kv_len_scalar);
    const uint64_t rows = end > p.row_base ? end - p.row_base : 1;
    CUtensorMap mk, mv;
    if (g4a_status s = encode_kv_maps(ctx, p, C::KPS, rows, &mk, &mv)) return s;
    g4a_prof_scope ps(ctx, G4A_PROF_DECODE_SPLITKV);
    cudaError_t e =
        g4a_launch(decode_splitkv_kernel<HD, SHORT>, dim3(grid), dim3(kThreads), C::SMEM, ctx->stream, pdl, p, mk, mv);
    if (e != cudaSuccess) return g4a_cuda_fail(e, "launch decode_splitkv_kernel");
  }
  // The merge kernel is needed when a problem can span several CTAs, for zero-length problems,
  // and always in partial mode.
  const bool need_merge = (mode == 1) || grid > 1 || stages_upper == 0 || P > 1;
  if (need_merge) {
    g4a_prof_scope ps(ctx, G4A_PROF_DECODE_MERGE);
    cudaError_t e = (P == 1)
                        ? g4a_launch(merge_segments_kernel<16>, dim3(P, kGroup, HD / 64), dim3(512), 0, ctx->stream,
                                     stages_upper > 0, p, mode, part_out)
                        : g4a_launch(merge_segments_kernel<2>, dim3(P, kGroup, HD / 64), dim3(64), 0, ctx->stream,
                               stages_upper > 0, p, mode, part_out);
    if (e != cudaSuccess) return g4a_cuda_fail(e, "launch merge_segments_kernel");
  }
  return G4A_OK;
}

// keys_upper: an upper bound on the total number of visible (problem, key) pairs.
g4a_status dispatch_fast(g4a_ctx* ctx, DecodeParams& p, long long keys_upper, int mode, float* part_out, bool pdl,
                         const FixedScratch* fixed = nullptr, bool balance = false) {
  switch (p.hd) {
    // Calls whose regular stages would leave SMs idle use the half-size stages.
    case 128: {
      const long long st = (keys_upper + Cfg<128>::KPS - 1) / Cfg<128>::KPS;
      if (st < ctx->num_sms)
        return launch_fast<128, true>(ctx, p, (keys_upper + Cfg<128, true>::KPS - 1) / Cfg<128, true>::KPS, mode,
                                      part_out, pdl, fixed, balance);
      return launch_fast<128, false>(ctx, p, st, mode, part_out, pdl, fixed, balance);
    }
    case 256: {
      const long long st = (keys_upper + Cfg<256>::KPS - 1) / Cfg<256>::KPS;
      if (st < ctx->num_sms)
        return launch_fast<256, true>(ctx, p, (keys_upper + Cfg<256, true>::KPS - 1) / Cfg<256, true>::KPS, mode,
                                      part_out, pdl, fixed, balance);
      return launch_fast<256, false>(ctx, p, st, mode, part_out, pdl, fixed, balance);
    }
    case 512:
      return launch_fast<512, false>(ctx, p, (keys_upper + Cfg<512>::KPS - 1) / Cfg<512>::KPS, mode, part_out, pdl,
                                     fixed, balance);
    default:
      return g4a_fail(G4A_EINVAL, "decode: unsupported head_dim %d", p.hd);
  }
}

int kps_of(uint32_t hd) { return hd == 512 ? Cfg<512>::KPS : hd == 256 ? Cfg<256>::KPS : Cfg<128>::KPS; }

g4a_status check_common(const char* fn, const void* q, const void* k, const void* v, const void* out, uint32_t nqh,
                        uint32_t nkh, uint32_t hd) {
  if (!q || !k || !v || !out) return g4a_fail(G4A_EINVAL, "%s: null pointer", fn);
  if (nqh == 0 || nkh == 0 || nkh > nqh) return g4a_fail(G4A_EINVAL, "%s: bad head counts nqh=%u nkh=%u", fn, nqh, nkh);
  if (hd == 0 || hd > 512 || (hd % 8) != 0)
    return g4a_fail(G4A_EINVAL, "%s: head_dim %u must be a multiple of 8 in [8, 512]", fn, hd);
  if (((uintptr_t)k | (uintptr_t)v) & 15u) return g4a_fail(G4A_EINVAL, "%s: cache pointers must be 16-byte aligned", fn);
  if ((uintptr_t)q & 15u) return g4a_fail(G4A_EINVAL, "%s: q must be 16-byte aligned", fn);
  return G4A_OK;
}

DecodeParams base_params(const float* q, const uint16_t* k, const uint16_t* v, uint32_t nqh, uint32_t nkh, uint32_t hd,
                         float scale, uint32_t window, float* out) {
  DecodeParams p = {};
  p.q = q;
  p.k = reinterpret_cast<const __half*>(k);
  p.v = reinterpret_cast<const __half*>(v);
  p.nqh = (int)nqh;
  p.nkh = (int)nkh;
  p.hd = (int)hd;
  p.scale_log2 = scale * kLog2e;
  p.window = window;
  p.row_base = 0;
  p.kv_end = 0xffffffffu;
  p.out = out;
  return p;
}

g4a_status decode_contiguous(g4a_ctx* ctx, const float* q, const uint16_t* k, const uint16_t* v, float* out,
                             uint32_t nqh, uint32_t nkh, uint32_t hd, uint32_t kv_len, float scale, uint32_t window,
                             bool after_producer, const FixedScratch* fixed = nullptr) {
  DecodeParams p = base_params(q, k, v, nqh, nkh, hd, scale, window, out);
  p.B = 1;
  p.kv_len_scalar = kv_len;
  p.err = ctx->dev_err_dev;
  const uint32_t ws = (window != 0u && kv_len > window) ? kv_len - window : 0u;
  const long long keys = (long long)(kv_len - ws);
  if (fast_path_ok(nqh, nkh, hd))
    return dispatch_fast(ctx, p, keys * nkh + (long long)(nkh - 1) * kps_of(hd), 0, nullptr, true, fixed,
                         !after_producer);
  g4a_prof_scope ps(ctx, G4A_PROF_DECODE_GENERIC);
  decode_generic_kernel<<<nqh, 256, 0, ctx->stream>>>(p, 0, nullptr);
  return g4a_check_launch("decode_generic_kernel");
}

}  // namespace

// Fixed split-KV scratch of g4a_decode_attn_noalloc: enough for every single-sequence decode
// with num_kv_heads <= 64 at head_dim <= 512 on a 148-SM B200 ((148 + 64 + 1) rows of
// 8 * 514 floats, plus 64 segment ranges).  It occupies this much device memory on every device
// the library's module is loaded on.
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g4a_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::atomic<void*> g_noalloc_address[kMaxDevices];

// Device address of g4a_noalloc_scratch on `device`, looked up once per device with that device
// current (the caller's current device is restored afterwards, and a failure to restore it is
// reported).  The address is cached for the life of the process; it does not survive a
// cudaDeviceReset of that device.
g4a_status noalloc_scratch_address(int device, void** out) {
  if (device < 0 || device >= kMaxDevices) return g4a_fail(G4A_EINVAL, "noalloc scratch: device %d out of range", device);
  void* ptr = g_noalloc_address[device].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    int prev = -1;
    G4A_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != device) G4A_CUDA_TRY(cudaSetDevice(device));
    cudaError_t e = cudaGetSymbolAddress(&ptr, g4a_noalloc_scratch);
    const cudaError_t restore = (prev != device) ? cudaSetDevice(prev) : cudaSuccess;
    if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaGetSymbolAddress(g4a_noalloc_scratch)");
    if (restore != cudaSuccess) return g4a_cuda_fail(restore, "cudaSetDevice (restoring the caller's device)");
    if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 255u) != 0)
      return g4a_fail(G4A_ECUDA, "noalloc scratch: unexpected symbol address %p", ptr);
    g_noalloc_address[device].store(ptr, std::memory_order_release);
  }
  *out = ptr;
  return G4A_OK;
}

}  // namespace

// Prefill through the decode kernels, for shapes the tensor-core prefill kernel does not cover
// (head_dim 512 of Gemma's global layers, GQA ratios other than 8): prompt token i is one decode
// problem over the shared cache with kv_len = start_pos + i + 1 and the window measured from it,
// which is exactly the row the reference's per-token prefill (src/engine.ts:2460-2479) computes.
// The queries are read as f16.  Every problem re-reads its keys (from L2 for prompts whose cache
// fits), so this path is several times slower than the tensor-core kernel.
namespace {
__global__ void seq_lens_kernel(int* lens, uint32_t n, uint32_t first) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) lens[i] = (int)(first + i);
}
}  // namespace

g4a_status prefill_via_decode(g4a_ctx* ctx, const uint16_t* q16, const uint16_t* k, const uint16_t* v, float* out,
                              uint32_t T, uint32_t start_pos, uint32_t nqh, uint32_t nkh, uint32_t hd, float scale,
                              uint32_t window) {
  if (T > (uint32_t)0x7fffffff) return g4a_fail(G4A_EINVAL, "g4a_prefill_attn: T too large");
  if (ctx->seq_lens_cap < T) {
    // Growing must not free memory that queued kernels still read.
    G4A_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    if (ctx->seq_lens) cudaFree(ctx->seq_lens);
    ctx->seq_lens = nullptr;
    ctx->seq_lens_cap = 0;
    const size_t cap = std::max<size_t>(T, 4096);
    cudaError_t e = cudaMalloc((void**)&ctx->seq_lens, cap * sizeof(int));
    if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaMalloc(prefill sequence lengths)");
    ctx->seq_lens_cap = cap;
  }
  seq_lens_kernel<<<(T + 255) / 256, 256, 0, ctx->stream>>>(ctx->seq_lens, T, start_pos + 1u);
  if (g4a_status st = g4a_check_launch("seq_lens_kernel")) return st;
  DecodeParams p = base_params(nullptr, k, v, nqh, nkh, hd, scale, window, out);
  p.q16 = reinterpret_cast<const __half*>(q16);
  p.B = (int)T;
  p.kv_lens = ctx->seq_lens;
  p.kv_len_scalar = start_pos + T;  // rows of the cache the tensor maps cover
  p.err = ctx->dev_err_dev;
  if (fast_path_ok(nqh, nkh, hd)) {
    // visible keys: sum over L = start_pos + 1 .. start_pos + T of min(W, L)
    const long long a = (long long)start_pos + 1, b = (long long)start_pos + T;
    long long keys;
    if (window == 0u || (long long)window >= b) {
      keys = (a + b) * (long long)T / 2;
    } else if ((long long)window < a) {
      keys = (long long)window * T;
    } else {
      keys = (a + window) * ((long long)window - a + 1) / 2 + (long long)window * (b - window);
    }
    keys = keys * nkh + (long long)T * nkh * kps_of(hd);
    return dispatch_fast(ctx, p, keys, 0, nullptr, true);
  }
  g4a_prof_scope ps(ctx, G4A_PROF_DECODE_GENERIC);
  decode_generic_kernel<<<(unsigned)((size_t)T * nqh), 256, 0, ctx->stream>>>(p, 0, nullptr);
  return g4a_check_launch("decode_generic_kernel");
}

extern "C" {

g4a_status g4a_reserve_workspace(g4a_ctx* ctx, uint32_t max_batch, uint32_t head_dim, uint32_t num_q_heads) {
  G4A_CHECK_CTX(ctx);
  const size_t heads = num_q_heads < (uint32_t)kGroup ? (size_t)kGroup : num_q_heads;
  const size_t prow = heads * (head_dim + 2) * sizeof(float);
  const size_t segs = (size_t)ctx->num_sms + (size_t)max_batch * heads + 1;
  return g4a_ensure_workspace(ctx, ((segs * prow + 255) & ~size_t(255)) + (size_t)max_batch * heads * sizeof(int2) + 512);
}

g4a_status g4a_decode_attn(g4a_ctx* ctx, const float* q, const uint16_t* k_cache, const uint16_t* v_cache, float* out,
                           uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim, uint32_t kv_len,
                           float scale, uint32_t sliding_window) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_common(__func__, q, k_cache, v_cache, out, num_q_heads, num_kv_heads, head_dim)) return s;
  return decode_contiguous(ctx, q, k_cache, v_cache, out, num_q_heads, num_kv_heads, head_dim, kv_len, scale,
                           sliding_window, false);
}

g4a_status g4a_decode_attn_paged(g4a_ctx* ctx, const float* q, const uint16_t* k_pages, const uint16_t* v_pages,
                                 const int32_t* page_table, const int32_t* kv_lens, const int32_t* host_kv_lens,
                                 uint32_t batch, uint32_t page_size, uint32_t max_pages_per_seq, uint32_t num_pages,
                                 uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim, float scale,
                                 uint32_t sliding_window, float* out) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_common(__func__, q, k_pages, v_pages, out, num_q_heads, num_kv_heads, head_dim)) return s;
  if (batch == 0) return G4A_OK;
  if (!page_table || !kv_lens) return g4a_fail(G4A_EINVAL, "g4a_decode_attn_paged: null page_table or kv_lens");
  if (page_size == 0 || max_pages_per_seq == 0 || num_pages == 0)
    return g4a_fail(G4A_EINVAL, "g4a_decode_attn_paged: zero page_size / max_pages_per_seq / num_pages");
  if ((uint64_t)page_size * max_pages_per_seq > 0x7fffffffull)
    return g4a_fail(G4A_EINVAL, "g4a_decode_attn_paged: page_size * max_pages_per_seq exceeds 2^31");
  DecodeParams p = base_params(q, k_pages, v_pages, num_q_heads, num_kv_heads, head_dim, scale, sliding_window, out);
  p.B = (int)batch;
  p.kv_lens = kv_lens;
  p.page_table = page_table;
  p.page_size = (int)page_size;
  p.max_pages = (int)max_pages_per_seq;
  p.num_pages = (int)num_pages;
  p.err = ctx->dev_err_dev;
  if (fast_path_ok(num_q_heads, num_kv_heads, head_dim) && paged_fast_ok(page_size, head_dim)) {
    long long keys = 0;
    const uint64_t cap = (uint64_t)page_size * max_pages_per_seq;
    for (uint32_t b = 0; b < batch; b++) {
      uint64_t L = host_kv_lens ? (uint64_t)(host_kv_lens[b] < 0 ? 0 : host_kv_lens[b]) : cap;
      if (L > cap) L = cap;
      const uint64_t ws = (sliding_window != 0u && L > sliding_window) ? L - sliding_window : 0u;
      keys += (long long)(L - ws);
    }
    // Stages are counted per problem: pad one stage per problem for ragged tails.
    keys = keys * num_kv_heads + (long long)batch * num_kv_heads * kps_of(head_dim);
    return dispatch_fast(ctx, p, keys, 0, nullptr, true);
  }
  g4a_prof_scope ps(ctx, G4A_PROF_DECODE_GENERIC);
  decode_generic_kernel<<<batch * num_q_heads, 256, 0, ctx->stream>>>(p, 0, nullptr);
  return g4a_check_launch("decode_generic_kernel");
}

g4a_status g4a_decode_attn_partial(g4a_ctx* ctx, const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                   uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim, uint32_t kv_begin,
                                   uint32_t kv_end, uint32_t kv_len_total, float scale, uint32_t sliding_window,
                                   float* part) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_common(__func__, q, k_cache, v_cache, part, num_q_heads, num_kv_heads, head_dim)) return s;
  if (kv_end < kv_begin) return g4a_fail(G4A_EINVAL, "g4a_decode_attn_partial: kv_end < kv_begin");
  DecodeParams p = base_params(q, k_cache, v_cache, num_q_heads, num_kv_heads, head_dim, scale, sliding_window, nullptr);
  p.B = 1;
  p.kv_len_scalar = kv_len_total;
  p.row_base = kv_begin;
  p.kv_end = kv_end;
  p.err = ctx->dev_err_dev;
  const uint32_t ws = (sliding_window != 0u && kv_len_total > sliding_window) ? kv_len_total - sliding_window : 0u;
  const uint32_t lo = ws > kv_begin ? ws : kv_begin;
  const uint32_t hi = kv_len_total < kv_end ? kv_len_total : kv_end;
  const long long keys = hi > lo ? (long long)(hi - lo) : 0;
  if (num_kv_heads == 1 && fast_path_ok(num_q_heads, num_kv_heads, head_dim))
    return dispatch_fast(ctx, p, keys, 1, part, true, nullptr, true);
  g4a_prof_scope ps(ctx, G4A_PROF_DECODE_GENERIC);
  decode_generic_kernel<<<num_q_heads, 256, 0, ctx->stream>>>(p, 1, part);
  return g4a_check_launch("decode_generic_kernel(partial)");
}

g4a_status g4a_lse_merge(g4a_ctx* ctx, const float* parts, uint32_t n_parts, uint32_t num_q_heads, uint32_t head_dim,
                         float* out) {
  G4A_CHECK_CTX(ctx);
  if (!parts || !out) return g4a_fail(G4A_EINVAL, "g4a_lse_merge: null pointer");
  if (n_parts == 0 || num_q_heads == 0 || head_dim == 0)
    return g4a_fail(G4A_EINVAL, "g4a_lse_merge: n_parts, num_q_heads and head_dim must be > 0");
  g4a_prof_scope ps(ctx, G4A_PROF_LSE_MERGE);
  lse_merge_kernel<<<num_q_heads, 256, 0, ctx->stream>>>(parts, (int)n_parts, (int)num_q_heads, (int)head_dim, out);
  return g4a_check_launch("lse_merge_kernel");
}

// Allocation-free variant of g4a_decode_attn (no counterpart in the reference).  The split-KV
// partial rows and segment ranges live in g4a_noalloc_scratch below instead of the context's
// workspace, which g4a_decode_attn grows with cudaMalloc on first use and for larger shapes.
// Nothing in the scratch needs to start at zero: the main kernel writes every partial row and
// segment range before the merge kernel reads it.  The first call on each device looks up the
// scratch address (cudaGetSymbolAddress, with that device current); make that first call
// before capturing a stream.  Calls that overlap in time on one device share the scratch and
// race.
g4a_status g4a_decode_attn_noalloc(g4a_ctx* ctx, const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                   float* out, uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim,
                                   uint32_t kv_len, float scale, uint32_t sliding_window) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_common(__func__, q, k_cache, v_cache, out, num_q_heads, num_kv_heads, head_dim)) return s;
  if (ctx->prof_enabled)
    return g4a_fail(G4A_EINVAL, "%s: the per-launch profiler creates CUDA events; disable it for this call", __func__);
  void* scratch = nullptr;
  if (g4a_status s = noalloc_scratch_address(ctx->device, &scratch)) return s;
  const FixedScratch fixed = {scratch, kNoAllocScratchBytes, __func__};
  return decode_contiguous(ctx, q, k_cache, v_cache, out, num_q_heads, num_kv_heads, head_dim, kv_len, scale,
                           sliding_window, false, &fixed);
}

}  // extern "C"

// Producer stage launcher lives in g4a_producers.cu.
g4a_status g4a_launch_decode_prep(g4a_ctx* ctx, const float* sq, const float* sk, const float* sv, float* q,
                                  float* k, float* v, const uint16_t* qw, const uint16_t* kw,
                                  const uint16_t* rope_freqs, uint16_t* k_cache, uint16_t* v_cache, uint32_t nqh,
                                  uint32_t nkh, uint32_t hd, float eps, uint32_t position, uint32_t slot, float theta,
                                  uint32_t apply_div, bool is_producer);

extern "C" g4a_status g4a_attn_decode_layer(g4a_ctx* ctx, float* q, float* k, float* v, const uint16_t* q_norm_w,
                                            const uint16_t* k_norm_w, const uint16_t* rope_freqs, uint16_t* k_cache,
                                            uint16_t* v_cache, float* out, uint32_t num_q_heads,
                                            uint32_t num_kv_heads, uint32_t head_dim, float eps, uint32_t position,
                                            uint32_t slot, uint32_t kv_len, uint32_t max_seq_len, float theta,
                                            uint32_t apply_divisor, float scale, uint32_t sliding_window,
                                            uint32_t is_producer) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_common(__func__, q, k_cache, v_cache, out, num_q_heads, num_kv_heads, head_dim)) return s;
  if (!q_norm_w || (is_producer && (!k || !v || !k_norm_w)))
    return g4a_fail(G4A_EINVAL, "g4a_attn_decode_layer: null norm weight or k/v");
  if (apply_divisor && !rope_freqs)
    return g4a_fail(G4A_EINVAL, "g4a_attn_decode_layer: apply_divisor without rope_freqs");
  if (is_producer && slot >= max_seq_len)
    return g4a_fail(G4A_EINVAL, "g4a_attn_decode_layer: slot %u >= max_seq_len %u", slot, max_seq_len);
  if (kv_len > max_seq_len)
    return g4a_fail(G4A_EINVAL, "g4a_attn_decode_layer: kv_len %u > max_seq_len %u", kv_len, max_seq_len);
  if (g4a_status s = g4a_launch_decode_prep(ctx, nullptr, nullptr, nullptr, q, k, v, q_norm_w, k_norm_w, rope_freqs,
                                            k_cache, v_cache,
                                            num_q_heads, num_kv_heads, head_dim, eps, position, slot, theta,
                                            apply_divisor, is_producer != 0))
    return s;
  return decode_contiguous(ctx, q, k_cache, v_cache, out, num_q_heads, num_kv_heads, head_dim, kv_len, scale,
                           sliding_window, true);
}

namespace {

// Copies n4 float4 between device memory and pinned host memory mapped into the device's
// address space, as a kernel on the context's stream instead of a copy-engine transfer (which
// would break the programmatic-launch chain of the layer's kernels).  Host to device: the host
// data does not depend on the preceding kernel, so it is loaded before the wait, and stored to
// the device buffer (which the preceding call's kernels may still read) after it.  Device to
// host: the wait comes first (the source is the preceding kernel's output).
__global__ void __launch_bounds__(256) io_copy_kernel(const float4* __restrict__ src, float4* __restrict__ dst,
                                                      uint32_t n4, int src_is_host) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (src_is_host) {
    if (i < n4) v = src[i];
    g4a::pdl_wait_primary();
  } else {
    g4a::pdl_wait_primary();
    if (i < n4) v = __ldcg(src + i);
  }
  if (i < n4) dst[i] = v;
  g4a::pdl_launch_dependents();
}

// The device address of `host` if it is pinned host memory the device can reach, else nullptr.
void* mapped_host_address(const void* host) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, host) != cudaSuccess) {
    (void)cudaGetLastError();  // clear the (non-sticky) error of the query
    return nullptr;
  }
  return (a.type == cudaMemoryTypeHost && a.devicePointer) ? a.devicePointer : nullptr;
}

// dst <- src (bytes) on the context's stream: the copy kernel when the host side is mapped
// pinned memory and both sides are 16-byte aligned, else cudaMemcpyAsync.  (Used by
// g4a_attn_decode_layer_io when only one of its host buffers is mapped.)
g4a_status io_copy(g4a_ctx* ctx, void* dst, const void* src, size_t bytes, bool to_device) {
  const void* host = to_device ? src : dst;
  void* mapped = mapped_host_address(host);
  const bool aligned = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | bytes) & 15u) == 0;
  if (mapped && aligned && bytes / 16 <= 0xffffffffull) {
    const uint32_t n4 = (uint32_t)(bytes / 16);
    const void* s = to_device ? mapped : src;
    void* d = to_device ? dst : mapped;
    const cudaError_t e = g4a_launch(io_copy_kernel, dim3((n4 + 255) / 256), dim3(256), 0, ctx->stream, true,
                                     reinterpret_cast<const float4*>(s), reinterpret_cast<float4*>(d), n4,
                                     to_device ? 1 : 0);
    if (e != cudaSuccess) return g4a_cuda_fail(e, "launch io_copy_kernel");
    return G4A_OK;
  }
  G4A_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, to_device ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost,
                               ctx->stream));
  return G4A_OK;
}

}  // namespace

extern "C" g4a_status g4a_attn_decode_layer_io(g4a_ctx* ctx, const float* qkv_host, float* qkv_dev, float* out_dev,
                                               float* out_host, const uint16_t* q_norm_w, const uint16_t* k_norm_w,
                                               const uint16_t* rope_freqs, uint16_t* k_cache, uint16_t* v_cache,
                                               uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim,
                                               float eps, uint32_t position, uint32_t slot, uint32_t kv_len,
                                               uint32_t max_seq_len, float theta, uint32_t apply_divisor,
                                               float scale, uint32_t sliding_window, uint32_t is_producer) {
  G4A_CHECK_CTX(ctx);
  if (!qkv_host || !qkv_dev || !out_dev || !out_host)
    return g4a_fail(G4A_EINVAL, "g4a_attn_decode_layer_io: null host or device buffer");
  const size_t q_elems = (size_t)num_q_heads * head_dim, kv_elems = (size_t)num_kv_heads * head_dim;
  const size_t in_elems = q_elems + (is_producer ? 2 * kv_elems : 0);
  float* q = qkv_dev;
  float* k = qkv_dev + q_elems;
  float* v = k + kv_elems;
  // Validate before anything is enqueued, so a rejected call leaves the stream untouched.
  if (g4a_status s = check_common(__func__, q, k_cache, v_cache, out_dev, num_q_heads, num_kv_heads, head_dim))
    return s;
  if (!q_norm_w || (is_producer && !k_norm_w)) return g4a_fail(G4A_EINVAL, "g4a_attn_decode_layer_io: null norm weight");
  if (apply_divisor && !rope_freqs)
    return g4a_fail(G4A_EINVAL, "g4a_attn_decode_layer_io: apply_divisor without rope_freqs");
  if ((is_producer && slot >= max_seq_len) || kv_len > max_seq_len)
    return g4a_fail(G4A_EINVAL, "g4a_attn_decode_layer_io: slot %u / kv_len %u vs max_seq_len %u", slot, kv_len,
                    max_seq_len);
  // Mapped pinned host buffers: the producer kernel reads the inputs straight from host memory
  // (before its programmatic-launch wait) and the attention writes its output straight into
  // host memory, so the call is the layer's own launches and nothing else.
  void* in_map = mapped_host_address(qkv_host);
  void* out_map = in_map ? mapped_host_address(out_host) : nullptr;
  if (in_map && out_map && ((reinterpret_cast<uintptr_t>(in_map) | reinterpret_cast<uintptr_t>(out_map)) & 15u) == 0) {
    const float* sq = static_cast<const float*>(in_map);
    if (g4a_status s = g4a_launch_decode_prep(ctx, sq, sq + q_elems, sq + q_elems + kv_elems, q, k, v, q_norm_w,
                                              k_norm_w, rope_freqs, k_cache, v_cache, num_q_heads, num_kv_heads,
                                              head_dim, eps, position, slot, theta, apply_divisor, is_producer != 0))
      return s;
    return decode_contiguous(ctx, q, k_cache, v_cache, static_cast<float*>(out_map), num_q_heads, num_kv_heads,
                             head_dim, kv_len, scale, sliding_window, true);
  }
  if (g4a_status s = io_copy(ctx, qkv_dev, qkv_host, in_elems * sizeof(float), true)) return s;
  if (g4a_status s = g4a_attn_decode_layer(ctx, q, k, v, q_norm_w, k_norm_w, rope_freqs, k_cache, v_cache, out_dev,
                                           num_q_heads, num_kv_heads, head_dim, eps, position, slot, kv_len,
                                           max_seq_len, theta, apply_divisor, scale, sliding_window, is_producer))
    return s;
  return io_copy(ctx, out_host, out_dev, q_elems * sizeof(float), false);
}
