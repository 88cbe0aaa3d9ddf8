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
// Fast path (NQH = 8 * NKH, HD in {128, 256, 512}): persistent CTAs, one per SM, 8 warps.
// The flattened list of 32-key (16 for HD 512) "stages" of every (sequence, kv head) problem is
// split evenly over the grid, so a CTA may cover the end of one problem and the start of the
// next.  Warp 0 is also the producer: it TMA-bulk-copies each stage's K and V rows (one copy per
// contiguous run of rows, no multicast) from HBM into a 4-deep shared-memory ring guarded by
// mbarriers.  All eight warps are consumers: each owns G = 4 keys of every stage and HPW q heads
// (8, or 4 for HD 512); a lane holds HD/32 dims of q and of the output accumulator for each of
// its heads in registers, so one 16-byte shared load feeds HPW*HD/64 packed f32x2 FMAs.  Scores
// are reduced across lanes with a transposing butterfly (31 shuffles per 4 keys for 8 heads),
// then an online softmax in base 2 with lazy rescaling (the running max is only raised when a
// score exceeds it by more than 2^8), and p*V accumulates into the registers.  At the end of
// each segment (a problem's stages inside one CTA) the 8 warps merge through shared memory and
// write either the final row (segment = whole problem) or an un-normalised partial (m, l, o)
// that the merge kernel combines.  Decode is a GEMV per KV row (8 FLOP per byte of f16 KV), so
// it stays on the CUDA cores, bound by HBM bandwidth.
#include <math.h>

#include <algorithm>

#include "g4a_internal.cuh"

namespace {

constexpr int kGroup = 8;  // q heads per kv head on the fast path
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;  // 2 warps per SM sub-partition: up to 255 registers each
constexpr int kStages = 4;
constexpr int kG = 4;                  // keys per consumer warp per stage
constexpr float kLazyRescale = 8.0f;   // log2 units
constexpr float kLog2e = 1.4426950408889634f;

enum : int { F_SEG_FIRST = 1, F_SEG_LAST = 2, F_PROB_FIRST = 4, F_PROB_LAST = 8 };

struct StageMeta {
  int problem;
  int key0;    // first key (position) of the stage
  int nvalid;  // valid keys in the stage
  int flags;
  int seg;
};

struct DecodeParams {
  const float* q;         // [P * 8 (fast) | B * nqh, hd] f32
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
};

__device__ __forceinline__ uint32_t seq_len_of(const DecodeParams& p, int seq) {
  return p.kv_lens ? (uint32_t)max(p.kv_lens[seq], 0) : p.kv_len_scalar;
}

// Visible key range [lo, hi) of a sequence (window measured from the full length).
__device__ __forceinline__ void key_range(const DecodeParams& p, int seq, uint32_t& lo, uint32_t& hi) {
  uint32_t L = seq_len_of(p, seq);
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

template <int HD>
struct Cfg {
  static constexpr int HPW = (HD <= 256) ? 8 : 4;  // q heads per consumer warp
  static constexpr int NHW = kGroup / HPW;         // head groups
  static constexpr int NKW = kWarps / NHW;         // key warps per head group
  static constexpr int KPS = kG * NKW;             // keys per stage
  static constexpr int DPL = HD / 32;              // dims per lane
  static constexpr int NV = HPW * kG;              // score partials per lane
  static constexpr int DUP = 32 / NV;              // lanes holding the same reduced score
  static constexpr int ROW_BYTES = HD * 2;
  static constexpr int STAGE_BYTES = KPS * ROW_BYTES;  // per tensor
  static constexpr int OBUF_FLOATS = kWarps * HPW * HD;
  static constexpr size_t SMEM = (size_t)kStages * 2 * STAGE_BYTES + OBUF_FLOATS * 4 + kWarps * HPW * 2 * 4 +
                                 kWarps * (NV + HPW) * 4 + kStages * sizeof(StageMeta) + 2 * kStages * 8 + 64;
  static_assert(NV == 32 || NV == 16, "reduction assumes 16 or 32 partials per lane");
};

// Number of stages of a problem.
template <int KPS>
__device__ __forceinline__ int stages_of(const DecodeParams& p, int prob) {
  uint32_t lo, hi;
  key_range(p, prob / p.nkh, lo, hi);
  return (int)((hi - lo + KPS - 1) / KPS);
}

// Fixed-width loads of DPL halves from shared memory.
template <int DPL>
struct HalfVec;
template <>
struct HalfVec<4> {
  uint32_t w[2];
  __device__ __forceinline__ void load(const __half* s) {
    uint2 t = *reinterpret_cast<const uint2*>(s);
    w[0] = t.x;
    w[1] = t.y;
  }
};
template <>
struct HalfVec<8> {
  uint32_t w[4];
  __device__ __forceinline__ void load(const __half* s) {
    uint4 t = *reinterpret_cast<const uint4*>(s);
    w[0] = t.x;
    w[1] = t.y;
    w[2] = t.z;
    w[3] = t.w;
  }
};
template <>
struct HalfVec<16> {
  uint32_t w[8];
  __device__ __forceinline__ void load(const __half* s) {
    uint4 t = *reinterpret_cast<const uint4*>(s);
    uint4 u = *reinterpret_cast<const uint4*>(s + 8);
    w[0] = t.x;
    w[1] = t.y;
    w[2] = t.z;
    w[3] = t.w;
    w[4] = u.x;
    w[5] = u.y;
    w[6] = u.z;
    w[7] = u.w;
  }
};

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) decode_splitkv_kernel(const DecodeParams p) {
  using C = Cfg<HD>;
  constexpr int HPW = C::HPW, NKW = C::NKW, KPS = C::KPS, DPL = C::DPL, NV = C::NV, DUP = C::DUP;
  constexpr int ROW = C::ROW_BYTES;

  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* stage_base = smem;
  float* obuf = reinterpret_cast<float*>(smem + (size_t)kStages * 2 * C::STAGE_BYTES);
  float* mlbuf = obuf + C::OBUF_FLOATS;     // [warp][HPW][2]
  float* pbuf = mlbuf + kWarps * HPW * 2;   // [warp][NV + HPW]
  StageMeta* meta = reinterpret_cast<StageMeta*>(pbuf + kWarps * (NV + HPW));
  uint64_t* full = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(meta + kStages) + 7) & ~uintptr_t(7));
  uint64_t* empty = full + kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int P = p.B * p.nkh;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; s++) {
      g4a::mbar_init(&full[s], 1);
      g4a::mbar_init(&empty[s], kWarps);
    }
    g4a::fence_mbar_init();
  }
  __syncthreads();

  // Inputs (q, cache rows) may come from the preceding producer kernel.
  g4a::pdl_wait_primary();
  g4a::pdl_launch_dependents();

  // ---- stage range [s0, s1) of this CTA over the flattened stage list (every warp computes it)
  long long S = 0;
  for (int base = 0; base < P; base += 32) {
    const int pr = base + lane;
    int n = (pr < P) ? stages_of<KPS>(p, pr) : 0;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
    S += n;
  }
  // Only the first min(grid, S) CTAs take part, so every active CTA owns at least one stage and
  // the segment ids blockIdx.x + problem of one problem form a gap-free range.
  const long long G = (long long)gridDim.x < S ? (long long)gridDim.x : S;
  if ((long long)blockIdx.x >= G) return;  // uniform across the CTA
  const long long s0 = (long long)blockIdx.x * S / G;
  const long long s1 = (long long)(blockIdx.x + 1) * S / G;
  const int my_stages = (int)(s1 - s0);

  // =========================== producer role (warp 0 issues the TMA copies)
  // Stage n of this CTA goes to slot n % kStages.  Warp 0 keeps the cursor (problem, stage
  // within problem) and, before consuming stage it, issues stage it + kStages - 1 once all
  // eight warps have released that slot.
  int prob = 0, j = 0, nprob = 0;
  uint32_t lo = 0, hi = 0;
  uint64_t pol = 0;
  if (warp == 0) {
    long long acc = 0;
    bool found = false;
    for (int base = 0; base < P && !found; base += 32) {
      const int pr = base + lane;
      const int n = (pr < P) ? stages_of<KPS>(p, pr) : 0;
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
        prob = __shfl_sync(0xffffffffu, pr, src);
        j = (int)(s0 - __shfl_sync(0xffffffffu, lane_start, src));
        found = true;
      }
      acc += __shfl_sync(0xffffffffu, incl, 31);
    }
    nprob = stages_of<KPS>(p, prob);
    key_range(p, prob / p.nkh, lo, hi);
    pol = g4a::l2_policy_evict_first();
  }
  auto issue = [&](int n) {
    const int slot = n % kStages;
    const uint32_t par = ((n / kStages) & 1) ^ 1;
    if (lane == 0) g4a::mbar_wait_bounded(&empty[slot], par, p.err, G4A_DEVERR_WAIT_EMPTY);
    __syncwarp();
    const int seq = prob / p.nkh, kvh = prob % p.nkh;
    const uint32_t key0 = lo + (uint32_t)j * KPS;
    const int nvalid = (int)min((uint32_t)KPS, hi - key0);
    const __half* krow = nullptr;
    bool ok = false;
    if (lane < nvalid) {
      krow = row_ptr(p, p.k, seq, kvh, key0 + lane);
      ok = krow != nullptr;
    }
    // A bad page id skips the row (its keys then read stale shared memory; the error is
    // reported through g4a_sync).
    const unsigned okmask = __ballot_sync(0xffffffffu, ok);
    if (lane < nvalid && !ok && p.err) atomicExch(p.err, G4A_DEVERR_PAGE);
    const unsigned long long prev = __shfl_up_sync(0xffffffffu, (unsigned long long)(uintptr_t)krow, 1);
    const bool start =
        ok && (lane == 0 || !((okmask >> (lane - 1)) & 1u) || (uintptr_t)krow != (uintptr_t)prev + ROW);
    const unsigned starts = __ballot_sync(0xffffffffu, start);
    if (lane == 0) {
      StageMeta& mt = meta[slot];
      mt.problem = prob;
      mt.key0 = (int)key0;
      mt.nvalid = nvalid;
      int fl = 0;
      if (n == 0 || j == 0) fl |= F_SEG_FIRST;
      if (n == my_stages - 1 || j == nprob - 1) fl |= F_SEG_LAST;
      if (j == 0) fl |= F_PROB_FIRST;
      if (j == nprob - 1) fl |= F_PROB_LAST;
      mt.flags = fl;
      mt.seg = (int)blockIdx.x + prob;
      g4a::mbar_arrive_expect_tx(&full[slot], (uint32_t)__popc(okmask) * ROW * 2u);
    }
    __syncwarp();
    if (start) {
      // This lane's run covers lanes [lane, next run start or first skipped lane).
      const unsigned above = (lane == 31) ? 0u : (0xffffffffu << (lane + 1));
      const unsigned stop = (starts & above) | (~okmask & above);
      int end = stop ? (__ffs(stop) - 1) : 32;
      end = min(end, nvalid);
      const uint32_t bytes = (uint32_t)(end - lane) * ROW;
      unsigned char* sK = stage_base + (size_t)slot * 2 * C::STAGE_BYTES + (size_t)lane * ROW;
      unsigned char* sV = sK + C::STAGE_BYTES;
      const __half* vrow = p.v + (krow - p.k);
      g4a::bulk_g2s_hint(sK, krow, bytes, &full[slot], pol);
      g4a::bulk_g2s_hint(sV, vrow, bytes, &full[slot], pol);
    }
    if (++j == nprob) {  // advance the cursor to the next problem with stages
      j = 0;
      if (n + 1 < my_stages) {
        do {
          prob++;
          nprob = stages_of<KPS>(p, prob);
        } while (nprob == 0 && prob < P - 1);
        key_range(p, prob / p.nkh, lo, hi);
      }
    }
  };
  if (warp == 0) {
    for (int n = 0; n < kStages - 1 && n < my_stages; n++) issue(n);
  }

  // =========================== consumer role (all warps)
  const int hg = warp / NKW;  // head group
  const int kw = warp % NKW;  // key slot group
  float2 q2[HPW][DPL / 2];
  float2 o2[HPW][DPL / 2];
  float m_run = -INFINITY;  // running max (base 2) of this lane's head
  float l_part = 0.0f;      // this lane's share of the running sum
  bool seg_whole_start = false;

  // This lane's reduced score slot.
  const int c_lane = lane / DUP;
  const int h_lane = c_lane / kG;
  const int g_lane = c_lane % kG;
  float* pw = pbuf + warp * (NV + HPW);

  for (int it = 0; it < my_stages; it++) {
    if (warp == 0 && it + kStages - 1 < my_stages) issue(it + kStages - 1);
    const int slot = it % kStages;
    const uint32_t par = (it / kStages) & 1;
    g4a::mbar_wait_bounded(&full[slot], par, p.err, G4A_DEVERR_WAIT_FULL);
    const StageMeta mt = meta[slot];

    if (mt.flags & F_SEG_FIRST) {
      const float* qp = p.q + ((size_t)mt.problem * kGroup + hg * HPW) * HD + lane * DPL;
#pragma unroll
      for (int h = 0; h < HPW; h++) {
#pragma unroll
        for (int j4 = 0; j4 < DPL / 4; j4++) {
          float4 t = *reinterpret_cast<const float4*>(qp + (size_t)h * HD + j4 * 4);
          q2[h][j4 * 2] = make_float2(t.x, t.y);
          q2[h][j4 * 2 + 1] = make_float2(t.z, t.w);
        }
#pragma unroll
        for (int jj = 0; jj < DPL / 2; jj++) o2[h][jj] = make_float2(0.f, 0.f);
      }
      m_run = -INFINITY;
      l_part = 0.0f;
      seg_whole_start = (mt.flags & F_PROB_FIRST) != 0;
    }

    const unsigned char* sK = stage_base + (size_t)slot * 2 * C::STAGE_BYTES;
    const unsigned char* sV = sK + C::STAGE_BYTES;

    // ---- scores: part[h*G + g] = q_h . k_g over this lane's DPL dims
    float part[NV];
#pragma unroll
    for (int g = 0; g < kG; g++) {
      const int kl = kw * kG + g;
      if (kl < mt.nvalid) {
        HalfVec<DPL> kv;
        kv.load(reinterpret_cast<const __half*>(sK + (size_t)kl * ROW) + lane * DPL);
        float2 kf[DPL / 2];
#pragma unroll
        for (int jj = 0; jj < DPL / 2; jj++) kf[jj] = g4a::h2_to_f2(kv.w[jj]);
#pragma unroll
        for (int h = 0; h < HPW; h++) {
          float2 acc = __fmul2_rn(q2[h][0], kf[0]);
#pragma unroll
          for (int jj = 1; jj < DPL / 2; jj++) acc = __ffma2_rn(q2[h][jj], kf[jj], acc);
          part[h * kG + g] = acc.x + acc.y;
        }
      } else {
#pragma unroll
        for (int h = 0; h < HPW; h++) part[h * kG + g] = 0.0f;
      }
    }
    // ---- transposing butterfly: lane ends with the full dot of slot c_lane
#pragma unroll
    for (int n = NV, mask = 16; n >= 2; n >>= 1, mask >>= 1) {
      const bool upper = (lane & mask) != 0;
#pragma unroll
      for (int jj = 0; jj < n / 2; jj++) {
        const float keep = upper ? part[jj + n / 2] : part[jj];
        const float send = upper ? part[jj] : part[jj + n / 2];
        part[jj] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
      }
    }
    float s = part[0];
    if (DUP == 2) s += __shfl_xor_sync(0xffffffffu, s, 1);

    // ---- online softmax (base 2, lazy rescale)
    const bool valid = (kw * kG + g_lane) < mt.nvalid;
    const float t = valid ? s * p.scale_log2 : -INFINITY;
    float mx = t;
#pragma unroll
    for (int o = DUP; o < DUP * kG; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const bool need = mx > m_run + kLazyRescale;
    if (__any_sync(0xffffffffu, need)) {
      const float m_new = need ? mx : m_run;
      const float alpha = (need && m_run != -INFINITY) ? g4a::fast_exp2(m_run - m_new) : (need ? 0.0f : 1.0f);
      m_run = m_new;
      l_part *= alpha;
      if (g_lane == 0) pw[NV + h_lane] = alpha;
      __syncwarp();
#pragma unroll
      for (int h = 0; h < HPW; h++) {
        const float a = pw[NV + h];
        const float2 a2 = make_float2(a, a);
#pragma unroll
        for (int jj = 0; jj < DPL / 2; jj++) o2[h][jj] = __fmul2_rn(o2[h][jj], a2);
      }
    }
    const float pr = valid ? g4a::fast_exp2(t - m_run) : 0.0f;
    l_part += (lane % DUP == 0) ? pr : 0.0f;
    pw[g_lane * HPW + h_lane] = pr;
    __syncwarp();

    // ---- o += p * V
#pragma unroll
    for (int g = 0; g < kG; g++) {
      const int kl = kw * kG + g;
      if (kl < mt.nvalid) {
        HalfVec<DPL> vv;
        vv.load(reinterpret_cast<const __half*>(sV + (size_t)kl * ROW) + lane * DPL);
        float pg[HPW];
#pragma unroll
        for (int h4 = 0; h4 < HPW / 4; h4++) {
          const float4 t4 = *reinterpret_cast<const float4*>(pw + g * HPW + h4 * 4);
          pg[h4 * 4 + 0] = t4.x;
          pg[h4 * 4 + 1] = t4.y;
          pg[h4 * 4 + 2] = t4.z;
          pg[h4 * 4 + 3] = t4.w;
        }
        float2 vf[DPL / 2];
#pragma unroll
        for (int jj = 0; jj < DPL / 2; jj++) vf[jj] = g4a::h2_to_f2(vv.w[jj]);
#pragma unroll
        for (int h = 0; h < HPW; h++) {
          const float2 p2 = make_float2(pg[h], pg[h]);
#pragma unroll
          for (int jj = 0; jj < DPL / 2; jj++) o2[h][jj] = __ffma2_rn(p2, vf[jj], o2[h][jj]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) g4a::mbar_arrive(&empty[slot]);

    if (mt.flags & F_SEG_LAST) {
      // ---- merge the 8 warps of this CTA for this segment
      float l_head = l_part;
#pragma unroll
      for (int o = DUP; o < DUP * kG; o <<= 1) l_head += __shfl_xor_sync(0xffffffffu, l_head, o);
      if (g_lane == 0 && (lane % DUP) == 0) {
        mlbuf[(warp * HPW + h_lane) * 2 + 0] = m_run;
        mlbuf[(warp * HPW + h_lane) * 2 + 1] = l_head;
      }
      float* ow = obuf + (size_t)warp * HPW * HD;
#pragma unroll
      for (int h = 0; h < HPW; h++) {
#pragma unroll
        for (int j4 = 0; j4 < DPL / 4; j4++) {
          *reinterpret_cast<float4*>(ow + h * HD + lane * DPL + j4 * 4) =
              make_float4(o2[h][j4 * 2].x, o2[h][j4 * 2].y, o2[h][j4 * 2 + 1].x, o2[h][j4 * 2 + 1].y);
        }
      }
      g4a::named_bar_sync(1, kThreads);
      const bool whole = seg_whole_start && (mt.flags & F_PROB_LAST);
      const int tid = threadIdx.x;
      float* part_row = p.part + (size_t)mt.seg * (kGroup * (HD + 2));
      for (int e = tid; e < kGroup * HD; e += kThreads) {
        const int h8 = e / HD, d = e % HD;
        const int g0 = h8 / HPW, hh = h8 % HPW;
        float M = -INFINITY;
#pragma unroll
        for (int k = 0; k < NKW; k++) M = fmaxf(M, mlbuf[((g0 * NKW + k) * HPW + hh) * 2]);
        float acc = 0.f, lsum = 0.f;
#pragma unroll
        for (int k = 0; k < NKW; k++) {
          const int cw = g0 * NKW + k;
          const float mk = mlbuf[(cw * HPW + hh) * 2];
          const float sc = (mk == -INFINITY) ? 0.f : g4a::fast_exp2(mk - M);
          acc += sc * obuf[((size_t)cw * HPW + hh) * HD + d];
          lsum += sc * mlbuf[(cw * HPW + hh) * 2 + 1];
        }
        if (whole && p.out != nullptr) {
          p.out[((size_t)mt.problem * kGroup + h8) * HD + d] = acc / lsum;
        } else {
          part_row[2 * kGroup + h8 * HD + d] = acc;
          if (d == 0) {
            part_row[h8] = M;
            part_row[kGroup + h8] = lsum;
          }
        }
      }
      if (tid == 0) {
        if (seg_whole_start) p.seg_range[mt.problem].x = mt.seg;
        if (mt.flags & F_PROB_LAST) p.seg_range[mt.problem].y = mt.seg;
      }
      g4a::named_bar_sync(1, kThreads);
    }
  }
}

// Merge the segments of each problem.  grid (P, 8, HD/64), 256 threads: 16 segment lanes x 16
// float4 columns.  mode 0: normalised output rows; mode 1: one merged partial per problem.
__global__ void __launch_bounds__(256) merge_segments_kernel(const DecodeParams p, int mode, float* part_out) {
  g4a::pdl_wait_primary();
  const int prob = blockIdx.x, h = blockIdx.y, dchunk = blockIdx.z;
  const int hd = p.hd;
  const int sg = threadIdx.x / 16, c4 = threadIdx.x % 16;
  const int d = dchunk * 64 + c4 * 4;
  const size_t prow = (size_t)kGroup * (hd + 2);
  uint32_t lo, hi;
  key_range(p, prob / p.nkh, lo, hi);
  if (hi <= lo) {  // no visible key: zeros (the reference's seq_len 0 output)
    if (mode == 0) {
      if (sg == 0) *reinterpret_cast<float4*>(p.out + ((size_t)prob * kGroup + h) * hd + d) = make_float4(0, 0, 0, 0);
    } else {
      float* po = part_out + (size_t)prob * prow;
      if (sg == 0) *reinterpret_cast<float4*>(po + 2 * kGroup + h * hd + d) = make_float4(0, 0, 0, 0);
      if (threadIdx.x == 0 && dchunk == 0) {
        po[h] = -INFINITY;
        po[kGroup + h] = 0.f;
      }
    }
    return;
  }
  const int2 r = p.seg_range[prob];
  if (mode == 0 && r.x == r.y) return;  // single segment: the main kernel wrote the row
  __shared__ float smax[16];
  __shared__ float4 sacc[16][16];
  __shared__ float sl[16];
  float M = -INFINITY;
  for (int s = r.x + sg; s <= r.y; s += 16) M = fmaxf(M, p.part[(size_t)s * prow + h]);
  if (c4 == 0) smax[sg] = M;
  __syncthreads();
  M = -INFINITY;
#pragma unroll
  for (int i = 0; i < 16; i++) M = fmaxf(M, smax[i]);
  float4 acc = make_float4(0, 0, 0, 0);
  float lsum = 0.f;
#pragma unroll 4
  for (int s = r.x + sg; s <= r.y; s += 16) {
    const float* row = p.part + (size_t)s * prow;
    const float ms = row[h];
    if (ms == -INFINITY) continue;  // empty segment: contributes nothing (its o is not read)
    const float sc = exp2f(ms - M);
    const float4 o = *reinterpret_cast<const float4*>(row + 2 * kGroup + h * hd + d);
    acc.x += sc * o.x;
    acc.y += sc * o.y;
    acc.z += sc * o.z;
    acc.w += sc * o.w;
    lsum += sc * row[kGroup + h];
  }
  sacc[sg][c4] = acc;
  if (c4 == 0) sl[sg] = lsum;
  __syncthreads();
  if (sg == 0) {
    float4 a = make_float4(0, 0, 0, 0);
    float L = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      a.x += sacc[i][c4].x;
      a.y += sacc[i][c4].y;
      a.z += sacc[i][c4].z;
      a.w += sacc[i][c4].w;
      L += sl[i];
    }
    if (mode == 0) {
      const float inv = 1.0f / L;
      *reinterpret_cast<float4*>(p.out + ((size_t)prob * kGroup + h) * hd + d) =
          make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
    } else {
      float* po = part_out + (size_t)prob * prow;
      *reinterpret_cast<float4*>(po + 2 * kGroup + h * hd + d) = a;
      if (c4 == 0 && dchunk == 0) {
        po[h] = M;
        po[kGroup + h] = L;
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
  const float* qh = p.q + ((size_t)seq * p.nqh + h) * p.hd;
  float qv[MAXD], o[MAXD];
#pragma unroll
  for (int i = 0; i < MAXD; i++) {
    const int d = lane + 32 * i;
    qv[i] = d < p.hd ? qh[d] : 0.f;
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

template <int HD>
g4a_status configure_kernel(g4a_ctx* ctx) {
  static bool done[64] = {false};
  if (ctx->device < 64 && done[ctx->device]) return G4A_OK;
  cudaError_t e = cudaFuncSetAttribute(decode_splitkv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)Cfg<HD>::SMEM);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaFuncSetAttribute(decode_splitkv_kernel)");
  if (ctx->device < 64) done[ctx->device] = true;
  return G4A_OK;
}

template <int HD>
g4a_status launch_fast(g4a_ctx* ctx, DecodeParams& p, long long stages_upper, int mode, float* part_out, bool pdl) {
  using C = Cfg<HD>;
  if (g4a_status s = configure_kernel<HD>(ctx)) return s;
  const int P = p.B * p.nkh;
  int grid = (int)std::min<long long>(stages_upper, (long long)ctx->num_sms);
  if (grid < 1) grid = 1;
  const size_t prow = (size_t)kGroup * (HD + 2) * sizeof(float);
  const size_t segs = (size_t)grid + (size_t)P + 1;
  const size_t part_bytes = (segs * prow + 255) & ~size_t(255);
  if (g4a_status s = g4a_ensure_workspace(ctx, part_bytes + (size_t)P * sizeof(int2) + 256)) return s;
  p.part = reinterpret_cast<float*>(ctx->workspace);
  p.seg_range = reinterpret_cast<int2*>(reinterpret_cast<char*>(ctx->workspace) + part_bytes);
  p.err = ctx->dev_err_dev;
  if (stages_upper > 0) {
    g4a_prof_scope ps(ctx, G4A_PROF_DECODE_SPLITKV);
    cudaError_t e = g4a_launch(decode_splitkv_kernel<HD>, dim3(grid), dim3(kThreads), C::SMEM, ctx->stream, pdl, p);
    if (e != cudaSuccess) return g4a_cuda_fail(e, "launch decode_splitkv_kernel");
  }
  // The merge kernel is needed when a problem can span several CTAs, for zero-length problems,
  // and always in partial mode.
  const bool need_merge = (mode == 1) || grid > 1 || stages_upper == 0 || P > 1;
  if (need_merge) {
    g4a_prof_scope ps(ctx, G4A_PROF_DECODE_MERGE);
    cudaError_t e = g4a_launch(merge_segments_kernel, dim3(P, kGroup, HD / 64), dim3(256), 0, ctx->stream,
                               stages_upper > 0, p, mode, part_out);
    if (e != cudaSuccess) return g4a_cuda_fail(e, "launch merge_segments_kernel");
  }
  return G4A_OK;
}

// keys_upper: an upper bound on the total number of visible (problem, key) pairs.
g4a_status dispatch_fast(g4a_ctx* ctx, DecodeParams& p, long long keys_upper, int mode, float* part_out, bool pdl) {
  switch (p.hd) {
    case 128:
      return launch_fast<128>(ctx, p, (keys_upper + Cfg<128>::KPS - 1) / Cfg<128>::KPS, mode, part_out, pdl);
    case 256:
      return launch_fast<256>(ctx, p, (keys_upper + Cfg<256>::KPS - 1) / Cfg<256>::KPS, mode, part_out, pdl);
    case 512:
      return launch_fast<512>(ctx, p, (keys_upper + Cfg<512>::KPS - 1) / Cfg<512>::KPS, mode, part_out, pdl);
    default:
      return g4a_fail(G4A_EINVAL, "decode: unsupported head_dim %d", p.hd);
  }
}

int kps_of(uint32_t hd) { return hd == 512 ? Cfg<512>::KPS : Cfg<256>::KPS; }

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
                             bool pdl) {
  DecodeParams p = base_params(q, k, v, nqh, nkh, hd, scale, window, out);
  p.B = 1;
  p.kv_len_scalar = kv_len;
  p.err = ctx->dev_err_dev;
  const uint32_t ws = (window != 0u && kv_len > window) ? kv_len - window : 0u;
  const long long keys = (long long)(kv_len - ws);
  if (fast_path_ok(nqh, nkh, hd)) return dispatch_fast(ctx, p, keys * nkh + (long long)(nkh - 1) * kps_of(hd), 0, nullptr, pdl);
  g4a_prof_scope ps(ctx, G4A_PROF_DECODE_GENERIC);
  decode_generic_kernel<<<nqh, 256, 0, ctx->stream>>>(p, 0, nullptr);
  return g4a_check_launch("decode_generic_kernel");
}

}  // namespace

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
  if (fast_path_ok(num_q_heads, num_kv_heads, head_dim)) {
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
    return dispatch_fast(ctx, p, keys, 0, nullptr, false);
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
    return dispatch_fast(ctx, p, keys, 1, part, false);
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

}  // extern "C"

// Producer stage launcher lives in g4a_producers.cu.
g4a_status g4a_launch_decode_prep(g4a_ctx* ctx, float* q, float* k, float* v, const uint16_t* qw, const uint16_t* kw,
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
  if (g4a_status s = g4a_launch_decode_prep(ctx, q, k, v, q_norm_w, k_norm_w, rope_freqs, k_cache, v_cache,
                                            num_q_heads, num_kv_heads, head_dim, eps, position, slot, theta,
                                            apply_divisor, is_producer != 0))
    return s;
  return decode_contiguous(ctx, q, k_cache, v_cache, out, num_q_heads, num_kv_heads, head_dim, kv_len, scale,
                           sliding_window, true);
}
