// Prefill attention on the tensor cores (tcgen05.mma, TMEM accumulators and operands, TMA tile
// loads).
//
// The reference has no prefill attention kernel: prefillBatched (src/engine.ts:2460-2479) runs
// one decode forward per prompt token, so row i of the result is decode attention
// (shaders/attn_score.wgsl, softmax.wgsl, attn_output.wgsl) at kv_len = start_pos + i + 1 with
// the window measured from that kv_len.  This kernel computes the same rows as one flash-
// attention pass.
//
// Tile: 128 query rows = 16 consecutive tokens x the 8 q heads that share one kv head (GQA 8:1),
// so every row of a tile reads the same K/V rows.  One CTA per tile, heaviest (latest) tiles
// first.  Q (one TMA load) and 2-stage rings of K and V blocks (64 keys per block, one TMA op
// per tensor per block, 128-byte swizzle) live in shared memory.  TMEM (HD 256): O [0, 256),
// two score buffers S0/S1 [256, 384), two P buffers (f16 pairs) [384, 448).
// Double-buffering S and P lets the score MMA of block j+1 and the softmax of block j overlap
// the PV MMA of block j-1, and keeps the softmax off the O-correction chain.
// Warp roles (512 threads):
//   warp 0 lane 0   TMA: Q once, then K blocks (a K stage is released when S_j is done).
//   warp 2 lane 0   TMA: V blocks (a V stage is released when PV_j is done).
//   warp 1          allocates TMEM; lane 0 issues S_j = Q K_j^T (M 128, N 64, K = HD, f16 in /
//                   f32 accumulate, both operands from shared memory) into S[j % 2].
//   warp 3 lane 0   issues O += P_j V_j (N = HD), A = P[j % 2] from TMEM.
//   warps 4-11      softmax, two threads per query row (TMEM lane = row; warps w and w+4 take
//                   keys 0-31 and 32-63 of a block and exchange row maxima through shared
//                   memory): scores from TMEM (handed back right after the load), window/causal
//                   mask (boundary blocks only), online softmax in base 2 with lazy rescaling
//                   (the running max is only raised when a row's max grows by more than 2^15,
//                   so P <= 2^15 stays in f16 range, and then to 2^8 above the new block max,
//                   which makes the next raise -- an O correction for the whole warp -- rarer:
//                   Gemma's unit-RMS q and k with scale 1 give scores with a spread of ~16, and
//                   at 2^0 headroom most 32-row warps needed a correction on most blocks),
//                   P rounded to f16 into TMEM.  Each thread
//                   sums the same f16-rounded P values in f32 for l (rescaled in registers when
//                   the max is raised), so numerator and denominator use identical weights.
//                   Epilogue: the two halves add their l, then O / l from TMEM to the f32 output.
//   warps 12-15     correction: when a row's running max was raised, scale its O in TMEM by
//                   2^(m_old - m_new) after PV_{j-1} and before PV_j.
// Every mbarrier wait is bounded; after a timeout the CTA records an error, stops waiting and
// frees its TMEM.  Barriers that complete once per block come in pairs (one per block parity)
// wherever a consumer could otherwise fall two phases behind its producer.
//
// Head dim 512 (Gemma's global layers), the PAIR instance: one CTA cannot hold a 128-row tile
// (the f32 O accumulator alone would fill the 512 TMEM columns, the f16 Q tile 128 KB of shared
// memory), so a cluster of two CTAs computes each tile and CTA c owns head dims [256 c, 256 c +
// 256): its columns of Q, its halves of every K and V block, its 256 columns of O.  Each CTA
// computes the partial scores of its dims, S_c = Q_c K_c^T; the two exchange them through
// distributed shared memory and both add own + partner's (IEEE addition commutes, so the two
// sums are bit-identical), run the same softmax on the same scores -- hence the same P, running
// max and l -- and accumulate O_c += P V_c.  No MMA work is duplicated, only the softmax.
// TMEM (512 columns): O [0, 256), two S buffers [256, 384), and Q [384, 512) (the A operand of
// the score MMA: one TMA load into the idle send and receive slots, which the exchange warps
// then copy into TMEM before the first exchange; the partner sends its first scores only after
// this CTA's exchange warps have read the slots, the same signal as for every later block).  P goes to shared memory (one 16 KB
// buffer, the A operand of the PV MMA).  Shared memory also holds the 2-stage K and V rings (64
// keys x 256 dims) and, per TMEM lane quarter, one 8 KB slot for the scores this CTA sends and
// one for the partner's it receives.  Warps 16-19 (640 threads) exchange the partial scores of
// their lane quarter: load S_c from TMEM, stage it in shared memory, send it with one bulk copy
// into the partner's receive slot (completing on the partner's barrier), wait for the
// partner's, add, and store the sum into TMEM for the softmax warps.  (Per-thread remote stores
// took 1.5 us per block for the 32 KB, and the exchange inside the softmax warps put it on their
// critical path.)  A warp stages block j only after the partner has read block j-1 (a remote
// arrival), which also tells it that its own previous copy has landed.  Every wait is bounded,
// and a CTA that gives up also sets its partner's abort flag; the two CTAs leave through one
// cluster barrier, so neither's shared memory goes away while the other may still copy into it.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "g4a_internal.cuh"

namespace {

constexpr int kRows = 128;                 // query rows per tile (TMEM lanes)
constexpr int kHeadsPerKv = 8;             // q heads per kv head handled by this kernel
constexpr int kTokPerTile = kRows / kHeadsPerKv;
constexpr int kKeys = 64;                  // keys per block
constexpr int kStagesP = 2;                // K and V ring depth
constexpr int kThreadsP = 512;
constexpr float kLog2eP = 1.4426950408889634f;
constexpr float kRescaleP = 15.0f;         // lazy rescale threshold (log2 units): P <= 2^15 stays in f16 range
constexpr float kHeadroomP = 8.0f;         // a raised running max is set this far above the block max

// HD = head dims held by one CTA (the pair instance: 256 of 512).
template <int HD, bool PAIR>
struct PCfg {
  static constexpr int THREADS = PAIR ? kThreadsP + 128 : kThreadsP;
  static constexpr int NCB = HD / 64;               // 64-dim chunks (128-byte swizzle rows)
  static constexpr int Q_CHUNK = kRows * 128;       // bytes of one chunk of the Q tile
  static constexpr int KV_CHUNK = kKeys * 128;      // bytes of one chunk of a K or V block
  static constexpr int Q_LOAD_BYTES = NCB * Q_CHUNK;        // one TMA load of this CTA's Q columns
  static constexpr int Q_BYTES = PAIR ? 0 : Q_LOAD_BYTES;    // a pair keeps Q in TMEM
  static constexpr int KV_BYTES = NCB * KV_CHUNK;
  static constexpr int X_BYTES = PAIR ? kRows * kKeys * 4 : 0;  // one block's partial scores (f32)
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + kStagesP * KV_BYTES;
  // pair: [4 quarters] x 8 KB ([16 four-key groups][32 lanes][4 floats]) of the scores this CTA
  // sends (OFF_XS) and of the partner's it receives (OFF_XR); P [128 rows][128 B] (OFF_P)
  static constexpr int OFF_XS = OFF_V + kStagesP * KV_BYTES;
  static constexpr int OFF_XR = OFF_XS + X_BYTES;
  static constexpr int OFF_P = OFF_XR + X_BYTES;
  static constexpr int OFF_LSUM = OFF_P + (PAIR ? kRows * kKeys * 2 : 0);  // [2 halves][128 rows] row sums
  static constexpr int OFF_RED = OFF_LSUM + 2 * kRows * 4;      // [2 parities][2 halves][128 rows] row maxima
  static constexpr int OFF_ALPHA = OFF_RED + 2 * 2 * kRows * 4; // [2 parities][128 rows] rescale factors
  static constexpr int OFF_FLAG = OFF_ALPHA + 2 * kRows * 4;    // [2 parities][4 quarters] rescale needed
  static constexpr int OFF_BAR = OFF_FLAG + 64;
  static constexpr int NBARS = 56;
  static constexpr size_t SMEM = 1024 + (size_t)OFF_BAR + NBARS * 8 + 16;
  // TMEM columns (32-bit each; P and Q hold two f16 per column)
  static constexpr uint32_t COL_O = 0;
  static constexpr uint32_t COL_S = HD;                          // S[b] at COL_S + 64 b
  static constexpr uint32_t COL_P = COL_S + 2 * kKeys;           // P[b] at COL_P + 32 b (pair: in shared memory)
  static constexpr uint32_t COL_Q = COL_S + 2 * kKeys;           // pair: the Q tile (HD / 2 columns)
  static constexpr uint32_t COL_END = PAIR ? COL_Q + HD / 2 : COL_P + kKeys;
  static constexpr uint32_t TMEM_COLS = COL_END <= 256 ? 256u : 512u;
  static_assert(OFF_K % 1024 == 0 && OFF_V % 1024 == 0 && OFF_P % 1024 == 0 && KV_BYTES % 1024 == 0,
                "1024-byte aligned operands");
  static_assert(COL_END <= TMEM_COLS, "TMEM budget");
  static_assert(!PAIR || 2 * X_BYTES >= Q_LOAD_BYTES, "pair: Q is staged in the send and receive slots");
  static_assert(SMEM <= 232448, "shared memory budget");
};

struct PrefillParams {
  float* out;            // [T, nqh, HD] f32
  int T;
  uint32_t start_pos;
  int nqh, nkh;
  int ntiles;            // tiles per kv head = ceil(T / 16)
  float scale_log2;      // scale * log2(e)
  uint32_t window;       // 0 = causal over the whole prefix
  int* err;
};

// --------------------------------------------------------------------------- tcgen05 helpers
// Shared-memory matrix descriptor (sm_100 UMMA format): start address, leading and stride byte
// offsets (all >> 4), descriptor version 1 at bits 46-47, 128-byte swizzle (2) at bits 61-63.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of kind::f16 with f16 A and B, f32 accumulate, M = 128.
__host__ __device__ constexpr uint32_t f16_idesc(int n, bool b_mn_major) {
  return (1u << 4)                              // D format f32
         | (0u << 7) | (0u << 10)               // A, B format f16
         | (0u << 15)                           // A K-major
         | ((b_mn_major ? 1u : 0u) << 16)       // B major-ness
         | ((uint32_t)(n >> 3) << 17)           // N >> 3
         | ((uint32_t)(128 >> 4) << 24);        // M >> 4
}

// D (+)= A B^T with A from TMEM (K-major: row i in lane i, two f16 per 32-bit column) and B a
// shared-memory descriptor.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   g4a::smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive TMEM columns of this warp's 32 lanes: thread i gets lane (base + i).  The
// wait is in the same asm statement, so no use of the registers can be scheduled before the
// data has arrived.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Tiled TMA store of a shared-memory box to global memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_load_4d_p(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                              uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(g4a::smem_u32(bar)), "l"(pol)
      : "memory");
}

// Bounded mbarrier wait that also gives up at once when another thread of the CTA already gave
// up (abort flag in shared memory), so a failure costs one timeout, not one per wait.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                              int code) {
  if (g4a::mbar_try_wait(bar, parity)) return true;
  if (*abort_flag) return false;
  const uint64_t t0 = g4a::globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (g4a::mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0u) {
      if (*abort_flag) return false;
      if (g4a::globaltimer_ns() - t0 > 2000000000ull) {
        *abort_flag = 1;
        if (err) atomicExch(err, code);
        return false;
      }
    }
  }
}

// D (+)= A B^T with both operands as shared-memory descriptors.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Warp-uniform bounded wait (the tcgen05.ld/st after it are warp-collective).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  return __all_sync(0xffffffffu, wait_or_abort(bar, parity, abort_flag, err, G4A_DEVERR_WAIT_MMA));
}

// ------------------------------------------------------------------ cluster (CTA pair) helpers
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Every thread of both CTAs: release this CTA's prior writes, acquire the partner's.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
// Arrive on a barrier of the partner CTA, with no ordering of this thread's prior memory
// operations (the caller has no writes to publish: the arrival only says that a slot was read).
// Bulk copy of `bytes` from this CTA's shared memory into the partner's (dst and bar are
// shared::cluster addresses from mapa), completing as transaction bytes on the partner's barrier.
__device__ __forceinline__ void bulk_s2s_cluster(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "r"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(g4a::smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the partner's arrivals (acquire at cluster scope), warp-uniform.
__device__ __forceinline__ bool warp_wait_peer(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  bool done = mbar_try_wait_cluster(bar, parity);
  if (!done && !*abort_flag) {
    const uint64_t t0 = g4a::globaltimer_ns();
    uint32_t spins = 0;
    while (!(done = mbar_try_wait_cluster(bar, parity))) {
      if ((++spins & 63u) == 0u) {
        if (*abort_flag) break;
        if (g4a::globaltimer_ns() - t0 > 2000000000ull) {
          *abort_flag = 1;
          if (err) atomicExch(err, G4A_DEVERR_WAIT_PEER);
          break;
        }
      }
    }
  }
  return __all_sync(0xffffffffu, done);
}

// --------------------------------------------------------------------------- the kernel
template <int HD, bool PAIR>
__global__ void __launch_bounds__(PCfg<HD, PAIR>::THREADS, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmo,
                        const PrefillParams p) {
  using C = PCfg<HD, PAIR>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* fullK = bars;           // [2] K block landed
  uint64_t* fullV = bars + 2;       // [2] V block landed
  uint64_t* emptyK = bars + 4;      // [2] K stage consumed by S_j (tcgen05.commit)
  uint64_t* emptyV = bars + 6;      // [2] V stage consumed by PV_j (tcgen05.commit)
  uint64_t* barQ = bars + 8;        // Q tile landed
  uint64_t* barS = bars + 9;        // [2] S_j in S[j % 2] (tcgen05.commit)
  uint64_t* barSfree = bars + 11;   // [2] S_j loaded by the softmax warps (8 warps)
  uint64_t* barP = bars + 13;       // [2] P_j in P[j % 2] (8 softmax warps)
  uint64_t* barPV = bars + 15;      // [2] PV_j done (tcgen05.commit)
  uint64_t* barEnd = bars + 17;     // every score MMA done
  uint64_t* barEnd2 = bars + 18;    // every PV MMA done
  uint64_t* barAlpha = bars + 19;   // [2] rescale factors of block j published (4 softmax warps)
  uint64_t* barCorr = bars + 21;    // [2] O rescaled for block j (4 correction warps)
  uint64_t* barXchg = bars + 23;    // [2 parities][4 quarters] row-max halves written (2 softmax warps)
  uint64_t* barLsum = bars + 31;    // [4 quarters] row-sum halves written (2 softmax warps)
  uint64_t* barRx = bars + 35;      // pair: [4 quarters] the partner's partial scores landed
  uint64_t* barOK = bars + 39;      // pair: [4 quarters] the partner has read this CTA's
  uint64_t* barSx = bars + 43;      // pair: [2 parities][4 quarters] the full scores of block j in S[j % 2]
  uint64_t* barQ2 = bars + 51;      // pair: Q copied from the slots into TMEM (4 exchange warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // pair: both CTAs of a cluster take the same tile; cr is this CTA's half of the head dims
  const uint32_t cr = PAIR ? cluster_ctarank() : 0u;
  const uint32_t peer = cr ^ 1u;
  const unsigned tile = PAIR ? (blockIdx.x >> 1) : blockIdx.x;
  const int kvh = (int)(tile % (unsigned)p.nkh);
  const int t0 = (p.ntiles - 1 - (int)(tile / (unsigned)p.nkh)) * kTokPerTile;
  const int t_last = min(t0 + kTokPerTile, p.T) - 1;
  const uint32_t hi_max = p.start_pos + (uint32_t)t_last + 1u;
  const uint32_t first_hi = p.start_pos + (uint32_t)t0 + 1u;
  const uint32_t lo_min = (p.window != 0u && first_hi > p.window) ? first_hi - p.window : 0u;
  const int kb0 = (int)(lo_min / kKeys);
  const int nb = (int)((hi_max - 1u) / kKeys) - kb0 + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; s++) {
      g4a::mbar_init(&fullK[s], 1);
      g4a::mbar_init(&fullV[s], 1);
      g4a::mbar_init(&emptyK[s], 1);
      g4a::mbar_init(&emptyV[s], 1);
      g4a::mbar_init(&barS[s], 1);
      g4a::mbar_init(&barSfree[s], 8);
      g4a::mbar_init(&barP[s], 8);
      g4a::mbar_init(&barPV[s], 1);
      g4a::mbar_init(&barAlpha[s], 4);
      g4a::mbar_init(&barCorr[s], 4);
      for (int q = 0; q < 4; q++) g4a::mbar_init(&barXchg[s * 4 + q], 2);
    }
    for (int q = 0; q < 4; q++) g4a::mbar_init(&barLsum[q], 2);
    if (PAIR) {
      for (int i = 0; i < 4; i++) {
        g4a::mbar_init(&barRx[i], 1);  // the exchange warp's expect_tx + the partner's copy
        g4a::mbar_init(&barOK[i], 1);  // the partner's exchange warp (remote arrival)
      }
      for (int i = 0; i < 8; i++) g4a::mbar_init(&barSx[i], 1);
      g4a::mbar_init(barQ2, 4);
    }
    g4a::mbar_init(barQ, 1);
    g4a::mbar_init(barEnd, 1);
    g4a::mbar_init(barEnd2, 1);
    *abort_flag = 0;
    g4a::fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmq)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmo)) : "memory");
  }
  g4a::fence_proxy_async_smem();
  if (warp == 1) {  // TMEM: one CTA per SM (shared memory), so the allocation never waits
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(g4a::smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncwarp();  // warp 0 was diverged by the initialisation above
  tc_fence_before();
  // pair: the partner's barriers are initialised before anyone arrives on them remotely
  if constexpr (PAIR) cluster_sync_all(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  g4a::pdl_launch_dependents();
  // q16 and the cache rows are written by the preceding prep kernel.
  g4a::pdl_wait_primary();

  const uint32_t sbase = g4a::smem_u32(smem);
  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------------ TMA producers
    if (lane == 0) {
      const bool kside = warp == 0;
      uint64_t pol_kv;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_kv));
      if (kside) {  // pair: this CTA's chunks of the Q tile, into the (still idle) exchange slots
        uint64_t pol_q;
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_q));
        g4a::mbar_arrive_expect_tx(barQ, (uint32_t)C::Q_LOAD_BYTES);
        tma_load_4d_p(sbase + (PAIR ? C::OFF_XS : C::OFF_Q), &tmq, 0, kvh * kHeadsPerKv, t0, (int)cr * C::NCB, barQ,
                      pol_q);
      }
      uint64_t* empty = kside ? emptyK : emptyV;
      uint64_t* full = kside ? fullK : fullV;
      const CUtensorMap* map = kside ? &tmk : &tmv;
      const uint32_t dst0 = sbase + (kside ? C::OFF_K : C::OFF_V);
      for (int j = 0; j < nb; j++) {
        const int s = j & 1;
        if (j >= 2 && !wait_or_abort(&empty[s], (uint32_t)((j >> 1) - 1) & 1u, abort_flag, p.err,
                                     G4A_DEVERR_WAIT_EMPTY))
          break;
        g4a::mbar_arrive_expect_tx(&full[s], (uint32_t)C::KV_BYTES);
        // pair: this CTA's 64-dim chunks [NCB cr, NCB cr + NCB) of the block
        tma_load_4d_p(dst0 + s * C::KV_BYTES, map, 0, kvh, (kb0 + j) * kKeys, (int)cr * C::NCB, &full[s], pol_kv);
      }
      // Loads still in flight land before the CTA retires (bounded).
      for (int j = max(0, nb - 2); j < nb; j++)
        (void)wait_or_abort(&full[j & 1], (uint32_t)(j >> 1) & 1u, abort_flag, p.err, G4A_DEVERR_WAIT_FULL);
      if (kside) (void)wait_or_abort(barQ, 0, abort_flag, p.err, G4A_DEVERR_WAIT_FULL);
    }
  } else if (warp == 1 || warp == 3) {
    // ------------------------------------------------------------------ MMA issuers
    // Two issuing threads, so that the waits of one never leave the tensor pipe without work:
    // warp 1 issues the score MMAs, warp 3 the PV MMAs.  Each commit tracks the MMAs of its
    // own thread.  Base descriptors are built once; a K step only adds a constant to the
    // start-address field (bits 0-13, in 16-byte units; every operand lies below 256 KB).
    if (lane == 0) {
      uint64_t* my_end = (warp == 1) ? barEnd : barEnd2;
      if (warp == 1) {
        constexpr uint32_t idesc_s = f16_idesc(kKeys, false);
        const uint64_t dq = sw128_desc(sbase + C::OFF_Q, 16, 1024);
        const uint64_t dk0 = sw128_desc(sbase + C::OFF_K, 16, 1024);
        bool ok = wait_or_abort(PAIR ? barQ2 : barQ, 0, abort_flag, p.err, G4A_DEVERR_WAIT_FULL);
        for (int j = 0; ok && j < nb; j++) {
          const int b = j & 1;
          // S[b] was last read out by the softmax of block j-2
          if (j >= 2 && !wait_or_abort(&barSfree[b], (uint32_t)((j >> 1) - 1) & 1u, abort_flag, p.err,
                                       G4A_DEVERR_WAIT_MMA))
            break;
          if (!wait_or_abort(&fullK[b], (uint32_t)(j >> 1) & 1u, abort_flag, p.err, G4A_DEVERR_WAIT_FULL)) break;
          tc_fence_after();
          const uint64_t dk = dk0 + (uint64_t)((b * C::KV_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < HD / 16; kk++) {
            // K step kk: 64-dim chunk kk / 4, 32 bytes (16 dims) per step along the swizzled row
            const uint64_t off = (uint64_t)(((kk & 3) * 32) >> 4);
            if constexpr (PAIR)  // Q columns 8 kk .. 8 kk + 7 (two dims per column) in TMEM
              umma_f16_ts(tmem + C::COL_S + (uint32_t)(b * kKeys), tmem + C::COL_Q + (uint32_t)(kk * 8),
                          dk + (uint64_t)(((kk >> 2) * C::KV_CHUNK) >> 4) + off, idesc_s, kk > 0 ? 1u : 0u);
            else
              umma_f16_ss(tmem + C::COL_S + (uint32_t)(b * kKeys),
                          dq + (uint64_t)(((kk >> 2) * C::Q_CHUNK) >> 4) + off,
                          dk + (uint64_t)(((kk >> 2) * C::KV_CHUNK) >> 4) + off, idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&barS[b]);
          umma_commit(&emptyK[b]);
        }
      } else {
        constexpr uint32_t idesc_pv = f16_idesc(HD, true);
        // V block as the MN-major B operand: 64 dims per 128-byte row (N), chunks C::KV_CHUNK apart
        // (leading offset), 8-key row groups 1024 bytes apart (stride offset).
        const uint64_t dv0 = sw128_desc(sbase + C::OFF_V, (uint32_t)C::KV_CHUNK, 1024);
        const uint64_t dp = sw128_desc(sbase + C::OFF_P, 16, 1024);  // pair: P [128 rows][64 keys], K-major
        for (int i = 0; i < nb; i++) {
          const int b = i & 1;
          if (!wait_or_abort(&fullV[b], (uint32_t)(i >> 1) & 1u, abort_flag, p.err, G4A_DEVERR_WAIT_FULL)) break;
          // O rescaled for block i (after PV_{i-1}, which the correction warps waited for)
          if (!wait_or_abort(&barCorr[b], (uint32_t)(i >> 1) & 1u, abort_flag, p.err, G4A_DEVERR_WAIT_MMA)) break;
          if (!wait_or_abort(&barP[b], (uint32_t)(i >> 1) & 1u, abort_flag, p.err, G4A_DEVERR_WAIT_MMA)) break;
          tc_fence_after();
          const uint64_t dv = dv0 + (uint64_t)((b * C::KV_BYTES) >> 4);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; kk++) {
            if constexpr (PAIR) {  // 16 keys = 32 bytes along P's swizzled rows
              umma_f16_ss(tmem + C::COL_O, dp + (uint64_t)((kk * 32) >> 4), dv + (uint64_t)((kk * 2048) >> 4), idesc_pv,
                          (i > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint32_t a = tmem + C::COL_P + (uint32_t)(b * (kKeys / 2) + kk * 8);  // 16 keys = 8 columns
              umma_f16_ts(tmem + C::COL_O, a, dv + (uint64_t)((kk * 2048) >> 4), idesc_pv,
                          (i > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&barPV[b]);
          umma_commit(&emptyV[b]);
        }
      }
      // No MMA may still be running when TMEM is freed, also after an abort (bounded wait).
      umma_commit(my_end);
      (void)g4a::mbar_wait_bounded(my_end, 0, p.err, G4A_DEVERR_WAIT_MMA);
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------------ softmax, epilogue
    const int quarter = warp & 3;                               // TMEM lane quarter of this warp
    const int half = (warp - 4) >> 2;                           // keys [32*half, 32*half + 32) of a block
    const int r = quarter * 32 + lane;                          // tile row = TMEM lane
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const int tok = t0 + r / kHeadsPerKv;
    const uint32_t hi = p.start_pos + (uint32_t)tok + 1u;
    const uint32_t lo = (p.window != 0u && hi > p.window) ? hi - p.window : 0u;
    float* red = reinterpret_cast<float*>(smem + C::OFF_RED);     // [parity][half][row]
    float* alpha_buf = reinterpret_cast<float*>(smem + C::OFF_ALPHA);
    int* flag_buf = reinterpret_cast<int*>(smem + C::OFF_FLAG);
    const float c2 = p.scale_log2;
    float m = -INFINITY;
    float lsum = 0.f;  // this half's share of the row sum, relative to m
    bool ok = true;
    for (int j = 0; j < nb; j++) {
      const int b = j & 1;
      // pair: the full scores (own + partner's partial) from the exchange warp of this quarter
      ok = warp_wait(PAIR ? &barSx[b * 4 + quarter] : &barS[b], (uint32_t)(j >> 1) & 1u, abort_flag, p.err);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[32];
      tmem_ld32(tmem + lane_addr + C::COL_S + (uint32_t)(b * kKeys + 32 * half), sv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) g4a::mbar_arrive(&barSfree[b]);  // S[b] may be overwritten now
      const uint32_t key0 = (uint32_t)(kb0 + j) * kKeys + 32u * half;
      // Interior blocks (every key visible to every row of the warp) skip the mask.
      const bool interior = __all_sync(0xffffffffu, key0 >= lo && key0 + 32u <= hi) && c2 > 0.f;
      float x[32];
      float mx;
      if (interior) {  // raw scores; max scales with c2 > 0
#pragma unroll
        for (int c = 0; c < 32; c++) x[c] = __uint_as_float(sv[c]);
      } else {
#pragma unroll
        for (int c = 0; c < 32; c++) {
          float v = __uint_as_float(sv[c]) * c2;
          if (!(key0 + (uint32_t)c >= lo && key0 + (uint32_t)c < hi)) v = -INFINITY;
          x[c] = v;
        }
      }
      {
        float mq[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          mq[q] = fmaxf(fmaxf(x[q], x[q + 4]), fmaxf(x[q + 8], x[q + 12]));
          mq[q] = fmaxf(mq[q], fmaxf(fmaxf(x[q + 16], x[q + 20]), fmaxf(x[q + 24], x[q + 28])));
        }
        mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
        if (interior) mx *= c2;
      }
      // The row's other half (warp w +- 4, same lanes): exchange through shared memory with a
      // bounded handshake.  The slots alternate with the block parity; a warp writes slot b again
      // (block j+2) only after the exchange of block j+1, for which its partner had to arrive
      // after reading block j's value.
      red[(b * 2 + half) * kRows + r] = mx;
      __syncwarp();
      if (lane == 0) g4a::mbar_arrive(&barXchg[b * 4 + quarter]);
      ok = warp_wait(&barXchg[b * 4 + quarter], (uint32_t)(j >> 1) & 1u, abort_flag, p.err);
      if (!ok) break;
      mx = fmaxf(mx, red[(b * 2 + (half ^ 1)) * kRows + r]);
      // lazy rescale: the running max is only raised when it grows by more than 2^kRescaleP
      const bool grow = mx > m + kRescaleP;
      const float m_new = grow ? mx + kHeadroomP : m;
      const float alpha = grow ? ((m == -INFINITY) ? 0.f : g4a::fast_exp2(m - m_new)) : 1.f;
      lsum *= alpha;
      if (half == 0) {  // publish the row's factor for the correction warps (both halves agree)
        // slot b was read by the correction of block j-2
        if (j >= 2) {
          ok = warp_wait(&barCorr[b], (uint32_t)((j >> 1) - 1) & 1u, abort_flag, p.err);
          if (!ok) break;
        }
        const bool need = __any_sync(0xffffffffu, grow && m != -INFINITY);
        alpha_buf[b * kRows + r] = alpha;
        if (lane == 0) flag_buf[b * 4 + quarter] = need ? 1 : 0;
        __syncwarp();
        if (lane == 0) g4a::mbar_arrive(&barAlpha[b]);
      }
      m = m_new;
      // P = 2^(x - m) rounded to f16 pairs
      uint32_t pw[16];
      if (m == -INFINITY) {  // no visible key yet in this row
#pragma unroll
        for (int e = 0; e < 16; e++) pw[e] = 0u;
      } else if (interior) {
        const float nm = -m;
#pragma unroll
        for (int e = 0; e < 16; e++) {
          const float a = g4a::fast_exp2(fmaf(x[2 * e], c2, nm));
          const float bb = g4a::fast_exp2(fmaf(x[2 * e + 1], c2, nm));
          const __half2 h = __floats2half2_rn(a, bb);
          pw[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; e++) {
          const float a = g4a::fast_exp2(x[2 * e] - m);
          const float bb = g4a::fast_exp2(x[2 * e + 1] - m);
          const __half2 h = __floats2half2_rn(a, bb);
          pw[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
      }
      {  // l: the f16-rounded weights, summed in f32
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 16; e++) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&pw[e]));
          s4[e & 3] += f.x + f.y;
        }
        lsum += (s4[0] + s4[1]) + (s4[2] + s4[3]);
      }
      if constexpr (PAIR) {
        // the single P buffer was read by PV_{j-1}
        if (j >= 1) {
          ok = warp_wait(&barPV[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u, abort_flag, p.err);
          if (!ok) break;
        }
        // row r, keys 32 half .. 32 half + 31 = 16-byte chunks 4 half .. 4 half + 3 of the row's
        // 128 bytes, chunk c stored at c ^ (r & 7) (the 128-byte swizzle of the MMA descriptor)
        const uint32_t prow = sbase + C::OFF_P + (uint32_t)r * 128u;
#pragma unroll
        for (int cc = 0; cc < 4; cc++)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                           prow + (uint32_t)(((4 * half + cc) ^ (r & 7)) << 4)),
                       "r"(pw[4 * cc]), "r"(pw[4 * cc + 1]), "r"(pw[4 * cc + 2]), "r"(pw[4 * cc + 3])
                       : "memory");
        g4a::fence_proxy_async_smem();  // visible to the tensor core's reads
      } else {
        // P[b] was read by PV_{j-2}
        if (j >= 2) {
          ok = warp_wait(&barPV[b], (uint32_t)((j >> 1) - 1) & 1u, abort_flag, p.err);
          if (!ok) break;
          tc_fence_after();
        }
        tmem_st16(tmem + lane_addr + C::COL_P + (uint32_t)(b * (kKeys / 2) + 16 * half), pw);
        tmem_wait_st();
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) g4a::mbar_arrive(&barP[b]);
    }
    // pair: a warp that gave up stops the partner's waits too (the partner is still resident: it
    // leaves only through the cluster barrier at the end)
    if (PAIR && !ok && lane == 0)
      asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(mapa_shared(g4a::smem_u32((const void*)abort_flag), peer)),
                   "r"(1u)
                   : "memory");
    // epilogue: l = both halves' sums (added in the same order by both), then O / l, each half
    // of the row's threads storing half of the columns
    float* lsum_buf = reinterpret_cast<float*>(smem + C::OFF_LSUM);  // [half][row]
    lsum_buf[half * kRows + r] = lsum;
    __syncwarp();
    if (lane == 0) g4a::mbar_arrive(&barLsum[quarter]);
    if (ok) ok = warp_wait(&barLsum[quarter], 0u, abort_flag, p.err);
    const float l = ok ? lsum_buf[r] + lsum_buf[kRows + r] : 0.f;
    if (ok) ok = warp_wait(&barPV[(nb - 1) & 1], (uint32_t)((nb - 1) >> 1) & 1u, abort_flag, p.err);
    tc_fence_after();
    // O / l is staged in shared memory (the K and V rings are idle now: every MMA is done) as
    // HD/32 column boxes of [128 rows x 128 B] with the 128-byte swizzle (16-byte chunk q of row
    // r at q ^ (r & 7), so the 32 rows a warp writes spread over the banks), then written by
    // HD/32 TMA stores: the tile's rows are 16 tokens x 8 consecutive heads, a box of the
    // [T, nqh, HD] output, and rows past T are clipped.  (Per-thread stores of 32 different
    // rows per instruction took ~6 us per tile.)
    const float inv = (l > 0.f) ? 1.0f / l : 0.f;
    const uint32_t obox = sbase + C::OFF_K;  // HD/32 boxes of 16 KB
    g4a::fence_proxy_async_smem();  // after the async-proxy use of the rings
    static_assert(kRows * HD * 4 <= 2 * kStagesP * C::KV_BYTES, "the O tile fits the K and V rings");
#pragma unroll 1
    for (int c = 0; c < HD / 64; c++) {
      const int chunk = half * (HD / 64) + c;  // 32-column box
      uint32_t o[32];
      tmem_ld32(tmem + lane_addr + (uint32_t)(C::COL_O + chunk * 32), o);
      const uint32_t row = obox + (uint32_t)chunk * (kRows * 128) + (uint32_t)r * 128;
#pragma unroll
      for (int q = 0; q < 8; q++) {
        const uint32_t addr = row + (uint32_t)((q ^ (r & 7)) * 16);
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(__uint_as_float(o[4 * q]) * inv),
                     "f"(__uint_as_float(o[4 * q + 1]) * inv), "f"(__uint_as_float(o[4 * q + 2]) * inv),
                     "f"(__uint_as_float(o[4 * q + 3]) * inv)
                     : "memory");
      }
    }
    g4a::fence_proxy_async_smem();  // the generic-proxy writes are visible to the TMA store
    g4a::named_bar_sync(1, 8 * 32);  // every softmax warp reaches this, also after an abort
    if (warp == 4 && lane == 0 && ok) {
#pragma unroll 1
      for (int chunk = 0; chunk < HD / 32; chunk++)
        tma_store_3d(&tmo, obox + (uint32_t)chunk * (kRows * 128), chunk * 32 + (int)cr * HD, kvh * kHeadsPerKv, t0);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // shared memory read before exit
    }
  } else if (warp < 16) {  // warps 12-15 (the pair's exchange warps are 16-19)
    // ------------------------------------------------------------------ O correction
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const float* alpha_buf = reinterpret_cast<const float*>(smem + C::OFF_ALPHA);
    const volatile int* flag_buf = reinterpret_cast<const volatile int*>(smem + C::OFF_FLAG);
    for (int j = 0; j < nb; j++) {
      const int b = j & 1;
      if (!warp_wait(&barAlpha[b], (uint32_t)(j >> 1) & 1u, abort_flag, p.err)) break;
      // (block 0: the flag is clear, nothing has been accumulated yet)
      const float alpha = alpha_buf[b * kRows + r];
      const bool need = flag_buf[b * 4 + quarter] != 0;
      if (need) {
        // O holds PV_0 .. PV_{j-1}: wait for the last of them
        if (!warp_wait(&barPV[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u, abort_flag, p.err)) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HD / 32; c += 2) {  // two 32-column chunks in flight
          uint32_t o0[32], o1[32];
          tmem_ld32(tmem + lane_addr + (uint32_t)(C::COL_O + c * 32), o0);
          tmem_ld32(tmem + lane_addr + (uint32_t)(C::COL_O + c * 32 + 32), o1);
#pragma unroll
          for (int i = 0; i < 32; i++) {
            o0[i] = __float_as_uint(__uint_as_float(o0[i]) * alpha);
            o1[i] = __float_as_uint(__uint_as_float(o1[i]) * alpha);
          }
          tmem_st32(tmem + lane_addr + (uint32_t)(C::COL_O + c * 32), o0);
          tmem_st32(tmem + lane_addr + (uint32_t)(C::COL_O + c * 32 + 32), o1);
        }
        tmem_wait_st();
      }
      // barCorr[b] may only complete again (block j) once the PV issuer has consumed its
      // previous phase (block j-2), or the issuer could find the parity flipped back and wait for
      // good: wait until PV_{j-2} is done, which the issuer started after that phase.  (Without
      // this, corrections with nothing to rescale could run two blocks ahead of the issuer.)
      if (j >= 2 && !warp_wait(&barPV[b], (uint32_t)((j >> 1) - 1) & 1u, abort_flag, p.err)) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) g4a::mbar_arrive(&barCorr[b]);
    }
  } else if (PAIR) {
    // ------------------------------------------------------------------ score exchange (pair)
    // Warp 16 + q: rows 32 q .. 32 q + 31 (TMEM lane quarter q), all 64 keys of a block.
    const int quarter = warp & 3;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t xs = sbase + C::OFF_XS + (uint32_t)quarter * 8192u;
    const uint32_t xr = sbase + C::OFF_XR + (uint32_t)quarter * 8192u;
    const uint32_t xr_peer = mapa_shared(xr, peer);
    const uint32_t rx_peer = mapa_shared(g4a::smem_u32(&barRx[quarter]), peer);
    const uint32_t ok_peer = mapa_shared(g4a::smem_u32(&barOK[quarter]), peer);
    // Q into TMEM: row r = 32 quarter + lane (token t0 + r / 8, head kvh * 8 + r % 8), this CTA's
    // 64-dim chunks c = 0..3 as landed by the TMA load ([chunk][128 rows][128 B], 16-byte unit k
    // of row r at k ^ (r & 7)); dims 64 c + 8 k .. + 7 go to TMEM columns 32 c + 4 k .. + 3.
    bool ok = warp_wait(barQ, 0u, abort_flag, p.err);
    if (ok) {
      const int r = quarter * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < C::NCB; c++) {
        uint32_t w[32];
        const uint32_t row = sbase + C::OFF_XS + (uint32_t)c * C::Q_CHUNK + (uint32_t)r * 128u;
#pragma unroll
        for (int k = 0; k < 8; k++)
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(w[4 * k]), "=r"(w[4 * k + 1]), "=r"(w[4 * k + 2]), "=r"(w[4 * k + 3])
                       : "r"(row + (uint32_t)((k ^ (r & 7)) << 4))
                       : "memory");
        tmem_st32(tmem + lane_addr + C::COL_Q + (uint32_t)(32 * c), w);
      }
      tmem_wait_st();
      tc_fence_before();
    }
    // every exchange warp has read the slots before any of them stages scores there, and the
    // partner may copy its first scores into this CTA's receive slot (barOK phase 0)
    g4a::named_bar_sync(2, 4 * 32);
    if (ok && lane == 0) {
      g4a::mbar_arrive(barQ2);
      mbar_arrive_remote_relaxed(ok_peer);
    }
    for (int j = 0; ok && j < nb; j++) {
      const int b = j & 1;
      ok = warp_wait(&barS[b], (uint32_t)(j >> 1) & 1u, abort_flag, p.err);
      if (!ok) break;
      tc_fence_after();
      const uint32_t scol = tmem + lane_addr + C::COL_S + (uint32_t)(b * kKeys);
      // the partner has read block j-1 from its slot (phase 0: its Q), so its receive slot is free
      // and the copy from xs has landed
      ok = warp_wait_peer(&barOK[quarter], (uint32_t)j & 1u, abort_flag, p.err);
      if (!ok) break;
#pragma unroll 1
      for (int h = 0; h < 2; h++) {  // 32 keys at a time (registers)
        uint32_t own[32];
        tmem_ld32(scol + 32u * h, own);
#pragma unroll
        for (int g = 0; g < 8; g++)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(xs + (uint32_t)((8 * h + g) * 512 + lane * 16)),
                       "r"(own[4 * g]), "r"(own[4 * g + 1]), "r"(own[4 * g + 2]), "r"(own[4 * g + 3])
                       : "memory");
      }
      g4a::fence_proxy_async_smem();  // the staged scores are visible to the copy engine
      __syncwarp();
      if (lane == 0) {
        g4a::mbar_arrive_expect_tx(&barRx[quarter], 8192u);  // the partner's block j, into xr
        bulk_s2s_cluster(xr_peer, xs, 8192u, rx_peer);
      }
      ok = warp_wait_peer(&barRx[quarter], (uint32_t)j & 1u, abort_flag, p.err);
      if (!ok) break;
#pragma unroll 1
      for (int h = 0; h < 2; h++) {  // own partial again from TMEM, + the partner's, back into TMEM
        uint32_t own[32];
        tmem_ld32(scol + 32u * h, own);
#pragma unroll
        for (int g = 0; g < 8; g++) {
          float4 v;
          asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                       : "r"(xr + (uint32_t)((8 * h + g) * 512 + lane * 16))
                       : "memory");
          own[4 * g] = __float_as_uint(__uint_as_float(own[4 * g]) + v.x);
          own[4 * g + 1] = __float_as_uint(__uint_as_float(own[4 * g + 1]) + v.y);
          own[4 * g + 2] = __float_as_uint(__uint_as_float(own[4 * g + 2]) + v.z);
          own[4 * g + 3] = __float_as_uint(__uint_as_float(own[4 * g + 3]) + v.w);
        }
        tmem_st32(scol + 32u * h, own);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();  // every lane has read the slot and stored its sums
      if (lane == 0) {
        g4a::mbar_arrive(&barSx[b * 4 + quarter]);
        mbar_arrive_remote_relaxed(ok_peer);  // the slot's values are in registers already
      }
    }
    if (!ok && lane == 0)  // stop the partner's waits too
      asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(mapa_shared(g4a::smem_u32((const void*)abort_flag), peer)),
                   "r"(1u)
                   : "memory");
  }
  // The single-lane roles above leave their warps diverged: reconverge every warp before the
  // CTA barrier, so that it waits for each lane (an aligned barrier reached by part of a warp
  // is not a barrier for the rest of it).
  __syncwarp();
  tc_fence_before();
  if constexpr (PAIR) cluster_sync_all(); else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
  }
}

g4a_status get_encoder_p(g4a_ctx* ctx, PFN_cuTensorMapEncodeTiled_v12000* out) {
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

// {64, heads, rows, chunks} f16 map with the chunk index outermost (stride 128 B), 128-byte
// swizzle, box {64, box_heads, box_rows, box_chunks}: one TMA op lands a tile as `box_chunks`
// column boxes of [box_heads * box_rows rows x 128 B].
// The f32 output [T, nqh, HD] as {HD, nqh, T} with 128-byte swizzle and box {32, 8, 16}: one
// TMA store writes 32 columns of a tile's 16 tokens x 8 heads; rows past T are not written.
g4a_status encode_out_map(g4a_ctx* ctx, CUtensorMap* map, float* base, uint32_t hd, uint32_t nqh, uint32_t T) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (g4a_status s = get_encoder_p(ctx, &enc)) return s;
  cuuint64_t dims[3] = {hd, nqh, T};
  cuuint64_t strides[2] = {(cuuint64_t)hd * 4, (cuuint64_t)nqh * hd * 4};
  cuuint32_t box[3] = {32, (cuuint32_t)kHeadsPerKv, (cuuint32_t)kTokPerTile};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return g4a_fail(G4A_ECUDA, "cuTensorMapEncodeTiled failed (%d) for the output", (int)r);
  return G4A_OK;
}

g4a_status encode_rows_map(g4a_ctx* ctx, CUtensorMap* map, const void* base, uint32_t hd, uint32_t heads,
                           uint64_t rows, uint32_t box_heads, uint32_t box_rows, uint32_t box_chunks,
                           const char* what) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  if (g4a_status s = get_encoder_p(ctx, &enc)) return s;
  const cuuint64_t ncb = hd / 64;
  cuuint64_t dims[4] = {64, heads, rows, ncb};
  cuuint64_t strides[3] = {(cuuint64_t)hd * 2, (cuuint64_t)heads * hd * 2, 128};
  cuuint32_t box[4] = {64, box_heads, box_rows, box_chunks};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return g4a_fail(G4A_ECUDA, "cuTensorMapEncodeTiled failed (%d) for %s", (int)r, what);
  return G4A_OK;
}

// HD = head dims of the layer; the pair instance (HD 512) gives each CTA of a cluster 256.
template <int HD>
g4a_status launch_prefill(g4a_ctx* ctx, const uint16_t* q16, const uint16_t* k, const uint16_t* v, float* out,
                          uint32_t T, uint32_t start_pos, uint32_t nqh, uint32_t nkh, float scale, uint32_t window) {
  constexpr bool kPair = HD == 512;
  constexpr int kHdCta = kPair ? HD / 2 : HD;
  using C = PCfg<kHdCta, kPair>;
  auto kernel = prefill_attn_kernel<kHdCta, kPair>;
  static std::atomic<bool> configured[64];
  if (ctx->device >= 64 || !configured[ctx->device].load()) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    if (e != cudaSuccess) return g4a_cuda_fail(e, "cudaFuncSetAttribute(prefill_attn_kernel)");
    if (ctx->device < 64) configured[ctx->device].store(true);
  }
  CUtensorMap mq, mk, mv;
  const uint64_t rows = (uint64_t)start_pos + T;
  // pair: each CTA loads its NCB of the HD / 64 chunks of a K or V block (Q is read into TMEM)
  if (g4a_status s = encode_rows_map(ctx, &mk, k, HD, nkh, rows, 1, kKeys, C::NCB, "the K cache")) return s;
  if (g4a_status s = encode_rows_map(ctx, &mv, v, HD, nkh, rows, 1, kKeys, C::NCB, "the V cache")) return s;
  // pair: each CTA loads its NCB of the HD / 64 chunks of the Q tile
  if (g4a_status s = encode_rows_map(ctx, &mq, q16, HD, nqh, T, kHeadsPerKv, kTokPerTile, C::NCB, "q16")) return s;
  CUtensorMap mo;
  if (g4a_status s = encode_out_map(ctx, &mo, out, HD, nqh, T)) return s;
  PrefillParams p = {};
  p.out = out;
  p.T = (int)T;
  p.start_pos = start_pos;
  p.nqh = (int)nqh;
  p.nkh = (int)nkh;
  p.ntiles = (int)((T + kTokPerTile - 1) / kTokPerTile);
  p.scale_log2 = scale * kLog2eP;
  p.window = window;
  p.err = ctx->dev_err_dev;
  g4a_prof_scope ps(ctx, G4A_PROF_PREFILL_ATTN);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.ntiles * p.nkh * (kPair ? 2 : 1)));
  cfg.blockDim = dim3((unsigned)C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;  // pair: the two CTAs of a tile
  attr[1].val.clusterDim.x = kPair ? 2 : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = kPair ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, mq, mk, mv, mo, p);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "launch prefill_attn_kernel");
  return G4A_OK;
}

}  // namespace

extern "C" g4a_status g4a_prefill_attn(g4a_ctx* ctx, const uint16_t* q16, const uint16_t* k_cache,
                                       const uint16_t* v_cache, float* out, uint32_t T, uint32_t start_pos,
                                       uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim, float scale,
                                       uint32_t sliding_window) {
  G4A_CHECK_CTX(ctx);
  if (!q16 || !k_cache || !v_cache || !out) return g4a_fail(G4A_EINVAL, "g4a_prefill_attn: null pointer");
  if (num_q_heads == 0 || num_kv_heads == 0 || num_kv_heads > num_q_heads)
    return g4a_fail(G4A_EINVAL, "g4a_prefill_attn: bad head counts nqh=%u nkh=%u", num_q_heads, num_kv_heads);
  if (head_dim == 0 || head_dim > 512 || (head_dim % 8) != 0)
    return g4a_fail(G4A_EINVAL, "g4a_prefill_attn: head_dim %u must be a multiple of 8 in [8, 512]", head_dim);
  if ((((uintptr_t)q16) | ((uintptr_t)k_cache) | ((uintptr_t)v_cache) | ((uintptr_t)out)) & 15u)
    return g4a_fail(G4A_EINVAL, "g4a_prefill_attn: pointers must be 16-byte aligned");
  if ((uint64_t)start_pos + T > 0xffffffffull) return g4a_fail(G4A_EINVAL, "g4a_prefill_attn: start_pos + T overflows");
  if (T == 0) return G4A_OK;
  // The tcgen05 kernel covers GQA 8:1 at head_dim 128 and 256, and at head_dim 512 (Gemma's
  // global layers) as CTA pairs; every other shape runs through the decode kernels.
  if (num_q_heads != (uint32_t)kHeadsPerKv * num_kv_heads || (head_dim != 128 && head_dim != 256 && head_dim != 512))
    return prefill_via_decode(ctx, q16, k_cache, v_cache, out, T, start_pos, num_q_heads, num_kv_heads, head_dim,
                              scale, sliding_window);
  if (head_dim == 512)
    return launch_prefill<512>(ctx, q16, k_cache, v_cache, out, T, start_pos, num_q_heads, num_kv_heads, scale,
                               sliding_window);
  if (head_dim == 256)
    return launch_prefill<256>(ctx, q16, k_cache, v_cache, out, T, start_pos, num_q_heads, num_kv_heads, scale,
                               sliding_window);
  return launch_prefill<128>(ctx, q16, k_cache, v_cache, out, T, start_pos, num_q_heads, num_kv_heads, scale,
                             sliding_window);
}
