// Projection GEMVs around attention: out[m] = sum_k W[m, k] * input[k] with the weight in the
// reference's f16, Q8 or 4-bit block-affine storage (shaders/matmul_quant.wgsl,
// matmul_quant_mr4.wgsl, matmul_q8.wgsl, matmul_q8_mr.wgsl, matmul_q4k.wgsl, matmul_q4k_mr.wgsl;
// dispatched at src/engine.ts:2043-2053 and :2096).
//
// Arithmetic order.  Every one of those shaders computes a row with a 256-thread workgroup:
// thread t sums term(k) for k = t, t + 256, t + 512, ... in that order from 0.0, then the
// partials fold with `for stride = 128; stride > 0; stride >>= 1: p[t] += p[t + stride]`
// (e.g. matmul_quant.wgsl:30-50, matmul_q8_mr.wgsl:49-85).  The per-element terms are
//   f16 : f32(w) * x                          (matmul_quant.wgsl:34)
//   Q8  : (f32(q) * f32(scale)) * x            (matmul_q8.wgsl:49, matmul_q8_mr.wgsl:58-61)
//   Q4K : (f32(scale) * f32(nib) + f32(min)) * x (matmul_q4k.wgsl:54, matmul_q4k_mr.wgsl:74-81)
// with every product and sum rounded separately (no contraction).  Here one warp computes a
// row: lane l plays the eight workgroup threads t = 8l .. 8l+7, so one 16-byte (f16), 8-byte
// (Q8) or 4-byte (Q4K) load per lane per 256-element step brings the lane exactly its threads'
// elements, and a warp load is one contiguous 512 / 256 / 128-byte run of the row.  The tree
// levels 128 .. 8 pair thread t with t + stride = 8(l + stride/8) + e, i.e. lane l + stride/8
// with the same e (done as a butterfly that halves the values per lane at each level).  The
// result is bit-identical to the shader's order.  The f16 path for N % 8 != 0 (or an unaligned
// weight) uses the other natural layout, threads t = l + 32e, with scalar 2-byte loads.
//
// Roofline: HBM-bound streaming of the weight (2 / 1.0625 / 0.625 bytes per element); the
// input vector is staged once per CTA in shared memory.  The kernel waits for the previous
// kernel (programmatic dependent launch) only before it reads `input`: the weight does not
// depend on it, so each warp loads its first row's weights before the wait.
#include <cuda_fp16.h>

#include "g4a_internal.cuh"

namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr uint32_t kMaxGemvN = 49152;  // input staged in shared memory (192 KB)

struct GemvJob {
  const void* w;
  const __half* s;
  float* out;
  uint32_t M;
  uint32_t row0;  // first virtual row of this job
};
struct GemvJobs {
  GemvJob j[G4A_MATMUL_MAX_JOBS];
  int n;
  uint32_t rows;  // sum of M
};

// Streaming loads of the (read-only, read-once) weight.  Not volatile: the compiler may batch
// them ahead of the arithmetic that consumes them.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream4(const void* p) {
  uint32_t v;
  asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Byte i (0..3) of `w` as the float 2^23 + byte, built by one byte permute: the float's low
// byte is the data byte and its top byte is 0x4B (2^23 has exponent byte 0x4B, mantissa 0), so
// subtracting the bias is exact and gives small integers without the conversion unit.
template <int I>
__device__ __forceinline__ float byte_biased(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)I));
}

__device__ __forceinline__ const GemvJob& job_of(const GemvJobs& jobs, uint32_t r, uint32_t& m) {
  int q = 0;
#pragma unroll
  for (int i = 1; i < G4A_MATMUL_MAX_JOBS; i++)
    if (i < jobs.n && r >= jobs.j[i].row0) q = i;
  m = r - jobs.j[q].row0;
  return jobs.j[q];
}

// Weight bytes of the 256-element step j of row m as seen by `lane`.
template <uint32_t FMT>
__device__ __forceinline__ const void* step_ptr(const GemvJob& jb, uint32_t m, uint32_t N, uint32_t j, int lane) {
  const size_t k = (size_t)m * N + 256u * j + 8u * (uint32_t)lane;  // first element of the lane
  if constexpr (FMT == G4A_WEIGHT_F16) return reinterpret_cast<const __half*>(jb.w) + k;
  if constexpr (FMT == G4A_WEIGHT_Q8) return reinterpret_cast<const uint8_t*>(jb.w) + k;
  return reinterpret_cast<const uint32_t*>(jb.w) + k / 8;
}

// One 256-element step of a row as one lane sees it: its eight weights (and their scales).
template <uint32_t FMT>
struct StepRaw;
template <>
struct StepRaw<G4A_WEIGHT_F16> {
  uint4 w;
};
template <>
struct StepRaw<G4A_WEIGHT_Q8> {
  uint2 w;
  __half sc;
};
template <>
struct StepRaw<G4A_WEIGHT_Q4K> {
  uint32_t w;
  __half sc, mn;
};
// Steps whose loads are issued together before any of them is consumed: 8 steps hold a whole
// row of the reference's projections (N <= 2048) in one round trip.
constexpr int kStepBatch = 8;

template <uint32_t FMT>
__device__ __forceinline__ StepRaw<FMT> load_step(const GemvJob& jb, uint32_t m, uint32_t N, uint32_t j, int lane) {
  StepRaw<FMT> r;
  const uint32_t k0 = 256u * j + 8u * (uint32_t)lane;
  if constexpr (FMT == G4A_WEIGHT_F16) {
    r.w = ld_stream16(step_ptr<FMT>(jb, m, N, j, lane));
  } else if constexpr (FMT == G4A_WEIGHT_Q8) {
    r.w = ld_stream8(step_ptr<FMT>(jb, m, N, j, lane));
    // the lane's 8 elements lie in one 32-element block: (m N + k0) / 32
    r.sc = __ldg(jb.s + (size_t)m * (N / 32u) + (k0 >> 5));
  } else {
    r.w = ld_stream4(step_ptr<FMT>(jb, m, N, j, lane));
    // super-block j = k0 >> 8, sub-block (k0 & 255) >> 5 = lane / 4
    const __half* meta = jb.s + (size_t)m * (N / 256u) * 16u + 16u * j;
    r.sc = __ldg(meta + (lane >> 2));
    r.mn = __ldg(meta + 8 + (lane >> 2));
  }
  return r;
}

// Packed pairs of f32 for the sm_100 two-lane FP32 instructions (add / sub / mul / fma .rn.f32x2):
// each rounds both halves exactly like the scalar instruction, so pairing elements halves the
// instruction count of the per-element terms without changing a bit.  Low half = first element.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// The partial sums of a lane's eight threads t = 8 lane + e, as pairs (e = 2i, 2i + 1).
struct Acc8 {
  uint64_t p[4];
};

// The lane's eight input elements of step j (256 j + 8 lane .. + 7) as four pairs.
__device__ __forceinline__ void load_x_pairs(const float* xs, uint32_t j, int lane, uint64_t (&x)[4]) {
  const uint32_t k0 = 256u * j + 8u * (uint32_t)lane;
  const ulonglong2 xa = *reinterpret_cast<const ulonglong2*>(xs + k0);
  const ulonglong2 xb = *reinterpret_cast<const ulonglong2*>(xs + k0 + 4);
  x[0] = xa.x;
  x[1] = xa.y;
  x[2] = xb.x;
  x[3] = xb.y;
}

// acc[e] += term(element 256 j + 8 lane + e) for the lane's eight threads, two elements per
// instruction (every product and sum still separately rounded, in the shader's order); x holds
// the lane's eight input elements of the step.
template <uint32_t FMT>
__device__ __forceinline__ void consume_step_x(const StepRaw<FMT>& r, const uint64_t (&x)[4], Acc8& acc) {
  if constexpr (FMT == G4A_WEIGHT_F16) {
    // scalar: this path streams at the copy rate already, and the paired form of f32(w) * x + acc
    // did not keep the shader's separate roundings
    const uint32_t w4[4] = {r.w.x, r.w.y, r.w.z, r.w.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float2 w = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
      const float2 xv = f2_unpack(x[i]);
      float2 a = f2_unpack(acc.p[i]);
      a.x = __fadd_rn(a.x, __fmul_rn(w.x, xv.x));
      a.y = __fadd_rn(a.y, __fmul_rn(w.y, xv.y));
      acc.p[i] = f2_pack(a.x, a.y);
    }
  } else if constexpr (FMT == G4A_WEIGHT_Q8) {
    // int8 q as the byte u = q + 128 (flip the sign bit of every byte): 2^23 + u - (2^23 + 128)
    const float sc = __half2float(r.sc);
    const uint64_t sc2 = f2_pack(sc, sc), bias2 = f2_pack(8388736.0f, 8388736.0f);
    const uint32_t u0 = r.w.x ^ 0x80808080u, u1 = r.w.y ^ 0x80808080u;
    const uint64_t q[4] = {f2_pack(byte_biased<0>(u0), byte_biased<1>(u0)),
                           f2_pack(byte_biased<2>(u0), byte_biased<3>(u0)),
                           f2_pack(byte_biased<0>(u1), byte_biased<1>(u1)),
                           f2_pack(byte_biased<2>(u1), byte_biased<3>(u1))};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float2 t = f2_unpack(f2_mul(f2_mul(f2_sub(q[i], bias2), sc2), x[i]));
      float2 a = f2_unpack(acc.p[i]);
      a.x = __fadd_rn(a.x, t.x);
      a.y = __fadd_rn(a.y, t.y);
      acc.p[i] = f2_pack(a.x, a.y);
    }
  } else {
    // Nibbles 0, 2, 4, 6 are the bytes of `lo`, nibbles 1, 3, 5, 7 those of `hi`.
    const uint32_t lo = r.w & 0x0F0F0F0Fu, hi = (r.w >> 4) & 0x0F0F0F0Fu;
    const uint64_t nb[4] = {f2_pack(byte_biased<0>(lo), byte_biased<0>(hi)),
                            f2_pack(byte_biased<1>(lo), byte_biased<1>(hi)),
                            f2_pack(byte_biased<2>(lo), byte_biased<2>(hi)),
                            f2_pack(byte_biased<3>(lo), byte_biased<3>(hi))};
    const float sc = __half2float(r.sc), mn = __half2float(r.mn);
    const uint64_t sc2 = f2_pack(sc, sc), mn2 = f2_pack(mn, mn), bias2 = f2_pack(8388608.0f, 8388608.0f);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      // The shader's RN(RN(scale * nib) + min) is one fused multiply-add here: scale is an f16
      // value and nib an integer below 16, so their product has at most 15 significant bits
      // within the f32 normal range and is exact; the fma's single rounding is then the sum's.
      const uint64_t wv = f2_fma(sc2, f2_sub(nb[i], bias2), mn2);
      const float2 t = f2_unpack(f2_mul(wv, x[i]));
      float2 a = f2_unpack(acc.p[i]);
      a.x = __fadd_rn(a.x, t.x);
      a.y = __fadd_rn(a.y, t.y);
      acc.p[i] = f2_pack(a.x, a.y);
    }
  }
}

template <uint32_t FMT>
__device__ __forceinline__ void consume_step(const StepRaw<FMT>& r, uint32_t j, int lane, const float* xs,
                                             Acc8& acc) {
  uint64_t x[4];
  load_x_pairs(xs, j, lane, x);
  consume_step_x<FMT>(r, x, acc);
}

__device__ __forceinline__ void acc_unpack(const Acc8& acc, float (&a)[8]) {
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 v = f2_unpack(acc.p[i]);
    a[2 * i] = v.x;
    a[2 * i + 1] = v.y;
  }
}

// The 256-thread tree for threads t = 8 lane + e, as a butterfly that halves the values each
// lane holds at every level, so 12 shuffles do what 40 would in the direct form.  Each add
// pairs exactly the shader's operands p[t] and p[t + stride]; only which lane computes it (and
// so the operand order) changes, and IEEE addition is commutative.  Every lane returns p[0].
//   stride 128: lanes L and L^16 (t = 8(L&15) + e): the lower lane keeps e 0-3, the upper 4-7;
//               then lane L holds t = 8(L&15) + 4(L>>4) + e, e < 4.
//   stride  64: lanes L and L^8: lower keeps e 0-1, upper 2-3 -> t = 8(L&7) + 4(L>>4) + 2((L>>3)&1) + e.
//   stride  32: lanes L and L^4: lower keeps e 0, upper 1 -> one value, t = 8(L&3) + 4(L>>4) +
//               2((L>>3)&1) + ((L>>2)&1).
//   strides 16, 8, 4, 2, 1: partners at lane bits 1, 0, 4, 3, 2 (both lanes form the sum).
__device__ __forceinline__ float tree_butterfly(const float (&a)[8], int lane) {
  const bool u16 = (lane & 16) != 0, u8 = (lane & 8) != 0, u4 = (lane & 4) != 0;
  float b[4];
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const float keep = u16 ? a[e + 4] : a[e];
    const float send = u16 ? a[e] : a[e + 4];
    b[e] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
  float c[2];
#pragma unroll
  for (int e = 0; e < 2; e++) {
    const float keep = u8 ? b[e + 2] : b[e];
    const float send = u8 ? b[e] : b[e + 2];
    c[e] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
  float d;
  {
    const float keep = u4 ? c[1] : c[0];
    const float send = u4 ? c[0] : c[1];
    d = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 2));   // stride 16
  d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 1));   // stride 8
  d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 16));  // stride 4
  d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 8));   // stride 2
  d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 4));   // stride 1
  return d;
}

// Stage input[0, N) into shared memory (after the PDL wait).
__device__ __forceinline__ void stage_input(const float* __restrict__ x, uint32_t N, float* xs, uint32_t padded) {
  const int t = threadIdx.x;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (N & 3u) == 0) {
    for (uint32_t i = t; i < N / 4; i += kGemvThreads)
      reinterpret_cast<float4*>(xs)[i] = __ldg(reinterpret_cast<const float4*>(x) + i);
  } else {
    for (uint32_t i = t; i < N; i += kGemvThreads) xs[i] = __ldg(x + i);
  }
  for (uint32_t i = N + t; i < padded; i += kGemvThreads) xs[i] = 0.f;
}

// Vector path: N % 8 == 0 (Q8: N % 32, Q4K: N % 256), 16-byte aligned weights.
template <uint32_t FMT>
__global__ void __launch_bounds__(kGemvThreads, 3) gemv_kernel(const float* __restrict__ x, uint32_t N,
                                                            const __grid_constant__ GemvJobs jobs) {
  extern __shared__ float4 gemv_smem[];
  float* xs = reinterpret_cast<float*>(gemv_smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t steps = (N + 255u) / 256u;
  const uint32_t stride = gridDim.x * kGemvWarps;
  // A lane's steps: all 256-element steps, and the partial last one where its 8 elements lie
  // below N.  Threads past N keep a zero partial, as in the shader (their loop never runs).
  const uint32_t mine = steps - ((steps > N / 256u && 256u * (steps - 1) + 8u * lane >= N) ? 1u : 0u);
  constexpr int B = kStepBatch;
  // Software pipeline over a warp's rows (Q8, Q4K: a batch is 24-32 registers): the first
  // batch of the next row is loaded while the current row is summed.  f16 batches are twice as
  // large, and two of them would halve the CTAs an SM holds, so f16 loads each row's batch at
  // the row's start.  The weight does not depend on the preceding kernel, so the first row's
  // batch is loaded before the programmatic-launch wait, overlapping that kernel's tail.
  constexpr bool kPipe = FMT != G4A_WEIGHT_F16;
  StepRaw<FMT> nxt[B];
  uint32_t r = blockIdx.x * kGemvWarps + warp;
  auto load_batch = [&](StepRaw<FMT>(&raw)[B], uint32_t row, uint32_t j0) {
    uint32_t m;
    const GemvJob& jb = job_of(jobs, row, m);
#pragma unroll
    for (int u = 0; u < B; u++)
      if (j0 + u < mine) raw[u] = load_step<FMT>(jb, m, N, j0 + u, lane);
  };
  if (r < jobs.rows) load_batch(nxt, r, 0);
  g4a::pdl_wait_primary();  // `input` is written by the preceding kernel
  stage_input(x, N, xs, steps * 256u);
  __syncthreads();
  g4a::pdl_launch_dependents();
  // Sums row `row` whose first batch is in `raw` (the array is reused for later batches).
  auto sum_row = [&](StepRaw<FMT>(&raw)[B], uint32_t row) {
    uint32_t m;
    const GemvJob& jb = job_of(jobs, row, m);
    Acc8 acc = {{0, 0, 0, 0}};  // +0.0f pairs
#pragma unroll
    for (int u = 0; u < B; u++)
      if ((uint32_t)u < mine) consume_step<FMT>(raw[u], u, lane, xs, acc);
    for (uint32_t j = B; j < mine; j += B) {  // rows longer than one batch
      load_batch(raw, row, j);
#pragma unroll
      for (int u = 0; u < B; u++)
        if (j + u < mine) consume_step<FMT>(raw[u], j + u, lane, xs, acc);
    }
    float a[8];
    acc_unpack(acc, a);
    const float v = tree_butterfly(a, lane);
    if (lane == 0) jb.out[m] = v;
  };
  if constexpr (kPipe) {
    for (; r < jobs.rows; r += stride) {
      StepRaw<FMT> cur[B];
#pragma unroll
      for (int u = 0; u < B; u++) cur[u] = nxt[u];
      if (r + stride < jobs.rows) load_batch(nxt, r + stride, 0);
      sum_row(cur, r);
    }
  } else {
    for (bool first = true; r < jobs.rows; r += stride, first = false) {
      if (!first) load_batch(nxt, r, 0);
      sum_row(nxt, r);
    }
  }
}

// Rows of exactly S full 256-element steps (N = 256 S, S <= 8: every projection of the
// reference model): a lane's row pointer is formed once and every step is a compile-time
// offset from it, with no per-step bounds predicate.  Q8 and Q4K load the next row's steps
// while the current row is summed; f16 (twice the registers per step) loads at the row start.
template <uint32_t FMT, int S, bool XREG = false>
__global__ void __launch_bounds__(kGemvThreads, XREG ? 2 : 3) gemv_fixed_kernel(const float* __restrict__ x,
                                                                     const __grid_constant__ GemvJobs jobs) {
  constexpr uint32_t N = 256u * S;
  extern __shared__ float4 gemv_smem[];
  float* xs = reinterpret_cast<float*>(gemv_smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * kGemvWarps;
  auto load_row = [&](StepRaw<FMT>(&raw)[S], uint32_t row) {
    uint32_t m;
    const GemvJob& jb = job_of(jobs, row, m);
    if constexpr (FMT == G4A_WEIGHT_F16) {
      const __half* w = reinterpret_cast<const __half*>(jb.w) + (size_t)m * N + 8u * lane;
#pragma unroll
      for (int u = 0; u < S; u++) raw[u].w = ld_stream16(w + 256 * u);
    } else if constexpr (FMT == G4A_WEIGHT_Q8) {
      const uint8_t* w = reinterpret_cast<const uint8_t*>(jb.w) + (size_t)m * N + 8u * lane;
      const __half* sc = jb.s + (size_t)m * (N / 32u) + (lane >> 2);  // block 8 u + lane / 4
#pragma unroll
      for (int u = 0; u < S; u++) {
        raw[u].w = ld_stream8(w + 256 * u);
        raw[u].sc = __ldg(sc + 8 * u);
      }
    } else {
      const uint32_t* w = reinterpret_cast<const uint32_t*>(jb.w) + (size_t)m * (N / 8u) + lane;
      const __half* meta = jb.s + (size_t)m * (16u * S) + (lane >> 2);  // super-block u, sub lane / 4
#pragma unroll
      for (int u = 0; u < S; u++) {
        raw[u].w = ld_stream4(w + 32 * u);
        raw[u].sc = __ldg(meta + 16 * u);
        raw[u].mn = __ldg(meta + 16 * u + 8);
      }
    }
  };
  // XREG (Q8 and Q4K with many rows): the lane's S x 8 input elements stay in registers across
  // the warp's rows (the input is the same for every row), so the inner loop reads no shared
  // memory, at two CTAs per SM instead of three.  Few rows (the per-layer projections) are
  // latency-bound and keep the shared-memory form.
  static_assert(!XREG || FMT != G4A_WEIGHT_F16, "XREG is for the quantised formats");
  uint64_t xr[XREG ? S : 1][4];
  auto sum_row = [&](const StepRaw<FMT>(&raw)[S], uint32_t row) {
    Acc8 acc = {{0, 0, 0, 0}};  // +0.0f pairs
#pragma unroll
    for (int u = 0; u < S; u++) {
      if constexpr (XREG)
        consume_step_x<FMT>(raw[u], xr[u], acc);
      else
        consume_step<FMT>(raw[u], (uint32_t)u, lane, xs, acc);
    }
    float a[8];
    acc_unpack(acc, a);
    const float v = tree_butterfly(a, lane);
    uint32_t m;
    const GemvJob& jb = job_of(jobs, row, m);
    if (lane == 0) jb.out[m] = v;
  };
  uint32_t r = blockIdx.x * kGemvWarps + warp;
  StepRaw<FMT> nxt[S];
  if (r < jobs.rows) load_row(nxt, r);  // independent of the preceding kernel
  g4a::pdl_wait_primary();              // `input` is written by the preceding kernel
  stage_input(x, N, xs, N);
  __syncthreads();
  g4a::pdl_launch_dependents();
  if constexpr (XREG) {
#pragma unroll
    for (int u = 0; u < S; u++) load_x_pairs(xs, (uint32_t)u, lane, xr[u]);
  }
  if constexpr (FMT != G4A_WEIGHT_F16) {
    for (; r < jobs.rows; r += stride) {
      StepRaw<FMT> cur[S];
#pragma unroll
      for (int u = 0; u < S; u++) cur[u] = nxt[u];
      if (r + stride < jobs.rows) load_row(nxt, r + stride);
      if constexpr (XREG) {
        // Many rows: pull the row after the next one into L2, one 128-byte line per lane (lane
        // 31 takes the line where the row's scales start), so that the register loads of the
        // next pass find it there; no registers are held for it.  Q8 lm-head 262144 x 1536:
        // 117 -> 106.5 us; the 4-bit kernel is issue-bound and unchanged.
        const uint32_t rr = r + 2u * stride;
        if (rr < jobs.rows && rr > r) {
          uint32_t m2;
          const GemvJob& jb2 = job_of(jobs, rr, m2);
          constexpr uint32_t RB = FMT == G4A_WEIGHT_Q8 ? N : N / 2u;  // weight bytes of a row
          const char* w = reinterpret_cast<const char*>(jb2.w) + (size_t)m2 * RB;
          if ((uint32_t)lane * 128u < RB) asm volatile("prefetch.global.L2 [%0];" ::"l"(w + lane * 128) : "memory");
          const __half* sp = jb2.s + (size_t)m2 * (FMT == G4A_WEIGHT_Q8 ? N / 32u : 16u * S);
          if (lane == 31) asm volatile("prefetch.global.L2 [%0];" ::"l"(sp) : "memory");
        }
      }
      sum_row(cur, r);
    }
  } else {
    for (bool first = true; r < jobs.rows; r += stride, first = false) {
      if (!first) load_row(nxt, r);
      sum_row(nxt, r);
    }
  }
}

// Scalar f16 path for any N and 2-byte aligned weights: threads t = lane + 32 e.
__global__ void __launch_bounds__(kGemvThreads) gemv_f16_scalar_kernel(const float* __restrict__ x, uint32_t N,
                                                                       const __grid_constant__ GemvJobs jobs) {
  extern __shared__ float4 gemv_smem[];
  float* xs = reinterpret_cast<float*>(gemv_smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  g4a::pdl_wait_primary();
  stage_input(x, N, xs, N);
  __syncthreads();
  g4a::pdl_launch_dependents();
  for (uint32_t r = blockIdx.x * kGemvWarps + warp; r < jobs.rows; r += gridDim.x * kGemvWarps) {
    uint32_t m;
    const GemvJob& jb = job_of(jobs, r, m);
    const __half* w = reinterpret_cast<const __half*>(jb.w) + (size_t)m * N;
    float p[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (uint32_t base = 0; base < N; base += 256u) {
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const uint32_t k = base + (uint32_t)lane + 32u * e;
        if (k < N) p[e] = __fadd_rn(p[e], __fmul_rn(__half2float(w[k]), xs[k]));
      }
    }
    // strides 128, 64, 32 pair e with e + 4, e + 2, e + 1 in the same lane
#pragma unroll
    for (int e = 0; e < 4; e++) p[e] = __fadd_rn(p[e], p[e + 4]);
    p[0] = __fadd_rn(p[0], p[2]);
    p[1] = __fadd_rn(p[1], p[3]);
    float v = __fadd_rn(p[0], p[1]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, off));
    if (lane == 0) jb.out[m] = v;
  }
}

}  // namespace

extern "C" {

g4a_status g4a_matmul_group(g4a_ctx* ctx, uint32_t weight_format, const float* input, uint32_t N,
                            const g4a_matmul_job* jobs, uint32_t num_jobs) {
  G4A_CHECK_CTX(ctx);
  if (weight_format > G4A_WEIGHT_Q4K) return g4a_fail(G4A_EINVAL, "g4a_matmul: unknown weight_format %u", weight_format);
  if (num_jobs == 0 || num_jobs > G4A_MATMUL_MAX_JOBS || !jobs)
    return g4a_fail(G4A_EINVAL, "g4a_matmul_group: num_jobs %u not in [1, %d]", num_jobs, G4A_MATMUL_MAX_JOBS);
  if (N > kMaxGemvN) return g4a_fail(G4A_EINVAL, "g4a_matmul: N %u > %u", N, kMaxGemvN);
  if (weight_format == G4A_WEIGHT_Q8 && (N % 32u) != 0)
    return g4a_fail(G4A_EINVAL, "g4a_matmul: Q8 needs N %% 32 == 0 (N = %u)", N);
  if (weight_format == G4A_WEIGHT_Q4K && (N % 256u) != 0)
    return g4a_fail(G4A_EINVAL, "g4a_matmul: Q4K needs N %% 256 == 0 (N = %u)", N);
  GemvJobs J = {};
  bool vec = (N % 8u) == 0;
  uint64_t rows = 0;
  for (uint32_t i = 0; i < num_jobs; i++) {
    const g4a_matmul_job& s = jobs[i];
    if (s.M == 0) continue;
    if (!s.weight || !s.out) return g4a_fail(G4A_EINVAL, "g4a_matmul: job %u: null weight or out", i);
    if (weight_format != G4A_WEIGHT_F16 && !s.scales)
      return g4a_fail(G4A_EINVAL, "g4a_matmul: job %u: null scales", i);
    const uintptr_t wa = reinterpret_cast<uintptr_t>(s.weight);
    if (weight_format == G4A_WEIGHT_F16) {
      if (wa & 1u) return g4a_fail(G4A_EINVAL, "g4a_matmul: job %u: f16 weight not 2-byte aligned", i);
      if (wa & 15u) vec = false;
    } else if (wa & 15u) {
      return g4a_fail(G4A_EINVAL, "g4a_matmul: job %u: quantised weight not 16-byte aligned", i);
    }
    if (s.scales && (reinterpret_cast<uintptr_t>(s.scales) & 1u))
      return g4a_fail(G4A_EINVAL, "g4a_matmul: job %u: scales not 2-byte aligned", i);
    J.j[J.n] = GemvJob{s.weight, reinterpret_cast<const __half*>(s.scales), s.out, s.M, (uint32_t)rows};
    J.n++;
    rows += s.M;
  }
  if (rows == 0) return G4A_OK;
  if (rows > 0xffffffffull - 2u * 148u * kGemvWarps) return g4a_fail(G4A_EINVAL, "g4a_matmul: too many rows");
  if (!input) return g4a_fail(G4A_EINVAL, "g4a_matmul: null input");
  J.rows = (uint32_t)rows;
  const uint32_t padded = (N + 255u) / 256u * 256u;
  const size_t smem = (size_t)(vec ? padded : (N ? N : 1u)) * sizeof(float);
  // Up to 8 CTAs of 8 warps per SM, one row per warp per pass.
  const uint64_t want = (rows + kGemvWarps - 1) / kGemvWarps;
  const uint64_t cap = (uint64_t)ctx->num_sms * 8u;
  const dim3 grid((unsigned)(want < cap ? want : cap));
  g4a_prof_scope ps(ctx, G4A_PROF_MATMUL);
  cudaError_t e;
  if (!vec) {
    if (smem > 48u * 1024u) {
      const cudaError_t a =
          cudaFuncSetAttribute(gemv_f16_scalar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (a != cudaSuccess) return g4a_cuda_fail(a, "cudaFuncSetAttribute(gemv)");
    }
    e = g4a_launch(gemv_f16_scalar_kernel, grid, dim3(kGemvThreads), smem, ctx->stream, true, input, N, J);
  } else {
    const uint32_t S = N / 256u;
    if (N % 256u == 0 && S >= 1 && S <= 8) {
      using FixedKernel = void (*)(const float*, GemvJobs);
      static const FixedKernel fixed[3][8] = {
          {gemv_fixed_kernel<G4A_WEIGHT_F16, 1>, gemv_fixed_kernel<G4A_WEIGHT_F16, 2>,
           gemv_fixed_kernel<G4A_WEIGHT_F16, 3>, gemv_fixed_kernel<G4A_WEIGHT_F16, 4>,
           gemv_fixed_kernel<G4A_WEIGHT_F16, 5>, gemv_fixed_kernel<G4A_WEIGHT_F16, 6>,
           gemv_fixed_kernel<G4A_WEIGHT_F16, 7>, gemv_fixed_kernel<G4A_WEIGHT_F16, 8>},
          {gemv_fixed_kernel<G4A_WEIGHT_Q8, 1>, gemv_fixed_kernel<G4A_WEIGHT_Q8, 2>,
           gemv_fixed_kernel<G4A_WEIGHT_Q8, 3>, gemv_fixed_kernel<G4A_WEIGHT_Q8, 4>,
           gemv_fixed_kernel<G4A_WEIGHT_Q8, 5>, gemv_fixed_kernel<G4A_WEIGHT_Q8, 6>,
           gemv_fixed_kernel<G4A_WEIGHT_Q8, 7>, gemv_fixed_kernel<G4A_WEIGHT_Q8, 8>},
          {gemv_fixed_kernel<G4A_WEIGHT_Q4K, 1>, gemv_fixed_kernel<G4A_WEIGHT_Q4K, 2>,
           gemv_fixed_kernel<G4A_WEIGHT_Q4K, 3>, gemv_fixed_kernel<G4A_WEIGHT_Q4K, 4>,
           gemv_fixed_kernel<G4A_WEIGHT_Q4K, 5>, gemv_fixed_kernel<G4A_WEIGHT_Q4K, 6>,
           gemv_fixed_kernel<G4A_WEIGHT_Q4K, 7>, gemv_fixed_kernel<G4A_WEIGHT_Q4K, 8>}};
      static const FixedKernel fixed_xreg[2][8] = {
          {gemv_fixed_kernel<G4A_WEIGHT_Q8, 1, true>, gemv_fixed_kernel<G4A_WEIGHT_Q8, 2, true>,
           gemv_fixed_kernel<G4A_WEIGHT_Q8, 3, true>, gemv_fixed_kernel<G4A_WEIGHT_Q8, 4, true>,
           gemv_fixed_kernel<G4A_WEIGHT_Q8, 5, true>, gemv_fixed_kernel<G4A_WEIGHT_Q8, 6, true>,
           gemv_fixed_kernel<G4A_WEIGHT_Q8, 7, true>, gemv_fixed_kernel<G4A_WEIGHT_Q8, 8, true>},
          {gemv_fixed_kernel<G4A_WEIGHT_Q4K, 1, true>, gemv_fixed_kernel<G4A_WEIGHT_Q4K, 2, true>,
           gemv_fixed_kernel<G4A_WEIGHT_Q4K, 3, true>, gemv_fixed_kernel<G4A_WEIGHT_Q4K, 4, true>,
           gemv_fixed_kernel<G4A_WEIGHT_Q4K, 5, true>, gemv_fixed_kernel<G4A_WEIGHT_Q4K, 6, true>,
           gemv_fixed_kernel<G4A_WEIGHT_Q4K, 7, true>, gemv_fixed_kernel<G4A_WEIGHT_Q4K, 8, true>}};
      // streaming-sized row counts: the register-resident input (see gemv_fixed_kernel)
      const bool xreg = weight_format != G4A_WEIGHT_F16 && rows >= 65536u;
      e = g4a_launch(xreg ? fixed_xreg[weight_format - 1][S - 1] : fixed[weight_format][S - 1], grid,
                     dim3(kGemvThreads), smem, ctx->stream, true, input, J);
    } else {
      auto kern = weight_format == G4A_WEIGHT_F16 ? gemv_kernel<G4A_WEIGHT_F16>
                  : weight_format == G4A_WEIGHT_Q8 ? gemv_kernel<G4A_WEIGHT_Q8>
                                                   : gemv_kernel<G4A_WEIGHT_Q4K>;
      if (smem > 48u * 1024u) {
        const cudaError_t a = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (a != cudaSuccess) return g4a_cuda_fail(a, "cudaFuncSetAttribute(gemv)");
      }
      e = g4a_launch(kern, grid, dim3(kGemvThreads), smem, ctx->stream, true, input, N, J);
    }
  }
  if (e != cudaSuccess) return g4a_cuda_fail(e, "launch gemv");
  return G4A_OK;
}

g4a_status g4a_matmul(g4a_ctx* ctx, uint32_t weight_format, const float* input, const void* weight,
                      const uint16_t* scales, float* out, uint32_t M, uint32_t N) {
  const g4a_matmul_job job = {weight, scales, out, M};
  return g4a_matmul_group(ctx, weight_format, input, N, &job, 1);
}

}  // extern "C"
