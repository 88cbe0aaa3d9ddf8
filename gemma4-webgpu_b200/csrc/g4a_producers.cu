// Producer kernels of the attention block: per-head RMSNorm(+weight) + RoPE for q and k, the
// weightless v_norm, and the f16 KV-cache store.
//
// Reference arithmetic (paths relative to the reference project root):
//   shaders/fused_per_head_norm_rope.wgsl:26-63    per-head norm * w, then NeoX RoPE
//   shaders/per_head_rms_norm_no_weight.wgsl:17-36  v / sqrt(mean(v^2) + eps)
//   shaders/kv_cache_store.wgsl:13-17               cache[slot, kvh, d] = x[kvh, d]
// One 256-thread CTA per head, like the reference's one workgroup per head.  The sum of
// squares uses the same per-thread partials and the same stride-halving tree (strides 128..1)
// as the WGSL `shared_sum` reduction, and every product/quotient is an explicit IEEE
// round-to-nearest intrinsic (no contraction), so the results are bit-identical to the CPU
// restatement.  The RoPE frequency is 1/RN32(theta^(2i/HD)) with the power evaluated in double
// and rounded once -- on the host, once per launch, and passed to the kernels as a table
// (it depends only on theta and HD) -- and cos/sin are the double-precision values of the f32
// angle rounded to f32: a fixed definition of the WGSL built-ins whose precision the reference
// leaves to the WebGPU implementation.
//
// These kernels move a few KB per token; they are launch-bound, which is why the decode path
// runs q, k and v through one launch (g4a_attn_decode_layer) and prefill runs all T tokens
// through one launch (g4a_prefill_qkv_prep).
#include <math.h>

#include "g4a_internal.cuh"

namespace {

constexpr int kWG = 256;           // threads per head, as the WGSL workgroup_size
constexpr int kMaxHeadDim = 1024;  // smem staging bound

// Sum over the 256 threads with the WGSL tree order; returns the total to every thread.
__device__ __forceinline__ float wg_tree_sum(float partial, float* red) {
  const int t = threadIdx.x;
  red[t] = partial;
  __syncthreads();
#pragma unroll
  for (int stride = 128; stride >= 32; stride >>= 1) {
    if (t < stride) red[t] = __fadd_rn(red[t], red[t + stride]);
    __syncthreads();
  }
  if (t < 32) {
    float v = red[t];
#pragma unroll
    for (int stride = 16; stride >= 1; stride >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, stride));
    if (t == 0) red[0] = v;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float head_rms(const float* x, int hd, float eps, float* red) {
  float partial = 0.0f;
  for (int i = threadIdx.x; i < hd; i += kWG) partial = __fadd_rn(partial, __fmul_rn(x[i], x[i]));
  float ss = wg_tree_sum(partial, red);
  return __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), eps));
}

// RN32(theta^(2i/HD)) for the pairs of a head, evaluated on the host (double pow, rounded once).
struct RopePow {
  float p[kMaxHeadDim / 2];
};

RopePow make_rope_pow(float theta, uint32_t hd) {
  RopePow t;
  for (uint32_t i = 0; i < hd / 2 && i < (uint32_t)(kMaxHeadDim / 2); i++) {
    const float e = (float)(i * 2u) / (float)hd;
    t.p[i] = (float)pow((double)theta, (double)e);
  }
  return t;
}

// RoPE inverse frequency of pair i (fused_per_head_norm_rope.wgsl:50-54).
__device__ __forceinline__ float rope_freq(int i, const RopePow& tab, const __half* rope_freqs, uint32_t apply_div) {
  float freq = __fdiv_rn(1.0f, tab.p[i]);
  if (apply_div != 0u) freq = __fdiv_rn(freq, __half2float(rope_freqs[i]));
  return freq;
}

// Normalise one head (x * w / rms) and rotate it.  `in` may alias `out_f32`.  Either output may
// be null.  xs is hd floats of shared memory, red 256 floats.
__device__ void norm_rope_head(const float* in, float* out_f32, __half* out_f16, const __half* w,
                               const __half* rope_freqs, int hd, float eps, uint32_t position, const RopePow& tab,
                               uint32_t apply_div, float* xs, float* red) {
  for (int i = threadIdx.x; i < hd; i += kWG) xs[i] = in[i];
  __syncthreads();
  const float rms = head_rms(xs, hd, eps, red);
  for (int i = threadIdx.x; i < hd; i += kWG) xs[i] = __fdiv_rn(__fmul_rn(xs[i], __half2float(w[i])), rms);
  __syncthreads();
  const int half_dim = hd / 2;
  const float posf = __uint2float_rn(position);
  for (int i = threadIdx.x; i < half_dim; i += kWG) {
    float freq = rope_freq(i, tab, rope_freqs, apply_div);
    float angle = __fmul_rn(posf, freq);
    double s, c;
    sincos((double)angle, &s, &c);
    float sin_a = __double2float_rn(s), cos_a = __double2float_rn(c);
    float x0 = xs[i], x1 = xs[i + half_dim];
    float y0 = __fsub_rn(__fmul_rn(x0, cos_a), __fmul_rn(x1, sin_a));
    float y1 = __fadd_rn(__fmul_rn(x0, sin_a), __fmul_rn(x1, cos_a));
    if (out_f32) {
      out_f32[i] = y0;
      out_f32[i + half_dim] = y1;
    }
    if (out_f16) {
      out_f16[i] = __float2half_rn(y0);
      out_f16[i + half_dim] = __float2half_rn(y1);
    }
  }
  __syncthreads();
}

// Weightless RMSNorm of one head (or a plain copy when normalise == false).
__device__ void vnorm_head(const float* in, float* out_f32, __half* out_f16, int hd, float eps, bool normalise,
                           float* xs, float* red) {
  for (int i = threadIdx.x; i < hd; i += kWG) xs[i] = in[i];
  __syncthreads();
  float rms = 1.0f;
  if (normalise) rms = head_rms(xs, hd, eps, red);
  for (int i = threadIdx.x; i < hd; i += kWG) {
    float y = normalise ? __fdiv_rn(xs[i], rms) : xs[i];
    if (out_f32) out_f32[i] = y;
    if (out_f16) out_f16[i] = __float2half_rn(y);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kWG) norm_rope_kernel(float* x, const __half* w, const __half* rope_freqs, int hd,
                                                         float eps, uint32_t position,
                                                         const __grid_constant__ RopePow tab, uint32_t apply_div) {
  __shared__ float xs[kMaxHeadDim];
  __shared__ float red[kWG];
  float* xh = x + (size_t)blockIdx.x * hd;
  norm_rope_head(xh, xh, nullptr, w, rope_freqs, hd, eps, position, tab, apply_div, xs, red);
}

__global__ void __launch_bounds__(kWG) rms_norm_no_weight_kernel(float* x, int hd, float eps) {
  __shared__ float xs[kMaxHeadDim];
  __shared__ float red[kWG];
  float* xh = x + (size_t)blockIdx.x * hd;
  vnorm_head(xh, xh, nullptr, hd, eps, true, xs, red);
}

// One CTA per kv head: k -> f16 cache row; v -> (v_norm) -> f16 cache row (+ in place).
__global__ void __launch_bounds__(kWG) kv_store_kernel(const float* k, float* v, __half* k_cache, __half* v_cache,
                                                        int nkh, int hd, uint32_t slot, float eps, int fuse) {
  __shared__ float xs[kMaxHeadDim];
  __shared__ float red[kWG];
  const int j = blockIdx.x;
  const size_t row = ((size_t)slot * nkh + j) * hd;
  const float* kh = k + (size_t)j * hd;
  for (int i = threadIdx.x; i < hd; i += kWG) k_cache[row + i] = __float2half_rn(kh[i]);
  float* vh = v + (size_t)j * hd;
  vnorm_head(vh, fuse ? vh : nullptr, v_cache + row, hd, eps, fuse != 0, xs, red);
}

// Whole decode-producer stage of one layer in a single launch: CTAs [0, nqh) norm+RoPE the q
// heads; CTAs [nqh, nqh+nkh) (producer layers only) norm+RoPE the k head, v_norm the v head,
// and write both as f16 to cache row `slot`.  Results go to q / k / v (in place, the
// reference's work buffers).  With sq != nullptr the inputs are read from sq / sk / sv instead
// (e.g. mapped host memory that nothing on the device writes): those loads are issued before
// the programmatic-launch wait, so their latency overlaps the preceding kernel.
__global__ void __launch_bounds__(kWG) decode_prep_kernel(const float* sq, const float* sk, const float* sv,
                                                           float* q, float* k, float* v, const __half* qw,
                                                           const __half* kw, const __half* rope_freqs,
                                                           __half* k_cache, __half* v_cache, int nqh, int nkh,
                                                           int hd, float eps, uint32_t position, uint32_t slot,
                                                           const __grid_constant__ RopePow tab, uint32_t apply_div) {
  __shared__ float xs[kMaxHeadDim];
  __shared__ float red[kWG];
  __shared__ float xin[kMaxHeadDim];  // staged input of a separate-source call
  constexpr int kPer = kMaxHeadDim / kWG;
  const int b = blockIdx.x;
  const bool staged = sq != nullptr;
  float p0[kPer], p1[kPer];
  if (staged) {
    const float* s0 = (b < nqh) ? sq + (size_t)b * hd : sk + (size_t)(b - nqh) * hd;
#pragma unroll
    for (int u = 0; u < kPer; u++) {
      const int i = threadIdx.x + u * kWG;
      p0[u] = i < hd ? s0[i] : 0.f;
    }
    if (b >= nqh) {
      const float* s1 = sv + (size_t)(b - nqh) * hd;
#pragma unroll
      for (int u = 0; u < kPer; u++) {
        const int i = threadIdx.x + u * kWG;
        p1[u] = i < hd ? s1[i] : 0.f;
      }
    }
  }
  // Launched as a programmatic dependent of the preceding kernel: everything it writes (q / k /
  // v, the cache rows a previous attention may still read) and every in-place input waits for
  // that kernel to finish; only the launch and the separate-source loads overlap it.
  g4a::pdl_wait_primary();
  auto stage = [&](const float (&pv)[kPer]) {
#pragma unroll
    for (int u = 0; u < kPer; u++) {
      const int i = threadIdx.x + u * kWG;
      if (i < hd) xin[i] = pv[u];
    }
    __syncthreads();
  };
  if (b < nqh) {
    float* qh = q + (size_t)b * hd;
    if (staged) stage(p0);
    norm_rope_head(staged ? xin : qh, qh, nullptr, qw, rope_freqs, hd, eps, position, tab, apply_div, xs, red);
  } else {
    const int j = b - nqh;
    const size_t row = ((size_t)slot * nkh + j) * hd;
    float* kh = k + (size_t)j * hd;
    if (staged) stage(p0);
    norm_rope_head(staged ? xin : kh, kh, k_cache + row, kw, rope_freqs, hd, eps, position, tab, apply_div, xs,
                   red);
    float* vh = v + (size_t)j * hd;
    // (norm_rope_head copied xin into xs behind a CTA barrier, so xin can take the v head)
    if (staged) stage(p1);
    vnorm_head(staged ? xin : vh, vh, v_cache + row, hd, eps, true, xs, red);
  }
  // Let a programmatically-dependent attention launch start its prologue.
  g4a::pdl_launch_dependents();
}

// Prefill input stage: one CTA per token (grid T), one warp per head (q heads, then k heads,
// then v heads).  Token i is at position start_pos + i and is stored at cache row start_pos + i;
// inputs are left untouched.  The RoPE sin/cos of the position are computed once per token, and
// the two norm weights are widened to f32 once per token, both into shared memory.  A
// warp reproduces the 256-thread WGSL sum-of-squares tree exactly: lane l holds elements
// l + 32j, so thread t = l + 32j's partial sum (its elements t, t + 256, ... added from 0 in
// order) and the first three halving levels (128, 64, 32) are lane-local adds in the same order,
// and the last five levels are the same shuffles as in wg_tree_sum.  RoPE pairs (p, p + hd/2) are
// lane-local too.  Every output is bit-identical to the single-head kernels.  head_dim must be
// a multiple of 64 and at most 512; NJ = head_dim / 32 is a template argument, so every index
// into the lane's elements is a compile-time constant and they stay in registers.
constexpr int kPrepMaxHd = 512;
constexpr int kPrepMaxWarps = 32;

template <int NJ>
__global__ void __launch_bounds__(1024) prefill_prep_kernel(const float* q, const float* k, const float* v,
                                                             const __half* qw, const __half* kw,
                                                             const __half* rope_freqs, __half* q16, __half* k_cache,
                                                             __half* v_cache, int nqh, int nkh, int hd, float eps,
                                                             uint32_t start_pos, const __grid_constant__ RopePow tab,
                                                             uint32_t apply_div) {
  __shared__ float sn[kPrepMaxHd / 2], cs[kPrepMaxHd / 2];
  __shared__ float sw[2][kPrepMaxHd];  // q_norm and k_norm weights as f32
  const int t = threadIdx.x, lane = t & 31;
  const uint32_t i = blockIdx.x;
  const uint32_t pos = start_pos + i;
  const int half_dim = hd / 2;
  const float posf = __uint2float_rn(pos);
  for (int p = t; p < half_dim; p += blockDim.x) {
    const float angle = __fmul_rn(posf, rope_freq(p, tab, rope_freqs, apply_div));
    double s_, c_;
    sincos((double)angle, &s_, &c_);
    sn[p] = __double2float_rn(s_);
    cs[p] = __double2float_rn(c_);
  }
  for (int p = t; p < hd; p += blockDim.x) {
    sw[0][p] = __half2float(qw[p]);
    sw[1][p] = __half2float(kw[p]);
  }
  __syncthreads();
  const int H = nqh + 2 * nkh;
  for (int h = t >> 5; h < H; h += blockDim.x >> 5) {
    const bool is_q = h < nqh, is_k = !is_q && h < nqh + nkh;
    const float* src = is_q ? q + ((size_t)i * nqh + h) * hd
                       : is_k ? k + ((size_t)i * nkh + (h - nqh)) * hd
                              : v + ((size_t)i * nkh + (h - nqh - nkh)) * hd;
    float x[NJ];
#pragma unroll
    for (int j = 0; j < NJ; j++) x[j] = src[lane + 32 * j];
    // thread t = lane + 32j of the WGSL workgroup: partial over elements t, t + 256
    float s8[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      // (j % NJ) keeps every index in range at compile time; the guards select the live terms.
      float part = 0.f;
      if (j < NJ) part = __fmul_rn(x[j % NJ], x[j % NJ]);  // 0 + x*x
      if (j + 8 < NJ) part = __fadd_rn(part, __fmul_rn(x[(j + 8) % NJ], x[(j + 8) % NJ]));
      s8[j] = part;
    }
#pragma unroll
    for (int j = 0; j < 4; j++) s8[j] = __fadd_rn(s8[j], s8[j + 4]);  // stride 128
#pragma unroll
    for (int j = 0; j < 2; j++) s8[j] = __fadd_rn(s8[j], s8[j + 2]);  // stride 64
    float val = __fadd_rn(s8[0], s8[1]);                              // stride 32
#pragma unroll
    for (int stride = 16; stride >= 1; stride >>= 1) val = __fadd_rn(val, __shfl_down_sync(0xffffffffu, val, stride));
    const float ss = __shfl_sync(0xffffffffu, val, 0);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), eps));
    __half* dst;
    if (is_q || is_k) {
      const float* w = sw[is_q ? 0 : 1];
      dst = is_q ? q16 + ((size_t)i * nqh + h) * hd : k_cache + ((size_t)pos * nkh + (h - nqh)) * hd;
      constexpr int pj = NJ / 2;  // pair partner of element j is j + pj
#pragma unroll
      for (int j = 0; j < pj; j++) {
        const int p = lane + 32 * j;
        const float x0 = __fdiv_rn(__fmul_rn(x[j], w[p]), rms);
        const float x1 = __fdiv_rn(__fmul_rn(x[j + pj], w[p + half_dim]), rms);
        dst[p] = __float2half_rn(__fsub_rn(__fmul_rn(x0, cs[p]), __fmul_rn(x1, sn[p])));
        dst[p + half_dim] = __float2half_rn(__fadd_rn(__fmul_rn(x0, sn[p]), __fmul_rn(x1, cs[p])));
      }
    } else {
      dst = v_cache + ((size_t)pos * nkh + (h - nqh - nkh)) * hd;
#pragma unroll
      for (int j = 0; j < NJ; j++) dst[lane + 32 * j] = __float2half_rn(__fdiv_rn(x[j], rms));
    }
  }
  g4a::pdl_launch_dependents();
}

g4a_status check_head_dim(const char* fn, uint32_t hd, bool need_even) {
  if (hd == 0 || hd > (uint32_t)kMaxHeadDim)
    return g4a_fail(G4A_EINVAL, "%s: head_dim %u not in [1, %d]", fn, hd, kMaxHeadDim);
  if (need_even && (hd & 1u)) return g4a_fail(G4A_EINVAL, "%s: head_dim %u must be even for RoPE", fn, hd);
  return G4A_OK;
}

}  // namespace

extern "C" {

g4a_status g4a_norm_rope(g4a_ctx* ctx, float* x, const uint16_t* weight, const uint16_t* rope_freqs,
                         uint32_t num_heads, uint32_t head_dim, float eps, uint32_t position, float theta,
                         uint32_t apply_divisor) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_head_dim(__func__, head_dim, true)) return s;
  if (num_heads == 0) return G4A_OK;
  if (!x || !weight) return g4a_fail(G4A_EINVAL, "g4a_norm_rope: null x or weight");
  if (apply_divisor && !rope_freqs)
    return g4a_fail(G4A_EINVAL, "g4a_norm_rope: apply_divisor set but rope_freqs is null");
  g4a_prof_scope ps(ctx, G4A_PROF_NORM_ROPE);
  norm_rope_kernel<<<num_heads, kWG, 0, ctx->stream>>>(x, (const __half*)weight, (const __half*)rope_freqs,
                                                       (int)head_dim, eps, position,
                                                       make_rope_pow(theta, head_dim), apply_divisor);
  return g4a_check_launch("norm_rope_kernel");
}

g4a_status g4a_rms_norm_no_weight(g4a_ctx* ctx, float* x, uint32_t num_heads, uint32_t head_dim, float eps) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_head_dim(__func__, head_dim, false)) return s;
  if (num_heads == 0) return G4A_OK;
  if (!x) return g4a_fail(G4A_EINVAL, "g4a_rms_norm_no_weight: null x");
  g4a_prof_scope ps(ctx, G4A_PROF_RMS_NORM);
  rms_norm_no_weight_kernel<<<num_heads, kWG, 0, ctx->stream>>>(x, (int)head_dim, eps);
  return g4a_check_launch("rms_norm_no_weight_kernel");
}

g4a_status g4a_kv_store(g4a_ctx* ctx, const float* k, float* v, uint16_t* k_cache, uint16_t* v_cache,
                        uint32_t num_kv_heads, uint32_t head_dim, uint32_t slot, uint32_t max_seq_len, float eps,
                        uint32_t fuse_v_norm) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_head_dim(__func__, head_dim, false)) return s;
  if (num_kv_heads == 0) return G4A_OK;
  if (!k || !v || !k_cache || !v_cache) return g4a_fail(G4A_EINVAL, "g4a_kv_store: null pointer");
  if (slot >= max_seq_len) return g4a_fail(G4A_EINVAL, "g4a_kv_store: slot %u >= max_seq_len %u", slot, max_seq_len);
  g4a_prof_scope ps(ctx, G4A_PROF_KV_STORE);
  kv_store_kernel<<<num_kv_heads, kWG, 0, ctx->stream>>>(k, v, (__half*)k_cache, (__half*)v_cache, (int)num_kv_heads,
                                                         (int)head_dim, slot, eps, fuse_v_norm ? 1 : 0);
  return g4a_check_launch("kv_store_kernel");
}

g4a_status g4a_prefill_qkv_prep(g4a_ctx* ctx, const float* q, const float* k, const float* v,
                                const uint16_t* q_norm_w, const uint16_t* k_norm_w, const uint16_t* rope_freqs,
                                uint16_t* q16_out, uint16_t* k_cache, uint16_t* v_cache, uint32_t T,
                                uint32_t start_pos, uint32_t max_seq_len, uint32_t num_q_heads,
                                uint32_t num_kv_heads, uint32_t head_dim, float eps, float theta,
                                uint32_t apply_divisor) {
  G4A_CHECK_CTX(ctx);
  if (g4a_status s = check_head_dim(__func__, head_dim, true)) return s;
  if (T == 0) return G4A_OK;
  if (!q || !k || !v || !q_norm_w || !k_norm_w || !q16_out || !k_cache || !v_cache)
    return g4a_fail(G4A_EINVAL, "g4a_prefill_qkv_prep: null pointer");
  if (apply_divisor && !rope_freqs)
    return g4a_fail(G4A_EINVAL, "g4a_prefill_qkv_prep: apply_divisor without rope_freqs");
  if ((uint64_t)start_pos + T > max_seq_len)
    return g4a_fail(G4A_EINVAL, "g4a_prefill_qkv_prep: start_pos %u + T %u exceeds max_seq_len %u", start_pos, T,
                    max_seq_len);
  if (head_dim > (uint32_t)kPrepMaxHd || (head_dim % 64) != 0)
    return g4a_fail(G4A_EINVAL, "g4a_prefill_qkv_prep: head_dim %u must be a multiple of 64 and <= %d", head_dim,
                    kPrepMaxHd);
  const uint32_t heads = num_q_heads + 2 * num_kv_heads;
  if (heads == 0) return G4A_OK;
  const uint32_t warps = heads < (uint32_t)kPrepMaxWarps ? heads : (uint32_t)kPrepMaxWarps;
  decltype(&prefill_prep_kernel<2>) kern = nullptr;
  switch (head_dim / 32) {
    case 2: kern = prefill_prep_kernel<2>; break;
    case 4: kern = prefill_prep_kernel<4>; break;
    case 6: kern = prefill_prep_kernel<6>; break;
    case 8: kern = prefill_prep_kernel<8>; break;
    case 10: kern = prefill_prep_kernel<10>; break;
    case 12: kern = prefill_prep_kernel<12>; break;
    case 14: kern = prefill_prep_kernel<14>; break;
    default: kern = prefill_prep_kernel<16>; break;
  }
  g4a_prof_scope ps(ctx, G4A_PROF_PREFILL_PREP);
  kern<<<T, warps * 32, 0, ctx->stream>>>(q, k, v, (const __half*)q_norm_w, (const __half*)k_norm_w,
                                          (const __half*)rope_freqs, (__half*)q16_out, (__half*)k_cache,
                                          (__half*)v_cache, (int)num_q_heads, (int)num_kv_heads, (int)head_dim, eps,
                                          start_pos, make_rope_pow(theta, head_dim), apply_divisor);
  return g4a_check_launch("prefill_prep_kernel");
}

}  // extern "C"

// Internal entry used by g4a_attn_decode_layer (g4a_decode.cu).
g4a_status g4a_launch_decode_prep(g4a_ctx* ctx, const float* sq, const float* sk, const float* sv, float* q,
                                  float* k, float* v, const uint16_t* qw,
                                  const uint16_t* kw, const uint16_t* rope_freqs, uint16_t* k_cache,
                                  uint16_t* v_cache, uint32_t nqh, uint32_t nkh, uint32_t hd, float eps,
                                  uint32_t position, uint32_t slot, float theta, uint32_t apply_div,
                                  bool is_producer) {
  if (g4a_status s = check_head_dim("g4a_attn_decode_layer", hd, true)) return s;
  uint32_t blocks = nqh + (is_producer ? nkh : 0u);
  if (blocks == 0) return G4A_OK;
  g4a_prof_scope ps(ctx, G4A_PROF_DECODE_PREP);
  const cudaError_t e = g4a_launch(decode_prep_kernel, dim3(blocks), dim3(kWG), 0, ctx->stream, true, sq, sk, sv,
                                   q, k, v,
                                   (const __half*)qw, (const __half*)kw, (const __half*)rope_freqs, (__half*)k_cache,
                                   (__half*)v_cache, (int)nqh, (int)nkh, (int)hd, eps, position, slot,
                                   make_rope_pow(theta, hd), apply_div);
  if (e != cudaSuccess) return g4a_cuda_fail(e, "launch decode_prep_kernel");
  return G4A_OK;
}
