/*
 * CPU oracle for the gemma4-webgpu attention hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of the reference's six WGSL compute
 * shaders that make up the per-layer attention chain.  It is the parity checker for the
 * CUDA library and the timed CPU baseline; nothing in the product links it.  Only the
 * test-suite, the smoke check and the CPU-baseline leg of the benchmark load it.
 *
 * Reference shaders restated (paths relative to the reference project root):
 *   shaders/fused_per_head_norm_rope.wgsl:20-64   -> orc_norm_rope
 *   shaders/per_head_rms_norm_no_weight.wgsl:13-38 -> orc_rms_norm_no_weight
 *   shaders/kv_cache_store.wgsl:8-18              -> orc_kv_cache_store_f32 / _f16
 *   shaders/attn_score.wgsl:15-40                 -> orc_attn_score
 *   shaders/softmax.wgsl:7-46                     -> orc_softmax
 *   shaders/attn_output.wgsl:7-23                 -> orc_attn_output
 *   shaders/matmul_quant.wgsl, matmul_quant_mr4.wgsl -> orc_matmul_f16
 *   shaders/matmul_q8.wgsl, matmul_q8_mr.wgsl      -> orc_matmul_q8
 *   shaders/matmul_q4k.wgsl, matmul_q4k_mr.wgsl    -> orc_matmul_q4k
 * and the dispatch order of src/engine.ts:2061-2094 (v_norm, norm+RoPE, store, score,
 * softmax, output) in orc_decode_chain_f32.
 *
 * Operation order.  Each WGSL kernel runs one 256-thread workgroup per head for its
 * reductions (`shared_sum[tid]` + a stride-halving tree, e.g. softmax.wgsl:13-40).  The
 * restatement reproduces that exact per-thread partial order and tree, so f32 results of
 * reductions are reproducible bit for bit.  Products and sums are kept as separate
 * roundings (this file must be compiled with -ffp-contract=off): WGSL leaves contraction
 * to the implementation, and the un-contracted form is the one this oracle pins.
 *
 * Transcendentals.  WGSL leaves the precision of pow/sin/cos/exp/sqrt to the WebGPU
 * implementation (Dawn/Tint + vendor driver); no reference test pins it.  This oracle fixes
 * one definition: sqrt is IEEE (correctly rounded); the RoPE frequency is
 * 1/RN32(theta^(2i/HD)) with the power correctly rounded to f32 (computed in double);
 * cos/sin of the f32 angle are RN32 of the double-precision results; exp is glibc expf.
 * The CUDA library uses the same frequency / sin / cos definition, which makes the
 * norm+RoPE and KV-store kernels bit-exact against this file.
 *
 * f16 KV cache.  The reference caches are f32 (kv_cache_store.wgsl:4-5); the B200 build
 * stores f16.  orc_kv_cache_store_f16 rounds to nearest-even, and the attention functions
 * take the f16 cache so that parity compares kernel error, not cache quantisation.
 *
 * fp64 golden.  orc_decode_attn_f64 evaluates the same attention (mask, scale, GQA map) with
 * double accumulation; it is the tolerance golden (max abs <= 2e-3, per-head cosine >=
 * 0.9999) the GPU kernels are checked against.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define WG 256u /* workgroup_size of every reduction shader */

/* ---------------------------------------------------------------- f16 <-> f32 */

float orc_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t expo = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (expo == 0) {
    if (mant == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { mant <<= 1; e++; } while ((mant & 0x400u) == 0);
      mant &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
    }
  } else if (expo == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((expo + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Round-to-nearest-even f32 -> f16 (IEEE binary16), with overflow to inf and subnormals. */
uint16_t orc_float_to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) { /* inf or nan */
    return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
  }
  if (absx >= 0x477ff000u) { /* >= 65520 rounds to inf */
    return (uint16_t)(sign | 0x7c00u);
  }
  if (absx < 0x38800000u) { /* below 2^-14: subnormal half (or zero) */
    if (absx < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to 0 */
    uint32_t mant = (absx & 0x7fffffu) | 0x800000u;
    int shift = 126 - (int)(absx >> 23); /* 14..24 */
    uint32_t q = mant >> (shift);
    uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (absx >> 23) - 127 + 15;
  uint32_t mant = absx & 0x7fffffu;
  uint32_t q = (e << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

void orc_f32_to_f16_array(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = orc_float_to_half(in[i]);
}

void orc_f16_to_f32_array(const uint16_t* in, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = orc_half_to_float(in[i]);
}

/* ------------------------------------------------------------- reductions */

/* Sum of squares of one head as the 256-thread workgroup computes it:
 * thread t accumulates x[t], x[t+256], ... (partial += val*val), then
 * `for stride = 128; stride > 0; stride >>= 1: s[t] += s[t+stride]`.
 * fused_per_head_norm_rope.wgsl:27-39, per_head_rms_norm_no_weight.wgsl:19-31. */
static float wg_sum_squares(const float* x, uint32_t n) {
  float s[WG];
  for (uint32_t t = 0; t < WG; t++) {
    float partial = 0.0f;
    for (uint32_t i = t; i < n; i += WG) {
      float sq = x[i] * x[i];
      partial = partial + sq;
    }
    s[t] = partial;
  }
  for (uint32_t stride = WG / 2; stride > 0; stride >>= 1)
    for (uint32_t t = 0; t < stride; t++) s[t] = s[t] + s[t + stride];
  return s[0];
}

/* RoPE inverse frequency for pair i: 1 / RN32(theta^(2i/hd)).
 * fused_per_head_norm_rope.wgsl:50 (`1.0 / pow(theta, f32(i*2u) / f32(head_dim))`). */
float orc_rope_base_freq(float theta, uint32_t i, uint32_t head_dim) {
  float e = (float)(i * 2u) / (float)head_dim;
  float p = (float)pow((double)theta, (double)e);
  return 1.0f / p;
}

/* ------------------------------------------------------------- producers */

/* fused_per_head_norm_rope.wgsl:20-64: per head, x*w/rms, then NeoX half-split RoPE. */
void orc_norm_rope(float* data, const uint16_t* weight, const uint16_t* rope_freqs,
                   uint32_t num_heads, uint32_t head_dim, float eps, uint32_t position,
                   float theta, uint32_t apply_divisor) {
  uint32_t half_dim = head_dim / 2u;
  for (uint32_t head = 0; head < num_heads; head++) {
    float* x = data + (size_t)head * head_dim;
    float ss = wg_sum_squares(x, head_dim);
    float rms = sqrtf(ss / (float)head_dim + eps);
    for (uint32_t i = 0; i < head_dim; i++) {
      float xw = x[i] * orc_half_to_float(weight[i]);
      x[i] = xw / rms;
    }
    for (uint32_t i = 0; i < half_dim; i++) {
      float freq = orc_rope_base_freq(theta, i, head_dim);
      if (apply_divisor != 0u) freq = freq / orc_half_to_float(rope_freqs[i]);
      float angle = (float)position * freq;
      float cos_a = (float)cos((double)angle);
      float sin_a = (float)sin((double)angle);
      float x0 = x[i];
      float x1 = x[i + half_dim];
      float a = x0 * cos_a, b = x1 * sin_a;
      float c = x0 * sin_a, d = x1 * cos_a;
      x[i] = a - b;
      x[i + half_dim] = c + d;
    }
  }
}

/* per_head_rms_norm_no_weight.wgsl:13-38: v / sqrt(mean(v^2) + eps), in place. */
void orc_rms_norm_no_weight(float* data, uint32_t num_heads, uint32_t head_dim, float eps) {
  for (uint32_t head = 0; head < num_heads; head++) {
    float* x = data + (size_t)head * head_dim;
    float ss = wg_sum_squares(x, head_dim);
    float rms = sqrtf(ss / (float)head_dim + eps);
    for (uint32_t i = 0; i < head_dim; i++) x[i] = x[i] / rms;
  }
}

/* kv_cache_store.wgsl:8-18 (f32 cache, as in the reference). */
void orc_kv_cache_store_f32(const float* k_in, const float* v_in, float* k_cache, float* v_cache,
                            uint32_t num_kv_heads, uint32_t head_dim, uint32_t position) {
  size_t total = (size_t)num_kv_heads * head_dim;
  for (size_t i = 0; i < total; i++) {
    k_cache[(size_t)position * total + i] = k_in[i];
    v_cache[(size_t)position * total + i] = v_in[i];
  }
}

/* Same store into the build's f16 cache (round to nearest even). */
void orc_kv_cache_store_f16(const float* k_in, const float* v_in, uint16_t* k_cache,
                            uint16_t* v_cache, uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t slot) {
  size_t total = (size_t)num_kv_heads * head_dim;
  for (size_t i = 0; i < total; i++) {
    k_cache[(size_t)slot * total + i] = orc_float_to_half(k_in[i]);
    v_cache[(size_t)slot * total + i] = orc_float_to_half(v_in[i]);
  }
}

/* ------------------------------------------------------------- attention (f32, WGSL order) */

static uint32_t window_start(uint32_t seq_len, uint32_t sliding_window) {
  /* attn_score.wgsl:23-25 */
  if (sliding_window == 0u || seq_len == 0u) return 0u;
  uint32_t current_pos = seq_len - 1u;
  return (current_pos + 1u > sliding_window) ? current_pos + 1u - sliding_window : 0u;
}

uint32_t orc_window_start(uint32_t seq_len, uint32_t sliding_window) {
  return window_start(seq_len, sliding_window);
}

/* attn_score.wgsl:15-40.  scores is [num_q_heads, seq_len]; k_cache is an f32 view. */
void orc_attn_score(const float* q, const float* k_cache, float* scores, uint32_t num_q_heads,
                    uint32_t num_kv_heads, uint32_t head_dim, uint32_t seq_len, float scale,
                    uint32_t sliding_window) {
  uint32_t ws = window_start(seq_len, sliding_window);
  size_t kv_stride = (size_t)num_kv_heads * head_dim;
  int64_t total = (int64_t)num_q_heads * seq_len;
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; idx++) {
    uint32_t head = (uint32_t)(idx / seq_len);
    uint32_t pos = (uint32_t)(idx % seq_len);
    if (sliding_window != 0u && pos < ws) {
      scores[idx] = -1e30f;
      continue;
    }
    uint32_t kv_head = head * num_kv_heads / num_q_heads;
    const float* qh = q + (size_t)head * head_dim;
    const float* kp = k_cache + (size_t)pos * kv_stride + (size_t)kv_head * head_dim;
    float dot = 0.0f;
    for (uint32_t d = 0; d < head_dim; d++) {
      float pr = qh[d] * kp[d];
      dot = dot + pr;
    }
    scores[idx] = dot * scale;
  }
}

/* softmax.wgsl:7-46, one 256-thread workgroup per head, in place. */
void orc_softmax(float* scores, uint32_t num_heads, uint32_t seq_len) {
#pragma omp parallel for schedule(static)
  for (int64_t hh = 0; hh < (int64_t)num_heads; hh++) {
    float* s = scores + (size_t)hh * seq_len;
    float red[WG];
    for (uint32_t t = 0; t < WG; t++) {
      float m = -1e30f;
      for (uint32_t i = t; i < seq_len; i += WG) m = fmaxf(m, s[i]);
      red[t] = m;
    }
    for (uint32_t stride = WG / 2; stride > 0; stride >>= 1)
      for (uint32_t t = 0; t < stride; t++) red[t] = fmaxf(red[t], red[t + stride]);
    float max_val = red[0];
    for (uint32_t t = 0; t < WG; t++) {
      float sum = 0.0f;
      for (uint32_t i = t; i < seq_len; i += WG) {
        float e = expf(s[i] - max_val);
        s[i] = e;
        sum = sum + e;
      }
      red[t] = sum;
    }
    for (uint32_t stride = WG / 2; stride > 0; stride >>= 1)
      for (uint32_t t = 0; t < stride; t++) red[t] = red[t] + red[t + stride];
    float sum_val = red[0];
    for (uint32_t i = 0; i < seq_len; i++) s[i] = s[i] / sum_val;
  }
}

/* attn_output.wgsl:7-23: out[h,d] = sum_pos probs[h,pos] * V[pos,kvh,d], sequential in pos. */
void orc_attn_output(const float* probs, const float* v_cache, float* out, uint32_t num_q_heads,
                     uint32_t num_kv_heads, uint32_t head_dim, uint32_t seq_len) {
  size_t kv_stride = (size_t)num_kv_heads * head_dim;
  int64_t total = (int64_t)num_q_heads * head_dim;
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < total; idx++) {
    uint32_t head = (uint32_t)(idx / head_dim);
    uint32_t d = (uint32_t)(idx % head_dim);
    uint32_t kv_head = head * num_kv_heads / num_q_heads;
    float sum = 0.0f;
    for (uint32_t pos = 0; pos < seq_len; pos++) {
      float pr = probs[(size_t)head * seq_len + pos] *
                 v_cache[(size_t)pos * kv_stride + (size_t)kv_head * head_dim + d];
      sum = sum + pr;
    }
    out[idx] = sum;
  }
}

/* The reference's decode attention chain on f32 caches: score -> softmax -> output
 * (src/engine.ts:2092-2094).  scores_work must hold num_q_heads*seq_len floats. */
void orc_decode_chain_f32(const float* q, const float* k_cache, const float* v_cache, float* out,
                          float* scores_work, uint32_t num_q_heads, uint32_t num_kv_heads,
                          uint32_t head_dim, uint32_t seq_len, float scale,
                          uint32_t sliding_window) {
  if (seq_len == 0u) { /* no dispatch covers any score; attn_output's loop is empty */
    memset(out, 0, sizeof(float) * (size_t)num_q_heads * head_dim);
    return;
  }
  orc_attn_score(q, k_cache, scores_work, num_q_heads, num_kv_heads, head_dim, seq_len, scale,
                 sliding_window);
  orc_softmax(scores_work, num_q_heads, seq_len);
  orc_attn_output(scores_work, v_cache, out, num_q_heads, num_kv_heads, head_dim, seq_len);
}

/* ------------------------------------------------------------- fp64 golden */

/* Decode attention over an f16 cache with double accumulation.  Same semantics as the WGSL
 * chain: window [max(0, L-W), L) measured from kv_len (attn_score.wgsl:23-30), kvh =
 * h*NKH/NQH (attn_score.wgsl:31), scale multiplies the dot (attn_score.wgsl:39). */
void orc_decode_attn_f64(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                         float* out, uint32_t num_q_heads, uint32_t num_kv_heads,
                         uint32_t head_dim, uint32_t kv_len, float scale,
                         uint32_t sliding_window) {
  uint32_t ws = window_start(kv_len, sliding_window);
  size_t kv_stride = (size_t)num_kv_heads * head_dim;
#pragma omp parallel for schedule(static)
  for (int64_t hh = 0; hh < (int64_t)num_q_heads; hh++) {
    uint32_t head = (uint32_t)hh;
    uint32_t kv_head = head * num_kv_heads / num_q_heads;
    const float* qh = q + (size_t)head * head_dim;
    double* acc = (double*)calloc(head_dim, sizeof(double));
    double mx = -INFINITY;
    uint32_t n = kv_len - ws;
    double* sc = (double*)malloc(sizeof(double) * (n ? n : 1));
    for (uint32_t p = ws; p < kv_len; p++) {
      const uint16_t* kp = k_cache + (size_t)p * kv_stride + (size_t)kv_head * head_dim;
      double dot = 0.0;
      for (uint32_t d = 0; d < head_dim; d++) dot += (double)qh[d] * (double)orc_half_to_float(kp[d]);
      dot *= (double)scale;
      sc[p - ws] = dot;
      if (dot > mx) mx = dot;
    }
    double l = 0.0;
    for (uint32_t p = ws; p < kv_len; p++) {
      double e = exp(sc[p - ws] - mx);
      l += e;
      const uint16_t* vp = v_cache + (size_t)p * kv_stride + (size_t)kv_head * head_dim;
      for (uint32_t d = 0; d < head_dim; d++) acc[d] += e * (double)orc_half_to_float(vp[d]);
    }
    for (uint32_t d = 0; d < head_dim; d++)
      out[(size_t)head * head_dim + d] = (n == 0) ? 0.0f : (float)(acc[d] / l);
    free(sc);
    free(acc);
  }
}

/* Partial (unnormalised) attention over key range [kv_begin, kv_end) of a kv_len-long
 * cache, in double: per head m = max score, l = sum exp(s - m), o = sum exp(s - m) v.
 * The window is still measured from kv_len.  Used to check split-KV partials and the
 * log-sum-exp merge.  Heads with no visible key get m = -inf, l = 0, o = 0. */
void orc_decode_partial_f64(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                            uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim,
                            uint32_t kv_begin, uint32_t kv_end, uint32_t kv_len, float scale,
                            uint32_t sliding_window, double* m_out, double* l_out,
                            double* o_out) {
  uint32_t ws = window_start(kv_len, sliding_window);
  uint32_t b = kv_begin > ws ? kv_begin : ws;
  uint32_t e_ = kv_end < kv_len ? kv_end : kv_len;
  size_t kv_stride = (size_t)num_kv_heads * head_dim;
  for (uint32_t head = 0; head < num_q_heads; head++) {
    uint32_t kv_head = head * num_kv_heads / num_q_heads;
    const float* qh = q + (size_t)head * head_dim;
    double mx = -INFINITY;
    for (uint32_t p = b; p < e_; p++) {
      const uint16_t* kp = k_cache + (size_t)p * kv_stride + (size_t)kv_head * head_dim;
      double dot = 0.0;
      for (uint32_t d = 0; d < head_dim; d++) dot += (double)qh[d] * (double)orc_half_to_float(kp[d]);
      dot *= (double)scale;
      if (dot > mx) mx = dot;
    }
    double l = 0.0;
    double* o = o_out + (size_t)head * head_dim;
    for (uint32_t d = 0; d < head_dim; d++) o[d] = 0.0;
    for (uint32_t p = b; p < e_; p++) {
      const uint16_t* kp = k_cache + (size_t)p * kv_stride + (size_t)kv_head * head_dim;
      double dot = 0.0;
      for (uint32_t d = 0; d < head_dim; d++) dot += (double)qh[d] * (double)orc_half_to_float(kp[d]);
      dot *= (double)scale;
      double e = exp(dot - mx);
      l += e;
      const uint16_t* vp = v_cache + (size_t)p * kv_stride + (size_t)kv_head * head_dim;
      for (uint32_t d = 0; d < head_dim; d++) o[d] += e * (double)orc_half_to_float(vp[d]);
    }
    m_out[head] = mx;
    l_out[head] = l;
  }
}

/* Causal / sliding prefill as the reference computes it: prefillBatched (src/engine.ts:
 * 2460-2479) runs one decode step per token, so row i is decode attention with kv_len =
 * start_pos + i + 1 over the cache that holds every earlier row.  q is [T, NQH, HD] f32
 * (already f16-valued when the GPU side takes f16 Q); out is [T, NQH, HD]. */
void orc_prefill_attn_f64(const float* q, const uint16_t* k_cache, const uint16_t* v_cache,
                          float* out, uint32_t T, uint32_t start_pos, uint32_t num_q_heads,
                          uint32_t num_kv_heads, uint32_t head_dim, float scale,
                          uint32_t sliding_window) {
  size_t row = (size_t)num_q_heads * head_dim;
  for (uint32_t i = 0; i < T; i++)
    orc_decode_attn_f64(q + i * row, k_cache, v_cache, out + i * row, num_q_heads, num_kv_heads,
                        head_dim, start_pos + i + 1u, scale, sliding_window);
}

/* ------------------------------------------------------------- projection matmuls */

/* One output row as a 256-thread workgroup of the matmul shaders computes it: thread t
 * accumulates term(k) for k = t, t + 256, ... from 0.0 in order (acc = acc + term), then
 * the partials fold with the stride-halving tree; output = p[0].  matmul_quant.wgsl:29-52,
 * matmul_q8.wgsl:42-66, matmul_q4k.wgsl:41-71 (the _mr variants, matmul_quant_mr4.wgsl:55-89,
 * matmul_q8_mr.wgsl:49-86 and matmul_q4k_mr.wgsl:54-96, keep the same per-row order). */
#define ROW_TREE(TERM)                                         \
  do {                                                         \
    float p_[WG];                                              \
    for (uint32_t t = 0; t < WG; t++) {                        \
      float acc = 0.0f;                                        \
      for (uint32_t k = t; k < N; k += WG) acc = acc + (TERM); \
      p_[t] = acc;                                             \
    }                                                          \
    for (uint32_t st = WG / 2; st > 0; st >>= 1)               \
      for (uint32_t t = 0; t < st; t++) p_[t] = p_[t] + p_[t + st]; \
    out[m] = p_[0];                                            \
  } while (0)

/* f16 weight [M, N]: term = f32(weight[m N + k]) * input[k]   (matmul_quant.wgsl:34) */
void orc_matmul_f16(const float* input, const uint16_t* weight, float* out, uint32_t M, uint32_t N) {
#pragma omp parallel for schedule(static)
  for (int64_t mm = 0; mm < (int64_t)M; mm++) {
    const uint32_t m = (uint32_t)mm;
    const uint16_t* w = weight + (size_t)m * N;
    ROW_TREE(orc_half_to_float(w[k]) * input[k]);
  }
}

/* int8 of the packed word, as unpack_i8 (matmul_q8.wgsl:25-28) */
static int32_t unpack_i8(uint32_t packed, uint32_t lane) {
  uint32_t b = (packed >> (lane * 8u)) & 0xffu;
  return b >= 128u ? (int32_t)b - 256 : (int32_t)b;
}

/* Q8: term = f32(q) * f32(scale[m N/32 + k/32]) * input[k]   (matmul_q8.wgsl:45-50) */
void orc_matmul_q8(const float* input, const uint32_t* qweight, const uint16_t* qscale, float* out, uint32_t M,
                   uint32_t N) {
  const uint32_t nblocks = N / 32u;
#pragma omp parallel for schedule(static)
  for (int64_t mm = 0; mm < (int64_t)M; mm++) {
    const uint32_t m = (uint32_t)mm;
    const size_t qb = (size_t)m * N, sb = (size_t)m * nblocks;
    ROW_TREE((float)unpack_i8(qweight[(qb + k) >> 2], (uint32_t)((qb + k) & 3u)) *
             orc_half_to_float(qscale[sb + (k >> 5)]) * input[k]);
  }
}

/* 4-bit block-affine: nib = nibble (m N + k) % 8 of word (m N + k) / 8; with sb = k / 256 and
 * sub = (k % 256) / 32, term = (f32(meta[sb*16 + sub]) * f32(nib) + f32(meta[sb*16 + 8 + sub]))
 * * input[k]   (matmul_q4k.wgsl:44-55) */
void orc_matmul_q4k(const float* input, const uint32_t* qweight, const uint16_t* qmeta, float* out, uint32_t M,
                    uint32_t N) {
  const uint32_t nsblk = N / 256u;
#pragma omp parallel for schedule(static)
  for (int64_t mm = 0; mm < (int64_t)M; mm++) {
    const uint32_t m = (uint32_t)mm;
    const size_t qb = (size_t)m * N, mb = (size_t)m * nsblk * 16u;
    ROW_TREE((orc_half_to_float(qmeta[mb + (k >> 8) * 16u + ((k & 255u) >> 5)]) *
                  (float)((qweight[(qb + k) >> 3] >> (((qb + k) & 7u) * 4u)) & 0xfu) +
              orc_half_to_float(qmeta[mb + (k >> 8) * 16u + 8u + ((k & 255u) >> 5)])) *
             input[k]);
  }
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  omp_set_num_threads(n);
#else
  (void)n;
#endif
}
