// Prefill attention on the tensor cores (tcgen05.mma + TMEM).  The reference has no prefill
// attention kernel: prefillBatched (src/engine.ts:2460-2479) runs one decode forward per token,
// so row i equals decode attention at kv_len = start_pos + i + 1.
#include "g4a_internal.cuh"

extern "C" g4a_status g4a_prefill_attn(g4a_ctx* ctx, const uint16_t* q16, const uint16_t* k_cache,
                                       const uint16_t* v_cache, float* out, uint32_t T, uint32_t start_pos,
                                       uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t head_dim, float scale,
                                       uint32_t sliding_window) {
  G4A_CHECK_CTX(ctx);
  (void)q16; (void)k_cache; (void)v_cache; (void)out; (void)T; (void)start_pos; (void)num_q_heads;
  (void)num_kv_heads; (void)head_dim; (void)scale; (void)sliding_window;
  return g4a_fail(G4A_EUNSUPPORTED, "g4a_prefill_attn: tensor-core prefill kernel not built yet");
}
