// Chunked-prefill MoE path (placeholder until the grouped dequant-GEMM lands).
#include "finch_internal.cuh"

extern "C" int finch_encode_moe_prefill(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, const void *h_post,
                                        const int32_t *expert_ids, const float *weights, const uint8_t *valid,
                                        const finch_shared *shared, const float *h_mid, float *hidden_out, int T) {
    if (!ctx) return FINCH_E_ARG;
    if ((size_t)T * ctx->cfg.top_k <= FINCH_MAX_PAIRS)
        return finch_encode_moe_decode(ctx, stream, pool, layer, h_post, expert_ids, weights, valid, shared, h_mid, hidden_out, T);
    return finch_fail(ctx, FINCH_E_UNSUPPORTED, "prefill chunks above %d pairs are not built yet", FINCH_MAX_PAIRS);
}
