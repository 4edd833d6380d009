// Chunked-prefill MoE entry point (prefill_chunk_cmd3 / _batch_general,
// finchmoe/infer.m:10704-11241).
//
// A chunk of T tokens is cut into sub-batches of at most eight tokens and each
// sub-batch goes through the decode kernels (moe_decode.cu), which already read
// every expert selected inside a sub-batch once for all of its tokens.  This is
// the reference's own scheme -- per-position dispatch of the decode kernels,
// with the GGUF path de-duplicating experts inside a group of positions
// (infer.m:12424-12532) -- with the group size fixed at eight.  Every output
// row is bit-identical to what the decode entry point gives for the same token,
// the property the reference claims for its chunked prefill (README.md:25).
#include "finch_internal.cuh"

extern "C" int finch_encode_moe_prefill(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, const void *h_post,
                                        const int32_t *expert_ids, const float *weights, const uint8_t *valid,
                                        const finch_shared *shared, const float *h_mid, float *hidden_out, int T) {
    if (!ctx || !h_post || !expert_ids || !weights || !hidden_out || T < 1) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    int sub = FINCH_MAX_PAIRS / c.top_k;
    if (sub > 8) sub = 8;
    if (sub > c.max_tokens) sub = c.max_tokens;
    const size_t elt = c.act_dtype == FINCH_BF16 ? 2 : 4;
    for (int t0 = 0; t0 < T; t0 += sub) {
        const int n = T - t0 < sub ? T - t0 : sub;
        finch_shared sh;
        if (shared) {
            sh = *shared;
            sh.gate_score = shared->gate_score ? shared->gate_score + t0 : nullptr;
        }
        const int rc = finch_encode_moe_decode(ctx, stream, pool, layer, (const char *)h_post + (size_t)t0 * c.hidden * elt,
                                               expert_ids + (size_t)t0 * c.top_k, weights + (size_t)t0 * c.top_k,
                                               valid ? valid + (size_t)t0 * c.top_k : nullptr, shared ? &sh : nullptr,
                                               h_mid ? h_mid + (size_t)t0 * c.hidden : nullptr, hidden_out + (size_t)t0 * c.hidden, n);
        if (rc) return rc;
    }
    return FINCH_OK;
}
