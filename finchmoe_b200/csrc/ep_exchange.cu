// Device-side steps of the expert-parallel MoE layer.
//
// Experts are sharded in contiguous blocks (rank r owns experts [r * E / G, (r + 1) * E / G) of every
// layer); tokens stay with the rank that owns them.  One layer is
//   plan     which of my tokens go to which rank (a token goes at most once to a rank, with its whole
//            row of expert ids and router weights), positions inside each destination's list
//   pack     one record per (token, destination): activation row, ids, weights, valid mask
//   (exchange: the host layer runs an all-to-all over NCCL between pack and unpack)
//   unpack   records received -> contiguous activation / id / weight / mask arrays; the rank then runs
//            its ordinary MoE path on them: its pool holds only its own experts, so every other
//            expert of a row is skipped, and the result is the weighted sum over the local experts
//   (exchange back: fp32 rows)
//   combine  hidden[t] += partial sums in ascending rank order (deterministic)
// The reference has no multi-device path; these entry points extend its per-layer CMD3
// (finchmoe/infer.m:9597-9741) across GPUs.
#include "finch_internal.cuh"

namespace {

__host__ __device__ inline int rec_bytes_of(int hidden, int elt, int K) { return (hidden * elt + 9 * K + 15) & ~15; }

// One CTA of 1024 threads.  counts[d], offs[d] (exclusive prefix, offs[G] = total), send_tok[offs[d] + p] =
// p-th token (ascending) that has a usable expert on rank d, slot_of[t * G + d] = p or -1.  Nothing goes to rank
// `skip` (the home rank, when it computes its own experts' share of its own tokens in place).
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t *ids, const uint8_t *valid, int T, int K, int n_experts, int G, int skip,
                                                       int *counts, int *offs, int *send_tok, int *slot_of) {
    __shared__ int warp_sum[32];
    __shared__ int run;        // tokens placed so far in the current destination's list
    __shared__ int base;       // offs[d]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = n_experts / G;
    if (tid == 0) base = 0;
    __syncthreads();
    for (int d = 0; d < G; d++) {
        if (tid == 0) run = 0;
        __syncthreads();
        for (int t0 = 0; t0 < T; t0 += 1024) {
            const int t = t0 + tid;
            bool go = false;
            if (t < T && d != skip)
                for (int k = 0; k < K; k++) {
                    const int e = ids[t * K + k];
                    if ((!valid || valid[t * K + k]) && e >= 0 && e < n_experts && e / per == d) go = true;
                }
            const unsigned bal = __ballot_sync(0xffffffffu, go);
            if (lane == 0) warp_sum[warp] = __popc(bal);
            __syncthreads();
            int before = run;
            for (int w = 0; w < warp; w++) before += warp_sum[w];
            const int pos = before + __popc(bal & ((1u << lane) - 1u));
            if (t < T) {
                slot_of[t * G + d] = go ? pos : -1;
                if (go) send_tok[base + pos] = t;
            }
            __syncthreads();
            if (tid == 0) {
                int s = 0;
                for (int w = 0; w < 32; w++) s += warp_sum[w];
                run += s;
            }
            __syncthreads();
        }
        if (tid == 0) {
            counts[d] = run;
            offs[d] = base;
            base += run;
            if (d == G - 1) offs[G] = base;
        }
        __syncthreads();
    }
}

// grid: one CTA per record; record = [activation row | ids K x int32 | weights K x fp32 | valid K bytes | pad]
__global__ void ep_pack_kernel(const uint8_t *x, const int32_t *ids, const float *weights, const uint8_t *valid, int row_bytes, int K, int rec_bytes,
                               const int *offs, int G, const int *send_tok, uint8_t *out) {
    const int i = blockIdx.x;
    if (i >= offs[G]) return;
    const int t = send_tok[i];
    uint8_t *rec = out + (size_t)i * rec_bytes;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)t * row_bytes);
    uint4 *dst = reinterpret_cast<uint4 *>(rec);
    for (int j = threadIdx.x; j < row_bytes / 16; j += blockDim.x) dst[j] = src[j];
    if (threadIdx.x < K) {
        const int k = threadIdx.x;
        reinterpret_cast<int32_t *>(rec + row_bytes)[k] = ids[t * K + k];
        reinterpret_cast<float *>(rec + row_bytes + 4 * K)[k] = weights[t * K + k];
        rec[row_bytes + 8 * K + k] = valid ? valid[t * K + k] : (uint8_t)1;
    }
}

__global__ void ep_unpack_kernel(const uint8_t *in, int n, int row_bytes, int K, int rec_bytes, uint8_t *x, int32_t *ids, float *weights, uint8_t *valid) {
    const int i = blockIdx.x;
    if (i >= n) return;
    const uint8_t *rec = in + (size_t)i * rec_bytes;
    const uint4 *src = reinterpret_cast<const uint4 *>(rec);
    uint4 *dst = reinterpret_cast<uint4 *>(x + (size_t)i * row_bytes);
    for (int j = threadIdx.x; j < row_bytes / 16; j += blockDim.x) dst[j] = src[j];
    if (threadIdx.x < K) {
        const int k = threadIdx.x;
        ids[i * K + k] = reinterpret_cast<const int32_t *>(rec + row_bytes)[k];
        weights[i * K + k] = reinterpret_cast<const float *>(rec + row_bytes + 4 * K)[k];
        valid[i * K + k] = rec[row_bytes + 8 * K + k];
    }
}

// grid (hidden / 256, T)
__global__ void __launch_bounds__(256) ep_combine_kernel(float *hidden_out, const float *back, const int *slot_of, const int *offs, int G, int hidden) {
    const int t = blockIdx.y, row = blockIdx.x * 256 + threadIdx.x;
    if (row >= hidden) return;
    float h = hidden_out[(size_t)t * hidden + row];
    for (int d = 0; d < G; d++) {
        const int p = slot_of[t * G + d];
        if (p >= 0) h += back[(size_t)(offs[d] + p) * hidden + row];
    }
    hidden_out[(size_t)t * hidden + row] = h;
}

}  // namespace

extern "C" int finch_ep_record_bytes(const finch_ctx *ctx) {
    if (!ctx) return 0;
    return rec_bytes_of(ctx->cfg.hidden, ctx->cfg.act_dtype == FINCH_BF16 ? 2 : 4, ctx->cfg.top_k);
}

extern "C" int finch_encode_ep_plan(finch_ctx *ctx, finch_stream stream, const int32_t *expert_ids, const uint8_t *valid, int T, int world,
                                    int skip_rank, int *counts, int *offs, int *send_tok, int *slot_of) {
    if (!ctx || !expert_ids || !counts || !offs || !send_tok || !slot_of || T < 1 || world < 1) return FINCH_E_ARG;
    if (ctx->cfg.n_experts % world) return finch_fail(ctx, FINCH_E_ARG, "%d experts do not split over %d ranks", ctx->cfg.n_experts, world);
    cudaSetDevice(ctx->cfg.device);
    ep_plan_kernel<<<1, 1024, 0, finch_pick_stream(ctx, stream)>>>(expert_ids, valid, T, ctx->cfg.top_k, ctx->cfg.n_experts, world, skip_rank, counts, offs,
                                                                    send_tok, slot_of);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_pack(finch_ctx *ctx, finch_stream stream, const void *h_post, const int32_t *expert_ids, const float *weights,
                                    const uint8_t *valid, int T, int world, const int *offs, const int *send_tok, void *records) {
    if (!ctx || !h_post || !expert_ids || !weights || !offs || !send_tok || !records || T < 1 || world < 1) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    const int elt = c.act_dtype == FINCH_BF16 ? 2 : 4, row_bytes = c.hidden * elt;
    if (row_bytes % 16) return finch_fail(ctx, FINCH_E_ARG, "activation rows must be multiples of 16 bytes");
    cudaSetDevice(c.device);
    ep_pack_kernel<<<T * world, 128, 0, finch_pick_stream(ctx, stream)>>>((const uint8_t *)h_post, expert_ids, weights, valid, row_bytes, c.top_k,
                                                                          rec_bytes_of(c.hidden, elt, c.top_k), offs, world, send_tok, (uint8_t *)records);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_unpack(finch_ctx *ctx, finch_stream stream, const void *records, int n, void *h_post, int32_t *expert_ids, float *weights,
                                      uint8_t *valid) {
    if (!ctx || n < 0) return FINCH_E_ARG;
    if (n == 0) return FINCH_OK;   // a rank that received nothing (its buffers may be NULL)
    if (!records || !h_post || !expert_ids || !weights || !valid) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    const int elt = c.act_dtype == FINCH_BF16 ? 2 : 4;
    cudaSetDevice(c.device);
    ep_unpack_kernel<<<n, 128, 0, finch_pick_stream(ctx, stream)>>>((const uint8_t *)records, n, c.hidden * elt, c.top_k, rec_bytes_of(c.hidden, elt, c.top_k),
                                                                    (uint8_t *)h_post, expert_ids, weights, valid);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_combine(finch_ctx *ctx, finch_stream stream, float *hidden_out, const float *back_rows, const int *slot_of, const int *offs,
                                       int T, int world) {
    if (!ctx || !hidden_out || !back_rows || !slot_of || !offs || T < 1 || world < 1) return FINCH_E_ARG;
    cudaSetDevice(ctx->cfg.device);
    ep_combine_kernel<<<dim3((ctx->cfg.hidden + 255) / 256, T), 256, 0, finch_pick_stream(ctx, stream)>>>(hidden_out, back_rows, slot_of, offs, world,
                                                                                                           ctx->cfg.hidden);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}
