// Host-pointer entry point of the MoE layer: packs the caller's CPU buffers
// into one pinned staging block, moves it to the device in one transfer (a kernel
// that reads the block over the bus for decode-sized calls, a copy otherwise), encodes
// (or, for a shape seen before, replays from a captured graph)
// the decode or prefill path (decode-sized calls write their result rows straight
// into the pinned block; larger ones copy them back) and waits.
#include <chrono>

#include "finch_internal.cuh"

int finch_stage_reserve(finch_ctx *ctx, size_t bytes);

static inline size_t up256(size_t n) { return (n + 255) & ~(size_t)255; }

// The inputs of a decode-sized call, read from the pinned block over the bus by a kernel instead of a copy
// operation: a few tens of KB, one 16-byte word per thread.  It lets the kernels behind it start at once
// (griddepcontrol.launch_dependents first), so the gate/up kernel's prologue runs while the words are in flight,
// which a copy operation in the stream does not allow.
__global__ void __launch_bounds__(256) host_stage_kernel(const uint4 *__restrict__ src, uint4 *__restrict__ dst, int n16) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n16) dst[i] = src[i];
}

extern "C" int finch_moe_forward_host(finch_ctx *ctx, finch_pool *pool, int layer, const void *h_post,
                                      const int32_t *expert_ids, const float *weights, const uint8_t *valid,
                                      const finch_shared *shared, const float *shared_gate_score_host, const float *h_mid,
                                      float *hidden_out, int T) {
    if (!ctx || !pool || !h_post || !expert_ids || !weights || !hidden_out || T < 1) return FINCH_E_ARG;
    if (shared && !shared_gate_score_host) return finch_fail(ctx, FINCH_E_ARG, "shared expert given without gate scores");
    const finch_config &c = ctx->cfg;
    const size_t elt = c.act_dtype == FINCH_BF16 ? 2 : 4;
    const size_t n_x = (size_t)T * c.hidden * elt, n_id = (size_t)T * c.top_k * 4, n_w = n_id, n_v = valid ? (size_t)T * c.top_k : 0;
    const size_t n_s = shared ? (size_t)T * 4 : 0, n_h = h_mid ? (size_t)T * c.hidden * 4 : 0, n_o = (size_t)T * c.hidden * 4;
    // o_q: the completion value of this call, staged with the inputs
    const size_t o_x = 0, o_id = o_x + up256(n_x), o_w = o_id + up256(n_id), o_v = o_w + up256(n_w), o_s = o_v + up256(n_v),
                 o_h = o_s + up256(n_s), o_q = o_h + up256(n_h), o_o = o_q + 256, o_st = o_o + up256(n_o), total = o_st + 256;
    int rc = finch_stage_reserve(ctx, total);
    if (rc) return rc;
    cudaSetDevice(c.device);
    char *hs = (char *)ctx->stage_host, *ds = (char *)ctx->stage_dev;
    memcpy(hs + o_x, h_post, n_x);
    memcpy(hs + o_id, expert_ids, n_id);
    memcpy(hs + o_w, weights, n_w);
    if (valid) memcpy(hs + o_v, valid, n_v);
    if (shared) memcpy(hs + o_s, shared_gate_score_host, n_s);
    if (h_mid) memcpy(hs + o_h, h_mid, n_h);
    // what finch_encode_moe_decode accepts; everything else goes through the prefill entry (which splits)
    const bool small = T <= 8 && T <= c.max_tokens && (size_t)T * c.top_k <= FINCH_MAX_PAIRS;
    // The inputs cross the bus in one copy into device memory: every CTA of the gate/up kernel reads the
    // activations and the routing.  The result of a decode-sized call is a few tens of KB: the combine kernel
    // writes its rows straight into the pinned staging block, which saves the copy back and its stream
    // dependency (it costs more than moving the bytes), and a kernel fetches the inputs from the pinned block instead
    // of a copy operation (measured: 61.2 against 62.7 us per layer; 58.3 with the graph replay below).
    // FINCH_HOST_PATH=2 keeps plain launches, 1 also the copy operation for the inputs, 0 forces a copy back as well.
    static const int host_path = [] {
        const char *e = getenv("FINCH_HOST_PATH");
        return e ? atoi(e) : 3;
    }();
    char *in = ds, *out = ds;
    if (small && host_path >= 1) {
        void *m = nullptr;
        if (cudaHostGetDevicePointer(&m, hs, 0) == cudaSuccess && m) out = (char *)m;
        else cudaGetLastError();
    }
    // A decode-sized call whose result lands in the pinned block also reports there: the last CTA of the combine
    // kernel writes the status word and then this call's sequence number, and the host waits on that word instead
    // of on the stream (no copy operation for the status, no driver wake-up).
    const bool flagged = out != ds;
    volatile unsigned *done = reinterpret_cast<volatile unsigned *>(hs + o_st + 64);
    if (flagged) {
        ctx->hp_seq = ctx->hp_seq + 1 == 0 ? 1 : ctx->hp_seq + 1;
        *done = 0u;                      // the block is reused: whatever lay here is not a completion
        *reinterpret_cast<unsigned *>(hs + o_q) = ctx->hp_seq;
    }
    finch_shared sh;
    if (shared) {
        sh = *shared;
        sh.gate_score = (const float *)(in + o_s);
    }
    auto fn = small ? finch_encode_moe_decode : finch_encode_moe_prefill;
    // the launch sequence: the inputs' way to device memory, then the layer's kernels
    auto encode = [&]() -> int {
        if (flagged && host_path >= 2) {
            const int n16 = (int)(o_o / 16);
            host_stage_kernel<<<(n16 + 255) / 256, 256, 0, ctx->stream>>>(reinterpret_cast<const uint4 *>(out), reinterpret_cast<uint4 *>(ds), n16);
            FINCH_CUDA_OK(ctx, cudaGetLastError());
            ctx->launches++;
        } else {
            FINCH_CUDA_OK(ctx, cudaMemcpyAsync(ds, hs, o_o, cudaMemcpyHostToDevice, ctx->stream));
        }
        if (flagged) {
            ctx->hp_done = reinterpret_cast<unsigned *>(out + o_st + 64);
            ctx->hp_status = reinterpret_cast<int *>(out + o_st);
            ctx->hp_seq_src = reinterpret_cast<const unsigned *>(ds + o_q);
        }
        const int r = fn(ctx, ctx->stream, pool, layer, in + o_x, (const int32_t *)(in + o_id), (const float *)(in + o_w),
                         valid ? (const uint8_t *)(in + o_v) : nullptr, shared ? &sh : nullptr, h_mid ? (const float *)(in + o_h) : nullptr,
                         (float *)(out + o_o), T);
        ctx->hp_done = nullptr;
        return r;
    };
    // Decode-sized calls repeat with the same shape layer after layer, token after token: the second call of a shape
    // is captured into a CUDA graph (every address in it is a staging address) and later ones are one graph launch
    // instead of four kernel launches.  FINCH_HOST_PATH=2 keeps the plain launches.
    finch_ctx::HostGraph *hg = nullptr;
    if (flagged && host_path >= 3 && !ctx->profile) {
        finch_shared key{};   // zero, padding included; filled field by field so that it stays comparable byte by byte
        if (shared) {
            const finch_wdesc *from[3] = {&shared->gate, &shared->up, &shared->down};
            finch_wdesc *to[3] = {&key.gate, &key.up, &key.down};
            for (int i = 0; i < 3; i++) {
                to[i]->W = from[i]->W;
                to[i]->scales = from[i]->scales;
                to[i]->biases = from[i]->biases;
                to[i]->out_dim = from[i]->out_dim;
                to[i]->in_dim = from[i]->in_dim;
                to[i]->group_size = from[i]->group_size;
                to[i]->bits = from[i]->bits;
                to[i]->scale_dtype = from[i]->scale_dtype;
            }
        }
        for (auto &g : ctx->host_graphs)
            if (g.pool == pool && g.layer == layer && g.T == T && g.valid == (valid != nullptr) && g.h_mid == (h_mid != nullptr) &&
                g.has_shared == (shared != nullptr) && g.fault == ctx->fault && g.stage_gen == ctx->stage_gen && (!shared || !memcmp(&g.shared, &key, sizeof key))) {
                hg = &g;
                break;
            }
        if (!hg) {
            if (ctx->host_graphs.size() >= 256) {   // shapes that never repeat: start over rather than grow
                for (auto &g : ctx->host_graphs)
                    if (g.exec) cudaGraphExecDestroy(g.exec);
                ctx->host_graphs.clear();
            }
            ctx->host_graphs.push_back({pool, layer, T, valid != nullptr, h_mid != nullptr, shared != nullptr, ctx->fault, key, ctx->stage_gen, 0, nullptr});
            hg = &ctx->host_graphs.back();
        }
    }
    if (hg && hg->exec) {
        FINCH_CUDA_OK(ctx, cudaGraphLaunch(hg->exec, ctx->stream));
        ctx->launches += 4;
    } else if (hg && hg->seen == 1) {
        cudaGraph_t graph = nullptr;
        cudaGraphExec_t exec = nullptr;
        hg->seen = -1;   // unless everything below works out
        if (cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            rc = encode();
            const cudaError_t ce = cudaStreamEndCapture(ctx->stream, &graph);
            if (rc == FINCH_OK && ce == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
                hg->exec = exec;
                hg->seen = 2;
            }
        }
        if (!hg->exec) cudaGetLastError();
        if (graph) cudaGraphDestroy(graph);
        if (hg->exec) {
            FINCH_CUDA_OK(ctx, cudaGraphLaunch(hg->exec, ctx->stream));
        } else {
            rc = encode();   // nothing was launched by the failed capture
            if (rc) return rc;
        }
    } else {
        rc = encode();
        if (rc) return rc;
        if (hg && hg->seen == 0) hg->seen = 1;
    }
    bool waited = false;
    if (flagged) {
        const auto t0 = std::chrono::steady_clock::now();
        for (unsigned spins = 0;; spins++) {
            if (*done == ctx->hp_seq) {
                waited = true;
                break;
            }
            if ((spins & 0xfffu) == 0xfffu && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(2)) break;   // fall back to the stream
        }
    }
    if (!waited) {
        if (out == ds) FINCH_CUDA_OK(ctx, cudaMemcpyAsync(hs + o_o, ds + o_o, n_o, cudaMemcpyDeviceToHost, ctx->stream));
        // the device status word rides along (a bounded wait that ran out leaves the output undefined)
        FINCH_CUDA_OK(ctx, cudaMemcpyAsync(hs + o_st, ctx->dev_status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
        FINCH_CUDA_OK(ctx, cudaStreamSynchronize(ctx->stream));
    }
    memcpy(hidden_out, hs + o_o, n_o);
    const int dev_rc = *(const int *)(hs + o_st);
    if (dev_rc != FINCH_OK) return finch_fail(ctx, dev_rc, "device status %d after the MoE layer", dev_rc);
    return FINCH_OK;
}
