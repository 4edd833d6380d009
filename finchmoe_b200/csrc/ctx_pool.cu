// Context, device buffers, the HBM-resident expert pool with its slot table,
// events and the synthetic pool fill used by the benchmark.
#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <thread>

#include "finch_internal.cuh"
#include "tile_layout.h"

int finch_fail(finch_ctx *ctx, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->err = buf;
    return code;
}

extern "C" const char *finch_status_str(int s) {
    switch (s) {
        case FINCH_OK: return "ok";
        case FINCH_E_ARG: return "bad argument";
        case FINCH_E_NOSLOT: return "expert not resident";
        case FINCH_E_CUDA: return "CUDA error";
        case FINCH_E_NCCL: return "NCCL error";
        case FINCH_E_TIMEOUT: return "timeout";
        case FINCH_E_UNSUPPORTED: return "unsupported";
        case FINCH_E_NOMEM: return "out of memory";
    }
    return "unknown";
}

extern "C" const char *finch_last_error(const finch_ctx *ctx) { return ctx ? ctx->err.c_str() : ""; }
extern "C" size_t finch_expert_bytes(const finch_ctx *ctx) { return ctx ? ctx->expert_bytes : 0; }
extern "C" uint64_t finch_launch_count(const finch_ctx *ctx) { return ctx ? ctx->launches : 0; }

int finch_func_attr_once(finch_ctx *ctx, const void *func, int smem_bytes) {
    static std::mutex mu;
    static std::vector<std::pair<const void *, int>> done;
    std::lock_guard<std::mutex> lk(mu);
    const int dev = ctx->cfg.device;
    for (const auto &d : done)
        if (d.first == func && d.second == dev) return FINCH_OK;
    if (smem_bytes > 48 * 1024) FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes));
    done.push_back({func, dev});
    return FINCH_OK;
}

extern "C" int finch_ctx_create(const finch_config *cfg, finch_ctx **out) {
    if (!cfg || !out) return FINCH_E_ARG;
    *out = nullptr;
    const finch_config &c = *cfg;
    if (c.hidden <= 0 || c.hidden % 128 || c.moe_inter <= 0 || c.moe_inter % 128 || c.group_size != 64 ||
        c.top_k < 1 || c.top_k > 8 || c.n_experts < 1 || c.n_layers < 1 || c.max_tokens < 1 ||
        (c.expert_bits != 3) || (c.scale_dtype != FINCH_BF16 && c.scale_dtype != FINCH_FP16) ||
        (c.act_dtype != FINCH_F32 && c.act_dtype != FINCH_BF16) || (c.shared_inter % 64) || c.hidden > 8192 ||
        c.moe_inter > 8192 || c.moe_inter > c.hidden || c.shared_inter > c.hidden || c.shared_inter < 0)
        return FINCH_E_ARG;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || c.device < 0 || c.device >= ndev) return FINCH_E_CUDA;
    finch_ctx *ctx = new finch_ctx();
    ctx->cfg = c;
    ctx->no_pdl = getenv("FINCH_NO_PDL") && getenv("FINCH_NO_PDL")[0] == '1';
    auto bail = [&](int code) {
        finch_ctx_destroy(ctx);
        return code;
    };
    if (cudaSetDevice(c.device) != cudaSuccess) return bail(FINCH_E_CUDA);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, c.device) != cudaSuccess) return bail(FINCH_E_CUDA);
    ctx->sm_count = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess) return bail(FINCH_E_CUDA);
    if (cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking) != cudaSuccess || cudaStreamCreateWithFlags(&ctx->side2, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_fork2, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_join2, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ctx->ev_join, cudaEventDisableTiming) != cudaSuccess)
        return bail(FINCH_E_CUDA);
    const size_t gw = (size_t)c.moe_inter * c.hidden * 3 / 8, gs = (size_t)c.moe_inter * (c.hidden / 64) * 2;
    const size_t dw = gw, ds = (size_t)c.hidden * (c.moe_inter / 64) * 2;
    ctx->lay.gate_w = 0;
    ctx->lay.gate_s = gw;
    ctx->lay.gate_b = gw + gs;
    ctx->lay.up_w = gw + 2 * gs;
    ctx->lay.up_s = ctx->lay.up_w + gw;
    ctx->lay.up_b = ctx->lay.up_s + gs;
    ctx->lay.down_w = ctx->lay.up_b + gs;
    ctx->lay.down_s = ctx->lay.down_w + dw;
    ctx->lay.down_b = ctx->lay.down_s + ds;
    ctx->expert_bytes = ctx->lay.down_b + ds;
    const size_t pairs = (size_t)c.max_tokens * c.top_k;
    const int sh_inter = c.shared_inter > 0 ? c.shared_inter : 64;
    bool ok = cudaMalloc(&ctx->act, pairs * c.moe_inter * sizeof(float)) == cudaSuccess &&
              cudaMalloc(&ctx->shared_act, (size_t)c.max_tokens * sh_inter * sizeof(float)) == cudaSuccess &&
              cudaMalloc(&ctx->partial, (pairs + c.max_tokens) * c.hidden * sizeof(float)) == cudaSuccess &&
              cudaMalloc(&ctx->dev_status, sizeof(int)) == cudaSuccess && cudaMalloc(&ctx->hp_ticket, sizeof(unsigned)) == cudaSuccess;
    if (!ok) return bail(FINCH_E_NOMEM);
    cudaMemset(ctx->dev_status, 0, sizeof(int));
    cudaMemset(ctx->hp_ticket, 0, sizeof(unsigned));
    cudaMemset(ctx->partial, 0, (pairs + c.max_tokens) * c.hidden * sizeof(float));
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(FINCH_E_CUDA);
    *out = ctx;
    return FINCH_OK;
}

extern "C" void finch_ctx_destroy(finch_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->cfg.device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->act);
    cudaFree(ctx->shared_act);
    cudaFree(ctx->partial);
    cudaFree(ctx->dev_status);
    cudaFree(ctx->hp_ticket);
    if (ctx->ev_fork) cudaEventDestroy(ctx->ev_fork);
    if (ctx->ev_join) cudaEventDestroy(ctx->ev_join);
    if (ctx->side) cudaStreamDestroy(ctx->side);
    if (ctx->ev_fork2) cudaEventDestroy(ctx->ev_fork2);
    if (ctx->ev_join2) cudaEventDestroy(ctx->ev_join2);
    if (ctx->side2) cudaStreamDestroy(ctx->side2);
    for (auto &e : ctx->shared_cache) cudaFree(e.tiles);
    for (auto &g : ctx->host_graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    cudaFree(ctx->stage_dev);
    cudaFree(ctx->pf_ws);
    cudaFree(ctx->gq_ws);
    cudaFree(ctx->gguf_ws);
    cudaFree(ctx->logits);
    if (ctx->stage_host) cudaFreeHost(ctx->stage_host);
    for (cudaEvent_t e : ctx->prof_events) cudaEventDestroy(e);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

extern "C" int finch_buf_alloc(finch_ctx *ctx, size_t bytes, void **dev) {
    if (!ctx || !dev || bytes == 0) return FINCH_E_ARG;
    cudaSetDevice(ctx->cfg.device);
    if (cudaMalloc(dev, bytes) != cudaSuccess) {
        cudaGetLastError();
        return finch_fail(ctx, FINCH_E_NOMEM, "cudaMalloc(%zu) failed", bytes);
    }
    return FINCH_OK;
}

extern "C" int finch_weights_upload(finch_ctx *ctx, const void *host, size_t bytes, void **dev) {
    if (!ctx || !host || !dev) return FINCH_E_ARG;
    int rc = finch_buf_alloc(ctx, bytes, dev);
    if (rc) return rc;
    FINCH_CUDA_OK(ctx, cudaMemcpy(*dev, host, bytes, cudaMemcpyHostToDevice));
    return FINCH_OK;
}

extern "C" int finch_buf_free(finch_ctx *ctx, void *dev) {
    if (!ctx) return FINCH_E_ARG;
    cudaSetDevice(ctx->cfg.device);
    FINCH_CUDA_OK(ctx, cudaFree(dev));
    return FINCH_OK;
}

extern "C" int finch_sync(finch_ctx *ctx) {
    if (!ctx) return FINCH_E_ARG;
    cudaSetDevice(ctx->cfg.device);
    FINCH_CUDA_OK(ctx, cudaDeviceSynchronize());
    return FINCH_OK;
}

extern "C" int finch_device_status(finch_ctx *ctx, int *status_out) {
    if (!ctx || !status_out) return FINCH_E_ARG;
    FINCH_CUDA_OK(ctx, cudaMemcpy(status_out, ctx->dev_status, sizeof(int), cudaMemcpyDeviceToHost));
    return FINCH_OK;
}

extern "C" int finch_device_status_clear(finch_ctx *ctx) {
    if (!ctx) return FINCH_E_ARG;
    cudaSetDevice(ctx->cfg.device);
    FINCH_CUDA_OK(ctx, cudaDeviceSynchronize());
    FINCH_CUDA_OK(ctx, cudaMemset(ctx->dev_status, 0, sizeof(int)));
    return FINCH_OK;
}

// ------------------------------------------------------------------ events
extern "C" int finch_event_create(finch_ctx *ctx, finch_event **out) {
    if (!ctx || !out) return FINCH_E_ARG;
    finch_event *e = new finch_event();
    e->ctx = ctx;
    if (cudaEventCreateWithFlags(&e->ev, cudaEventDisableTiming) != cudaSuccess) {
        delete e;
        return finch_fail(ctx, FINCH_E_CUDA, "cudaEventCreate failed");
    }
    *out = e;
    return FINCH_OK;
}
extern "C" int finch_event_record(finch_event *ev, finch_stream stream) {
    if (!ev) return FINCH_E_ARG;
    FINCH_CUDA_OK(ev->ctx, cudaEventRecord(ev->ev, finch_pick_stream(ev->ctx, stream)));
    return FINCH_OK;
}
extern "C" int finch_event_wait(finch_event *ev, int timeout_ms) {
    if (!ev) return FINCH_E_ARG;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t q = cudaEventQuery(ev->ev);
        if (q == cudaSuccess) return FINCH_OK;
        if (q != cudaErrorNotReady) return finch_fail(ev->ctx, FINCH_E_CUDA, "cudaEventQuery: %s", cudaGetErrorString(q));
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (timeout_ms >= 0 && ms >= timeout_ms) return finch_fail(ev->ctx, FINCH_E_TIMEOUT, "event not complete after %d ms", timeout_ms);
        std::this_thread::yield();
    }
}
extern "C" void finch_event_destroy(finch_event *ev) {
    if (!ev) return;
    cudaEventDestroy(ev->ev);
    delete ev;
}

// -------------------------------------------------------------------- pool
extern "C" int finch_pool_create(finch_ctx *ctx, int n_layers, int n_experts, int max_slots, finch_pool **out) {
    if (!ctx || !out || n_layers < 1 || n_experts < 1 || max_slots < 0) return FINCH_E_ARG;
    cudaSetDevice(ctx->cfg.device);
    finch_pool *p = new finch_pool();
    p->ctx = ctx;
    p->n_layers = n_layers;
    p->n_experts = n_experts;
    const size_t total = (size_t)n_layers * n_experts;
    p->slots = max_slots == 0 ? (int)total : (int)std::min<size_t>(max_slots, total);
    p->slot_bytes = (ctx->expert_bytes + 255) / 256 * 256;
    p->slot_of.assign(total, -1);
    p->owner.assign(p->slots, -1);
    p->last_used.assign(p->slots, 0);
    if (cudaMalloc(&p->base, (size_t)p->slots * p->slot_bytes) != cudaSuccess ||
        cudaMalloc(&p->slot_table_dev, total * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        finch_pool_destroy(p);
        return finch_fail(ctx, FINCH_E_NOMEM, "pool of %d slots x %zu bytes does not fit", p->slots, p->slot_bytes);
    }
    cudaMemset(p->slot_table_dev, 0xff, total * sizeof(int32_t));
    *out = p;
    return FINCH_OK;
}

extern "C" void finch_pool_destroy(finch_pool *p) {
    if (!p) return;
    cudaSetDevice(p->ctx->cfg.device);
    cudaDeviceSynchronize();
    // launch sequences captured for this pool carry its addresses
    for (auto &g : p->ctx->host_graphs)
        if (g.pool == p) {
            if (g.exec) cudaGraphExecDestroy(g.exec);
            g.exec = nullptr;
            g.pool = nullptr;
            g.seen = -1;
        }
    cudaFree(p->base);
    cudaFree(p->slot_table_dev);
    delete p;
}

static int pool_claim_slot(finch_pool *p, int key) {
    int slot = p->slot_of[key];
    if (slot >= 0) return slot;
    if (p->used < p->slots) {
        while (p->owner[p->cursor] >= 0) p->cursor = (p->cursor + 1) % p->slots;
        slot = p->cursor;
        p->used++;
    } else {  // evict the least recently used entry (linear scan, as the reference does)
        slot = 0;
        for (int s = 1; s < p->slots; s++)
            if (p->last_used[s] < p->last_used[slot]) slot = s;
        const int old = p->owner[slot];
        p->slot_of[old] = -1;
        const int32_t neg = -1;
        cudaMemcpy(p->slot_table_dev + old, &neg, sizeof neg, cudaMemcpyHostToDevice);
        p->evictions++;
    }
    p->owner[slot] = key;
    p->slot_of[key] = slot;
    return slot;
}

extern "C" int finch_pool_put(finch_pool *p, int layer, int expert, const void *block) {
    if (!p || !block || layer < 0 || layer >= p->n_layers || expert < 0 || expert >= p->n_experts) return FINCH_E_ARG;
    finch_ctx *ctx = p->ctx;
    cudaSetDevice(ctx->cfg.device);
    const int key = layer * p->n_experts + expert;
    // A put may overwrite a slot (a full pool evicts) and edits the slot table that queued kernels resolve ids
    // with.  The copies below are synchronous on the legacy stream, which does not order them against the
    // context's non-blocking stream or a caller's stream: wait for what is queued on this device first, so that no
    // kernel in flight reads a slot or a table entry while it changes.  (With every expert resident, the
    // intended mode here, puts happen before the first layer call and this costs nothing.)
    if (p->slot_of[key] >= 0 || p->used >= p->slots) FINCH_CUDA_OK(ctx, cudaDeviceSynchronize());
    const int slot = pool_claim_slot(p, key);
    p->last_used[slot] = ++p->clock;
    p->tmp.resize(ctx->expert_bytes);
    finch_retile(ctx->cfg.hidden, ctx->cfg.moe_inter, (const uint8_t *)block, p->tmp.data(), 1);
    FINCH_CUDA_OK(ctx, cudaMemcpy(p->base + (size_t)slot * p->slot_bytes, p->tmp.data(), ctx->expert_bytes, cudaMemcpyHostToDevice));
    const int32_t s32 = slot;
    FINCH_CUDA_OK(ctx, cudaMemcpy(p->slot_table_dev + key, &s32, sizeof s32, cudaMemcpyHostToDevice));
    return FINCH_OK;
}

extern "C" int finch_pool_lookup(finch_pool *p, int layer, int expert, int *slot_out, void **dev_ptr_out) {
    if (!p || layer < 0 || layer >= p->n_layers || expert < 0 || expert >= p->n_experts) return FINCH_E_ARG;
    const int slot = p->slot_of[layer * p->n_experts + expert];
    if (slot < 0) {
        p->misses++;
        return FINCH_E_NOSLOT;
    }
    p->hits++;
    p->last_used[slot] = ++p->clock;
    if (slot_out) *slot_out = slot;
    if (dev_ptr_out) *dev_ptr_out = p->base + (size_t)slot * p->slot_bytes;
    return FINCH_OK;
}

extern "C" int finch_pool_get(finch_pool *p, int layer, int expert, void *out) {
    if (!p || !out || layer < 0 || layer >= p->n_layers || expert < 0 || expert >= p->n_experts) return FINCH_E_ARG;
    const int slot = p->slot_of[layer * p->n_experts + expert];
    if (slot < 0) return FINCH_E_NOSLOT;
    cudaSetDevice(p->ctx->cfg.device);
    p->tmp.resize(p->ctx->expert_bytes);
    FINCH_CUDA_OK(p->ctx, cudaMemcpy(p->tmp.data(), p->base + (size_t)slot * p->slot_bytes, p->ctx->expert_bytes, cudaMemcpyDeviceToHost));
    finch_retile(p->ctx->cfg.hidden, p->ctx->cfg.moe_inter, p->tmp.data(), (uint8_t *)out, 0);
    return FINCH_OK;
}

extern "C" int finch_pool_get_stats(const finch_pool *p, finch_pool_stats *out) {
    if (!p || !out) return FINCH_E_ARG;
    out->hits = p->hits;
    out->misses = p->misses;
    out->evictions = p->evictions;
    out->slots = p->slots;
    out->used = p->used;
    out->slot_bytes = p->slot_bytes;
    return FINCH_OK;
}

// ---- synthetic fill ------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// One thread per 32-bit word of a block (tiled layout, tile_layout.h).  Code
// words get random bits; a scale word holds two scales = |N(0, 0.01)|
// (Box-Muller) and the matching bias word holds -4 * the stored (rounded) scale.
__device__ __forceinline__ uint16_t synth_scale16(uint64_t key, int scale_dtype, bool bias) {
    const uint64_t r = mix64(key);
    const float u1 = ((r >> 40) + 1) * (1.0f / 16777217.0f), u2 = ((r >> 8) & 0xffffff) * (1.0f / 16777216.0f);
    const float s = fabsf(0.01f * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
    if (scale_dtype == FINCH_FP16) {
        const __half h = __float2half_rn(s);
        return bias ? __half_as_ushort(__float2half_rn(-4.0f * __half2float(h))) : __half_as_ushort(h);
    }
    const __nv_bfloat16 h = __float2bfloat16_rn(s);
    return bias ? __bfloat16_as_ushort(__float2bfloat16_rn(-4.0f * __bfloat162float(h))) : __bfloat16_as_ushort(h);
}

// The contents depend on the expert's key (layer * n_experts + expert), not on the slot that stores it.
__global__ void pool_fill_kernel(uint8_t *base, size_t slot_bytes, int first_slot, int first_key, uint64_t seed, FinchTile T, int scale_dtype) {
    const size_t words = T.total / 4;
    const int slot = first_key + blockIdx.y;   // the name the generator mixes in
    uint32_t *blk = reinterpret_cast<uint32_t *>(base + (size_t)(first_slot + blockIdx.y) * slot_bytes);
    for (size_t w = (size_t)blockIdx.x * blockDim.x + threadIdx.x; w < words; w += (size_t)gridDim.x * blockDim.x) {
        const size_t off = w * 4;
        const bool isB = off >= T.b_base;
        const size_t o2 = isB ? off - T.b_base : off;
        const int tsz = isB ? T.tileB : T.tileA, sb0 = isB ? T.sbB : T.sbA;
        const int tile = (int)(o2 / tsz), rel = (int)(o2 % tsz);
        uint32_t out;
        if (rel < sb0) {
            out = (uint32_t)mix64(seed ^ ((uint64_t)slot << 32) ^ (uint64_t)w);
        } else {
            const int e = (rel - sb0) / 4, field = e & 3, g = (e >> 2) & 7, u = e >> 5;
            const bool bias = field >= 2;
            const uint64_t id = (((((uint64_t)tile * 8 + g) * 2 + (field & 1)) * 128 + u) * 2) | ((uint64_t)isB << 40);
            const uint64_t key = seed ^ 0xabcdefull ^ ((uint64_t)slot << 42);
            out = (uint32_t)synth_scale16(key ^ id, scale_dtype, bias) | ((uint32_t)synth_scale16(key ^ (id + 1), scale_dtype, bias) << 16);
        }
        blk[w] = out;
    }
}

extern "C" int finch_pool_fill_synthetic(finch_pool *p, int layer0, int layer1, uint64_t seed) {
    if (!p || layer0 < 0 || layer1 > p->n_layers || layer0 >= layer1) return FINCH_E_ARG;
    finch_ctx *ctx = p->ctx;
    if (p->slots != p->n_layers * p->n_experts) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "synthetic fill needs a fully resident pool");
    cudaSetDevice(ctx->cfg.device);
    const FinchTile T = finch_tile(ctx->cfg.hidden, ctx->cfg.moe_inter);
    for (int l = layer0; l < layer1; l++) {
        // identity slot assignment: slot = layer * n_experts + expert
        for (int e = 0; e < p->n_experts; e++) {
            const int key = l * p->n_experts + e;
            if (p->slot_of[key] < 0) {
                p->slot_of[key] = key;
                p->owner[key] = key;
                p->last_used[key] = ++p->clock;
            } else if (p->slot_of[key] != key) {
                return finch_fail(ctx, FINCH_E_UNSUPPORTED, "pool already holds experts in non-identity slots");
            }
        }
        dim3 grid(64, p->n_experts);
        pool_fill_kernel<<<grid, 256, 0, ctx->stream>>>(p->base, p->slot_bytes, l * p->n_experts, l * p->n_experts, seed + (uint64_t)l * 0x10001ull, T,
                                                        ctx->cfg.scale_dtype);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
    }
    p->used = 0;
    for (int s = 0; s < p->slots; s++) p->used += p->owner[s] >= 0;
    FINCH_CUDA_OK(ctx, cudaMemcpyAsync(p->slot_table_dev, p->slot_of.data(), p->slot_of.size() * sizeof(int32_t),
                                       cudaMemcpyHostToDevice, ctx->stream));
    FINCH_CUDA_OK(ctx, cudaStreamSynchronize(ctx->stream));
    return FINCH_OK;
}

// The same generator for one shard of the experts (expert-parallel ranks): experts [e0, e1) of layers
// [layer0, layer1) get exactly the contents finch_pool_fill_synthetic gives them in a full pool, stored in
// slots layer * (e1 - e0) + (expert - e0).
extern "C" int finch_pool_fill_synthetic_range(finch_pool *p, int layer0, int layer1, int e0, int e1, uint64_t seed) {
    if (!p || layer0 < 0 || layer1 > p->n_layers || layer0 >= layer1 || e0 < 0 || e1 > p->n_experts || e0 >= e1) return FINCH_E_ARG;
    finch_ctx *ctx = p->ctx;
    const int per = e1 - e0;
    if (p->slots < p->n_layers * per) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "pool has %d slots, the shard needs %d", p->slots, p->n_layers * per);
    cudaSetDevice(ctx->cfg.device);
    const FinchTile T = finch_tile(ctx->cfg.hidden, ctx->cfg.moe_inter);
    for (int l = layer0; l < layer1; l++) {
        for (int e = e0; e < e1; e++) {
            const int key = l * p->n_experts + e, slot = l * per + (e - e0);
            if (p->slot_of[key] < 0 && p->owner[slot] < 0) {
                p->slot_of[key] = slot;
                p->owner[slot] = key;
                p->last_used[slot] = ++p->clock;
            } else if (p->slot_of[key] != slot) {
                return finch_fail(ctx, FINCH_E_UNSUPPORTED, "pool already holds experts in other slots");
            }
        }
        pool_fill_kernel<<<dim3(64, per), 256, 0, ctx->stream>>>(p->base, p->slot_bytes, l * per, l * p->n_experts + e0,
                                                                 seed + (uint64_t)l * 0x10001ull, T, ctx->cfg.scale_dtype);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
    }
    p->used = 0;
    for (int s = 0; s < p->slots; s++) p->used += p->owner[s] >= 0;
    FINCH_CUDA_OK(ctx, cudaMemcpyAsync(p->slot_table_dev, p->slot_of.data(), p->slot_of.size() * sizeof(int32_t),
                                       cudaMemcpyHostToDevice, ctx->stream));
    FINCH_CUDA_OK(ctx, cudaStreamSynchronize(ctx->stream));
    return FINCH_OK;
}
