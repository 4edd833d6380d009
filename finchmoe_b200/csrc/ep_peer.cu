// The fixed-capacity exchange of the expert-parallel layer over NVLink peer memory: the ranks' own kernels
// store records and partial rows straight into each other's receive areas, every payload word beside the
// sender's epoch, and the receiving kernels read word pairs until they carry the epoch they expect.  No
// collective library call and no host step per layer, so a decode layer is a fixed sequence of launches on
// one stream (and can sit in a CUDA graph).
//
//   dispatch   every token's record -> slot [my rank][t] of every rank's area (my own included)
//   receive    read the world * T records addressed to me as they arrive and spread them into the row arrays
//              the MoE entry points take; on request the block of my own tokens is masked out
//   return     the partial rows of source s's tokens -> slot [my rank][t] of rank s's area (a kernel of its own, or
//              the last kernel of the decode pass when the layer runs through finch_encode_ep_peer_decode)
//   combine    read every other rank's partial rows of my tokens as they arrive, add them to the layer output
//              in ascending rank order, and advance this rank's epoch
//
// Why one buffer per slot is enough: a rank dispatches layer l + 1 only after its combine of layer l, which read
// every peer's return of layer l, which each peer issued after its receive of layer l had read the slots.  The
// same chain orders the partial-row slots.  All ranks must therefore call the four steps in the same order the
// same number of times (that also keeps their epochs equal).
//
// Every wait is bounded: when a word pair does not arrive within the limit the kernel records FINCH_E_TIMEOUT
// in the device status word, treats the slot as empty and goes on; once the status word is set no later wait
// spins again.  Plain peer stores and local loads only (no multicast objects).
// The reference runs on one device; this extends its per-layer path (finchmoe/infer.m:9597-9741).
#include <cstring>

#include "finch_internal.cuh"

struct finch_ep_peer {
    finch_ctx *ctx = nullptr;
    int rank = 0, world = 0, T = 0;
    size_t bytes = 0, off_back = 0;      // the area: records [world * T] (each word beside its epoch), then partial rows likewise
    uint32_t *sync = nullptr;            // this rank's own {epoch, ticket of the combine kernel}
    uint8_t *area = nullptr;             // this rank's receive area
    uint8_t *remote[16] = {};            // every rank's area as this process addresses it (remote[rank] == area)
    bool opened[16] = {};                // mapped through an IPC handle (to be closed)
    long long limit = 4000000;           // polls of ~100 ns before a wait gives up
};

namespace {

constexpr int MAXW = 16;
struct Areas {
    uint8_t *p[MAXW];
};

__host__ __device__ inline int rec_bytes_of(int hidden, int elt, int K) { return (hidden * elt + 9 * K + 15) & ~15; }
inline size_t up256(size_t n) { return (n + 255) & ~(size_t)255; }

// Programmatic dependent launch: a kernel of the chain may be scheduled while its predecessor still runs.  Every
// kernel here executes dep_wait() before it exits, so "my predecessor has completed" holds transitively along the
// stream; a kernel that needs nothing its predecessor wrote does its work first and waits last.
__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- data and flag in the same word pair -------------------------------------------------------------
// Every 16-byte store carries two payload words and, beside each, the sender's epoch: {w0, epoch, w1, epoch}.  An
// aligned 8-byte half of it arrives whole, so a receiver that reads a pair with the epoch it expects has the
// payload word that came with it: no fence and no separate flag round trip on the sending side, one NVLink
// crossing per hop.  The epoch is a word in each rank's own memory that the combine kernel advances once per layer;
// all ranks run the same sequence, so sender and receiver agree on it, and a slot's previous contents carry an
// older epoch (zeroed memory: 0, which no epoch takes).
__device__ __forceinline__ void ll_store(uint4 *p, uint32_t w0, uint32_t w1, uint32_t e) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(w0), "r"(e), "r"(w1), "r"(e) : "memory");
}
__device__ __forceinline__ uint4 ll_peek(const uint4 *p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}
// False: the pair did not arrive within the limit (recorded in the status word).  Once the status word is set,
// nothing spins again.
__device__ __forceinline__ bool ll_load(const uint4 *p, uint32_t e, uint32_t &w0, uint32_t &w1, int *status, long long limit) {
    for (long long i = 0;; i++) {
        uint32_t a, b, c, d;
        asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "l"(p) : "memory");
        if (b == e && d == e) {
            w0 = a;
            w1 = c;
            return true;
        }
        if (i >= limit || (i == 0 && *reinterpret_cast<volatile int *>(status) != 0)) break;
        __nanosleep(40);
    }
    atomicCAS(status, 0, FINCH_E_TIMEOUT);
    w0 = w1 = 0u;
    return false;
}

// grid (T, world), 128 threads: record of token t -> rank d's area (d == rank: my own; the rank's tokens take the same route)
__global__ void __launch_bounds__(128) peer_dispatch_kernel(Areas areas, int rank, int T, const uint8_t *x, const int32_t *ids, const float *weights,
                                                            const uint8_t *valid, int row_bytes, int K, int rec_bytes, const uint32_t *epoch) {
    __shared__ __align__(16) uint32_t tail[32];      // ids, weights, mask bytes, padding: the part of the record after the row
    const int t = blockIdx.x, d = blockIdx.y;
    dep_wait();        // the activations are the work of what ran before (and the epoch that of the previous layer's combine)
    const uint32_t e = *epoch;
    dep_launch();
    if (threadIdx.x < 32) tail[threadIdx.x] = 0u;
    __syncthreads();
    if (threadIdx.x < K) {
        const int k = threadIdx.x;
        tail[k] = (uint32_t)ids[t * K + k];
        tail[K + k] = __float_as_uint(weights[t * K + k]);
        reinterpret_cast<uint8_t *>(tail + 2 * K)[k] = valid ? valid[t * K + k] : (uint8_t)1;
    }
    __syncthreads();
    uint4 *dst = reinterpret_cast<uint4 *>(areas.p[d]) + (size_t)(rank * T + t) * (rec_bytes / 8);
    const uint2 *row = reinterpret_cast<const uint2 *>(x + (size_t)t * row_bytes);
    for (int q = threadIdx.x; q < rec_bytes / 8; q += blockDim.x) {
        uint2 w;
        if (q < row_bytes / 8) w = row[q];
        else w = make_uint2(tail[2 * (q - row_bytes / 8)], tail[2 * (q - row_bytes / 8) + 1]);
        ll_store(dst + q, w.x, w.y, e);
    }
}

// grid world * T, 128 threads, rec_bytes of dynamic shared memory: slot i = [source][t] of my area -> row i of the arrays
__global__ void __launch_bounds__(128) peer_receive_kernel(const uint8_t *area, int rank, int T, int row_bytes, int K, int rec_bytes, uint8_t *x, int32_t *ids,
                                                           float *weights, uint8_t *valid, int *status, long long limit, int mask_own, const uint32_t *epoch) {
    extern __shared__ __align__(16) uint32_t srec[];
    const int i = blockIdx.x, src_rank = i / T;
    const bool masked = mask_own && src_rank == rank;   // my own tokens are served in place by the caller: their rows select nothing
    const uint32_t e = *epoch;
    dep_launch();
    // The records are ordered by the epochs they carry, and the row arrays were last read by kernels that completed
    // before the dispatch kernel passed its wait (which is before this grid could start): no wait up front.
    const uint4 *src = reinterpret_cast<const uint4 *>(area) + (size_t)i * (rec_bytes / 8);
    int bad = 0;
    // a thread's word pairs are requested together; those that have not arrived yet are then waited for one by one
    constexpr int RQ = 10;      // 128 threads x 10 pairs x 8 payload bytes covers a record of 10 KB
    uint4 v[RQ];
#pragma unroll
    for (int r = 0; r < RQ; r++) {
        const int q = threadIdx.x + r * 128;
        if (q < rec_bytes / 8) v[r] = ll_peek(src + q);
    }
#pragma unroll
    for (int r = 0; r < RQ; r++) {
        const int q = threadIdx.x + r * 128;
        if (q < rec_bytes / 8) {
            uint32_t w0 = v[r].x, w1 = v[r].z;
            if (v[r].y != e || v[r].w != e)
                if (!ll_load(src + q, e, w0, w1, status, limit)) bad = 1;
            srec[2 * q] = w0;
            srec[2 * q + 1] = w1;
        }
    }
    for (int q = threadIdx.x + RQ * 128; q < rec_bytes / 8; q += blockDim.x) {     // longer records: the plain loop
        uint32_t w0, w1;
        if (!ll_load(src + q, e, w0, w1, status, limit)) bad = 1;
        srec[2 * q] = w0;
        srec[2 * q + 1] = w1;
    }
    bad = __syncthreads_or(bad);
    if (bad) {          // incomplete: the row selects nothing
        if (threadIdx.x < K) valid[i * K + threadIdx.x] = 0;
        dep_wait();
        return;
    }
    const uint4 *s4 = reinterpret_cast<const uint4 *>(srec);
    uint4 *dst = reinterpret_cast<uint4 *>(x + (size_t)i * row_bytes);
    for (int j = threadIdx.x; j < row_bytes / 16; j += blockDim.x) dst[j] = s4[j];
    if (threadIdx.x < K) {
        const int k = threadIdx.x;
        const uint32_t *tail = srec + row_bytes / 4;
        ids[i * K + k] = (int32_t)tail[k];
        weights[i * K + k] = __uint_as_float(tail[K + k]);
        valid[i * K + k] = masked ? (uint8_t)0 : reinterpret_cast<const uint8_t *>(tail + 2 * K)[k];
    }
    dep_wait();
}

// grid (T, world), 256 threads: partial row of source s's token t -> rank s's area
__global__ void __launch_bounds__(256) peer_return_kernel(Areas areas, int rank, int T, const float *rows, int hidden, size_t off_back, const uint32_t *epoch) {
    const int t = blockIdx.x, s = blockIdx.y;
    dep_wait();        // the rows are the predecessor's output
    const uint32_t e = *epoch;
    dep_launch();
    if (s == rank) return;
    const uint2 *src = reinterpret_cast<const uint2 *>(rows + (size_t)(s * T + t) * hidden);
    uint4 *dst = reinterpret_cast<uint4 *>(areas.p[s] + off_back) + (size_t)(rank * T + t) * (hidden / 2);
    for (int q = threadIdx.x; q < hidden / 2; q += blockDim.x) {
        const uint2 w = src[q];
        ll_store(dst + q, w.x, w.y, e);
    }
}

// grid (T, hidden / 512), 256 threads, a thread per pair of outputs: hidden_out[t] += partial rows of ranks
// 0 .. world - 1 (not mine), ascending; the last CTA to finish advances the epoch.
__global__ void __launch_bounds__(256) peer_combine_kernel(const uint8_t *area, int rank, int world, int T, float *hidden_out, int hidden, size_t off_back,
                                                           int *status, long long limit, uint32_t *epoch, unsigned *ticket) {
    const int t = blockIdx.x, q = blockIdx.y * 256 + threadIdx.x;
    const uint32_t e = *epoch;
    dep_launch();
    // The peers' rows are ordered by the epochs they carry: they are requested before anything else.  hidden_out is
    // the work of the kernel before this one (the decode pass that also returned the other ranks' rows): it is read
    // only after the wait.
    const bool mine = q < hidden / 2;
    const uint4 *back = reinterpret_cast<const uint4 *>(area + off_back) + (size_t)t * (hidden / 2) + q;
    const size_t dstride = (size_t)T * (hidden / 2);
    uint4 v[MAXW];
    if (mine) {
#pragma unroll
        for (int d = 0; d < MAXW; d++)
            if (d < world && d != rank) v[d] = ll_peek(back + d * dstride);      // all peers' words requested together
    }
    dep_wait();
    if (mine) {
        float2 *out = reinterpret_cast<float2 *>(hidden_out + (size_t)t * hidden) + q;
        float2 h = *out;
#pragma unroll
        for (int d = 0; d < MAXW; d++)
            if (d < world && d != rank) {
                uint32_t w0 = v[d].x, w1 = v[d].z;
                if (v[d].y != e || v[d].w != e) ll_load(back + d * dstride, e, w0, w1, status, limit);
                h.x += __uint_as_float(w0);
                h.y += __uint_as_float(w1);
            }
        *out = h;
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(ticket, 1u) == gridDim.x * gridDim.y - 1) {
        *ticket = 0u;
        *epoch = e + 1u == 0u ? 1u : e + 1u;
        __threadfence();
    }
}

template <typename... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), dim3 grid, int threads, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

Areas areas_of(const finch_ep_peer *p) {
    Areas a{};
    for (int r = 0; r < p->world; r++) a.p[r] = p->remote[r];
    return a;
}

int connected(finch_ep_peer *p) {
    for (int r = 0; r < p->world; r++)
        if (!p->remote[r]) return finch_fail(p->ctx, FINCH_E_ARG, "rank %d's receive area has not been imported", r);
    return FINCH_OK;
}

}  // namespace

extern "C" int finch_ep_peer_create(finch_ctx *ctx, int rank, int world, int tokens_per_rank, finch_ep_peer **out) {
    if (!ctx || !out || world < 1 || world > MAXW || rank < 0 || rank >= world || tokens_per_rank < 1) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    if (c.n_experts % world) return finch_fail(ctx, FINCH_E_ARG, "%d experts do not split over %d ranks", c.n_experts, world);
    if (c.hidden % 4) return finch_fail(ctx, FINCH_E_ARG, "hidden must be a multiple of 4");
    cudaSetDevice(c.device);
    finch_ep_peer *p = new finch_ep_peer();
    p->ctx = ctx;
    p->rank = rank;
    p->world = world;
    p->T = tokens_per_rank;
    const int elt = c.act_dtype == FINCH_BF16 ? 2 : 4;
    const size_t slots = (size_t)world * tokens_per_rank;
    p->off_back = up256(slots * 2 * rec_bytes_of(c.hidden, elt, c.top_k));
    p->bytes = p->off_back + up256(slots * 2 * c.hidden * 4);
    if (cudaMalloc(&p->area, p->bytes) != cudaSuccess || cudaMalloc(&p->sync, 2 * sizeof(uint32_t)) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p->area);
        const size_t bytes = p->bytes;
        delete p;
        return finch_fail(ctx, FINCH_E_NOMEM, "peer receive area (%zu bytes)", bytes);
    }
    cudaMemset(p->area, 0, p->bytes);
    const uint32_t init[2] = {1u, 0u};          // epochs start at 1: zeroed slots match none
    cudaMemcpy(p->sync, init, sizeof(init), cudaMemcpyHostToDevice);
    cudaDeviceSynchronize();
    p->remote[rank] = p->area;
    *out = p;
    return FINCH_OK;
}

extern "C" int finch_ep_peer_export(finch_ep_peer *p, void *handle64) {
    if (!p || !handle64) return FINCH_E_ARG;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "handle size");
    cudaIpcMemHandle_t h;
    cudaSetDevice(p->ctx->cfg.device);
    FINCH_CUDA_OK(p->ctx, cudaIpcGetMemHandle(&h, p->area));
    memcpy(handle64, &h, 64);
    return FINCH_OK;
}

extern "C" int finch_ep_peer_import(finch_ep_peer *p, int src_rank, const void *handle64) {
    if (!p || !handle64 || src_rank < 0 || src_rank >= p->world) return FINCH_E_ARG;
    if (src_rank == p->rank) return FINCH_OK;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, 64);
    void *ptr = nullptr;
    cudaSetDevice(p->ctx->cfg.device);
    FINCH_CUDA_OK(p->ctx, cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    p->remote[src_rank] = (uint8_t *)ptr;
    p->opened[src_rank] = true;
    return FINCH_OK;
}

extern "C" void *finch_ep_peer_area(finch_ep_peer *p) { return p ? p->area : nullptr; }

extern "C" int finch_ep_peer_attach(finch_ep_peer *p, int src_rank, void *area) {
    if (!p || !area || src_rank < 0 || src_rank >= p->world || src_rank == p->rank) return FINCH_E_ARG;
    p->remote[src_rank] = (uint8_t *)area;
    p->opened[src_rank] = false;
    return FINCH_OK;
}

extern "C" int finch_ep_peer_set_wait_limit(finch_ep_peer *p, long long polls) {
    if (!p || polls < 1) return FINCH_E_ARG;
    p->limit = polls;
    return FINCH_OK;
}

extern "C" int finch_ep_peer_reset(finch_ep_peer *p) {
    if (!p) return FINCH_E_ARG;
    cudaSetDevice(p->ctx->cfg.device);
    FINCH_CUDA_OK(p->ctx, cudaDeviceSynchronize());
    FINCH_CUDA_OK(p->ctx, cudaMemset(p->area, 0, p->bytes));
    const uint32_t init[2] = {1u, 0u};
    FINCH_CUDA_OK(p->ctx, cudaMemcpy(p->sync, init, sizeof(init), cudaMemcpyHostToDevice));
    FINCH_CUDA_OK(p->ctx, cudaDeviceSynchronize());
    return FINCH_OK;
}

extern "C" int finch_ep_peer_destroy(finch_ep_peer *p) {
    if (!p) return FINCH_E_ARG;
    cudaSetDevice(p->ctx->cfg.device);
    cudaDeviceSynchronize();
    for (int r = 0; r < p->world; r++)
        if (p->opened[r]) cudaIpcCloseMemHandle(p->remote[r]);
    cudaFree(p->area);
    cudaFree(p->sync);
    delete p;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_peer_dispatch(finch_ctx *ctx, finch_stream stream, finch_ep_peer *p, const void *h_post, const int32_t *expert_ids,
                                             const float *weights, const uint8_t *valid) {
    if (!ctx || !p || p->ctx != ctx || !h_post || !expert_ids || !weights) return FINCH_E_ARG;
    int rc = connected(p);
    if (rc) return rc;
    const finch_config &c = ctx->cfg;
    const int elt = c.act_dtype == FINCH_BF16 ? 2 : 4, row_bytes = c.hidden * elt;
    if (row_bytes % 16) return finch_fail(ctx, FINCH_E_ARG, "activation rows must be multiples of 16 bytes");
    cudaSetDevice(c.device);
    FINCH_CUDA_OK(ctx, launch_pdl(peer_dispatch_kernel, dim3(p->T, p->world), 128, 0, finch_pick_stream(ctx, stream), areas_of(p), p->rank, p->T,
                                  (const uint8_t *)h_post, expert_ids, weights, valid, row_bytes, c.top_k, rec_bytes_of(c.hidden, elt, c.top_k),
                                  (const uint32_t *)p->sync));
    ctx->launches++;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_peer_receive(finch_ctx *ctx, finch_stream stream, finch_ep_peer *p, void *h_post, int32_t *expert_ids, float *weights,
                                            uint8_t *valid, int mask_own) {
    if (!ctx || !p || p->ctx != ctx || !h_post || !expert_ids || !weights || !valid) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    const int elt = c.act_dtype == FINCH_BF16 ? 2 : 4;
    cudaSetDevice(c.device);
    const int rec = rec_bytes_of(c.hidden, elt, c.top_k);
    FINCH_CUDA_OK(ctx, launch_pdl(peer_receive_kernel, dim3(p->world * p->T), 128, (size_t)rec, finch_pick_stream(ctx, stream), (const uint8_t *)p->area, p->rank,
                                  p->T, c.hidden * elt, c.top_k, rec, (uint8_t *)h_post, expert_ids, weights, valid, ctx->dev_status, p->limit, mask_own,
                                  (const uint32_t *)p->sync));
    ctx->launches++;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_peer_return(finch_ctx *ctx, finch_stream stream, finch_ep_peer *p, const float *rows) {
    if (!ctx || !p || p->ctx != ctx || !rows) return FINCH_E_ARG;
    int rc = connected(p);
    if (rc) return rc;
    if (p->world == 1) return FINCH_OK;
    cudaSetDevice(ctx->cfg.device);
    FINCH_CUDA_OK(ctx, launch_pdl(peer_return_kernel, dim3(p->T, p->world), 256, 0, finch_pick_stream(ctx, stream), areas_of(p), p->rank, p->T, rows,
                                  ctx->cfg.hidden, p->off_back, (const uint32_t *)p->sync));
    ctx->launches++;
    return FINCH_OK;
}

// One launch sequence for the whole layer on this rank: batch c = the T rows received from rank c (the receive step's
// arrays), of which the experts held here are computed; the rank's own batch also gets h_mid and the shared expert and
// lands in hidden_out, and the combine kernel of the decode path stores the other batches' rows straight into their
// ranks' partial-row slots (the return step, without a kernel of its own).  Then: finch_encode_ep_peer_combine.
extern "C" int finch_encode_ep_peer_decode(finch_ctx *ctx, finch_stream stream, finch_ep_peer *p, finch_pool *pool, int layer, const void *rows_x,
                                           const int32_t *rows_ids, const float *rows_weights, const uint8_t *rows_valid, const finch_shared *shared,
                                           const float *h_mid, float *hidden_out) {
    if (!ctx || !p || p->ctx != ctx || !pool || !rows_x || !rows_ids || !rows_weights || !hidden_out) return FINCH_E_ARG;
    int rc = connected(p);
    if (rc) return rc;
    finch_ret_info ret{};
    for (int r = 0; r < p->world; r++) ret.area[r] = p->remote[r];
    ret.off_back = p->off_back;
    ret.rank = p->rank;
    ret.T = p->T;
    ret.epoch = p->sync;
    return finch_encode_moe_decode_multi_ret(ctx, stream, pool, layer, p->world, p->T, rows_x, rows_ids, rows_weights, rows_valid, p->rank, shared, h_mid,
                                             hidden_out, &ret);
}

extern "C" int finch_encode_ep_peer_combine(finch_ctx *ctx, finch_stream stream, finch_ep_peer *p, float *hidden_out) {
    if (!ctx || !p || p->ctx != ctx || !hidden_out) return FINCH_E_ARG;
    // with one rank there is nothing to add, but the kernel still closes the layer: it advances the epoch
    cudaSetDevice(ctx->cfg.device);
    FINCH_CUDA_OK(ctx, launch_pdl(peer_combine_kernel, dim3(p->T, (ctx->cfg.hidden / 2 + 255) / 256), 256, 0, finch_pick_stream(ctx, stream), (const uint8_t *)p->area, p->rank, p->world, p->T,
                                  hidden_out, ctx->cfg.hidden, p->off_back, ctx->dev_status, p->limit, p->sync, (unsigned *)(p->sync + 1)));
    ctx->launches++;
    return FINCH_OK;
}
