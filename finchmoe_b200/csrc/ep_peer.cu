// The fixed-capacity exchange of the expert-parallel layer over NVLink peer memory: the ranks' own kernels
// store records and partial rows straight into each other's receive areas, one release flag per slot, and
// the receiving kernels wait for the flags.  No collective library call and no host step per layer, so a
// decode layer is a fixed sequence of launches on one stream (and can sit in a CUDA graph).
//
//   dispatch   every token's record -> slot [my rank][t] of every rank's area (my own included), then its flag
//   receive    wait for the world * T records addressed to me, spread them into the row arrays the MoE entry
//              points take, clear their flags; on request the block of my own tokens is masked out
//   return     the partial rows of source s's tokens -> slot [my rank][t] of rank s's area, then its flag
//   combine    wait for every other rank's partial rows of my tokens, add them to the layer output in
//              ascending rank order, clear their flags
//
// Why one buffer and a 0/1 flag per slot are enough: a rank dispatches layer l + 1 only after its combine
// of layer l, which waited for every peer's return of layer l, which each peer issued after its receive of
// layer l had read and cleared the slots.  The same chain orders the partial-row slots.  All ranks must
// therefore call the four steps in the same order the same number of times.
//
// Every wait is bounded: when a flag does not arrive within the limit the kernel records FINCH_E_TIMEOUT in
// the device status word, treats the slot as empty and returns; once the status word is set no later wait
// spins again.  Plain peer loads and stores only (no multicast objects).
// The reference runs on one device; this extends its per-layer path (finchmoe/infer.m:9597-9741).
#include <cstring>

#include "finch_internal.cuh"

struct finch_ep_peer {
    finch_ctx *ctx = nullptr;
    int rank = 0, world = 0, T = 0;
    size_t bytes = 0, off_rflag = 0, off_back = 0, off_bflag = 0;
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

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) { asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory"); }
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Programmatic dependent launch: a kernel of the chain may be scheduled while its predecessor still runs.  Every
// kernel here executes dep_wait() before it exits, so "my predecessor has completed" holds transitively along the
// stream; a kernel that needs nothing its predecessor wrote does its work first and waits last.
__device__ __forceinline__ void dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// One thread waits for a slot's flag.  False: it did not arrive (recorded), the slot is to be treated as empty.
__device__ bool wait_flag(const uint32_t *flag, int *status, long long limit) {
    if (ld_acquire_sys(flag) == 1u) return true;
    if (*reinterpret_cast<volatile int *>(status) != 0) return false;   // an earlier wait already ran out: do not spin again
    for (long long i = 0; i < limit; i++) {
        __nanosleep(64);
        if (ld_acquire_sys(flag) == 1u) return true;
    }
    atomicCAS(status, 0, FINCH_E_TIMEOUT);
    return false;
}

// grid (T, world), 128 threads: record of token t -> rank d's area
__global__ void __launch_bounds__(128) peer_dispatch_kernel(Areas areas, int rank, int T, const uint8_t *x, const int32_t *ids, const float *weights,
                                                            const uint8_t *valid, int row_bytes, int K, int rec_bytes, size_t off_rflag) {
    const int t = blockIdx.x, d = blockIdx.y;   // d == rank: my own area (the rank's tokens take the same route)
    dep_wait();        // the activations are the work of what ran before
    dep_launch();
    uint8_t *area = areas.p[d];
    uint8_t *rec = area + (size_t)(rank * T + t) * rec_bytes;
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)t * row_bytes);
    uint4 *dst = reinterpret_cast<uint4 *>(rec);
    for (int j = threadIdx.x; j < row_bytes / 16; j += blockDim.x) dst[j] = src[j];
    if (threadIdx.x < K) {
        const int k = threadIdx.x;
        reinterpret_cast<int32_t *>(rec + row_bytes)[k] = ids[t * K + k];
        reinterpret_cast<float *>(rec + row_bytes + 4 * K)[k] = weights[t * K + k];
        rec[row_bytes + 8 * K + k] = valid ? valid[t * K + k] : (uint8_t)1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t *>(area + off_rflag) + rank * T + t, 1u);
    }
}

// grid world * T, 128 threads: slot i = [source][t] of my area -> row i of the arrays
__global__ void __launch_bounds__(128) peer_receive_kernel(uint8_t *area, int rank, int T, int row_bytes, int K, int rec_bytes, size_t off_rflag, uint8_t *x,
                                                           int32_t *ids, float *weights, uint8_t *valid, int *status, long long limit, int mask_own) {
    __shared__ int ok;
    const int i = blockIdx.x, src_rank = i / T;
    const bool masked = mask_own && src_rank == rank;   // my own tokens are served in place by the caller: their rows select nothing
    uint32_t *flag = reinterpret_cast<uint32_t *>(area + off_rflag) + i;
    dep_launch();
    // The records are ordered by their flags, and the row arrays were last read by kernels that completed before the
    // dispatch kernel passed its wait (which is before this grid could start): no wait for the predecessor up front.
    if (threadIdx.x == 0) ok = wait_flag(flag, status, limit) ? 1 : 0;
    __syncthreads();
    if (!ok) {
        if (threadIdx.x < K) valid[i * K + threadIdx.x] = 0;
        dep_wait();
        return;
    }
    const uint8_t *rec = area + (size_t)i * rec_bytes;
    const uint4 *src = reinterpret_cast<const uint4 *>(rec);
    uint4 *dst = reinterpret_cast<uint4 *>(x + (size_t)i * row_bytes);
    for (int j = threadIdx.x; j < row_bytes / 16; j += blockDim.x) dst[j] = src[j];
    if (threadIdx.x < K) {
        const int k = threadIdx.x;
        ids[i * K + k] = reinterpret_cast<const int32_t *>(rec + row_bytes)[k];
        weights[i * K + k] = reinterpret_cast<const float *>(rec + row_bytes + 4 * K)[k];
        valid[i * K + k] = masked ? (uint8_t)0 : rec[row_bytes + 8 * K + k];
    }
    __syncthreads();
    if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t *>(flag) = 0u;
    dep_wait();
}

// grid (T, world), 256 threads: partial row of source s's token t -> rank s's area
__global__ void __launch_bounds__(256) peer_return_kernel(Areas areas, int rank, int T, const float *rows, int hidden, size_t off_back, size_t off_bflag) {
    const int t = blockIdx.x, s = blockIdx.y;
    dep_wait();        // the rows are the predecessor's output
    dep_launch();
    if (s == rank) return;
    uint8_t *area = areas.p[s];
    const float4 *src = reinterpret_cast<const float4 *>(rows + (size_t)(s * T + t) * hidden);
    float4 *dst = reinterpret_cast<float4 *>(area + off_back) + (size_t)(rank * T + t) * (hidden / 4);
    for (int j = threadIdx.x; j < hidden / 4; j += blockDim.x) dst[j] = src[j];
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(reinterpret_cast<uint32_t *>(area + off_bflag) + rank * T + t, 1u);
    }
}

// grid T, 256 threads: hidden_out[t] += partial rows of ranks 0 .. world - 1 (not mine), ascending
__global__ void __launch_bounds__(256) peer_combine_kernel(uint8_t *area, int rank, int world, int T, float *hidden_out, int hidden, size_t off_back,
                                                           size_t off_bflag, int *status, long long limit) {
    __shared__ int ok[MAXW];
    const int t = blockIdx.x;
    uint32_t *flags = reinterpret_cast<uint32_t *>(area + off_bflag);
    dep_launch();
    // hidden_out was written two kernels back; the return kernel in between passed its wait before this grid could
    // start, so that writer has completed.  The peers' rows are ordered by their flags.
    if (threadIdx.x < world) {
        const int d = threadIdx.x;
        ok[d] = d != rank && wait_flag(flags + d * T + t, status, limit);
    }
    __syncthreads();
    const float4 *back = reinterpret_cast<const float4 *>(area + off_back);
    float4 *out = reinterpret_cast<float4 *>(hidden_out + (size_t)t * hidden);
    for (int j = threadIdx.x; j < hidden / 4; j += blockDim.x) {
        float4 h = out[j];
        for (int d = 0; d < world; d++) {
            if (!ok[d]) continue;
            const float4 v = back[(size_t)(d * T + t) * (hidden / 4) + j];
            h.x += v.x;
            h.y += v.y;
            h.z += v.z;
            h.w += v.w;
        }
        out[j] = h;
    }
    __syncthreads();
    if (threadIdx.x < world && ok[threadIdx.x]) *reinterpret_cast<volatile uint32_t *>(flags + threadIdx.x * T + t) = 0u;
    dep_wait();
}

template <typename... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), dim3 grid, int threads, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
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
    p->off_rflag = up256(slots * rec_bytes_of(c.hidden, elt, c.top_k));
    p->off_back = p->off_rflag + up256(slots * 4);
    p->off_bflag = p->off_back + up256(slots * c.hidden * 4);
    p->bytes = p->off_bflag + up256(slots * 4);
    if (cudaMalloc(&p->area, p->bytes) != cudaSuccess) {
        cudaGetLastError();
        delete p;
        return finch_fail(ctx, FINCH_E_NOMEM, "peer receive area (%zu bytes)", p->bytes);
    }
    cudaMemset(p->area, 0, p->bytes);
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
    FINCH_CUDA_OK(p->ctx, cudaMemset(p->area + p->off_rflag, 0, p->off_back - p->off_rflag));
    FINCH_CUDA_OK(p->ctx, cudaMemset(p->area + p->off_bflag, 0, p->bytes - p->off_bflag));
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
    FINCH_CUDA_OK(ctx, launch_pdl(peer_dispatch_kernel, dim3(p->T, p->world), 128, finch_pick_stream(ctx, stream), areas_of(p), p->rank, p->T,
                                  (const uint8_t *)h_post, expert_ids, weights, valid, row_bytes, c.top_k, rec_bytes_of(c.hidden, elt, c.top_k), p->off_rflag));
    ctx->launches++;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_peer_receive(finch_ctx *ctx, finch_stream stream, finch_ep_peer *p, void *h_post, int32_t *expert_ids, float *weights,
                                            uint8_t *valid, int mask_own) {
    if (!ctx || !p || p->ctx != ctx || !h_post || !expert_ids || !weights || !valid) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    const int elt = c.act_dtype == FINCH_BF16 ? 2 : 4;
    cudaSetDevice(c.device);
    FINCH_CUDA_OK(ctx, launch_pdl(peer_receive_kernel, dim3(p->world * p->T), 128, finch_pick_stream(ctx, stream), p->area, p->rank, p->T, c.hidden * elt,
                                  c.top_k, rec_bytes_of(c.hidden, elt, c.top_k), p->off_rflag, (uint8_t *)h_post, expert_ids, weights, valid, ctx->dev_status,
                                  p->limit, mask_own));
    ctx->launches++;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_peer_return(finch_ctx *ctx, finch_stream stream, finch_ep_peer *p, const float *rows) {
    if (!ctx || !p || p->ctx != ctx || !rows) return FINCH_E_ARG;
    int rc = connected(p);
    if (rc) return rc;
    if (p->world == 1) return FINCH_OK;
    cudaSetDevice(ctx->cfg.device);
    FINCH_CUDA_OK(ctx, launch_pdl(peer_return_kernel, dim3(p->T, p->world), 256, finch_pick_stream(ctx, stream), areas_of(p), p->rank, p->T, rows,
                                  ctx->cfg.hidden, p->off_back, p->off_bflag));
    ctx->launches++;
    return FINCH_OK;
}

extern "C" int finch_encode_ep_peer_combine(finch_ctx *ctx, finch_stream stream, finch_ep_peer *p, float *hidden_out) {
    if (!ctx || !p || p->ctx != ctx || !hidden_out) return FINCH_E_ARG;
    if (p->world == 1) return FINCH_OK;
    cudaSetDevice(ctx->cfg.device);
    FINCH_CUDA_OK(ctx, launch_pdl(peer_combine_kernel, dim3(p->T), 256, finch_pick_stream(ctx, stream), p->area, p->rank, p->world, p->T, hidden_out,
                                  ctx->cfg.hidden, p->off_back, p->off_bflag, ctx->dev_status, p->limit));
    ctx->launches++;
    return FINCH_OK;
}
