// Chunked-prefill MoE entry point (prefill_chunk_cmd3 / _batch_general,
// finchmoe/infer.m:10704-11241) and the dense 4-bit projection GEMM
// (gpu_encode_prefill_matvec, infer.m:3672).
//
// Paths (finch_set_prefill_mode; by default chosen by chunk length):
//  * tensor-core paths (chunks of 80 tokens and more, or on request): the (token, k) pairs are sorted by expert and
//    the routed experts run as one of
//      - grouped mma.sync passes (moe_decode.cu, the default): a unit of codes is unpacked once for up to 16
//        tokens of its expert, same arithmetic as the decode kernels;
//      - two grouped dequant-GEMMs on tcgen05 (dqgemm_tc.cuh): gate/up with SiLU(gate)*up in the epilogue
//        (activation stored as two bf16 planes, value and remainder, about 16 bits together), then down -- both
//        planes against the same weight tile -- into one fp32 row per pair;
//      - two grouped tcgen05 GEMMs that take the packed codes themselves as the A operand (umma3.cuh);
//    the shared expert is three dense 4-bit GEMMs (dqgemm_tc.cuh) on a second stream; a last kernel applies the
//    router weights in ascending k, the shared gate and the residual (moe_combine_residual_prefill,
//    finchmoe/shaders.metal:2764-2802).  Every selected expert is read from HBM once per chunk of 512.
//  * sub-batch path (short chunks, or on request): groups of at most eight tokens go through the
//    decode kernels (moe_decode.cu) -- the reference's own scheme, per-position dispatch of the decode
//    kernels with expert de-duplication inside a group (infer.m:12424-12532).  Every output row is then
//    bit-identical to the decode entry point's, the property the reference claims (README.md:25).
//
// The dequantising path carries every operand as a bf16 value plus a bf16 remainder (16 significant bits:
// the dequantised weights, fp32 activations, SiLU(gate)*up; bf16 activations are exact as they are) and
// accumulates in fp32, so it agrees with the reference's arithmetic (exact fp32 weights and activations)
// to about 1e-5 of an output's scale; the other two multiply exact operands.  The parity tests hold all of
// them to the same bar as the decode path.
#include "dqgemm_tc.cuh"
#include "umma3.cuh"

// the grouped 3-bit passes on mma.sync (moe_decode.cu)
size_t finch_group3_ws_bytes(finch_ctx *ctx, int T);
int finch_group3_prefill(finch_ctx *ctx, cudaStream_t st, finch_pool *pool, int layer, const void *x, const int32_t *ids, const uint8_t *valid, int T, void *ws,
                         float *down_out);

namespace {

constexpr int CHUNK = 512;   // default tokens per tensor-core pass: 4096 pairs (finch_set_prefill_chunk changes it)
constexpr int TC_MIN_TOKENS = 80;    // shorter chunks are faster through the decode kernels (measured: 64 tokens 261 vs 299 us, 128 tokens 521 vs 327)

// One CTA: pairs -> expert histogram -> ranges -> order.  Pairs that are masked, out of range or not
// resident are left out (their rows are never produced and never combined).
// It also lists the (expert, first token) tiles of the two grouped GEMMs, tn_a / tn_b tokens per tile, so
// that their grids hold no CTA without work: items_a / items_b = [expert, first pair of the tile inside
// the expert's range], n_items[0 / 1] = how many.
// cap_a / cap_b: the most tiles the two GEMM grids were sized for (pairs / tile + experts resident when the call
// was encoded); more than that -- experts added to the pool between encode and execution -- is reported
// through status and the lists are cut there.
__global__ void __launch_bounds__(1024) pf_sort_kernel(const int32_t *ids, const uint8_t *valid, const int32_t *slot_row, int n_experts, int P,
                                                       int *seg, int *order, int tn_a, int tn_b, int2 *items_a, int2 *items_b, int *n_items,
                                                       int cap_a, int cap_b, int *status) {
    extern __shared__ int sm[];   // [n_experts] counts, cursors, first item of the expert in each list
    int *cnt = sm, *cur = sm + n_experts, *ia = cur + n_experts, *ib = ia + n_experts;
    const int tid = threadIdx.x;
    for (int e = tid; e < n_experts; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) {
        const int e = ids[p];
        if ((valid && !valid[p]) || e < 0 || e >= n_experts || slot_row[e] < 0) continue;
        atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    // exclusive scans over the experts (one thread each, n_experts <= 1024): pairs, tiles of each GEMM
    {
        __shared__ int wsum[3][32];
        const int lane = tid & 31, wid = tid >> 5;
        const int c0 = tid < n_experts ? cnt[tid] : 0;
        int v[3] = {c0, (c0 + tn_a - 1) / tn_a, (c0 + tn_b - 1) / tn_b}, inc[3];
#pragma unroll
        for (int q = 0; q < 3; q++) {
            inc[q] = v[q];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, inc[q], o);
                if (lane >= o) inc[q] += t;
            }
            if (lane == 31) wsum[q][wid] = inc[q];
        }
        __syncthreads();
        if (wid == 0) {
#pragma unroll
            for (int q = 0; q < 3; q++) {
                const int w = wsum[q][lane];
                int acc = w;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, acc, o);
                    if (lane >= o) acc += t;
                }
                wsum[q][lane] = acc - w;   // exclusive prefix of the warp totals
                if (lane == 31) {
                    if (q == 0) seg[n_experts] = acc;
                    else {
                        const int cap = q == 1 ? cap_a : cap_b;
                        if (acc > cap) atomicCAS(status, 0, FINCH_E_UNSUPPORTED);
                        n_items[q - 1] = acc < cap ? acc : cap;
                    }
                }
            }
        }
        __syncthreads();
        if (tid < n_experts) {
            const int e = tid;
            seg[e] = cur[e] = wsum[0][wid] + inc[0] - v[0];
            ia[e] = wsum[1][wid] + inc[1] - v[1];
            ib[e] = wsum[2][wid] + inc[2] - v[2];
        }
    }
    __syncthreads();
    for (int e = tid; e < n_experts; e += blockDim.x) {
        for (int i = 0, t0 = 0; t0 < cnt[e]; i++, t0 += tn_a)
            if (ia[e] + i < cap_a) items_a[ia[e] + i] = make_int2(e, t0);
        for (int i = 0, t0 = 0; t0 < cnt[e]; i++, t0 += tn_b)
            if (ib[e] + i < cap_b) items_b[ib[e] + i] = make_int2(e, t0);
    }
    // the order of the pairs inside an expert's range is arbitrary: every pair's output row is computed
    // from its own activation row only, so the results do not depend on it
    for (int p = tid; p < P; p += blockDim.x) {
        const int e = ids[p];
        if ((valid && !valid[p]) || e < 0 || e >= n_experts || slot_row[e] < 0) continue;
        order[atomicAdd(&cur[e], 1)] = p;
    }
}

// fp32 activations -> two bf16 planes: the value rounded to bf16 and the bf16-rounded remainder
__global__ void pf_to_bf16_kernel(const float *src, uint16_t *dst, uint16_t *dst_lo, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n / 2; i += (size_t)gridDim.x * blockDim.x) {
        uint32_t h, r;
        dqgemm::bf16x2_split(src[2 * i], src[2 * i + 1], h, r);
        reinterpret_cast<uint32_t *>(dst)[i] = h;
        reinterpret_cast<uint32_t *>(dst_lo)[i] = r;
    }
}

// act = SiLU(g) * u, stored as two bf16 planes: the value rounded to bf16 and the remainder (shared expert)
__global__ void pf_swiglu_kernel(const float *g, const float *u, uint16_t *act, uint16_t *act_lo, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float gv = g[i], v = (gv / (1.0f + expf(-gv))) * u[i];
        const uint32_t hi = dqgemm::bf16x2_rn(v, 0.f) & 0xffffu;
        act[i] = (uint16_t)hi;
        act_lo[i] = (uint16_t)(dqgemm::bf16x2_rn(v - __uint_as_float(hi << 16), 0.f) & 0xffffu);
    }
}

// hidden[t] = h_mid[t] + sum_{k ascending, usable} w[t][k] * down[t*K + k] + sigmoid(score[t]) * shared[t]
__global__ void __launch_bounds__(256) pf_combine_kernel(const int32_t *ids, const uint8_t *valid, const int32_t *slot_row, int n_experts,
                                                         const float *weights, int K, const float *down, const float *shared_out,
                                                         const float *gate_score, const float *h_mid, float *hidden_out, int hidden) {
    __shared__ int ok[8];
    __shared__ float wk[8];
    const int t = blockIdx.y, row = blockIdx.x * 256 + threadIdx.x;
    if (threadIdx.x < K) {
        const int p = t * K + threadIdx.x, e = ids[p];
        ok[threadIdx.x] = !(valid && !valid[p]) && e >= 0 && e < n_experts && slot_row[e] >= 0;
        wk[threadIdx.x] = weights[p];
    }
    __syncthreads();
    if (row >= hidden) return;
    float moe = 0.f;
    for (int k = 0; k < K; k++)
        if (ok[k]) moe = fmaf(wk[k], down[(size_t)(t * K + k) * hidden + row], moe);
    float h = h_mid ? h_mid[(size_t)t * hidden + row] : 0.f;
    h += moe;
    if (shared_out) {
        const float sg = 1.0f / (1.0f + expf(-gate_score[t]));
        h = fmaf(sg, shared_out[(size_t)t * hidden + row], h);
    }
    hidden_out[(size_t)t * hidden + row] = h;
}

inline size_t up256(size_t n) { return (n + 255) & ~(size_t)255; }

int tn_max_for(int tokens) {
    int t = (tokens + 15) & ~15;
    return t < 16 ? 16 : (t > 256 ? 256 : t);
}

// The kernel's opt-in to 227 KB of shared memory is a per-device function attribute: set once per device.
int gemm_attr_once(finch_ctx *ctx) {
    static std::mutex mu;
    static std::vector<int> done;
    std::lock_guard<std::mutex> lk(mu);
    for (int d : done)
        if (d == ctx->cfg.device) return FINCH_OK;
    FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(dqgemm::dqgemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(dqgemm::dqgemm_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    done.push_back(ctx->cfg.device);
    return FINCH_OK;
}
int launch_gemm(finch_ctx *ctx, cudaStream_t st, const dqgemm::Args &a, dim3 grid) {
    {
        const int rc = gemm_attr_once(ctx);
        if (rc) return rc;
    }
    const int smem = dqgemm::smem_bytes(a.tn_max, a.X2 ? 2 : 1, a.mode != dqgemm::DENSE4);
    if (smem > 227 * 1024) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "token tile %d needs %d bytes of shared memory", a.tn_max, smem);
    dqgemm::dqgemm_tc_kernel<<<grid, dqgemm::NTB, smem, st>>>(a);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

int dense4_checked(finch_ctx *ctx, const finch_wdesc *w, const char *what) {
    int rc = finch_validate_wdesc(ctx, w, what);
    if (rc) return rc;
    if (w->bits != 4 || w->group_size != 64 || w->in_dim % 128 || w->out_dim % 128)
        return finch_fail(ctx, FINCH_E_UNSUPPORTED, "%s: the tensor-core GEMM takes 4-bit g64 tensors with dims that are multiples of 128", what);
    return FINCH_OK;
}

// out[T][out_dim] (fp32) = X[T][in_dim] (bf16) * dequant(w)^T
int dense4_gemm(finch_ctx *ctx, cudaStream_t st, const finch_wdesc *w, const uint16_t *xb, const uint16_t *xb_lo, float *out, int T) {
    dqgemm::Args a{};
    a.mode = dqgemm::DENSE4;
    a.K = w->in_dim;
    // token tile: small enough that the grid covers the SMs, large enough not to dequantise a tile too often
    a.tn_max = tn_max_for((int)((long long)T * (w->out_dim / dqgemm::GM) / 148));
    if (xb_lo && a.tn_max > 128) a.tn_max = 128;   // two activation planes side by side: 2 x tokens accumulator columns (an MMA takes 256)
    a.X2 = xb_lo;
    a.scale_dtype = w->scale_dtype;
    a.W = (const uint32_t *)w->W;
    a.S = (const uint16_t *)w->scales;
    a.B = (const uint16_t *)w->biases;
    a.rows = w->out_dim;
    a.n_tokens = T;
    a.X = xb;
    a.out = out;
    a.status = ctx->dev_status;
    return launch_gemm(ctx, st, a, dim3(w->out_dim / dqgemm::GM, 1, (T + a.tn_max - 1) / a.tn_max));
}

int ensure_ws(finch_ctx *ctx, size_t bytes, cudaStream_t st) {
    if (ctx->pf_ws_bytes >= bytes) return FINCH_OK;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cap);
    if (cap != cudaStreamCaptureStatusNone)
        return finch_fail(ctx, FINCH_E_UNSUPPORTED, "the prefill workspace must be sized by one call outside stream capture first");
    if (ctx->pf_ws) {
        cudaStreamSynchronize(st);
        cudaFree(ctx->pf_ws);
        ctx->pf_ws = nullptr;
        ctx->pf_ws_bytes = 0;
    }
    if (cudaMalloc(&ctx->pf_ws, bytes) != cudaSuccess) {
        cudaGetLastError();
        return finch_fail(ctx, FINCH_E_NOMEM, "prefill workspace (%zu bytes)", bytes);
    }
    ctx->pf_ws_bytes = bytes;
    return FINCH_OK;
}

int umma_attr_once(finch_ctx *ctx) {
    static std::mutex mu;
    static std::vector<int> done;
    std::lock_guard<std::mutex> lk(mu);
    for (int d : done)
        if (d == ctx->cfg.device) return FINCH_OK;
    FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(umma3::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(umma3::gemm_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    done.push_back(ctx->cfg.device);
    return FINCH_OK;
}

// Which kernels take the routed experts of a chunk.
enum RoutedKind { ROUTED_DEQUANT = 0,   // two tcgen05 GEMMs over weights dequantised to bf16 planes (dqgemm_tc.cuh)
                  ROUTED_GROUPED = 1,   // grouped mma.sync passes (moe_decode.cu)
                  ROUTED_CODES = 2 };   // two tcgen05 GEMMs over the packed codes themselves (umma3.cuh)

int prefill_tc_chunk(finch_ctx *ctx, cudaStream_t st, finch_pool *pool, int layer, const void *h_post, const int32_t *ids,
                     const float *weights, const uint8_t *valid, const finch_shared *shared, const float *h_mid, float *hidden_out, int T, int kind) {
    const bool grouped = kind == ROUTED_GROUPED;
    const finch_config &c = ctx->cfg;
    const int P = T * c.top_k, H = c.hidden, I = c.moe_inter, Is = shared ? shared->gate.out_dim : 0;
    const int32_t *slot_row = pool->slot_table_dev + (size_t)layer * pool->n_experts;
    // workspace carve
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t r = off;
        off += up256(bytes);
        return r;
    };
    const size_t o_seg = take((c.n_experts + 1) * sizeof(int)), o_order = take((size_t)P * sizeof(int));
    const int max_items = P / 16 + c.n_experts + 1;   // tiles of at least 16 tokens, plus one ragged tile per expert
    const size_t o_ia = take((size_t)max_items * sizeof(int2)), o_ib = take((size_t)max_items * sizeof(int2)), o_ni = take(2 * sizeof(int));
    const size_t o_xb = take((size_t)T * H * 2), o_xl = take((size_t)T * H * 2), o_sg = take((size_t)T * Is * 4), o_su = take((size_t)T * Is * 4), o_sact = take((size_t)T * Is * 4);
    const size_t o_g3 = grouped ? take(finch_group3_ws_bytes(ctx, T)) : 0;
    const bool codes = kind == ROUTED_CODES;
    const int pl_a = c.act_dtype == FINCH_BF16 ? 1 : 2;   // activation columns per token of the gate/up GEMM (the down GEMM's fp32 input: 2)
    const size_t o_ra = codes ? take((size_t)T * (H / 64) * pl_a * umma3::REC) : 0, o_xa = codes ? take((size_t)T * (H / 64) * 4) : 0,
                 o_fa = codes ? take((size_t)T * 4) : 0, o_rb = codes ? take((size_t)P * (I / 64) * 2 * umma3::REC) : 0,
                 o_xsb = codes ? take((size_t)P * (I / 64) * 4) : 0, o_fb = codes ? take((size_t)P * 4) : 0;
    int rc = ensure_ws(ctx, off, st);
    if (rc) return rc;
    char *ws = (char *)ctx->pf_ws;
    int *seg = (int *)(ws + o_seg), *order = (int *)(ws + o_order), *n_items = (int *)(ws + o_ni);
    int2 *items_a = (int2 *)(ws + o_ia), *items_b = (int2 *)(ws + o_ib);
    uint16_t *xb = (uint16_t *)(ws + o_xb), *xl = (uint16_t *)(ws + o_xl), *sact = (uint16_t *)(ws + o_sact), *sact_lo = sact + (size_t)T * Is;
    float *sg = (float *)(ws + o_sg), *su = (float *)(ws + o_su);
    uint16_t *act = (uint16_t *)ctx->act, *act_lo = act + (size_t)P * I;   // two bf16 planes [P][I] inside the fp32-sized buffer
    float *down = ctx->partial, *shared_out = ctx->partial + (size_t)P * H;

    // token tiles: as many tokens as still let two CTAs share an SM (an expert's tile is dequantised once per token tile)
    const bool x_lo_needed = c.act_dtype != FINCH_BF16;   // fp32 activations travel as two bf16 planes
    if (grouped) {
        const uint16_t *x = (const uint16_t *)h_post, *x_lo = nullptr;
        if (x_lo_needed && shared) {
            pf_to_bf16_kernel<<<148, 256, 0, st>>>((const float *)h_post, xb, xl, (size_t)T * H);
            FINCH_CUDA_OK(ctx, cudaGetLastError());
            x = xb;
            x_lo = xl;
            ctx->launches++;
        }
        // The shared expert (three small dense GEMMs, each bounded by the latency of its K loop) runs on a second stream
        // beside the routed experts' passes and joins before the combine; both branches only read the inputs.
        cudaStream_t ss = st;
        if (shared) {
            ss = ctx->side;
            FINCH_CUDA_OK(ctx, cudaEventRecord(ctx->ev_fork, st));
            FINCH_CUDA_OK(ctx, cudaStreamWaitEvent(ss, ctx->ev_fork, 0));
            if ((rc = dense4_gemm(ctx, ss, &shared->gate, x, x_lo, sg, T))) return rc;
            if ((rc = dense4_gemm(ctx, ss, &shared->up, x, x_lo, su, T))) return rc;
            pf_swiglu_kernel<<<148, 256, 0, ss>>>(sg, su, sact, sact_lo, (size_t)T * Is);
            FINCH_CUDA_OK(ctx, cudaGetLastError());
            if ((rc = dense4_gemm(ctx, ss, &shared->down, sact, sact_lo, shared_out, T))) return rc;
            FINCH_CUDA_OK(ctx, cudaEventRecord(ctx->ev_join, ss));
            ctx->launches++;
        }
        if ((rc = finch_group3_prefill(ctx, st, pool, layer, h_post, ids, valid, T, ws + o_g3, down))) return rc;
        if (shared) FINCH_CUDA_OK(ctx, cudaStreamWaitEvent(st, ctx->ev_join, 0));
        pf_combine_kernel<<<dim3((H + 255) / 256, T), 256, 0, st>>>(ids, valid, slot_row, c.n_experts, weights, c.top_k, down, shared ? shared_out : nullptr,
                                                                    shared ? shared->gate_score : nullptr, h_mid, hidden_out, H);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        ctx->launches++;
        return FINCH_OK;
    }
    if (codes) {
        if ((rc = umma_attr_once(ctx))) return rc;
        int resident = 0;
        for (int e = 0; e < pool->n_experts; e++) resident += pool->slot_of[(size_t)layer * pool->n_experts + e] >= 0;
        const int tn_ga = umma3::tokens_per_cta(pl_a), tn_dn = umma3::tokens_per_cta(2);
        const int cap = P / tn_dn + resident + 1;
        pf_sort_kernel<<<1, 1024, 4 * c.n_experts * sizeof(int), st>>>(ids, valid, slot_row, c.n_experts, P, seg, order, tn_ga, tn_dn, items_a, items_b,
                                                                       n_items, cap, cap, ctx->dev_status);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        const uint16_t *x = (const uint16_t *)h_post, *x_lo = nullptr;
        if (x_lo_needed && shared) {
            pf_to_bf16_kernel<<<148, 256, 0, st>>>((const float *)h_post, xb, xl, (size_t)T * H);
            FINCH_CUDA_OK(ctx, cudaGetLastError());
            x = xb;
            x_lo = xl;
            ctx->launches++;
        }
        cudaStream_t ss = st;
        if (shared) {   // the shared expert's dense GEMMs beside the routed experts, as in the grouped branch
            ss = ctx->side;
            FINCH_CUDA_OK(ctx, cudaEventRecord(ctx->ev_fork, st));
            FINCH_CUDA_OK(ctx, cudaStreamWaitEvent(ss, ctx->ev_fork, 0));
            if ((rc = dense4_gemm(ctx, ss, &shared->gate, x, x_lo, sg, T))) return rc;
            if ((rc = dense4_gemm(ctx, ss, &shared->up, x, x_lo, su, T))) return rc;
            pf_swiglu_kernel<<<148, 256, 0, ss>>>(sg, su, sact, sact_lo, (size_t)T * Is);
            FINCH_CUDA_OK(ctx, cudaGetLastError());
            if ((rc = dense4_gemm(ctx, ss, &shared->down, sact, sact_lo, shared_out, T))) return rc;
            FINCH_CUDA_OK(ctx, cudaEventRecord(ctx->ev_join, ss));
            ctx->launches++;
        }
        uint8_t *ra = (uint8_t *)(ws + o_ra), *rb = (uint8_t *)(ws + o_rb);
        float *xa = (float *)(ws + o_xa), *fa = (float *)(ws + o_fa), *xsb = (float *)(ws + o_xsb), *fb = (float *)(ws + o_fb);
        if (pl_a == 1) umma3::records_kernel<true, false><<<(T + 7) / 8, 256, 0, st>>>(h_post, T, H, ra, xa, fa);
        else umma3::records_kernel<false, true><<<(T + 7) / 8, 256, 0, st>>>(h_post, T, H, ra, xa, fa);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        umma3::Args u{};
        u.K = H;
        u.planes = pl_a;
        u.scale_dtype = c.scale_dtype;
        u.pool_base = (const uint8_t *)pool->base;
        u.slot_bytes = pool->slot_bytes;
        u.slot_row = slot_row;
        u.hidden = H;
        u.inter = I;
        u.seg = seg;
        u.order = order;
        u.items = items_a;
        u.n_items = n_items;
        u.top_k = c.top_k;
        u.recs = ra;
        u.xsum = xa;
        u.fac = fa;
        u.act_out = ctx->act;
        u.status = ctx->dev_status;
        umma3::gemm_kernel<<<dim3(I / 64, cap), dqgemm::NTB, umma3::smem_bytes(H, pl_a), st>>>(u);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        umma3::records_kernel<false, true><<<(P + 7) / 8, 256, 0, st>>>(ctx->act, P, I, rb, xsb, fb);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        u.down = 1;
        u.K = I;
        u.planes = 2;
        u.items = items_b;
        u.n_items = n_items + 1;
        u.recs = rb;
        u.xsum = xsb;
        u.fac = fb;
        u.out = down;
        umma3::gemm_kernel<<<dim3(H / dqgemm::GM, cap), dqgemm::NTB, umma3::smem_bytes(I, 2), st>>>(u);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        ctx->launches += 5;
        if (shared) FINCH_CUDA_OK(ctx, cudaStreamWaitEvent(st, ctx->ev_join, 0));
        pf_combine_kernel<<<dim3((H + 255) / 256, T), 256, 0, st>>>(ids, valid, slot_row, c.n_experts, weights, c.top_k, down, shared ? shared_out : nullptr,
                                                                    shared ? shared->gate_score : nullptr, h_mid, hidden_out, H);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        ctx->launches++;
        return FINCH_OK;
    }
    const int tn_a = tn_max_for(T < 64 ? T : (x_lo_needed ? 32 : 64)), tn_b = 32;
    // the grids of the two grouped GEMMs hold one CTA row per possible (expert, token tile): at most one ragged tile
    // per expert that is resident now, plus the full tiles
    int resident = 0;
    for (int e = 0; e < pool->n_experts; e++) resident += pool->slot_of[(size_t)layer * pool->n_experts + e] >= 0;
    const int cap_a = P / tn_a + resident + 1, cap_b = P / tn_b + resident + 1;
    pf_sort_kernel<<<1, 1024, 4 * c.n_experts * sizeof(int), st>>>(ids, valid, slot_row, c.n_experts, P, seg, order, tn_a, tn_b, items_a, items_b,
                                                                   n_items, cap_a, cap_b, ctx->dev_status);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    const uint16_t *x = (const uint16_t *)h_post, *x_lo = nullptr;
    if (x_lo_needed) {
        pf_to_bf16_kernel<<<148, 256, 0, st>>>((const float *)h_post, xb, xl, (size_t)T * H);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        x = xb;
        x_lo = xl;
        ctx->launches++;
    }
    ctx->launches++;

    dqgemm::Args a{};
    a.K = H;
    a.tn_max = tn_a;
    a.scale_dtype = c.scale_dtype;
    a.pool_base = (const uint8_t *)pool->base;
    a.slot_bytes = pool->slot_bytes;
    a.slot_row = slot_row;
    a.hidden = H;
    a.inter = I;
    a.seg = seg;
    a.order = order;
    a.top_k = c.top_k;
    a.status = ctx->dev_status;
    a.mode = dqgemm::EXPERT_GATEUP;
    a.X = x;
    a.X2 = x_lo;
    a.act_out = act;
    a.act_out_lo = act_lo;
    a.items = items_a;
    a.n_items = n_items;
    // grid.y bounds the number of (expert, token tile) items; CTAs past the actual count return at once
    if ((rc = launch_gemm(ctx, st, a, dim3(I / 64, cap_a, 1)))) return rc;   // 64 gate + 64 up rows per tile
    a.mode = dqgemm::EXPERT_DOWN;
    a.K = I;
    a.X = act;
    a.X2 = act_lo;
    a.out = down;
    a.tn_max = tn_b;   // two activation planes per stage
    a.items = items_b;
    a.n_items = n_items + 1;
    if ((rc = launch_gemm(ctx, st, a, dim3(H / dqgemm::GM, cap_b, 1)))) return rc;

    if (shared) {
        if ((rc = dense4_gemm(ctx, st, &shared->gate, x, x_lo, sg, T))) return rc;
        if ((rc = dense4_gemm(ctx, st, &shared->up, x, x_lo, su, T))) return rc;
        pf_swiglu_kernel<<<148, 256, 0, st>>>(sg, su, sact, sact_lo, (size_t)T * Is);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        if ((rc = dense4_gemm(ctx, st, &shared->down, sact, sact_lo, shared_out, T))) return rc;
        ctx->launches++;
    }
    pf_combine_kernel<<<dim3((H + 255) / 256, T), 256, 0, st>>>(ids, valid, slot_row, c.n_experts, weights, c.top_k, down,
                                                                shared ? shared_out : nullptr, shared ? shared->gate_score : nullptr, h_mid,
                                                                hidden_out, H);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

}  // namespace

extern "C" int finch_set_prefill_mode(finch_ctx *ctx, int mode) {
    if (!ctx || mode < 0 || mode > 4) return FINCH_E_ARG;
    ctx->prefill_mode = mode;
    return FINCH_OK;
}

extern "C" int finch_set_prefill_chunk(finch_ctx *ctx, int tokens) {
    if (!ctx || tokens < 0) return FINCH_E_ARG;
    if (tokens > ctx->cfg.max_tokens) return finch_fail(ctx, FINCH_E_ARG, "chunk of %d tokens exceeds max_tokens=%d", tokens, ctx->cfg.max_tokens);
    ctx->prefill_chunk = tokens;
    return FINCH_OK;
}

extern "C" int finch_encode_moe_prefill(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, const void *h_post,
                                        const int32_t *expert_ids, const float *weights, const uint8_t *valid,
                                        const finch_shared *shared, const float *h_mid, float *hidden_out, int T) {
    if (!ctx || !pool || !h_post || !expert_ids || !weights || !hidden_out || T < 1) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    const size_t elt = c.act_dtype == FINCH_BF16 ? 2 : 4;
    bool tc = ctx->prefill_mode >= 2 || (ctx->prefill_mode == 0 && T >= TC_MIN_TOKENS);
    // which kernels serve the routed experts of a tensor-core chunk: the grouped mma.sync passes (mode 3) unpack a
    // unit once for up to 16 tokens and win while experts see few tokens; the tcgen05 GEMMs (mode 2) win when a tile
    // of 64 tokens fills (the rows an expert-parallel rank receives).  By chunk length: the former.
    const int kind = ctx->prefill_mode == 4 ? ROUTED_CODES : (ctx->prefill_mode == 3 || ctx->prefill_mode == 0) ? ROUTED_GROUPED : ROUTED_DEQUANT;
    // shapes the tensor-core kernels take: whole 128-row tiles, 128-value K blocks, a 3-bit pool
    if (c.expert_bits != 3 || c.hidden % 128 || c.moe_inter % 128 || c.top_k > 8 || c.n_experts > 1024) tc = false;
    if (tc && shared) {
        if (shared->gate.bits != 4 || shared->gate.out_dim % 128 || shared->gate.in_dim != c.hidden || !shared->gate_score) tc = false;
    }
    if (tc) {
        if (T > c.max_tokens) return finch_fail(ctx, FINCH_E_ARG, "T=%d exceeds max_tokens=%d", T, c.max_tokens);
        if (pool->ctx != ctx) return finch_fail(ctx, FINCH_E_ARG, "pool belongs to another context");
        if (layer < 0 || layer >= pool->n_layers) return finch_fail(ctx, FINCH_E_ARG, "layer %d out of range", layer);
        if (shared) {
            int rc;
            if ((rc = dense4_checked(ctx, &shared->gate, "shared gate")) || (rc = dense4_checked(ctx, &shared->up, "shared up")) ||
                (rc = dense4_checked(ctx, &shared->down, "shared down")))
                return rc;
        }
        cudaSetDevice(c.device);
        cudaStream_t st = finch_pick_stream(ctx, stream);
        const int chunk = ctx->prefill_chunk > 0 ? ctx->prefill_chunk : CHUNK;
        for (int t0 = 0; t0 < T; t0 += chunk) {
            const int n = T - t0 < chunk ? T - t0 : chunk;
            finch_shared sh;
            if (shared) {
                sh = *shared;
                sh.gate_score = shared->gate_score + t0;
            }
            const int rc = prefill_tc_chunk(ctx, st, pool, layer, (const char *)h_post + (size_t)t0 * c.hidden * elt,
                                            expert_ids + (size_t)t0 * c.top_k, weights + (size_t)t0 * c.top_k,
                                            valid ? valid + (size_t)t0 * c.top_k : nullptr, shared ? &sh : nullptr,
                                            h_mid ? h_mid + (size_t)t0 * c.hidden : nullptr, hidden_out + (size_t)t0 * c.hidden, n, kind);
            if (rc) return rc;
        }
        return FINCH_OK;
    }
    int sub = FINCH_MAX_PAIRS / c.top_k;
    if (sub > 8) sub = 8;
    if (sub > c.max_tokens) sub = c.max_tokens;
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

// Dense 4-bit g64 projection for M tokens on the tensor cores: out fp32 [M][out_dim] = x * dequant(w)^T,
// x bf16 [M][in_dim] on the device (gpu_encode_prefill_matvec, finchmoe/infer.m:3672, for M >= 16).
extern "C" int finch_encode_dense_gemm(finch_ctx *ctx, finch_stream stream, const finch_wdesc *w, const void *x_bf16, float *out, int M) {
    if (!ctx || !w || !x_bf16 || !out || M < 1) return FINCH_E_ARG;
    int rc = dense4_checked(ctx, w, "dense GEMM");
    if (rc) return rc;
    cudaSetDevice(ctx->cfg.device);
    return dense4_gemm(ctx, finch_pick_stream(ctx, stream), w, (const uint16_t *)x_bf16, nullptr, out, M);
}
