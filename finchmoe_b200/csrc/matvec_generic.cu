// Format-generic quantized matvec (every bit width of the reference's matvec
// seam), the bit-exact dequant probe and the router tail.
//
// These kernels decode eight consecutive weights at a time with the exact
// two-rounding arithmetic of the reference's CPU path and are the general,
// any-shape implementation behind finch_matvec / finch_encode_batch_matvec.
// The MoE decode path does not use them: it has its own tensor-core kernels
// (moe_decode.cu).
#include "finch_internal.cuh"

int finch_try_fast_matvec(finch_ctx *ctx, cudaStream_t st, const void *x, int x_dtype, const finch_wdesc *specs, float *const *outs, int n, int M);
int finch_try_stream_matvec(finch_ctx *ctx, cudaStream_t st, const void *x, int x_dtype, const finch_wdesc *specs, float *const *outs, int n, int M);
int finch_kq_stream_matvec(finch_ctx *ctx, cudaStream_t st, const finch_wdesc *w, const void *x, int x_dtype, float *out, int M);
int finch_try_gguf_mma(finch_ctx *ctx, cudaStream_t st, const void *x, int x_dtype, const finch_wdesc *specs, float *const *outs, int n, int M);

namespace {

// ---- decoders: eight weights starting at element i0 (multiple of 8) of one row ----
struct RowRef {
    const uint8_t *row;  // packed row
    const uint16_t *s;   // scale row (affine)
    const uint16_t *b;   // bias row (affine)
    int scale_dtype;
};

__device__ __forceinline__ float affine_w(unsigned q, float s, float b) {
    return __fadd_rn(__fmul_rn((float)q, s), b);  // fl32(fl32(q*s)+b): two roundings, no contraction
}

template <int BITS>
__device__ __forceinline__ void decode8(const RowRef &r, int i0, float (&w)[8], uint8_t (&q)[8]);

template <>
__device__ __forceinline__ void decode8<3>(const RowRef &r, int i0, float (&w)[8], uint8_t (&q)[8]) {
    const uint8_t *t = r.row + (i0 >> 3) * 3;
    const uint32_t pk = (uint32_t)t[0] | ((uint32_t)t[1] << 8) | ((uint32_t)t[2] << 16);
    const float s = finch_widen16(r.s[i0 >> 6], r.scale_dtype), b = finch_widen16(r.b[i0 >> 6], r.scale_dtype);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        q[j] = (pk >> (3 * j)) & 7u;
        w[j] = affine_w(q[j], s, b);
    }
}
template <>
__device__ __forceinline__ void decode8<4>(const RowRef &r, int i0, float (&w)[8], uint8_t (&q)[8]) {
    const uint32_t pk = *reinterpret_cast<const uint32_t *>(r.row + (i0 >> 3) * 4);
    const float s = finch_widen16(r.s[i0 >> 6], r.scale_dtype), b = finch_widen16(r.b[i0 >> 6], r.scale_dtype);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        q[j] = (pk >> (4 * j)) & 15u;
        w[j] = affine_w(q[j], s, b);
    }
}
template <>
__device__ __forceinline__ void decode8<8>(const RowRef &r, int i0, float (&w)[8], uint8_t (&q)[8]) {
    const uint2 pk = *reinterpret_cast<const uint2 *>(r.row + i0);
    const float s = finch_widen16(r.s[i0 >> 6], r.scale_dtype), b = finch_widen16(r.b[i0 >> 6], r.scale_dtype);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        q[j] = ((j < 4 ? pk.x : pk.y) >> (8 * (j & 3))) & 255u;
        w[j] = affine_w(q[j], s, b);
    }
}
template <>
__device__ __forceinline__ void decode8<0>(const RowRef &r, int i0, float (&w)[8], uint8_t (&q)[8]) {
    const uint4 v = *reinterpret_cast<const uint4 *>(r.row + (size_t)i0 * 2);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        w[2 * j] = __uint_as_float(u[j] << 16);
        w[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
        q[2 * j] = q[2 * j + 1] = 0;
    }
}
__device__ __forceinline__ float ld_half(const uint8_t *p) {
    return __half2float(__ushort_as_half((uint16_t)(p[0] | (p[1] << 8))));
}
// GGUF Q4_K: 144-byte block = d, dmin (fp16), 12 bytes of 6-bit (scale, min) x 8, 128 nibble bytes.
template <>
__device__ __forceinline__ void decode8<10>(const RowRef &r, int i0, float (&w)[8], uint8_t (&q)[8]) {
    const uint8_t *blk = r.row + (size_t)(i0 >> 8) * 144;
    const int within = i0 & 255, c = within >> 6, hi = (within >> 5) & 1, l0 = within & 31;
    const float d = ld_half(blk), dmin = ld_half(blk + 2);
    const uint8_t *sc12 = blk + 4;
    const int j = 2 * c + hi;
    unsigned sc, mn;
    if (j < 4) {
        sc = sc12[j] & 63u;
        mn = sc12[j + 4] & 63u;
    } else {
        sc = (sc12[j + 4] & 0x0fu) | ((unsigned)(sc12[j - 4] >> 6) << 4);
        mn = (sc12[j + 4] >> 4) | ((unsigned)(sc12[j] >> 6) << 4);
    }
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)mn);
    const uint2 qs = *reinterpret_cast<const uint2 *>(blk + 16 + 32 * c + l0);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const unsigned byte = ((k < 4 ? qs.x : qs.y) >> (8 * (k & 3))) & 255u;
        q[k] = hi ? (byte >> 4) : (byte & 15u);
        w[k] = __fsub_rn(__fmul_rn(d1, (float)q[k]), m1);
    }
}
// GGUF Q6_K: 210-byte block = ql[128], qh[64], int8 scales[16], d (fp16); only 2-byte aligned.
template <>
__device__ __forceinline__ void decode8<11>(const RowRef &r, int i0, float (&w)[8], uint8_t (&q)[8]) {
    const uint8_t *blk = r.row + (size_t)(i0 >> 8) * 210;
    const int within = i0 & 255, h = within >> 7, qd = (within >> 5) & 3, l0 = within & 31;
    const float d = ld_half(blk + 208);
    const uint8_t *ql = blk + 64 * h + ((qd & 1) ? 32 : 0) + l0, *qh = blk + 128 + 32 * h + l0;
    const int8_t sc = ((const int8_t *)(blk + 192))[8 * h + (l0 >> 4) + 2 * qd];
    const float ds = __fmul_rn(d, (float)sc);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const unsigned lo = (qd >= 2) ? (ql[k] >> 4) : (ql[k] & 15u);
        const unsigned v = lo | (((qh[k] >> (2 * qd)) & 3u) << 4);
        q[k] = v;
        w[k] = __fmul_rn(ds, (float)((int)v - 32));
    }
}

__host__ __device__ inline size_t row_bytes_for(int bits, int in_dim) {
    switch (bits) {
        case 0: return (size_t)in_dim * 2;
        case 10: return (size_t)(in_dim / 256) * 144;
        case 11: return (size_t)(in_dim / 256) * 210;
        default: return (size_t)in_dim * bits / 8;
    }
}

struct Spec {
    const uint8_t *W;
    const uint16_t *S, *B;
    float *out;
    int out_dim, in_dim, bits, scale_dtype;
};
#define FINCH_MAX_SPECS 8
struct SpecPack {
    Spec s[FINCH_MAX_SPECS];
    int n;
};

constexpr int MT = 8;  // tokens per pass

template <int BITS>
__device__ void row_dot(const Spec &sp, int row, const void *x, int x_dtype, int M, int lane) {
    const int groups = sp.in_dim / 64;
    RowRef r{sp.W + (size_t)row * row_bytes_for(BITS, sp.in_dim), sp.S ? sp.S + (size_t)row * groups : nullptr,
             sp.B ? sp.B + (size_t)row * groups : nullptr, sp.scale_dtype};
    for (int m0 = 0; m0 < M; m0 += MT) {
        const int mt = min(MT, M - m0);
        float acc[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) acc[m] = 0.f;
        for (int i0 = lane * 8; i0 < sp.in_dim; i0 += 32 * 8) {
            float w[8];
            uint8_t q[8];
            decode8<BITS>(r, i0, w, q);
#pragma unroll
            for (int m = 0; m < MT; m++) {
                if (m < mt) {
                    float xv[8];
                    if (x_dtype == FINCH_BF16) {
                        const uint4 v = *reinterpret_cast<const uint4 *>((const uint16_t *)x + (size_t)(m0 + m) * sp.in_dim + i0);
                        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            xv[2 * j] = __uint_as_float(u[j] << 16);
                            xv[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
                        }
                    } else {
                        const float4 a = *reinterpret_cast<const float4 *>((const float *)x + (size_t)(m0 + m) * sp.in_dim + i0);
                        const float4 b = *reinterpret_cast<const float4 *>((const float *)x + (size_t)(m0 + m) * sp.in_dim + i0 + 4);
                        xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
                        xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[m] = fmaf(w[j], xv[j], acc[m]);
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float v = acc[m];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && m < mt) sp.out[(size_t)(m0 + m) * sp.out_dim + row] = v;
        }
    }
}

// grid: (ceil(max_out / 4), n specs); block 128 = 4 warps, one output row per warp.
__global__ void __launch_bounds__(128) batch_matvec_kernel(SpecPack pack, const void *x, int x_dtype, int M) {
    const Spec &sp = pack.s[blockIdx.y];
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= sp.out_dim) return;
    switch (sp.bits) {
        case 0: row_dot<0>(sp, row, x, x_dtype, M, lane); break;
        case 3: row_dot<3>(sp, row, x, x_dtype, M, lane); break;
        case 4: row_dot<4>(sp, row, x, x_dtype, M, lane); break;
        case 8: row_dot<8>(sp, row, x, x_dtype, M, lane); break;
        case 10: row_dot<10>(sp, row, x, x_dtype, M, lane); break;
        case 11: row_dot<11>(sp, row, x, x_dtype, M, lane); break;
    }
}

template <int BITS>
__device__ void dequant_row(const Spec &sp, int row, uint8_t *codes, float *w32, uint16_t *w16, int w16_dtype, int lane) {
    const int groups = sp.in_dim / 64;
    RowRef r{sp.W + (size_t)row * row_bytes_for(BITS, sp.in_dim), sp.S ? sp.S + (size_t)row * groups : nullptr,
             sp.B ? sp.B + (size_t)row * groups : nullptr, sp.scale_dtype};
    for (int i0 = lane * 8; i0 < sp.in_dim; i0 += 256) {
        float w[8];
        uint8_t q[8];
        decode8<BITS>(r, i0, w, q);
        const size_t o = (size_t)row * sp.in_dim + i0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (codes) codes[o + j] = q[j];
            if (w32) w32[o + j] = w[j];
            if (w16)
                w16[o + j] = w16_dtype == FINCH_FP16 ? __half_as_ushort(__float2half_rn(w[j]))
                                                     : __bfloat16_as_ushort(__float2bfloat16_rn(w[j]));
        }
    }
}

__global__ void __launch_bounds__(128) dequant_kernel(Spec sp, uint8_t *codes, float *w32, uint16_t *w16, int w16_dtype) {
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= sp.out_dim) return;
    switch (sp.bits) {
        case 0: dequant_row<0>(sp, row, codes, w32, w16, w16_dtype, lane); break;
        case 3: dequant_row<3>(sp, row, codes, w32, w16, w16_dtype, lane); break;
        case 4: dequant_row<4>(sp, row, codes, w32, w16, w16_dtype, lane); break;
        case 8: dequant_row<8>(sp, row, codes, w32, w16, w16_dtype, lane); break;
        case 10: dequant_row<10>(sp, row, codes, w32, w16, w16_dtype, lane); break;
        case 11: dequant_row<11>(sp, row, codes, w32, w16, w16_dtype, lane); break;
    }
}

// Router tail: one warp per token.  softmax (max-subtracted, expf), then K
// rounds of arg-max with "earlier index wins" on ties -- the set the
// reference's replace-the-minimum scan selects -- then renormalise.
__global__ void __launch_bounds__(128) route_topk_kernel(const float *logits, int n_experts, int K, int32_t *ids,
                                                         float *weights, int T) {
    const int t = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= T) return;
    const float *lg = logits + (size_t)t * n_experts;
    constexpr int PER = 32;  // up to 1024 experts
    float p[PER];
    float mx = -INFINITY;
    for (int j = 0; j < PER; j++) {
        const int e = lane + 32 * j;
        p[j] = e < n_experts ? lg[e] : -INFINITY;
        mx = fmaxf(mx, p[j]);
    }
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // the reference sums exp() sequentially; the warp tree here differs in the last bits only
    float sum = 0.f;
    for (int j = 0; j < PER; j++) {
        const int e = lane + 32 * j;
        p[j] = e < n_experts ? expf(p[j] - mx) : -1.f;
        if (e < n_experts) sum += p[j];
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
    for (int j = 0; j < PER; j++)
        if (p[j] >= 0.f) p[j] *= inv;
    float wsum = 0.f, myw = 0.f;
    int myid = 0;
    for (int k = 0; k < K; k++) {
        float bv = -1.f;
        int bi = 0x7fffffff;
        for (int j = 0; j < PER; j++) {
            const int e = lane + 32 * j;
            if (p[j] > bv) {  // strictly greater: the lowest index among equals is kept
                bv = p[j];
                bi = e;
            }
        }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 31) == lane && bi < n_experts) p[bi >> 5] = -1.f;  // remove the winner
        if (lane == k) {
            myw = bv;
            myid = bi;
        }
        wsum += bv;
    }
    if (lane < K) {
        ids[(size_t)t * K + lane] = myid;
        weights[(size_t)t * K + lane] = wsum > 0.f ? myw * (1.0f / wsum) : myw;
    }
}

int ensure_stage(finch_ctx *ctx, size_t bytes) {
    if (ctx->stage_bytes >= bytes) return FINCH_OK;
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->stage_dev);
    if (ctx->stage_host) cudaFreeHost(ctx->stage_host);
    ctx->stage_dev = ctx->stage_host = nullptr;
    ctx->stage_bytes = 0;
    ctx->stage_gen++;   // launch sequences captured on the old blocks are stale
    const size_t want = (bytes + (1u << 20) - 1) & ~(size_t)((1u << 20) - 1);
    if (cudaMalloc(&ctx->stage_dev, want) != cudaSuccess || cudaMallocHost(&ctx->stage_host, want) != cudaSuccess) {
        cudaGetLastError();
        return finch_fail(ctx, FINCH_E_NOMEM, "staging buffer of %zu bytes", want);
    }
    ctx->stage_bytes = want;
    return FINCH_OK;
}

}  // namespace

int finch_stage_reserve(finch_ctx *ctx, size_t bytes) { return ensure_stage(ctx, bytes); }

int finch_validate_wdesc(finch_ctx *ctx, const finch_wdesc *w, const char *what) {
    if (!w || !w->W) return finch_fail(ctx, FINCH_E_ARG, "%s: null weight", what);
    const int b = w->bits;
    if (!(b == 0 || b == 3 || b == 4 || b == 8 || b == 10 || b == 11))
        return finch_fail(ctx, FINCH_E_UNSUPPORTED, "%s: bits=%d is not a supported tier", what, b);
    if (w->out_dim < 1 || w->in_dim < 1) return finch_fail(ctx, FINCH_E_ARG, "%s: bad dims", what);
    if (b == 3 || b == 4 || b == 8) {
        if (!w->scales || !w->biases) return finch_fail(ctx, FINCH_E_ARG, "%s: affine tier needs scales and biases", what);
        if (w->group_size != 64 || w->in_dim % 64) return finch_fail(ctx, FINCH_E_ARG, "%s: group size must be 64 and divide in_dim", what);
        if (w->scale_dtype != FINCH_BF16 && w->scale_dtype != FINCH_FP16) return finch_fail(ctx, FINCH_E_ARG, "%s: scale_dtype", what);
    } else if (b == 0) {
        if (w->in_dim % 8) return finch_fail(ctx, FINCH_E_ARG, "%s: BF16 rows must be a multiple of 8 wide", what);
    } else if (w->in_dim % 256) {
        return finch_fail(ctx, FINCH_E_ARG, "%s: GGUF K-quant rows are whole 256-value blocks", what);
    }
    if ((uintptr_t)w->W % 16 && b != 11) return finch_fail(ctx, FINCH_E_ARG, "%s: weight pointer must be 16-byte aligned", what);
    return FINCH_OK;
}

extern "C" int finch_encode_batch_matvec(finch_ctx *ctx, finch_stream stream, const void *x, int x_dtype,
                                         const finch_wdesc *specs, float *const *outs, int n, int M) {
    if (!ctx || !x || !specs || !outs || n < 1 || n > FINCH_MAX_SPECS || M < 1) return FINCH_E_ARG;
    if (x_dtype != FINCH_F32 && x_dtype != FINCH_BF16) return finch_fail(ctx, FINCH_E_ARG, "x_dtype");
    SpecPack pack;
    pack.n = n;
    int max_out = 0;
    for (int i = 0; i < n; i++) {
        int rc = finch_validate_wdesc(ctx, &specs[i], "batch_matvec spec");
        if (rc) return rc;
        if (specs[i].in_dim != specs[0].in_dim) return finch_fail(ctx, FINCH_E_ARG, "specs must share in_dim");
        if (!outs[i]) return finch_fail(ctx, FINCH_E_ARG, "null output");
        pack.s[i] = Spec{(const uint8_t *)specs[i].W, (const uint16_t *)specs[i].scales, (const uint16_t *)specs[i].biases,
                         outs[i], specs[i].out_dim, specs[i].in_dim, specs[i].bits, specs[i].scale_dtype};
        max_out = max_out > specs[i].out_dim ? max_out : specs[i].out_dim;
    }
    cudaSetDevice(ctx->cfg.device);
    {   // a large 4- or 8-bit tensor (lm_head, the big projections) at a few positions: the tensor-core streaming kernel (matvec_stream.cu)
        const int rc = finch_try_stream_matvec(ctx, finch_pick_stream(ctx, stream), x, x_dtype, specs, outs, n, M);
        if (rc >= 0) return rc;
    }
    if (n == 1) {   // a large Q6_K / Q4_K tensor (a GGUF model's output projection) at one position: matvec_kq_stream.cu
        const int rc = finch_kq_stream_matvec(ctx, finch_pick_stream(ctx, stream), &specs[0], x, x_dtype, outs[0], M);
        if (rc >= 0) return rc;
    }
    {   // 9 and more positions of Q4_K / Q6_K tensors: one pass over the weights on the tensor cores (matvec_gguf_mma.cu)
        const int rc = finch_try_gguf_mma(ctx, finch_pick_stream(ctx, stream), x, x_dtype, specs, outs, n, M);
        if (rc >= 0) return rc;
    }
    {   // 1..8 positions of a 3-bit / 4-bit / Q4_K tensor: the streaming kernel (matvec_fast.cu)
        const int rc = finch_try_fast_matvec(ctx, finch_pick_stream(ctx, stream), x, x_dtype, specs, outs, n, M);
        if (rc >= 0) return rc;
    }
    dim3 grid((max_out + 3) / 4, n);
    batch_matvec_kernel<<<grid, 128, 0, finch_pick_stream(ctx, stream)>>>(pack, x, x_dtype, M);
    ctx->launches++;
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    return FINCH_OK;
}

extern "C" int finch_matvec(finch_ctx *ctx, const finch_wdesc *w, const float *x_host, float *out_host, int M) {
    if (!ctx || !w || !x_host || !out_host || M < 1) return FINCH_E_ARG;
    int rc = finch_validate_wdesc(ctx, w, "matvec");
    if (rc) return rc;
    const size_t xb = (size_t)M * w->in_dim * sizeof(float), ob = (size_t)M * w->out_dim * sizeof(float);
    if ((rc = ensure_stage(ctx, xb + ob + 512))) return rc;
    cudaSetDevice(ctx->cfg.device);
    float *xd = (float *)ctx->stage_dev, *od = (float *)((char *)ctx->stage_dev + ((xb + 255) & ~(size_t)255));
    FINCH_CUDA_OK(ctx, cudaMemcpyAsync(xd, x_host, xb, cudaMemcpyHostToDevice, ctx->stream));
    float *outs[1] = {od};
    if ((rc = finch_encode_batch_matvec(ctx, ctx->stream, xd, FINCH_F32, w, outs, 1, M))) return rc;
    FINCH_CUDA_OK(ctx, cudaMemcpyAsync(out_host, od, ob, cudaMemcpyDeviceToHost, ctx->stream));
    int dev_rc = FINCH_OK;   // the device status word rides along: a synchronous call reports what the device recorded
    FINCH_CUDA_OK(ctx, cudaMemcpyAsync(&dev_rc, ctx->dev_status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    FINCH_CUDA_OK(ctx, cudaStreamSynchronize(ctx->stream));
    if (dev_rc != FINCH_OK) return finch_fail(ctx, dev_rc, "device status %d after the matvec", dev_rc);
    return FINCH_OK;
}

extern "C" int finch_encode_route_topk(finch_ctx *ctx, finch_stream stream, const float *logits, int n_experts, int K,
                                       int32_t *ids, float *weights, int T) {
    if (!ctx || !logits || !ids || !weights || T < 1) return FINCH_E_ARG;
    if (n_experts < K || n_experts > 1024 || K < 1 || K > 32) return finch_fail(ctx, FINCH_E_ARG, "route: n_experts=%d K=%d", n_experts, K);
    cudaSetDevice(ctx->cfg.device);
    route_topk_kernel<<<(T + 3) / 4, 128, 0, finch_pick_stream(ctx, stream)>>>(logits, n_experts, K, ids, weights, T);
    ctx->launches++;
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    return FINCH_OK;
}

extern "C" int finch_debug_dequant(finch_ctx *ctx, const finch_wdesc *w, uint8_t *codes, float *w_f32, uint16_t *w16,
                                   int w16_dtype) {
    if (!ctx) return FINCH_E_ARG;
    int rc = finch_validate_wdesc(ctx, w, "debug_dequant");
    if (rc) return rc;
    if (w16 && w16_dtype != FINCH_BF16 && w16_dtype != FINCH_FP16) return finch_fail(ctx, FINCH_E_ARG, "w16_dtype");
    cudaSetDevice(ctx->cfg.device);
    const size_t n = (size_t)w->out_dim * w->in_dim;
    uint8_t *dc = nullptr;
    float *d32 = nullptr;
    uint16_t *d16 = nullptr;
    auto cleanup = [&]() {
        cudaFree(dc);
        cudaFree(d32);
        cudaFree(d16);
    };
    if ((codes && cudaMalloc(&dc, n) != cudaSuccess) || (w_f32 && cudaMalloc(&d32, n * 4) != cudaSuccess) ||
        (w16 && cudaMalloc(&d16, n * 2) != cudaSuccess)) {
        cleanup();
        cudaGetLastError();
        return finch_fail(ctx, FINCH_E_NOMEM, "debug_dequant buffers");
    }
    Spec sp{(const uint8_t *)w->W, (const uint16_t *)w->scales, (const uint16_t *)w->biases, nullptr, w->out_dim, w->in_dim,
            w->bits, w->scale_dtype};
    dequant_kernel<<<(w->out_dim + 3) / 4, 128, 0, ctx->stream>>>(sp, dc, d32, d16, w16_dtype);
    ctx->launches++;
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && codes) e = cudaMemcpyAsync(codes, dc, n, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess && w_f32) e = cudaMemcpyAsync(w_f32, d32, n * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess && w16) e = cudaMemcpyAsync(w16, d16, n * 2, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cleanup();
    if (e != cudaSuccess) return finch_fail(ctx, FINCH_E_CUDA, "debug_dequant: %s", cudaGetErrorString(e));
    return FINCH_OK;
}

// ---- allocation-free matvec ----------------------------------------------
// Staging memory for finch_matvec_noalloc: the activations of a call are copied
// here from the host and the results are written here before they go back.  It
// is part of the library image, so every GPU that loads the library holds these
// 512 KiB until the process exits.
#define FINCH_NOALLOC_SCRATCH_BYTES (512 * 1024)
static __device__ __align__(256) unsigned char g_noalloc_scratch[FINCH_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
void *g_noalloc_ptr[kMaxDevices] = {nullptr};  // device address of g_noalloc_scratch, per device
std::mutex g_noalloc_mu;
}  // namespace

extern "C" int finch_matvec_noalloc(const finch_wdesc *w, const float *x_host, float *out_host, int M, finch_stream stream) {
    if (!w || !x_host || !out_host || M < 1) return FINCH_E_ARG;
    if (const int rc = finch_validate_wdesc(nullptr, w, "matvec_noalloc")) return rc;   // the code finch_matvec gives for the same tensor
    const size_t xb = (size_t)M * w->in_dim * sizeof(float), ob = (size_t)M * w->out_dim * sizeof(float);
    const size_t x_room = (xb + 255) & ~(size_t)255;
    if (x_room + ob > FINCH_NOALLOC_SCRATCH_BYTES) return FINCH_E_UNSUPPORTED;  // M * (in_dim + out_dim) floats must fit 512 KiB
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FINCH_E_CUDA;
    void *base = nullptr;
    {
        // The array's name is only a host-side handle; the kernel needs the address it has on the
        // current device.  Looked up once per device, on the first call made with that device current
        // (the address does not outlive a cudaDeviceReset: the entry point is not to be used across one).
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
                cudaGetLastError();
                return FINCH_E_CUDA;
            }
            g_noalloc_ptr[dev] = p;
        }
        base = g_noalloc_ptr[dev];
    }
    cudaStream_t st = (cudaStream_t)stream;
    float *xd = (float *)base, *od = (float *)((char *)base + x_room);
    if (cudaMemcpyAsync(xd, x_host, xb, cudaMemcpyHostToDevice, st) != cudaSuccess) return FINCH_E_CUDA;
    SpecPack pack;
    pack.n = 1;
    pack.s[0] = Spec{(const uint8_t *)w->W, (const uint16_t *)w->scales, (const uint16_t *)w->biases, od, w->out_dim, w->in_dim, w->bits,
                     w->scale_dtype};
    batch_matvec_kernel<<<dim3((w->out_dim + 3) / 4, 1), 128, 0, st>>>(pack, xd, FINCH_F32, M);
    if (cudaGetLastError() != cudaSuccess) return FINCH_E_CUDA;
    if (cudaMemcpyAsync(out_host, od, ob, cudaMemcpyDeviceToHost, st) != cudaSuccess) return FINCH_E_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return FINCH_E_CUDA;
    return FINCH_OK;
}

// Router front end of a layer (routing_batch_fused / the gemv_bf16 fallback + cpu_softmax / cpu_topk /
// cpu_normalize_weights, finchmoe/infer.m:9061-9105, 9285-9289): logits = gate * h_post, the shared expert's gate
// score = shared_gate * h_post, then softmax / top-K / renormalise on the device -- no host round trip.
extern "C" int finch_encode_router(finch_ctx *ctx, finch_stream stream, const finch_wdesc *gate, const finch_wdesc *shared_gate, const void *h_post,
                                   int32_t *ids, float *weights, float *shared_score, int T) {
    if (!ctx || !gate || !h_post || !ids || !weights || T < 1) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    if (gate->out_dim != c.n_experts || gate->in_dim != c.hidden) return finch_fail(ctx, FINCH_E_ARG, "router gate must be [n_experts x hidden]");
    if (shared_gate && (!shared_score || shared_gate->out_dim != 1 || shared_gate->in_dim != c.hidden))
        return finch_fail(ctx, FINCH_E_ARG, "shared gate must be [1 x hidden] with a score output");
    if (T > c.max_tokens) return finch_fail(ctx, FINCH_E_ARG, "T=%d exceeds max_tokens=%d", T, c.max_tokens);
    if (!ctx->logits) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(finch_pick_stream(ctx, stream), &cap);
        if (cap != cudaStreamCaptureStatusNone) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "first router call must be outside stream capture");
        if (cudaMalloc(&ctx->logits, (size_t)c.max_tokens * c.n_experts * sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return finch_fail(ctx, FINCH_E_NOMEM, "router logits");
        }
    }
    finch_wdesc specs[2] = {*gate, shared_gate ? *shared_gate : *gate};
    float *outs[2] = {ctx->logits, shared_score};
    int rc = finch_encode_batch_matvec(ctx, stream, h_post, c.act_dtype, specs, outs, shared_gate ? 2 : 1, T);
    if (rc) return rc;
    return finch_encode_route_topk(ctx, stream, ctx->logits, c.n_experts, c.top_k, ids, weights, T);
}

// Residual add + RMS norm either side of the MoE layer (residual_norm_fused, finchmoe/shaders.metal:1232-1263;
// rms_norm_sum_sq + rms_norm_apply_bf16 after the combine, finchmoe/infer.m:9705-9737): h = resid + oproj,
// h_post = h / sqrt(mean(h^2) + eps) * w.  One CTA of 256 threads per token.
namespace {
__global__ void __launch_bounds__(256) residual_norm_kernel(const float *resid, const float *oproj, const uint16_t *norm_w, int dim, float eps,
                                                            float *h_mid_out, void *h_post_out, int out_dtype) {
    __shared__ float red[8];
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *r = resid + (size_t)t * dim, *o = oproj ? oproj + (size_t)t * dim : nullptr;
    float s = 0.f;
    for (int i = tid; i < dim; i += 256) {
        const float h = o ? r[i] + o[i] : r[i];
        if (h_mid_out) h_mid_out[(size_t)t * dim + i] = h;
        s = fmaf(h, h, s);
    }
#pragma unroll
    for (int k = 16; k; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
    if ((tid & 31) == 0) red[tid >> 5] = s;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) tot += red[w];
    const float inv = 1.0f / sqrtf(tot / (float)dim + eps);
    for (int i = tid; i < dim; i += 256) {
        const float h = o ? r[i] + o[i] : r[i];
        const float v = h * inv * __uint_as_float((uint32_t)norm_w[i] << 16);
        if (out_dtype == FINCH_BF16) ((__nv_bfloat16 *)h_post_out)[(size_t)t * dim + i] = __float2bfloat16_rn(v);
        else ((float *)h_post_out)[(size_t)t * dim + i] = v;
    }
}
}  // namespace

extern "C" int finch_encode_residual_norm(finch_ctx *ctx, finch_stream stream, const float *resid, const float *oproj, const uint16_t *norm_w_bf16,
                                          float eps, float *h_mid_out, void *h_post_out, int T) {
    if (!ctx || !resid || !norm_w_bf16 || !h_post_out || T < 1) return FINCH_E_ARG;
    cudaSetDevice(ctx->cfg.device);
    residual_norm_kernel<<<T, 256, 0, finch_pick_stream(ctx, stream)>>>(resid, oproj, norm_w_bf16, ctx->cfg.hidden, eps, h_mid_out, h_post_out,
                                                                        ctx->cfg.act_dtype);
    ctx->launches++;
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    return FINCH_OK;
}
