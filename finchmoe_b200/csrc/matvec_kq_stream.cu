// Streaming matvecs for large GGUF K-quant tensors (Q6_K, Q4_K) at ONE position: the output projection of a GGUF model
// (lm_head tier, out_dim 248,320, finchmoe/infer.m:5728-5815; kernels dequant_matvec_q6k / dequant_matvec_q4k,
// finchmoe/shaders.metal:3216-3299).  HBM-bound: every byte of the tensor is read once, straight from the GGUF block
// layout.  A warp owns a row at a time and walks its 256-value blocks four at a time, the words of the next four already
// in flight.  A byte becomes a float with one byte permute (0x4B000000 | q is the float 2^23 + q) and one subtraction and
// meets four consecutive activations read from shared memory as a float4.  The arithmetic is the reference's:
// value = d * sc * (q - 32) (Q6_K), d * sc * q - dmin * m (Q4_K), summed in fp32.
//
// Q6_K (210-byte blocks, so only 2-byte alignment): lane j takes word j of the 128 bytes of low nibbles: four bytes =
// eight values, four from the low nibbles and four from the high ones, consecutive values of two sub-blocks; the high
// bits are added with word-wide logic.
// Q4_K (144-byte blocks, 16-byte aligned): eight lanes per block, a lane takes the block's 16-byte header and 16 bytes
// of nibbles = 16 values of each of two sub-blocks.
#include "finch_internal.cuh"

namespace {

constexpr int KNT = 256;        // threads per CTA; four CTAs per SM
constexpr int KQ_MAXK = 8192;   // activations of the position as floats in shared memory: 32 KB

struct KqArgs {
    const uint8_t *W;
    float *out;
    const void *x;
    int x_bf16;
    int out_dim, K;
};

// four bytes at a 2-byte aligned address (a Q6_K block is 210 bytes long)
__device__ __forceinline__ uint32_t ld_u16x2(const uint8_t *p) {
    const uint16_t *q = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)__ldg(q) | ((uint32_t)__ldg(q + 1) << 16);
}
// sum_i (byte i of q4 - off) * x_i
__device__ __forceinline__ float dot4(uint32_t q4, const float4 x, float off) {
    const float c = 8388608.0f + off;
    float a = (__uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7540)) - c) * x.x;
    a = fmaf(__uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7541)) - c, x.y, a);
    a = fmaf(__uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7542)) - c, x.z, a);
    return fmaf(__uint_as_float(__byte_perm(q4, 0x4B000000u, 0x7543)) - c, x.w, a);
}
__device__ __forceinline__ float half_bits(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// ---- Q6_K: block = ql[128] qh[64] scales[16] (int8) d (fp16) = 210 bytes -------------------------------------
struct Raw6 {
    uint32_t ql, qh, sc, d;
};
// A4: the block starts on a 4-byte boundary (every other block of a row whose byte length is a multiple of 4)
template <bool A4>
__device__ __forceinline__ Raw6 load6(const uint8_t *blk, int lane) {
    const int half = lane >> 4, w = lane & 15;
    Raw6 r;
    if (A4) {
        r.ql = __ldg(reinterpret_cast<const uint32_t *>(blk) + lane);
        r.qh = __ldg(reinterpret_cast<const uint32_t *>(blk + 128) + half * 8 + (w & 7));
    } else {
        r.ql = ld_u16x2(blk + 4 * lane);
        r.qh = ld_u16x2(blk + 128 + 4 * (half * 8 + (w & 7)));
    }
    const int is = 192 + half * 8 + ((w & 7) >> 2) + (w < 8 ? 0 : 2);   // sub-block of the low-nibble values; the high ones: + 4
    r.sc = (uint32_t)__ldg(blk + is) | ((uint32_t)__ldg(blk + is + 4) << 8);
    r.d = __ldg(reinterpret_cast<const uint16_t *>(blk + 208));
    return r;
}
// xb: the block's 256 activations (float4 units)
__device__ __forceinline__ float dot6(const Raw6 &r, const float4 *xb, int lane) {
    const int half = lane >> 4, w = lane & 15;
    const int s_lo = w < 8 ? 0 : 2;                                   // the high bits of the low-nibble values; the others: + 4
    const uint32_t lowq = (r.ql & 0x0F0F0F0Fu) | (((r.qh >> s_lo) & 0x03030303u) << 4);
    const uint32_t highq = ((r.ql >> 4) & 0x0F0F0F0Fu) | (((r.qh >> (s_lo + 4)) & 0x03030303u) << 4);
    const int v0 = half * 128 + (w < 8 ? 0 : 32) + 4 * (w & 7);       // first of the four low-nibble values; the others: + 64
    const float a = dot4(lowq, xb[v0 >> 2], 32.0f), b = dot4(highq, xb[(v0 + 64) >> 2], 32.0f);
    const float d = half_bits(r.d);
    return d * fmaf((float)(int)(signed char)(r.sc & 0xffu), a, (float)(int)(signed char)((r.sc >> 8) & 0xffu) * b);
}

// grid: any; block KNT.  Dynamic shared memory: K floats.
// A warp walks its rows in steps of UB blocks (UB divides the blocks of a row); the words of the next step are in
// flight while this one is computed.
template <int UB>
__global__ void __launch_bounds__(KNT, 4) kq_stream_kernel(const KqArgs a) {
    extern __shared__ __align__(16) float xs[];
    const int tid = threadIdx.x, lane = tid & 31;
    const int K = a.K, nb = K / 256, BS = 210;
    for (int i = tid; i < K; i += KNT)
        xs[i] = a.x_bf16 ? __uint_as_float((uint32_t) reinterpret_cast<const uint16_t *>(a.x)[i] << 16) : reinterpret_cast<const float *>(a.x)[i];
    __syncthreads();
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
    const int wpc = KNT / 32, gw = blockIdx.x * wpc + (tid >> 5), nw = gridDim.x * wpc;
    if (gw >= a.out_dim) return;
    using Raw = Raw6;
    const size_t row_bytes = (size_t)nb * BS, row_step = (size_t)nw * row_bytes;
    // position of the step being loaded: row and first block
    int lrow = gw, lb = 0;
    const uint8_t *lp = a.W + (size_t)gw * row_bytes;
    auto load_step = [&](Raw (&r)[UB]) {
        if (lrow < a.out_dim) {
#pragma unroll
            for (int k = 0; k < UB; k++) {
                // UB even: block lb + k starts 210 (lb + k) bytes into a row whose length is a multiple of 4
                if (UB % 2 == 0 && k % 2 == 0) r[k] = load6<true>(lp + (size_t)(lb + k) * BS, lane);
                else r[k] = load6<false>(lp + (size_t)(lb + k) * BS, lane);
            }
        }
        lb += UB;
        if (lb >= nb) {
            lb = 0;
            lrow += nw;
            lp += row_step;
        }
    };
    Raw nxt[UB];
#pragma unroll
    for (int k = 0; k < UB; k++) nxt[k] = Raw{};
    load_step(nxt);
    float acc = 0.f;
    for (int row = gw; row < a.out_dim; row += nw) {
        for (int b0 = 0; b0 < nb; b0 += UB) {
            Raw cur[UB];
#pragma unroll
            for (int k = 0; k < UB; k++) cur[k] = nxt[k];
            load_step(nxt);
#pragma unroll
            for (int k = 0; k < UB; k++) {
                acc += dot6(cur[k], xs4 + (b0 + k) * 64, lane);
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) a.out[row] = acc;
        acc = 0.f;
    }
}

// ---- Q4_K: block = d dmin (fp16) scales[12] (6-bit, packed) qs[128] = 144 bytes -------------------------------
// Eight lanes per block, four blocks per warp step: lane (bq, m) takes the 16-byte header of block bq and bytes
// 16 m .. 16 m + 15 of its nibbles = 16 low-nibble values of sub-block 2 c and 16 high-nibble values of sub-block
// 2 c + 1 (c = m / 2).  Each of the eight lanes unpacks ONE sub-block's 6-bit scale and min (get_scale_min_k4,
// finchmoe/infer.m:1595-1603) and shuffles hand every lane the two it needs.  Shared memory: the activations and
// their sums over 16.
__device__ __forceinline__ void scale_min4(uint32_t s0, uint32_t s1, uint32_t s2, int is, float &sc, float &mn) {
    const uint32_t lo = is < 4 ? s0 : s1;
    const uint32_t q_is = (lo >> (8 * (is & 3))) & 0xffu;               // byte is
    if (is < 4) {
        sc = (float)(q_is & 63u);
        mn = (float)((s1 >> (8 * is)) & 63u);                           // byte is + 4
    } else {
        const uint32_t q8 = (s2 >> (8 * (is - 4))) & 0xffu;             // byte is + 4
        const uint32_t qm4 = (s0 >> (8 * (is - 4))) & 0xffu;            // byte is - 4
        sc = (float)((q8 & 0xFu) | ((qm4 >> 6) << 4));
        mn = (float)((q8 >> 4) | ((q_is >> 6) << 4));
    }
}

__global__ void __launch_bounds__(KNT, 4) q4k_stream_kernel(const KqArgs a) {
    extern __shared__ __align__(16) float xs[];
    const int tid = threadIdx.x, lane = tid & 31;
    const int K = a.K, nb = K / 256;          // nb is a multiple of 4
    // Activation v sits at float v + 4 (v / 64): the eight lanes of a block read 16-byte words 64 bytes apart, which
    // would all fall into two groups of banks; the skew of one 16-byte word per 64 values spreads them over all 32.
    float *sx16 = xs + K + 4 * (K / 64);       // sums of 16 consecutive activations
    for (int i = tid; i < K; i += KNT)
        xs[i + 4 * (i >> 6)] = a.x_bf16 ? __uint_as_float((uint32_t) reinterpret_cast<const uint16_t *>(a.x)[i] << 16) : reinterpret_cast<const float *>(a.x)[i];
    __syncthreads();
    for (int i = tid; i < K / 16; i += KNT) {
        const float4 *p = reinterpret_cast<const float4 *>(xs + 16 * i + 4 * (i >> 2));
        const float4 u = p[0], v = p[1], w = p[2], z = p[3];
        sx16[i] = (((u.x + u.y) + (u.z + u.w)) + ((v.x + v.y) + (v.z + v.w))) + (((w.x + w.y) + (w.z + w.w)) + ((z.x + z.y) + (z.z + z.w)));
    }
    __syncthreads();
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
    const int wpc = KNT / 32, gw = blockIdx.x * wpc + (tid >> 5), nw = gridDim.x * wpc;
    if (gw >= a.out_dim) return;
    const int bq = lane >> 3, m = lane & 7, c = m >> 1, half = m & 1;
    const size_t row_bytes = (size_t)nb * 144, row_step = (size_t)nw * row_bytes;
    int lrow = gw, lb = 0;
    const uint8_t *lp = a.W + (size_t)gw * row_bytes;
    uint4 nh = make_uint4(0, 0, 0, 0), nq = make_uint4(0, 0, 0, 0);
    auto load_step = [&]() {
        if (lrow < a.out_dim) {
            const uint8_t *blk = lp + (size_t)(lb + bq) * 144;
            nh = __ldg(reinterpret_cast<const uint4 *>(blk));
            nq = __ldg(reinterpret_cast<const uint4 *>(blk + 16) + m);
        }
        lb += 4;
        if (lb >= nb) {
            lb = 0;
            lrow += nw;
            lp += row_step;
        }
    };
    load_step();
    float acc = 0.f;
    for (int row = gw; row < a.out_dim; row += nw) {
        for (int b0 = 0; b0 < nb; b0 += 4) {
            const uint4 h = nh, q = nq;
            load_step();
            float sc, mn;
            scale_min4(h.y, h.z, h.w, m, sc, mn);
            sc *= half_bits(h.x & 0xffffu);
            mn *= half_bits(h.x >> 16);
            const int src = (lane & 24) + 2 * c;     // the lane of my block that unpacked sub-block 2 c
            const float sc0 = __shfl_sync(0xffffffffu, sc, src), sc1 = __shfl_sync(0xffffffffu, sc, src + 1);
            const float m0 = __shfl_sync(0xffffffffu, mn, src), m1 = __shfl_sync(0xffffffffu, mn, src + 1);
            const int v0 = (b0 + bq) * 256 + 64 * c + 16 * half;      // my low-nibble values; the high-nibble ones: + 32
            const float4 *xl = xs4 + ((v0 + 4 * (v0 >> 6)) >> 2), *xh = xl + 8;   // + 32 values: the same 64-value stretch
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
            float A = 0.f, B = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                A += dot4(w[k] & 0x0F0F0F0Fu, xl[k], 0.0f);
                B += dot4((w[k] >> 4) & 0x0F0F0F0Fu, xh[k], 0.0f);
            }
            acc += fmaf(sc0, A, sc1 * B) - fmaf(m0, sx16[v0 >> 4], m1 * sx16[(v0 + 32) >> 4]);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) a.out[row] = acc;
        acc = 0.f;
    }
}

}  // namespace

// Returns FINCH_OK after launching, or -1 when the call is not one these kernels take (the caller goes on to the
// general kernels): a single Q6_K / Q4_K tensor with many rows at one position (Q4_K: blocks per row a multiple of 4).
int finch_kq_stream_matvec(finch_ctx *ctx, cudaStream_t st, const finch_wdesc *w, const void *x, int x_dtype, float *out, int M) {
    if (M != 1 || (w->bits != 10 && w->bits != 11) || w->out_dim < 32768 || w->in_dim % 256 || w->in_dim > KQ_MAXK) return -1;
    const int nb = w->in_dim / 256;
    if (w->bits == 10 && (nb % 4 || (uintptr_t)w->W & 15)) return -1;
    if ((uintptr_t)w->W & 3 || (uintptr_t)x & 3) return -1;
    KqArgs a{};
    a.W = (const uint8_t *)w->W;
    a.out = out;
    a.x = x;
    a.x_bf16 = x_dtype == FINCH_BF16;
    a.out_dim = w->out_dim;
    a.K = w->in_dim;
    const int grid = ctx->sm_count * 4;
    if (w->bits == 10) {
        q4k_stream_kernel<<<grid, KNT, (a.K + 4 * (a.K / 64)) * 4 + (a.K / 16) * 4, st>>>(a);
    } else {
        const int smem = a.K * 4;
        if (nb % 4 == 0) kq_stream_kernel<4><<<grid, KNT, smem, st>>>(a);   // (eight blocks per step, three CTAs per SM: 236 against 210 us)
        else if (nb % 2 == 0) kq_stream_kernel<2><<<grid, KNT, smem, st>>>(a);
        else kq_stream_kernel<1><<<grid, KNT, smem, st>>>(a);
    }
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}
