// Streaming matvec for large GGUF Q6_K tensors at ONE position: the output projection of a GGUF model (lm_head tier,
// out_dim 248,320, finchmoe/infer.m:5728-5815; kernel dequant_matvec_q6k, finchmoe/shaders.metal:3216-3299).
// HBM-bound: every byte of the tensor is read once, by exactly one lane (the high-bit words by two), straight from
// the GGUF block layout.
//
// A warp owns a row at a time and walks its 256-value blocks up to four at a time, the words of the next four already
// in flight.  Per block lane j takes word j of the 128 bytes of low nibbles (32 words): four bytes = eight values,
// four from the low nibbles and four from the high ones, which are consecutive values of two sub-blocks; it adds the
// high bits with word-wide logic, turns each byte into a float with one byte permute (0x4B000000 | q is the float
// 2^23 + q) and one subtraction, and multiplies by four consecutive activations read from shared memory as a float4.
// The arithmetic is the reference's: value = d * sc * (q - 32), summed in fp32.
// (Q4_K stays with the row-pair kernel of matvec_fast.cu: a lane that unpacks a whole 32-value sub-block pays for the
// 6-bit scale unpacking once per 32 values; the word-per-lane mapping used here measured 282 against 156 us.)
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

}  // namespace

// Returns FINCH_OK after launching, or -1 when the call is not one this kernel takes (the caller goes on to the
// general kernels): a single Q6_K tensor with many rows at one position.
int finch_kq_stream_matvec(finch_ctx *ctx, cudaStream_t st, const finch_wdesc *w, const void *x, int x_dtype, float *out, int M) {
    if (M != 1 || w->bits != 11 || w->out_dim < 32768 || w->in_dim % 256 || w->in_dim > KQ_MAXK) return -1;
    if ((uintptr_t)w->W & 3 || (uintptr_t)x & 3) return -1;
    KqArgs a{};
    a.W = (const uint8_t *)w->W;
    a.out = out;
    a.x = x;
    a.x_bf16 = x_dtype == FINCH_BF16;
    a.out_dim = w->out_dim;
    a.K = w->in_dim;
    const int smem = a.K * 4;
    const int grid = ctx->sm_count * 4;
    const int nb = a.K / 256;
    if (nb % 4 == 0) kq_stream_kernel<4><<<grid, KNT, smem, st>>>(a);   // (eight blocks per step, three CTAs per SM: 236 against 210 us)
    else if (nb % 2 == 0) kq_stream_kernel<2><<<grid, KNT, smem, st>>>(a);
    else kq_stream_kernel<1><<<grid, KNT, smem, st>>>(a);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}
