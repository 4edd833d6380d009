// Streaming matvec for large row-major affine tensors (4-bit / 8-bit, group 64) at 1..8 positions: the lm_head /
// embedding tier (out_dim 248,320, finchmoe/infer.m:5728-5815) and the big 4-bit projections behind the generic
// matvec seam (fast_dequant_matvec / gpu_encode_batch_matvec, infer.m:3369, 3528; kernels
// finchmoe/shaders.metal:374-533).  HBM-bound: every weight byte is read once, straight from the reference's
// tensor layout (u32 words, 16-bit scale and bias per group of 64 as separate tensors) -- nothing is re-tiled.
//
// A warp owns 16 rows at a time.  Per scale group (64 codes) lane (g, t) of the warp loads the 16 (8-bit) or
// 8 (4-bit) bytes of rows g and g + 8 that hold codes 16 t .. 16 t + 15 of the group -- whole 32-byte sectors
// per row, so DRAM traffic is the algorithmic traffic -- isolates the codes with ANDs (a code at bit p <= 7 of
// a 16-bit half is the fp16 subnormal q * 2^(p-24)) and feeds them as the A operand of four
// mma.sync.m16n8k16 (fp32 accumulate).  The B operand holds the activations, pre-scaled by 2^(7-p) / norm and
// laid out in shared memory once per CTA: an fp32 activation as fp16 hi and lo * 2^11 columns (no mantissa
// bit lost), a bf16 activation as its own hi column.  The four lanes of a quad cover exactly one scale group,
// so all eight columns carry positions: four (fp32) or eight (bf16) per pass.  Scale and bias are applied to
// the fp32 group sums: out = sum_g s_g * (sum q x) + b_g * (sum x).  Loads run four (8-bit) or eight (4-bit) groups
// ahead of the MMAs.
#include <algorithm>

#include "finch_internal.cuh"

namespace {

constexpr int SNT = 256;            // threads per CTA: 8 warps, three CTAs per SM
constexpr int SMAXK = 8192;

__device__ __forceinline__ float pow2b(int e) { return __uint_as_float((uint32_t)e << 23); }

__device__ __forceinline__ void mma16816s(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct StreamArgs {
    const uint8_t *W;
    const uint16_t *S, *B;
    float *out;          // [M][out_dim]
    const void *x;       // [M][K] bf16 or fp32
    int x_bf16;
    int out_dim, K, M;
    int scale_fp16;
};

// Shared memory: B fragments [group][MMA pair 0..1][column 0..ncol)[t][16 B], the group sums [column token][group]
// and the exponent of every position.
__host__ __device__ inline int stream_smem_bytes(int K, int ncol, int M) {
    return (K / 64) * 2 * ncol * 64 + M * (K / 64) * 4 + 64 + 128 + (SNT / 32) * (K / 64) * 64;   // + per warp: [group][g][scale A, scale B, bias A, bias B]
}

template <int BITS>
__device__ __forceinline__ int slot_code(int m, int slot) {
    // code number (0..15 within the lane's 16 codes) in k-slot `slot` (0: 2t, 1: 2t+1, 2: 2t+8, 3: 2t+9) of MMA m
    if (BITS == 8) return 4 * m + (slot == 0 ? 0 : slot == 1 ? 2 : slot == 2 ? 1 : 3);   // word m: (0,2) then (1,3)
    // 4-bit: word m >> 1; even m takes codes (0,4) (1,5), odd m (2,6) (3,7)
    const int base = 8 * (m >> 1) + ((m & 1) ? 2 : 0);
    return base + (slot == 0 ? 0 : slot == 1 ? 4 : slot == 2 ? 1 : 5);
}
template <int BITS>
__device__ __forceinline__ int slot_pos(int slot) { return BITS == 8 ? 0 : (slot < 2 ? 0 : 4); }

// HILO: fp32 activations (two columns per position), else bf16 (one column).
template <int BITS, bool HILO, bool FP16S>
__global__ void __launch_bounds__(SNT, 3) stream_matvec_kernel(const StreamArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int K = a.K, NG = K / 64, M = a.M;
    const int ncol = HILO ? 2 * M : M;                 // columns in use (<= 8)
    uint8_t *frag = smem;
    float *sums = reinterpret_cast<float *>(smem + NG * 2 * ncol * 64);   // [M][NG]
    int *expo = reinterpret_cast<int *>(sums + M * NG);                    // [M]
    uint8_t *zero = reinterpret_cast<uint8_t *>(expo + 16);               // 128 zero bytes
    uint8_t *sbw = zero + 128 + (size_t)warp * NG * 64;                    // this warp's scales and biases of the tile it works on

    // ---- the activations' fragments, once per CTA ----
    for (int i = tid; i < 32; i += SNT) reinterpret_cast<int *>(zero)[i] = 0;
    auto xval = [&](int m, int k) -> float {
        return a.x_bf16 ? __uint_as_float((uint32_t) reinterpret_cast<const uint16_t *>(a.x)[(size_t)m * K + k] << 16)
                        : reinterpret_cast<const float *>(a.x)[(size_t)m * K + k];
    };
    if (warp < M) {   // one warp per position: group sums and the largest magnitude
        float amax = 0.f;
        for (int gr = 0; gr < NG; gr++) {
            const float v0 = xval(warp, gr * 64 + lane), v1 = xval(warp, gr * 64 + 32 + lane);
            float s = v0 + v1;
            amax = fmaxf(amax, fmaxf(fabsf(v0), fabsf(v1)));
#pragma unroll
            for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) sums[warp * NG + gr] = s;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        int E = (int)(__float_as_uint(amax) >> 23) + 1;
        E = E < 30 ? 30 : (E > 230 ? 230 : E);
        if (lane == 0) expo[warp] = E;
    }
    __syncthreads();
    // entry (group, MMA m, position, t): four pre-scaled values -> hi (and lo) words
    for (int e = tid; e < NG * 4 * M * 4; e += SNT) {
        const int tt = e & 3, pos = (e >> 2) % M, m = ((e >> 2) / M) & 3, gr = (e >> 2) / (M * 4);
        const int E = expo[pos];
        float v[4];
#pragma unroll
        for (int s = 0; s < 4; s++) v[s] = xval(pos, gr * 64 + 16 * tt + slot_code<BITS>(m, s)) * pow2b(261 - E - slot_pos<BITS>(s));
        uint32_t h0, h1, l0 = 0, l1 = 0;
        if (HILO) {
            float hf[4], lf[4];
#pragma unroll
            for (int s = 0; s < 4; s++) {
                hf[s] = __half2float(__float2half_rn(v[s]));
                lf[s] = (v[s] - hf[s]) * 2048.0f;
            }
            h0 = finch_pack_h2(hf[0], hf[1]); h1 = finch_pack_h2(hf[2], hf[3]);
            l0 = finch_pack_h2(lf[0], lf[1]); l1 = finch_pack_h2(lf[2], lf[3]);
        } else {
            h0 = finch_pack_h2(v[0], v[1]); h1 = finch_pack_h2(v[2], v[3]);
        }
        // [group][MMA pair][column][t][16 B]: the two MMAs of a pair side by side
        const int col = HILO ? 2 * pos : pos;
        uint8_t *o = frag + ((size_t)(gr * 2 + (m >> 1)) * ncol + col) * 64 + tt * 16 + (m & 1) * 8;
        *reinterpret_cast<uint2 *>(o) = make_uint2(h0, h1);
        if (HILO) *reinterpret_cast<uint2 *>(o + 64) = make_uint2(l0, l1);
    }
    __syncthreads();

    // ---- rows ----
    const uint32_t frag32 = finch_smem_u32(frag), zero32 = finch_smem_u32(zero);
    const bool bact = g < ncol;                         // this lane's B column carries a position
    const uint32_t pb0 = bact ? frag32 + (uint32_t)(g * 64 + t * 16) : zero32 + (uint32_t)(t * 16);
    const uint32_t bstep = bact ? (uint32_t)(2 * ncol * 64) : 0u, bpair = bact ? (uint32_t)(ncol * 64) : 0u;
    // accumulator columns 2t, 2t + 1: HILO: position t (hi, lo); else positions 2t, 2t + 1
    const int p0 = HILO ? t : 2 * t, p1 = HILO ? t : 2 * t + 1;
    const float *x0s = sums + (p0 < M ? p0 : 0) * NG, *x1s = sums + (p1 < M ? p1 : 0) * NG;
    const int row_bytes = K * BITS / 8, lane_bytes = BITS == 8 ? 16 : 8;
    const int n_tiles = (a.out_dim + 15) / 16, wstride = gridDim.x * (SNT / 32);
    for (int tile = blockIdx.x * (SNT / 32) + warp; tile < n_tiles; tile += wstride) {
        const int rA = min(tile * 16 + g, a.out_dim - 1), rB = min(tile * 16 + 8 + g, a.out_dim - 1);   // rows past the end repeat the last one
        const uint8_t *wA = a.W + (size_t)rA * row_bytes + t * lane_bytes, *wB = a.W + (size_t)rB * row_bytes + t * lane_bytes;
        // The tile's scales and biases: 16 rows of NG 16-bit values in each of the two tensors.  Lane (g, t) loads eight groups'
        // worth of rows g and g + 8 at a time (16 bytes per row and tensor) and leaves them in shared memory as
        // [group][g][scale A, scale B, bias A, bias B]: four wide loads per 32 groups instead of four narrow ones per group.
        __syncwarp();
        for (int g0 = 8 * t; g0 < NG; g0 += 32) {
            const uint4 sa = __ldg(reinterpret_cast<const uint4 *>(a.S + (size_t)rA * NG + g0)), sb = __ldg(reinterpret_cast<const uint4 *>(a.S + (size_t)rB * NG + g0));
            const uint4 ba = __ldg(reinterpret_cast<const uint4 *>(a.B + (size_t)rA * NG + g0)), bb2 = __ldg(reinterpret_cast<const uint4 *>(a.B + (size_t)rB * NG + g0));
            const uint32_t sa4[4] = {sa.x, sa.y, sa.z, sa.w}, sb4[4] = {sb.x, sb.y, sb.z, sb.w}, ba4[4] = {ba.x, ba.y, ba.z, ba.w}, bb4[4] = {bb2.x, bb2.y, bb2.z, bb2.w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int sh = (i & 1) * 16;
                const uint32_t lo = ((sa4[i >> 1] >> sh) & 0xffffu) | (((sb4[i >> 1] >> sh) & 0xffffu) << 16);
                const uint32_t hi = ((ba4[i >> 1] >> sh) & 0xffffu) | (((bb4[i >> 1] >> sh) & 0xffffu) << 16);
                *reinterpret_cast<uint2 *>(sbw + (size_t)((g0 + i) * 8 + g) * 8) = make_uint2(lo, hi);
            }
        }
        __syncwarp();
        const uint32_t sbw32 = finch_smem_u32(sbw) + (uint32_t)(g * 8);
        float r[4] = {0.f, 0.f, 0.f, 0.f}, bias[4] = {0.f, 0.f, 0.f, 0.f};
        // DEPTH groups of this warp's rows are on their way while one is multiplied: with 24 warps on an SM that is
        // about 100 KB of loads in flight, what the HBM latency asks for
        constexpr int DEPTH = BITS == 8 ? 4 : 8;
        uint32_t qa[DEPTH][BITS == 8 ? 4 : 2], qb[DEPTH][BITS == 8 ? 4 : 2];
        auto load = [&](int gr, int j) {
            if (BITS == 8) {
                const uint4 u = __ldg(reinterpret_cast<const uint4 *>(wA + (size_t)gr * 64)), v = __ldg(reinterpret_cast<const uint4 *>(wB + (size_t)gr * 64));
                qa[j][0] = u.x; qa[j][1] = u.y; qa[j][BITS == 8 ? 2 : 0] = u.z; qa[j][BITS == 8 ? 3 : 1] = u.w;
                qb[j][0] = v.x; qb[j][1] = v.y; qb[j][BITS == 8 ? 2 : 0] = v.z; qb[j][BITS == 8 ? 3 : 1] = v.w;
            } else {
                const uint2 u = __ldg(reinterpret_cast<const uint2 *>(wA + (size_t)gr * 32)), v = __ldg(reinterpret_cast<const uint2 *>(wB + (size_t)gr * 32));
                qa[j][0] = u.x; qa[j][1] = u.y;
                qb[j][0] = v.x; qb[j][1] = v.y;
            }
        };
#pragma unroll
        for (int j = 0; j < DEPTH; j++)
            if (j < NG) load(j, j);
        uint32_t pb = pb0;
        for (int gr0 = 0; gr0 < NG; gr0 += DEPTH) {
#pragma unroll
            for (int j = 0; j < DEPTH; j++) {
                const int gr = gr0 + j;
                if (gr < NG) {
                    uint4 b01, b23;
                    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(b01.x), "=r"(b01.y), "=r"(b01.z), "=r"(b01.w) : "r"(pb));
                    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(b23.x), "=r"(b23.y), "=r"(b23.z), "=r"(b23.w) : "r"(pb + bpair));
                    pb += bstep;
                    const uint32_t bb[8] = {b01.x, b01.y, b01.z, b01.w, b23.x, b23.y, b23.z, b23.w};
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
                    if (BITS == 8) {
#pragma unroll
                        for (int m = 0; m < 4; m++)
                            mma16816s(acc, qa[j][m] & 0x00FF00FFu, qb[j][m] & 0x00FF00FFu, (qa[j][m] >> 8) & 0x00FF00FFu, (qb[j][m] >> 8) & 0x00FF00FFu,
                                      bb[2 * m], bb[2 * m + 1]);
                    } else {
#pragma unroll
                        for (int w2 = 0; w2 < 2; w2++) {
                            const uint32_t ua = qa[j][w2], ub = qb[j][w2], va = ua >> 8, vb = ub >> 8;
                            mma16816s(acc, ua & 0x000F000Fu, ub & 0x000F000Fu, ua & 0x00F000F0u, ub & 0x00F000F0u, bb[4 * w2], bb[4 * w2 + 1]);
                            mma16816s(acc, va & 0x000F000Fu, vb & 0x000F000Fu, va & 0x00F000F0u, vb & 0x00F000F0u, bb[4 * w2 + 2], bb[4 * w2 + 3]);
                        }
                    }
                    uint2 sbv;   // scale of row A | row B << 16, bias likewise
                    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(sbv.x), "=r"(sbv.y) : "r"(sbw32 + (uint32_t)gr * 64u));
                    float s0, s1, b0, b1;
                    finch_widen16x2(sbv.x, FP16S ? FINCH_FP16 : FINCH_BF16, s0, s1);
                    finch_widen16x2(sbv.y, FP16S ? FINCH_FP16 : FINCH_BF16, b0, b1);
                    const float x0 = x0s[gr], x1 = x1s[gr];
                    if (gr + DEPTH < NG) load(gr + DEPTH, j);   // this buffer is free again
                    r[0] = fmaf(s0, acc[0], r[0]);
                    r[1] = fmaf(s0, acc[1], r[1]);
                    r[2] = fmaf(s1, acc[2], r[2]);
                    r[3] = fmaf(s1, acc[3], r[3]);
                    bias[0] = fmaf(b0, x0, bias[0]);
                    bias[1] = fmaf(b0, x1, bias[1]);
                    bias[2] = fmaf(b1, x0, bias[2]);
                    bias[3] = fmaf(b1, x1, bias[3]);
                }
            }
        }
        const int rowA = tile * 16 + g, rowB = rowA + 8;
        const float f0 = pow2b(expo[p0 < M ? p0 : 0] + 17), f1 = pow2b(expo[p1 < M ? p1 : 0] + 17);
        if (HILO) {
            if (p0 < M) {
                if (rowA < a.out_dim) a.out[(size_t)p0 * a.out_dim + rowA] = fmaf(r[0] + r[1] * (1.0f / 2048.0f), f0, bias[0]);
                if (rowB < a.out_dim) a.out[(size_t)p0 * a.out_dim + rowB] = fmaf(r[2] + r[3] * (1.0f / 2048.0f), f0, bias[2]);
            }
        } else {
            if (p0 < M) {
                if (rowA < a.out_dim) a.out[(size_t)p0 * a.out_dim + rowA] = fmaf(r[0], f0, bias[0]);
                if (rowB < a.out_dim) a.out[(size_t)p0 * a.out_dim + rowB] = fmaf(r[2], f0, bias[2]);
            }
            if (p1 < M) {
                if (rowA < a.out_dim) a.out[(size_t)p1 * a.out_dim + rowA] = fmaf(r[1], f1, bias[1]);
                if (rowB < a.out_dim) a.out[(size_t)p1 * a.out_dim + rowB] = fmaf(r[3], f1, bias[3]);
            }
        }
    }
}

template <int BITS, bool HILO, bool FP16S>
int launch_stream(finch_ctx *ctx, cudaStream_t st, const StreamArgs &a, int smem) {
    static std::mutex mu;
    static std::vector<int> done;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (std::find(done.begin(), done.end(), ctx->cfg.device) == done.end()) {
            FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(stream_matvec_kernel<BITS, HILO, FP16S>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024));
            done.push_back(ctx->cfg.device);
        }
    }
    const int tiles = (a.out_dim + 15) / 16;
    int ctas = (tiles + SNT / 32 - 1) / (SNT / 32);
    ctas = std::min(ctas, 3 * ctx->sm_count);
    stream_matvec_kernel<BITS, HILO, FP16S><<<ctas, SNT, smem, st>>>(a);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

}  // namespace

// Returns FINCH_OK after launching, or -1 when the call is not one this kernel takes (the caller then tries the
// other matvec kernels): one affine 4- or 8-bit g64 tensor of at least 32,768 rows (a CTA takes 128 rows: fewer rows
// leave SMs without work, and the row-pair kernel of matvec_fast.cu is faster there), K a multiple of 512 up to 8192,
// 16-byte aligned rows, up to four fp32 or eight bf16 positions per pass (more run as further passes).
int finch_try_stream_matvec(finch_ctx *ctx, cudaStream_t st, const void *x, int x_dtype, const finch_wdesc *specs, float *const *outs, int n, int M) {
    if (n != 1) return -1;
    const finch_wdesc &w = specs[0];
    if ((w.bits != 4 && w.bits != 8) || w.group_size != 64 || w.out_dim < 32768 || w.in_dim % 512 || w.in_dim > SMAXK) return -1;
    if (((uintptr_t)w.scales & 15) || ((uintptr_t)w.biases & 15)) return -1;
    if (((uintptr_t)w.W & 15) || ((size_t)w.in_dim * w.bits / 8) % 16) return -1;
    const bool hilo = x_dtype != FINCH_BF16;
    const int per = hilo ? 4 : 8;
    if (M > 4 * per) return -1;
    const size_t xelt = hilo ? 4 : 2;
    for (int m0 = 0; m0 < M; m0 += per) {
        StreamArgs a{};
        a.W = (const uint8_t *)w.W;
        a.S = (const uint16_t *)w.scales;
        a.B = (const uint16_t *)w.biases;
        a.out = outs[0] + (size_t)m0 * w.out_dim;
        a.x = (const char *)x + (size_t)m0 * w.in_dim * xelt;
        a.x_bf16 = !hilo;
        a.out_dim = w.out_dim;
        a.K = w.in_dim;
        a.M = std::min(per, M - m0);
        a.scale_fp16 = w.scale_dtype == FINCH_FP16;
        const int smem = stream_smem_bytes(a.K, hilo ? 2 * a.M : a.M, a.M);
        if (smem > 100 * 1024) return -1;
        int rc;
        const bool f = a.scale_fp16;
        if (w.bits == 8) rc = hilo ? (f ? launch_stream<8, true, true>(ctx, st, a, smem) : launch_stream<8, true, false>(ctx, st, a, smem))
                                   : (f ? launch_stream<8, false, true>(ctx, st, a, smem) : launch_stream<8, false, false>(ctx, st, a, smem));
        else rc = hilo ? (f ? launch_stream<4, true, true>(ctx, st, a, smem) : launch_stream<4, true, false>(ctx, st, a, smem))
                       : (f ? launch_stream<4, false, true>(ctx, st, a, smem) : launch_stream<4, false, false>(ctx, st, a, smem));
        if (rc) return rc;
    }
    return FINCH_OK;
}
