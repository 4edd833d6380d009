// GGUF Q4_K / Q6_K matrices at 9 .. 128 positions in one pass over the weights (the reference folds the positions of a
// prefill chunk into one dispatch for these tensors: dequant_matvec_qk_prefill, finchmoe/shaders.metal:3372-3440; host
// side finchmoe/infer.m:10958-11165).  out[m][r] = sum over sub-blocks of  dl * (sum q x) - ml * (sum x)  (Q4_K) or
// ds * (sum q x - 32 sum x)  (Q6_K): the same algebra as the reference's row dequantisation (infer.m:1605-1674) with
// the scale applied to fp32 sub-block sums.
//
// The codes never become floats on the CUDA cores: a 4- or 6-bit code isolated at bit 0 of a 16-bit half reads as the
// fp16 subnormal q * 2^-24 and is the A operand of mma.sync.m16n8k16 (fp32 accumulate); the B operand holds the
// activations of up to 128 positions as fp16, scaled per position by a power of two so that they fit (plus a second
// plane with the remainder * 2^11 for fp32 activations), written once by a preparation kernel in the order the
// fragments want.  The k index inside an MMA is free as long as A and B agree, so a lane takes the four bytes of a
// row that it loads (codes 4t .. 4t+3 of a 16-code run) as k = 2t, 2t+8, 2t+1, 2t+9 and the activations are stored
// permuted to match: no shuffles, two logic operations per pair of codes.
//
// A warp owns 16 rows, a CTA of four warps 64; the CTA walks K in super-blocks of 256 values, the activations of the
// block double-buffered in shared memory (cp.async), the packed rows read straight from global memory by the lanes
// that use them.  Every weight byte is read once per launch whatever the number of positions.
#include "finch_internal.cuh"

namespace {

constexpr int GW = 4;            // warps per CTA
constexpr int GNT = GW * 32;
constexpr int ROWH = 256 + 16;   // halves per position per K block in shared memory (row stride = 8 banks mod 32: conflict-free 64-bit reads)

struct GSpec {
    const uint8_t *W;
    float *out;
    int out_dim;
};
struct GPack {
    GSpec s[8];
    int n;
};

// One CTA per position.  xh / xl: [Tp][K] fp16, value k of a row stored at (k & ~3) + {0, 2, 1, 3}[k & 3];
// sx16 / sx32: [K / 16][Tp], [K / 32][Tp] = (sum of x over the sub-block) / F[m]; F[m] = 2^24 / scale(m).
__global__ void __launch_bounds__(256) gguf_prep_kernel(const void *x, int x_dtype, int T, int Tp, int K, __half *xh, __half *xl, float *sx16, float *sx32,
                                                        float *F) {
    __shared__ float red[8];
    __shared__ float s_scale;
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    auto value = [&](int k) -> float {
        return x_dtype == FINCH_BF16 ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(x)[(size_t)m * K + k] << 16)
                                     : reinterpret_cast<const float *>(x)[(size_t)m * K + k];
    };
    if (m >= T) {   // padding positions: zero operands, nothing is stored for them
        for (int k = tid; k < K; k += 256) {
            xh[(size_t)m * K + k] = __float2half(0.f);
            if (xl) xl[(size_t)m * K + k] = __float2half(0.f);
        }
        for (int j = tid; j < K / 16; j += 256) sx16[(size_t)j * Tp + m] = 0.f;
        for (int j = tid; j < K / 32; j += 256) sx32[(size_t)j * Tp + m] = 0.f;
        if (tid == 0) F[m] = 0.f;
        return;
    }
    float mx = 0.f;
    for (int k = tid; k < K; k += 256) {
        const float v = fabsf(value(k));
        mx = v > mx ? v : mx;       // NaN compares false: a NaN input poisons the sums below, not the scale
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float a = 0.f;
        for (int i = 0; i < 8; i++) a = fmaxf(a, red[i]);
        int e = 0;
        if (a > 0.f && a < 3.0e38f) frexpf(a, &e);      // a = f * 2^e, f in [0.5, 1)
        e = e < -100 ? -100 : (e > 100 ? 100 : e);
        s_scale = ldexpf(1.0f, 7 - e);                  // |x * scale| <= 128
        F[m] = ldexpf(1.0f, 17 + e);                    // 2^24 / scale
    }
    __syncthreads();
    const float scale = s_scale, invF = 1.0f / F[m];    // powers of two: exact
    // a thread takes four consecutive values; four threads a 16-value sub-block
    for (int q = tid; q < K / 4; q += 256) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = value(4 * q + i);
        __half h[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float s = v[i] * scale;
            h[i] = __float2half_rn(s);
            l[i] = __float2half_rn((s - __half2float(h[i])) * 2048.0f);
        }
        __half *dh = xh + (size_t)m * K + 4 * q;
        dh[0] = h[0]; dh[1] = h[2]; dh[2] = h[1]; dh[3] = h[3];
        if (xl) {
            __half *dl = xl + (size_t)m * K + 4 * q;
            dl[0] = l[0]; dl[1] = l[2]; dl[2] = l[1]; dl[3] = l[3];
        }
        float s = (v[0] + v[1]) + (v[2] + v[3]);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if ((tid & 3) == 0) sx16[(size_t)(q >> 2) * Tp + m] = s * invF;
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        if ((tid & 7) == 0) sx32[(size_t)(q >> 3) * Tp + m] = s * invF;
    }
}

__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ uint32_t ldg_u16x2(const uint8_t *p) {   // four bytes at a 2-byte aligned address
    const uint16_t *q = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)__ldg(q) | ((uint32_t)__ldg(q + 1) << 16);
}
__device__ __forceinline__ float half_bits_to_float(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)(h & 0xffffu))); }

// TYPE: 10 = Q4_K, 11 = Q6_K.  NT: n-tiles of 8 positions.  HILO: a second activation plane (fp32 inputs).
template <int TYPE, int NT, bool HILO>
__global__ void __launch_bounds__(GNT) gguf_mma_kernel(GPack pack, const __half *xh, const __half *xl, const float *sxs, const float *F, int T, int Tp, int K) {
    extern __shared__ __align__(16) uint8_t sm[];
    constexpr int NP = 8 * NT;
    constexpr int SUBS = TYPE == 10 ? 8 : 16;          // scale sub-blocks per super-block
    constexpr int PLANE = NP * ROWH * 2;               // bytes of one activation plane of a K block
    constexpr int SXB = SUBS * NP * 4;
    constexpr int BUF = PLANE * (HILO ? 2 : 1) + SXB;
    const GSpec sp = pack.s[blockIdx.y];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int tile = blockIdx.x * GW + warp;
    const bool active = tile * 16 < sp.out_dim;        // warp-uniform
    const int row0 = tile * 16 + g, row1 = row0 + 8;
    const int r0 = row0 < sp.out_dim ? row0 : sp.out_dim - 1, r1 = row1 < sp.out_dim ? row1 : sp.out_dim - 1;   // rows past the end repeat the last one
    const int nkb = K / 256;
    const uint32_t sm32 = finch_smem_u32(sm);

    auto load_block = [&](int kb, int buf) {
        const uint32_t base = sm32 + buf * BUF;
        // activation rows: 512 bytes per position and plane
        for (int i = tid; i < NP * 32; i += GNT) {
            const int p = i >> 5, ch = i & 31;
            cp_async16(base + (p * ROWH + ch * 8) * 2, xh + (size_t)p * K + kb * 256 + ch * 8);
            if (HILO) cp_async16(base + PLANE + (p * ROWH + ch * 8) * 2, xl + (size_t)p * K + kb * 256 + ch * 8);
        }
        // sub-block sums: SUBS rows of NP floats (Tp >= NP, rows of the table are Tp apart)
        for (int i = tid; i < SUBS * (NP / 4); i += GNT) {
            const int s = i / (NP / 4), ch = i - s * (NP / 4);
            cp_async16(base + PLANE * (HILO ? 2 : 1) + (s * NP + ch * 4) * 4, sxs + (size_t)(kb * SUBS + s) * Tp + ch * 4);
        }
    };

    float out[NT][4];
#pragma unroll
    for (int n = 0; n < NT; n++) out[n][0] = out[n][1] = out[n][2] = out[n][3] = 0.f;

    load_block(0, 0);
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int kb = 0; kb < nkb; kb++) {
        if (kb + 1 < nkb) load_block(kb + 1, (kb + 1) & 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const uint32_t base = sm32 + (kb & 1) * BUF;
        const uint32_t sx32a = base + PLANE * (HILO ? 2 : 1);

        if constexpr (TYPE == 10) {
            // ---- Q4_K super-block: d, dmin (fp16), 12 bytes of 6-bit scales / mins, 128 bytes of nibbles ----
            uint4 hd[2];
            uint32_t w[2][4][2];
            {
                const uint8_t *b0 = sp.W + ((size_t)r0 * nkb + kb) * 144, *b1 = sp.W + ((size_t)r1 * nkb + kb) * 144;
                hd[0] = __ldg(reinterpret_cast<const uint4 *>(b0));
                hd[1] = __ldg(reinterpret_cast<const uint4 *>(b1));
#pragma unroll
                for (int c = 0; c < 4; c++)
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        w[0][c][h] = __ldg(reinterpret_cast<const uint32_t *>(b0 + 16 + 32 * c + 16 * h + 4 * t));
                        w[1][c][h] = __ldg(reinterpret_cast<const uint32_t *>(b1 + 16 + 32 * c + 16 * h + 4 * t));
                    }
            }
            asm volatile("cp.async.wait_group 1;" ::: "memory");
            __syncthreads();
            if (active) {
                float d[2], dmin[2];
#pragma unroll
                for (int r = 0; r < 2; r++) {
                    d[r] = half_bits_to_float(hd[r].x);
                    dmin[r] = half_bits_to_float(hd[r].x >> 16);
                }
#pragma unroll
                for (int j = 0; j < 8; j++) {            // sub-block j: values 32 j .. 32 j + 31
                    const int c = j >> 1, sb = j & 1;
                    float dl[2], ml[2];
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        auto byte = [&](int i) -> uint32_t { return ((i < 4 ? hd[r].y : i < 8 ? hd[r].z : hd[r].w) >> (8 * (i & 3))) & 255u; };
                        uint32_t sc, mn;
                        if (j < 4) {
                            sc = byte(j) & 63u;
                            mn = byte(j + 4) & 63u;
                        } else {
                            sc = (byte(j + 4) & 15u) | ((byte(j - 4) >> 6) << 4);
                            mn = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
                        }
                        dl[r] = d[r] * (float)sc;
                        ml[r] = -(dmin[r] * (float)mn);
                    }
                    uint32_t a[2][4];
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        a[h][0] = (w[0][c][h] >> (4 * sb)) & 0x000F000Fu;
                        a[h][1] = (w[1][c][h] >> (4 * sb)) & 0x000F000Fu;
                        a[h][2] = (w[0][c][h] >> (4 * sb + 8)) & 0x000F000Fu;
                        a[h][3] = (w[1][c][h] >> (4 * sb + 8)) & 0x000F000Fu;
                    }
#pragma unroll
                    for (int n = 0; n < NT; n++) {
                        float acc[4] = {0.f, 0.f, 0.f, 0.f};
                        float accl[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const int s16 = 4 * c + 2 * sb + h;     // the 16-value run inside the super-block
                            uint32_t b0, b1;
                            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(base + ((8 * n + g) * ROWH + 16 * s16 + 4 * t) * 2));
                            mma_f16(acc, a[h][0], a[h][1], a[h][2], a[h][3], b0, b1);
                            if (HILO) {
                                asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(base + PLANE + ((8 * n + g) * ROWH + 16 * s16 + 4 * t) * 2));
                                mma_f16(accl, a[h][0], a[h][1], a[h][2], a[h][3], b0, b1);
                            }
                        }
                        float sa, sb2;
                        asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(sa), "=f"(sb2) : "r"(sx32a + (j * NP + 8 * n + 2 * t) * 4));
                        if (HILO) {
#pragma unroll
                            for (int i = 0; i < 4; i++) acc[i] = fmaf(accl[i], 1.0f / 2048.0f, acc[i]);
                        }
                        out[n][0] = fmaf(dl[0], acc[0], fmaf(ml[0], sa, out[n][0]));
                        out[n][1] = fmaf(dl[0], acc[1], fmaf(ml[0], sb2, out[n][1]));
                        out[n][2] = fmaf(dl[1], acc[2], fmaf(ml[1], sa, out[n][2]));
                        out[n][3] = fmaf(dl[1], acc[3], fmaf(ml[1], sb2, out[n][3]));
                    }
                }
            }
        } else {
            // ---- Q6_K super-block (210 bytes, 2-byte aligned): ql[128] low nibbles, qh[64] high bit pairs, 16 int8 scales, d ----
            uint32_t ql[2][2][2][2], qh[2][2][2], sc[2][4];
            float d[2];
#pragma unroll
            for (int r = 0; r < 2; r++) {
                const uint8_t *b = sp.W + ((size_t)(r ? r1 : r0) * nkb + kb) * 210;
#pragma unroll
                for (int hh = 0; hh < 2; hh++)
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        ql[r][hh][0][u] = ldg_u16x2(b + 64 * hh + 16 * u + 4 * t);
                        ql[r][hh][1][u] = ldg_u16x2(b + 64 * hh + 32 + 16 * u + 4 * t);
                        qh[r][hh][u] = ldg_u16x2(b + 128 + 32 * hh + 16 * u + 4 * t);
                    }
#pragma unroll
                for (int i = 0; i < 4; i++) sc[r][i] = ldg_u16x2(b + 192 + 4 * i);
                d[r] = half_bits_to_float(__ldg(reinterpret_cast<const uint16_t *>(b + 208)));
            }
            asm volatile("cp.async.wait_group 1;" ::: "memory");
            __syncthreads();
            if (active) {
#pragma unroll
                for (int s16 = 0; s16 < 16; s16++) {     // values 16 s16 .. 16 s16 + 15: one scale each
                    const int hh = s16 >> 3, q = (s16 >> 1) & 3, u = s16 & 1;
                    float ds[2], m32[2];
                    uint32_t cb[2];
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        const int sv = (int)(signed char)((sc[r][s16 >> 2] >> (8 * (s16 & 3))) & 255u);
                        ds[r] = d[r] * (float)sv;
                        m32[r] = -32.0f * ds[r];
                        cb[r] = ((ql[r][hh][q & 1][u] >> (4 * (q >> 1))) & 0x0F0F0F0Fu) | (((qh[r][hh][u] >> (2 * q)) & 0x03030303u) << 4);
                    }
                    const uint32_t a0 = cb[0] & 0x00FF00FFu, a1 = cb[1] & 0x00FF00FFu, a2 = (cb[0] >> 8) & 0x00FF00FFu, a3 = (cb[1] >> 8) & 0x00FF00FFu;
#pragma unroll
                    for (int n = 0; n < NT; n++) {
                        float acc[4] = {0.f, 0.f, 0.f, 0.f};
                        uint32_t b0, b1;
                        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(base + ((8 * n + g) * ROWH + 16 * s16 + 4 * t) * 2));
                        mma_f16(acc, a0, a1, a2, a3, b0, b1);
                        if (HILO) {
                            float accl[4] = {0.f, 0.f, 0.f, 0.f};
                            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(b0), "=r"(b1) : "r"(base + PLANE + ((8 * n + g) * ROWH + 16 * s16 + 4 * t) * 2));
                            mma_f16(accl, a0, a1, a2, a3, b0, b1);
#pragma unroll
                            for (int i = 0; i < 4; i++) acc[i] = fmaf(accl[i], 1.0f / 2048.0f, acc[i]);
                        }
                        float sa, sb2;
                        asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(sa), "=f"(sb2) : "r"(sx32a + (s16 * NP + 8 * n + 2 * t) * 4));
                        out[n][0] = fmaf(ds[0], acc[0], fmaf(m32[0], sa, out[n][0]));
                        out[n][1] = fmaf(ds[0], acc[1], fmaf(m32[0], sb2, out[n][1]));
                        out[n][2] = fmaf(ds[1], acc[2], fmaf(m32[1], sa, out[n][2]));
                        out[n][3] = fmaf(ds[1], acc[3], fmaf(m32[1], sb2, out[n][3]));
                    }
                }
            }
        }
        __syncthreads();   // everybody is done with this buffer before the block after next is copied into it
    }
    if (!active) return;
#pragma unroll
    for (int n = 0; n < NT; n++) {
        const int m0 = 8 * n + 2 * t, m1 = m0 + 1;
        if (m0 < T) {
            const float f = F[m0];
            if (row0 < sp.out_dim) sp.out[(size_t)m0 * sp.out_dim + row0] = out[n][0] * f;
            if (row1 < sp.out_dim) sp.out[(size_t)m0 * sp.out_dim + row1] = out[n][2] * f;
        }
        if (m1 < T) {
            const float f = F[m1];
            if (row0 < sp.out_dim) sp.out[(size_t)m1 * sp.out_dim + row0] = out[n][1] * f;
            if (row1 < sp.out_dim) sp.out[(size_t)m1 * sp.out_dim + row1] = out[n][3] * f;
        }
    }
}

template <int TYPE, int NT, bool HILO>
int launch_gq(finch_ctx *ctx, cudaStream_t st, const GPack &pack, int max_out, const __half *xh, const __half *xl, const float *sxs, const float *F, int T,
              int Tp, int K) {
    constexpr int NP = 8 * NT, SUBS = TYPE == 10 ? 8 : 16;
    constexpr int smem = 2 * (NP * ROWH * 2 * (HILO ? 2 : 1) + SUBS * NP * 4);
    int rc = finch_func_attr_once(ctx, (const void *)gguf_mma_kernel<TYPE, NT, HILO>, smem);
    if (rc) return rc;
    gguf_mma_kernel<TYPE, NT, HILO><<<dim3((max_out + 16 * GW - 1) / (16 * GW), pack.n), GNT, smem, st>>>(pack, xh, xl, sxs, F, T, Tp, K);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

template <int TYPE>
int launch_type(finch_ctx *ctx, cudaStream_t st, const GPack &pack, int max_out, const __half *xh, const __half *xl, const float *sxs, const float *F, int T,
                int Tp, int K, bool hilo) {
    const int nt = (T + 7) / 8;
    if (hilo) {
        if (nt <= 4) return launch_gq<TYPE, 4, true>(ctx, st, pack, max_out, xh, xl, sxs, F, T, Tp, K);
        return launch_gq<TYPE, 8, true>(ctx, st, pack, max_out, xh, xl, sxs, F, T, Tp, K);
    }
    if (nt <= 4) return launch_gq<TYPE, 4, false>(ctx, st, pack, max_out, xh, nullptr, sxs, F, T, Tp, K);
    if (nt <= 8) return launch_gq<TYPE, 8, false>(ctx, st, pack, max_out, xh, nullptr, sxs, F, T, Tp, K);
    return launch_gq<TYPE, 16, false>(ctx, st, pack, max_out, xh, nullptr, sxs, F, T, Tp, K);
}

}  // namespace

// Returns FINCH_OK after launching, an error code, or -1 when the call is not one this kernel takes.
int finch_try_gguf_mma(finch_ctx *ctx, cudaStream_t st, const void *x, int x_dtype, const finch_wdesc *specs, float *const *outs, int n, int M) {
    if (M < 9 || n > 8) return -1;
    const int bits = specs[0].bits, K = specs[0].in_dim;
    if ((bits != 10 && bits != 11) || K % 256) return -1;
    int max_out = 0;
    for (int i = 0; i < n; i++) {
        if (specs[i].bits != bits || specs[i].in_dim != K) return -1;
        if ((uintptr_t)specs[i].W & (bits == 10 ? 15 : 1)) return -1;     // Q4_K super-blocks are read with 16-byte loads
        max_out = max_out > specs[i].out_dim ? max_out : specs[i].out_dim;
    }
    const bool hilo = x_dtype != FINCH_BF16;
    const int per = hilo ? 64 : 128;                         // positions per pass (two planes need twice the shared memory)
    const int Tp = per;
    // scratch: activation planes, sub-block sums, position factors
    const size_t plane = (size_t)Tp * K * sizeof(__half), sx16b = (size_t)(K / 16) * Tp * 4, sx32b = (size_t)(K / 32) * Tp * 4;
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t need = up(plane) * 2 + up(sx16b) + up(sx32b) + up((size_t)Tp * 4);
    if (ctx->gq_ws_bytes < need) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(st, &cap);
        if (cap != cudaStreamCaptureStatusNone)
            return finch_fail(ctx, FINCH_E_UNSUPPORTED, "the GGUF batched-matvec workspace must be sized by one call outside stream capture first");
        if (ctx->gq_ws) {
            cudaStreamSynchronize(st);
            cudaFree(ctx->gq_ws);
            ctx->gq_ws = nullptr;
            ctx->gq_ws_bytes = 0;
        }
        if (cudaMalloc(&ctx->gq_ws, need) != cudaSuccess) {
            cudaGetLastError();
            return finch_fail(ctx, FINCH_E_NOMEM, "GGUF batched-matvec workspace (%zu bytes)", need);
        }
        ctx->gq_ws_bytes = need;
    }
    char *ws = (char *)ctx->gq_ws;
    __half *xh = (__half *)ws, *xl = (__half *)(ws + up(plane));
    float *sx16 = (float *)(ws + 2 * up(plane)), *sx32 = (float *)((char *)sx16 + up(sx16b)), *F = (float *)((char *)sx32 + up(sx32b));
    const size_t xelt = x_dtype == FINCH_BF16 ? 2 : 4;
    for (int m0 = 0; m0 < M; m0 += per) {
        const int T = M - m0 < per ? M - m0 : per;
        const int np = ((T + 7) / 8 <= 4) ? 32 : ((T + 7) / 8 <= 8 ? 64 : 128);     // positions the chosen instantiation reads
        gguf_prep_kernel<<<np, 256, 0, st>>>((const char *)x + (size_t)m0 * K * xelt, x_dtype, T, Tp, K, xh, hilo ? xl : nullptr, sx16, sx32, F);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        ctx->launches++;
        GPack pack;
        pack.n = n;
        for (int i = 0; i < n; i++) pack.s[i] = GSpec{(const uint8_t *)specs[i].W, outs[i] + (size_t)m0 * specs[i].out_dim, specs[i].out_dim};
        const int rc = bits == 10 ? launch_type<10>(ctx, st, pack, max_out, xh, xl, sx32, F, T, Tp, K, hilo)
                                  : launch_type<11>(ctx, st, pack, max_out, xh, xl, sx16, F, T, Tp, K, hilo);
        if (rc) return rc;
    }
    return FINCH_OK;
}
