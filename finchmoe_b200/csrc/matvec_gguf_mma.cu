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
// A CTA of sixteen warps owns 64 rows: four row tiles of 16 rows, each shared by four warps that split the position
// tiles between them (every warp of a tile decodes the same A fragments, which costs little against its MMAs, and
// the SM gets sixteen warps to hide latencies with).  The CTA walks K in super-blocks of 256 values, the activations
// of the block double-buffered in shared memory (cp.async), the packed rows read straight from global memory by the
// lanes that use them, one super-block ahead.  Every weight byte leaves DRAM once per launch whatever the number of
// positions.
#include "finch_internal.cuh"

namespace {

constexpr int GW = 4;            // row tiles (16 rows each) per CTA
// NS (template parameter): warps per row tile, each taking 1 / NS of the position tiles; threads = GW * NS * 32
constexpr int ROWH = 256 + 16;   // halves per position per K block in shared memory (row stride = 8 banks mod 32: conflict-free 64-bit reads)

struct GSpec {
    const uint8_t *W;
    float *out;
    int out_dim;
};
// items != NULL: grouped mode.  Work item blockIdx.y = (expert, first position, positions): the tensor of spec
// blockIdx.z starts at W + slab[spec] * expert, the activations, sums, factors and output rows at `first`.
struct GPack {
    GSpec s[8];
    int n;
    const int4 *items;
    const int *n_items;
    size_t slab[2];
};

// One CTA per position.  xh / xl: [Tp][K] fp16, value k of a row stored at (k & ~3) + {0, 2, 1, 3}[k & 3];
// sx16 / sx32: [K / 16][Tp], [K / 32][Tp] = (sum of x over the sub-block) / F[m]; F[m] = 2^24 / scale(m).
// Grouped mode (src != NULL): position m takes row src[m] of x (identity: row m), or is a padding position when
// src[m] < 0; positions at and beyond *total do nothing.
__global__ void __launch_bounds__(256) gguf_prep_kernel(const void *x, int x_dtype, int T, int Tp, int K, __half *xh, __half *xl, float *sx16, float *sx32,
                                                        float *F, const int *src, int identity, const int *total) {
    __shared__ float red[8];
    __shared__ float s_scale;
    const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (total && m >= *total) return;
    const int srow = src ? src[m] : m;
    const size_t xrow = (size_t)(src && !identity ? (srow < 0 ? 0 : srow) : m);
    auto value = [&](int k) -> float {
        return x_dtype == FINCH_BF16 ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(x)[xrow * K + k] << 16)
                                     : reinterpret_cast<const float *>(x)[xrow * K + k];
    };
    if (m >= T || srow < 0) {   // padding positions: zero operands, nothing is stored for them
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
template <int TYPE, int NT, bool HILO, int NS>
__global__ void __launch_bounds__(GW * NS * 32) gguf_mma_kernel(GPack pack, const __half *xh, const __half *xl, const float *sxs, const float *F, int T, int Tp, int K) {
    extern __shared__ __align__(16) uint8_t sm[];
    constexpr int NP = 8 * NT, GNT = GW * NS * 32;
    constexpr int SUBS = TYPE == 10 ? 8 : 16;          // scale sub-blocks per super-block
    constexpr int PLANE = NP * ROWH * 2;               // bytes of one activation plane of a K block
    constexpr int SXB = SUBS * NP * 4;
    constexpr int BUF = PLANE * (HILO ? 2 : 1) + SXB;
    GSpec sp = pack.s[pack.items ? blockIdx.z : blockIdx.y];
    if (pack.items) {       // CTA-uniform: the whole CTA leaves before any barrier
        if ((int)blockIdx.y >= *pack.n_items) return;
        const int4 it = pack.items[blockIdx.y];
        sp.W += pack.slab[blockIdx.z] * (size_t)it.x;
        sp.out += (size_t)it.y * sp.out_dim;
        xh += (size_t)it.y * K;
        if (HILO) xl += (size_t)it.y * K;
        sxs += it.y;
        F += it.y;
        T = it.z;
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int tile = blockIdx.x * GW + warp / NS, ns = warp % NS;
    constexpr int NTW = NT / NS;                       // position tiles of this warp: ns * NTW .. ns * NTW + NTW - 1
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

    float out[NTW][4];
#pragma unroll
    for (int n = 0; n < NTW; n++) out[n][0] = out[n][1] = out[n][2] = out[n][3] = 0.f;

    // packed rows of one super-block, as this lane uses them (rows g and g + 8 of the tile)
    struct W4 {
        uint4 hd[2];
        uint32_t w[2][4][2];
    } cur4;
    struct W6 {
        uint32_t ql[2][2][2][2], qh[2][2][2], sc[2][4], d[2];
    } cur6;
    auto load4 = [&](int kb, W4 &o) {
        const uint8_t *b0 = sp.W + ((size_t)r0 * nkb + kb) * 144, *b1 = sp.W + ((size_t)r1 * nkb + kb) * 144;
        o.hd[0] = __ldg(reinterpret_cast<const uint4 *>(b0));
        o.hd[1] = __ldg(reinterpret_cast<const uint4 *>(b1));
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                o.w[0][c][h] = __ldg(reinterpret_cast<const uint32_t *>(b0 + 16 + 32 * c + 16 * h + 4 * t));
                o.w[1][c][h] = __ldg(reinterpret_cast<const uint32_t *>(b1 + 16 + 32 * c + 16 * h + 4 * t));
            }
    };
    auto load6 = [&](int kb, W6 &o) {
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint8_t *b = sp.W + ((size_t)(r ? r1 : r0) * nkb + kb) * 210;
#pragma unroll
            for (int hh = 0; hh < 2; hh++)
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    o.ql[r][hh][0][u] = ldg_u16x2(b + 64 * hh + 16 * u + 4 * t);
                    o.ql[r][hh][1][u] = ldg_u16x2(b + 64 * hh + 32 + 16 * u + 4 * t);
                    o.qh[r][hh][u] = ldg_u16x2(b + 128 + 32 * hh + 16 * u + 4 * t);
                }
#pragma unroll
            for (int i = 0; i < 4; i++) o.sc[r][i] = ldg_u16x2(b + 192 + 4 * i);
            o.d[r] = __ldg(reinterpret_cast<const uint16_t *>(b + 208));
        }
    };
    if constexpr (TYPE == 10) load4(0, cur4);
    else load6(0, cur6);

    load_block(0, 0);
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int kb = 0; kb < nkb; kb++) {
        if (kb + 1 < nkb) load_block(kb + 1, (kb + 1) & 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        const uint32_t base = sm32 + (kb & 1) * BUF;
        const uint32_t sx32a = base + PLANE * (HILO ? 2 : 1);

        if constexpr (TYPE == 10) {
            // ---- Q4_K super-block: d, dmin (fp16), 12 bytes of 6-bit scales / mins, 128 bytes of nibbles ----
            const uint4 hd[2] = {cur4.hd[0], cur4.hd[1]};
            uint32_t w[2][4][2];
#pragma unroll
            for (int r = 0; r < 2; r++)
#pragma unroll
                for (int c = 0; c < 4; c++)
#pragma unroll
                    for (int h = 0; h < 2; h++) w[r][c][h] = cur4.w[r][c][h];
            if (kb + 1 < nkb) load4(kb + 1, cur4);      // the next super-block's rows travel while this one is computed
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
                    for (int nn = 0; nn < NTW; nn++) {
                        const int n = ns * NTW + nn;
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
                        out[nn][0] = fmaf(dl[0], acc[0], fmaf(ml[0], sa, out[nn][0]));
                        out[nn][1] = fmaf(dl[0], acc[1], fmaf(ml[0], sb2, out[nn][1]));
                        out[nn][2] = fmaf(dl[1], acc[2], fmaf(ml[1], sa, out[nn][2]));
                        out[nn][3] = fmaf(dl[1], acc[3], fmaf(ml[1], sb2, out[nn][3]));
                    }
                }
            }
        } else {
            // ---- Q6_K super-block (210 bytes, 2-byte aligned): ql[128] low nibbles, qh[64] high bit pairs, 16 int8 scales, d ----
            uint32_t ql[2][2][2][2], qh[2][2][2], sc[2][4];
            float d[2];
#pragma unroll
            for (int r = 0; r < 2; r++) {
#pragma unroll
                for (int hh = 0; hh < 2; hh++)
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        ql[r][hh][0][u] = cur6.ql[r][hh][0][u];
                        ql[r][hh][1][u] = cur6.ql[r][hh][1][u];
                        qh[r][hh][u] = cur6.qh[r][hh][u];
                    }
#pragma unroll
                for (int i = 0; i < 4; i++) sc[r][i] = cur6.sc[r][i];
                d[r] = half_bits_to_float(cur6.d[r]);
            }
            if (kb + 1 < nkb) load6(kb + 1, cur6);      // the next super-block's rows travel while this one is computed
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
                    for (int nn = 0; nn < NTW; nn++) {
                        const int n = ns * NTW + nn;
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
                        out[nn][0] = fmaf(ds[0], acc[0], fmaf(m32[0], sa, out[nn][0]));
                        out[nn][1] = fmaf(ds[0], acc[1], fmaf(m32[0], sb2, out[nn][1]));
                        out[nn][2] = fmaf(ds[1], acc[2], fmaf(m32[1], sa, out[nn][2]));
                        out[nn][3] = fmaf(ds[1], acc[3], fmaf(m32[1], sb2, out[nn][3]));
                    }
                }
            }
        }
        __syncthreads();   // everybody is done with this buffer before the block after next is copied into it
    }
    if (!active) return;
#pragma unroll
    for (int nn = 0; nn < NTW; nn++) {
        const int m0 = 8 * (ns * NTW + nn) + 2 * t, m1 = m0 + 1;
        if (m0 < T) {
            const float f = F[m0];
            if (row0 < sp.out_dim) sp.out[(size_t)m0 * sp.out_dim + row0] = out[nn][0] * f;
            if (row1 < sp.out_dim) sp.out[(size_t)m0 * sp.out_dim + row1] = out[nn][2] * f;
        }
        if (m1 < T) {
            const float f = F[m1];
            if (row0 < sp.out_dim) sp.out[(size_t)m1 * sp.out_dim + row0] = out[nn][1] * f;
            if (row1 < sp.out_dim) sp.out[(size_t)m1 * sp.out_dim + row1] = out[nn][3] * f;
        }
    }
}

template <int TYPE, int NT, bool HILO, int NS>
int launch_gq(finch_ctx *ctx, cudaStream_t st, const GPack &pack, int max_out, const __half *xh, const __half *xl, const float *sxs, const float *F, int T,
              int Tp, int K) {
    constexpr int NP = 8 * NT, SUBS = TYPE == 10 ? 8 : 16;
    constexpr int smem = 2 * (NP * ROWH * 2 * (HILO ? 2 : 1) + SUBS * NP * 4);
    int rc = finch_func_attr_once(ctx, (const void *)gguf_mma_kernel<TYPE, NT, HILO, NS>, smem);
    if (rc) return rc;
    const dim3 grid = pack.items ? dim3((max_out + 16 * GW - 1) / (16 * GW), T /* item bound */, pack.n) : dim3((max_out + 16 * GW - 1) / (16 * GW), pack.n);
    gguf_mma_kernel<TYPE, NT, HILO, NS><<<grid, GW * NS * 32, smem, st>>>(pack, xh, xl, sxs, F, T, Tp, K);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

template <int TYPE>
int launch_type(finch_ctx *ctx, cudaStream_t st, const GPack &pack, int max_out, const __half *xh, const __half *xl, const float *sxs, const float *F, int T,
                int Tp, int K, bool hilo) {
    const int nt = (T + 7) / 8;
    if (hilo) {
        if (nt <= 4) return launch_gq<TYPE, 4, true, 4>(ctx, st, pack, max_out, xh, xl, sxs, F, T, Tp, K);
        return launch_gq<TYPE, 8, true, 4>(ctx, st, pack, max_out, xh, xl, sxs, F, T, Tp, K);
    }
    if (nt <= 4) return launch_gq<TYPE, 4, false, 4>(ctx, st, pack, max_out, xh, nullptr, sxs, F, T, Tp, K);
    if (nt <= 8) return launch_gq<TYPE, 8, false, 4>(ctx, st, pack, max_out, xh, nullptr, sxs, F, T, Tp, K);
    return launch_gq<TYPE, 16, false, 4>(ctx, st, pack, max_out, xh, nullptr, sxs, F, T, Tp, K);
}

}  // namespace

namespace {

int ensure_gq_ws(finch_ctx *ctx, cudaStream_t st, size_t need) {
    if (ctx->gq_ws_bytes >= need) return FINCH_OK;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cap);
    if (cap != cudaStreamCaptureStatusNone)
        return finch_fail(ctx, FINCH_E_UNSUPPORTED, "the GGUF many-position workspace must be sized by one call outside stream capture first");
    if (ctx->gq_ws) {
        cudaStreamSynchronize(st);
        cudaFree(ctx->gq_ws);
        ctx->gq_ws = nullptr;
        ctx->gq_ws_bytes = 0;
    }
    if (cudaMalloc(&ctx->gq_ws, need) != cudaSuccess) {
        cudaGetLastError();
        return finch_fail(ctx, FINCH_E_NOMEM, "GGUF many-position workspace (%zu bytes)", need);
    }
    ctx->gq_ws_bytes = need;
    return FINCH_OK;
}

// ---- grouped expert MLP: the (token, expert) pairs of a chunk sorted by expert, so that an expert's rows leave
// memory once per chunk however many tokens chose it (the reference's pool de-duplication, finchmoe/infer.m:12424-12532).
// One CTA.  An expert's pairs get consecutive positions that start at a multiple of 8 (the padding positions carry
// src = -1).  Work items (expert, first position, positions): at most 32 positions in `small`, chunks of at most
// `cap` in `large`.  counts = {small items, large items, positions used}.
__global__ void __launch_bounds__(1024) gq_sort_kernel(const int32_t *ids, const uint8_t *valid, int P, int Kx, int n_experts, int cap, int *pos_of_pair,
                                                       int *src_tok, int maxpos, int4 *small, int4 *large, int *counts) {
    extern __shared__ int ssm[];
    int *cnt = ssm, *base = ssm + n_experts, *cur = base + n_experts;
    const int tid = threadIdx.x;
    for (int e = tid; e < n_experts; e += 1024) cnt[e] = 0;
    for (int i = tid; i < maxpos; i += 1024) src_tok[i] = -1;
    __syncthreads();
    for (int p = tid; p < P; p += 1024) {
        const int e = ids[p];
        if ((valid && !valid[p]) || e < 0 || e >= n_experts) continue;
        atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int pos = 0, ns = 0, nl = 0;
        for (int e = 0; e < n_experts; e++) {
            base[e] = cur[e] = pos;
            const int c = cnt[e];
            if (c == 0) continue;
            if (c <= 32) small[ns++] = make_int4(e, pos, c, 0);
            else
                for (int o = 0; o < c; o += cap) large[nl++] = make_int4(e, pos + o, c - o < cap ? c - o : cap, 0);
            pos += (c + 7) & ~7;
        }
        counts[0] = ns;
        counts[1] = nl;
        counts[2] = pos;
    }
    __syncthreads();
    for (int p = tid; p < P; p += 1024) {
        const int e = ids[p];
        if ((valid && !valid[p]) || e < 0 || e >= n_experts) {
            pos_of_pair[p] = -1;
            continue;
        }
        const int pos = atomicAdd(&cur[e], 1);     // the order inside an expert's range is arbitrary: a pair's row depends on its own input only
        pos_of_pair[p] = pos;
        src_tok[pos] = p / Kx;
    }
}

__global__ void gq_swiglu_kernel(const float *g, const float *u, float *act, const int *counts, int inter) {
    const size_t n = (size_t)counts[2] * inter;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float gv = g[i];
        act[i] = (gv / (1.0f + expf(-gv))) * u[i];
    }
}

// The reference's guarded combine (finchmoe/infer.m:3334-3347), one CTA of 256 threads per token: the experts whose
// output energy is finite and below 1e20 count, and their weights are renormalised when they sum to less than 0.99.
__global__ void __launch_bounds__(256) gq_combine_kernel(const float *outs, const int *pos_of_pair, const float *weights, int Kx, int hidden,
                                                         const float *h_mid, float *hidden_out) {
    __shared__ float red[8];
    __shared__ float wk[8];
    __shared__ int pk[8];
    __shared__ float total;
    const int tok = blockIdx.x, tid = threadIdx.x;
    if (tid == 0) total = 0.f;
    for (int k = 0; k < Kx; k++) {
        const int pos = pos_of_pair[tok * Kx + k];
        float er = 0.f;
        if (pos >= 0)
            for (int j = tid; j < hidden; j += 256) {
                const float v = outs[(size_t)pos * hidden + j];
                er += v * v;
            }
#pragma unroll
        for (int o = 16; o; o >>= 1) er += __shfl_xor_sync(0xffffffffu, er, o);
        if ((tid & 31) == 0) red[tid >> 5] = er;
        __syncthreads();
        if (tid == 0) {
            float sum = 0.f;
            for (int w = 0; w < 8; w++) sum += red[w];
            const bool ok = pos >= 0 && isfinite(sum) && sum < 1e20f;
            wk[k] = ok ? weights[tok * Kx + k] : 0.f;
            pk[k] = pos;
            if (ok) total += weights[tok * Kx + k];
        }
        __syncthreads();
    }
    const float tw = total, inv = (tw > 0.f && tw < 0.99f) ? 1.0f / tw : 1.0f;
    for (int j = tid; j < hidden; j += 256) {
        float m = 0.f;
        for (int k = 0; k < Kx; k++)
            if (wk[k] != 0.f) m = fmaf(wk[k], outs[(size_t)pk[k] * hidden + j], m);
        hidden_out[(size_t)tok * hidden + j] = (h_mid ? h_mid[(size_t)tok * hidden + j] : 0.f) + m * inv;
    }
}

template <int TYPE>
int launch_items(finch_ctx *ctx, cudaStream_t st, GPack pack, int max_out, const __half *xh, const __half *xl, const float *sxs, const float *F, int Tp, int K,
                 bool hilo, const int4 *small, const int4 *large, const int *counts, int bound_small, int bound_large) {
    int rc;
    pack.items = small;
    pack.n_items = counts;
    if (hilo) rc = launch_gq<TYPE, 4, true, 1>(ctx, st, pack, max_out, xh, xl, sxs, F, bound_small, Tp, K);
    else rc = launch_gq<TYPE, 4, false, 1>(ctx, st, pack, max_out, xh, nullptr, sxs, F, bound_small, Tp, K);
    if (rc) return rc;
    pack.items = large;
    pack.n_items = counts + 1;
    if (hilo) return launch_gq<TYPE, 8, true, 2>(ctx, st, pack, max_out, xh, xl, sxs, F, bound_large, Tp, K);
    return launch_gq<TYPE, 8, false, 2>(ctx, st, pack, max_out, xh, nullptr, sxs, F, bound_large, Tp, K);
}

}  // namespace

// The GGUF expert MLP for a chunk of B tokens (gate, up, SiLU, down, guarded combine), grouped by expert.
int finch_gguf_experts_grouped(finch_ctx *ctx, cudaStream_t st, const finch_gguf_experts *ex, const void *h_post, const int32_t *expert_ids, const float *weights,
                               const uint8_t *valid, const float *h_mid, float *hidden_out, int B) {
    const finch_config &c = ctx->cfg;
    const int H = c.hidden, I = c.moe_inter, Kx = c.top_k, P = B * Kx, E = c.n_experts;
    if (E > 1024) return -1;
    if (((uintptr_t)ex->gate & 15) || ((uintptr_t)ex->up & 15) || ((uintptr_t)ex->down & 15) || (ex->gate_slab & 15) || (ex->up_slab & 15) || (ex->down_slab & 1))
        return -1;
    constexpr int CAP = 64;
    const int maxpos = ((P + 7 * (E < P ? E : P)) + 7) & ~7;            // every touched expert pads its range to a multiple of 8
    const int bound_small = E < P ? E : P, bound_large = P / 33 + 1;   // large items hold at least 33 pairs of one expert... per chunk of CAP: see below
    const int n_large_max = P / CAP + (P / 33 + 1);                     // full chunks + one ragged chunk per expert with more than 32 pairs
    (void)bound_large;
    const int Kmax = H > I ? H : I;
    auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
    const size_t plane = up((size_t)maxpos * Kmax * sizeof(__half)), sx16b = up((size_t)(Kmax / 16) * maxpos * 4), sx32b = up((size_t)(Kmax / 32) * maxpos * 4);
    const size_t fb = up((size_t)maxpos * 4), gib = up((size_t)maxpos * I * 4), ob = up((size_t)maxpos * H * 4);
    const size_t ib = up((size_t)P * 4) + up((size_t)maxpos * 4) + up((size_t)bound_small * 16) + up((size_t)n_large_max * 16) + 256;
    int rc = ensure_gq_ws(ctx, st, 2 * plane + sx16b + sx32b + fb + 3 * gib + ob + ib);
    if (rc) return rc;
    char *w = (char *)ctx->gq_ws;
    auto take = [&](size_t bytes) {
        char *r = w;
        w += bytes;
        return r;
    };
    __half *xh = (__half *)take(plane), *xl = (__half *)take(plane);
    float *sx16 = (float *)take(sx16b), *sx32 = (float *)take(sx32b), *F = (float *)take(fb);
    float *g = (float *)take(gib), *u = (float *)take(gib), *act = (float *)take(gib), *outs = (float *)take(ob);
    int *pos_of_pair = (int *)take(up((size_t)P * 4)), *src_tok = (int *)take(up((size_t)maxpos * 4));
    int4 *small = (int4 *)take(up((size_t)bound_small * 16)), *large = (int4 *)take(up((size_t)n_large_max * 16));
    int *counts = (int *)take(256);

    gq_sort_kernel<<<1, 1024, 3 * E * sizeof(int), st>>>(expert_ids, valid, P, Kx, E, CAP, pos_of_pair, src_tok, maxpos, small, large, counts);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    const bool hilo = c.act_dtype != FINCH_BF16;
    gguf_prep_kernel<<<maxpos, 256, 0, st>>>(h_post, c.act_dtype, maxpos, maxpos, H, xh, hilo ? xl : nullptr, sx16, sx32, F, src_tok, 0, counts + 2);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches += 2;
    // gate and up: one launch pair when their types agree, else one pair each
    for (int which = 0; which < 2; which++) {
        const bool both = ex->gate_type == ex->up_type;
        if (both && which == 1) break;
        GPack pk{};
        pk.n = both ? 2 : 1;
        if (both || which == 0) {
            pk.s[0] = GSpec{(const uint8_t *)ex->gate, g, I};
            pk.slab[0] = ex->gate_slab;
            if (both) {
                pk.s[1] = GSpec{(const uint8_t *)ex->up, u, I};
                pk.slab[1] = ex->up_slab;
            }
        } else {
            pk.s[0] = GSpec{(const uint8_t *)ex->up, u, I};
            pk.slab[0] = ex->up_slab;
        }
        const int type = (both || which == 0) ? ex->gate_type : ex->up_type;
        rc = type == 10 ? launch_items<10>(ctx, st, pk, I, xh, xl, sx32, F, maxpos, H, hilo, small, large, counts, bound_small, n_large_max)
                        : launch_items<11>(ctx, st, pk, I, xh, xl, sx16, F, maxpos, H, hilo, small, large, counts, bound_small, n_large_max);
        if (rc) return rc;
    }
    gq_swiglu_kernel<<<296, 256, 0, st>>>(g, u, act, counts, I);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    gguf_prep_kernel<<<maxpos, 256, 0, st>>>(act, FINCH_F32, maxpos, maxpos, I, xh, xl, sx16, sx32, F, src_tok, 1, counts + 2);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches += 2;
    {
        GPack pk{};
        pk.n = 1;
        pk.s[0] = GSpec{(const uint8_t *)ex->down, outs, H};
        pk.slab[0] = ex->down_slab;
        rc = ex->down_type == 10 ? launch_items<10>(ctx, st, pk, H, xh, xl, sx32, F, maxpos, I, true, small, large, counts, bound_small, n_large_max)
                                 : launch_items<11>(ctx, st, pk, H, xh, xl, sx16, F, maxpos, I, true, small, large, counts, bound_small, n_large_max);
        if (rc) return rc;
    }
    gq_combine_kernel<<<B, 256, 0, st>>>(outs, pos_of_pair, weights, Kx, H, h_mid, hidden_out);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

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
    {
        const int rc = ensure_gq_ws(ctx, st, need);
        if (rc) return rc;
    }
    char *ws = (char *)ctx->gq_ws;
    __half *xh = (__half *)ws, *xl = (__half *)(ws + up(plane));
    float *sx16 = (float *)(ws + 2 * up(plane)), *sx32 = (float *)((char *)sx16 + up(sx16b)), *F = (float *)((char *)sx32 + up(sx32b));
    const size_t xelt = x_dtype == FINCH_BF16 ? 2 : 4;
    for (int m0 = 0; m0 < M; m0 += per) {
        const int T = M - m0 < per ? M - m0 : per;
        const int np = ((T + 7) / 8 <= 4) ? 32 : ((T + 7) / 8 <= 8 ? 64 : 128);     // positions the chosen instantiation reads
        gguf_prep_kernel<<<np, 256, 0, st>>>((const char *)x + (size_t)m0 * K * xelt, x_dtype, T, Tp, K, xh, hilo ? xl : nullptr, sx16, sx32, F, nullptr, 0,
                                             nullptr);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        ctx->launches++;
        GPack pack{};
        pack.n = n;
        for (int i = 0; i < n; i++) pack.s[i] = GSpec{(const uint8_t *)specs[i].W, outs[i] + (size_t)m0 * specs[i].out_dim, specs[i].out_dim};
        const int rc = bits == 10 ? launch_type<10>(ctx, st, pack, max_out, xh, xl, sx32, F, T, Tp, K, hilo)
                                  : launch_type<11>(ctx, st, pack, max_out, xh, xl, sx16, F, T, Tp, K, hilo);
        if (rc) return rc;
    }
    return FINCH_OK;
}
