// Streaming quantized matvec for 1..8 positions: 3-, 4- and 8-bit affine g64 and GGUF Q4_K / Q6_K tensors in the
// reference's own layouts (dequant_matvec_3bit / _4bit_v3 / dequant_matvec_qk, finchmoe/shaders.metal:
// 544-612, 374-463, 3216-3299; cpu twins finchmoe/infer.m:1660-1763).
//
//   out[m][r] = sum_g  s_rg * (sum_{k in g} q_rk x_mk)  +  b_rg * (sum_{k in g} x_mk)
//
// The codes never become integers: one AND isolates a code at bits [p, p+4) of a 16-bit half, which read
// as fp16 is the subnormal q * 2^(p-24); the half -> float widening is exact, and the activations are
// staged once per CTA in shared memory pre-multiplied by 2^(24-p) of their position (exact), so a plain
// FFMA accumulates q * x in fp32.  Scale and bias are applied once per 32-value chunk to fp32 sums.
// A warp streams two rows at a time with 16-byte (12-byte for 3-bit) loads per lane, 32 values per lane,
// so every load instruction covers 512 (384) contiguous bytes of a row; the pre-scaled activations are laid
// out so that the lanes' float4 reads are conflict-free.  The format-generic kernel (matvec_generic.cu)
// stays the fallback for the other tiers, larger batches and rows that do not fit shared memory.
#include "finch_internal.cuh"

namespace {

struct FSpec {
    const uint8_t *W;
    const uint16_t *S, *B;
    float *out;
    int out_dim, scale_dtype;
    // stacked expert slabs (GGUF ffn_*_exps): the tensor starts at W + slab * ids[id_index] and the spec is
    // skipped when that id is negative, out of range or masked; eid == NULL: W as given
    const int32_t *eid;
    const uint8_t *evalid;
    int id_index, n_ids;
    size_t slab;
    size_t x_off;   // first activation element of this spec inside x (specs of one launch may have different inputs)
};
struct FPack {
    FSpec s[16];
    int n;
};

constexpr int FM = 8;        // positions per launch
constexpr int FNT = 512;     // threads per CTA

// bit position, inside its 16-bit half, of code i (0..31) of the 3-bit period after the 18 masks of decode_chunk<3>
__device__ __forceinline__ int pos3_of(int i) { return (3 * i) & 7; }

__device__ __forceinline__ float h_lo(uint32_t r) { return __low2float(*reinterpret_cast<const __half2 *>(&r)); }
__device__ __forceinline__ float h_hi(uint32_t r) { return __high2float(*reinterpret_cast<const __half2 *>(&r)); }

// Packed words of one 32-code chunk of a row (loaded one iteration ahead of their use).
template <int BITS>
struct Raw {
    uint32_t w[BITS == 4 ? 4 : BITS == 3 ? 3 : (BITS == 10 || BITS == 8) ? 8 : 16];
};
template <int BITS>
__device__ __forceinline__ Raw<BITS> load_raw(const FSpec &sp, size_t row, int K, int c);
// 32 consecutive codes of one row -> qf[32] = q * 2^(p-24), plus the chunk's scale and bias.
template <int BITS>
__device__ __forceinline__ void decode_chunk(const FSpec &sp, size_t row, int K, int c, const Raw<BITS> &raw, float (&qf)[32], float &s, float &b);

template <>
__device__ __forceinline__ Raw<4> load_raw<4>(const FSpec &sp, size_t row, int K, int c) {
    const uint4 v = __ldg(reinterpret_cast<const uint4 *>(sp.W + row * (size_t)(K / 2)) + c);
    return Raw<4>{{v.x, v.y, v.z, v.w}};
}
template <>
__device__ __forceinline__ Raw<3> load_raw<3>(const FSpec &sp, size_t row, int K, int c) {
    const uint32_t *p = reinterpret_cast<const uint32_t *>(sp.W + row * (size_t)(K * 3 / 8)) + 3 * c;
    return Raw<3>{{__ldg(p), __ldg(p + 1), __ldg(p + 2)}};
}
template <>
__device__ __forceinline__ Raw<10> load_raw<10>(const FSpec &sp, size_t row, int K, int c) {
    const uint8_t *blk = sp.W + (row * (size_t)(K / 256) + (c >> 3)) * 144;
    const uint4 *q = reinterpret_cast<const uint4 *>(blk + 16 + 32 * ((c & 7) >> 1));
    const uint4 a = __ldg(q), bb = __ldg(q + 1);
    return Raw<10>{{a.x, a.y, a.z, a.w, bb.x, bb.y, bb.z, bb.w}};
}

template <>
__device__ __forceinline__ void decode_chunk<4>(const FSpec &sp, size_t row, int K, int c, const Raw<4> &raw, float (&qf)[32], float &s, float &b) {
    const uint32_t (&w)[4] = raw.w;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t x = w[i] >> 8;
        const uint32_t e0 = w[i] & 0x000F000Fu, e1 = w[i] & 0x00F000F0u, e2 = x & 0x000F000Fu, e3 = x & 0x00F000F0u;
        qf[8 * i + 0] = h_lo(e0); qf[8 * i + 4] = h_hi(e0);
        qf[8 * i + 1] = h_lo(e1); qf[8 * i + 5] = h_hi(e1);
        qf[8 * i + 2] = h_lo(e2); qf[8 * i + 6] = h_hi(e2);
        qf[8 * i + 3] = h_lo(e3); qf[8 * i + 7] = h_hi(e3);
    }
    const size_t g = row * (size_t)(K / 64) + (c >> 1);
    s = finch_widen16(__ldg(sp.S + g), sp.scale_dtype);
    b = finch_widen16(__ldg(sp.B + g), sp.scale_dtype);
}

template <>
__device__ __forceinline__ void decode_chunk<3>(const FSpec &sp, size_t row, int K, int c, const Raw<3> &raw, float (&qf)[32], float &s, float &b) {
    constexpr int IDX[36] = {0, 6, 1, 7, 2, -1, 3, 8, 4, 9, 5, 10, 11, 16, 12, 17, 13, 18,
                             14, 19, 15, 20, -1, 21, 22, 27, 23, 28, -1, 29, 24, 30, 25, 31, 26, -1};
    const uint32_t w0 = raw.w[0], w1 = raw.w[1], w2 = raw.w[2];
    const uint32_t v1 = __funnelshift_r(w0, w1, 8), v3 = __funnelshift_r(w1, w2, 8), v5 = w2 >> 8;
    uint32_t e[18];
    e[0] = w0 & 0x001C0007u;  e[1] = w0 & 0x00E00038u;  e[2] = w0 & 0x000001C0u;
    e[3] = v1 & 0x0007000Eu;  e[4] = v1 & 0x00380070u;  e[5] = v1 & 0x01C00380u;
    e[6] = w1 & 0x0007000Eu;  e[7] = w1 & 0x00380070u;  e[8] = w1 & 0x01C00380u;
    e[9] = v3 & 0x000E001Cu;  e[10] = v3 & 0x007000E0u; e[11] = v3 & 0x03800000u;
    e[12] = w2 & 0x000E001Cu; e[13] = w2 & 0x007000E0u; e[14] = w2 & 0x03800000u;
    e[15] = v5 & 0x001C0007u; e[16] = v5 & 0x00E00038u; e[17] = v5 & 0x000001C0u;
#pragma unroll
    for (int k = 0; k < 36; k++) {
        if (IDX[k] < 0) continue;
        qf[IDX[k]] = (k & 1) ? h_hi(e[k >> 1]) : h_lo(e[k >> 1]);
    }
    const size_t g = row * (size_t)(K / 64) + (c >> 1);
    s = finch_widen16(__ldg(sp.S + g), sp.scale_dtype);
    b = finch_widen16(__ldg(sp.B + g), sp.scale_dtype);
}

template <>
__device__ __forceinline__ Raw<8> load_raw<8>(const FSpec &sp, size_t row, int K, int c) {
    const uint4 *q = reinterpret_cast<const uint4 *>(sp.W + row * (size_t)K) + 2 * c;
    const uint4 a = __ldg(q), bb = __ldg(q + 1);
    return Raw<8>{{a.x, a.y, a.z, a.w, bb.x, bb.y, bb.z, bb.w}};
}
// 8-bit affine g64 (dequant_matvec_8bit, finchmoe/shaders.metal:473-533): a byte at bits [0, 8) of a half is the fp16
// subnormal q * 2^-24 as well.
template <>
__device__ __forceinline__ void decode_chunk<8>(const FSpec &sp, size_t row, int K, int c, const Raw<8> &raw, float (&qf)[32], float &s, float &b) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t e0 = raw.w[i] & 0x00FF00FFu, e1 = (raw.w[i] >> 8) & 0x00FF00FFu;   // bytes (0, 2) and (1, 3)
        qf[4 * i + 0] = h_lo(e0); qf[4 * i + 2] = h_hi(e0);
        qf[4 * i + 1] = h_lo(e1); qf[4 * i + 3] = h_hi(e1);
    }
    const size_t g = row * (size_t)(K / 64) + (c >> 1);
    s = finch_widen16(__ldg(sp.S + g), sp.scale_dtype);
    b = finch_widen16(__ldg(sp.B + g), sp.scale_dtype);
}

// GGUF Q4_K: 144-byte block of 256 values = d, dmin (fp16), 12 bytes of 6-bit (scale, min) x 8, 128 nibble
// bytes; chunk c = sub-block j of block c / 8: 32 bytes, low nibbles for even j, high nibbles for odd j
// (get_scale_min_k4 and gguf_dequant_row, finchmoe/infer.m:1595-1630).
template <>
__device__ __forceinline__ void decode_chunk<10>(const FSpec &sp, size_t row, int K, int c, const Raw<10> &raw, float (&qf)[32], float &s, float &b) {
    const uint8_t *blk = sp.W + (row * (size_t)(K / 256) + (c >> 3)) * 144;
    const int j = c & 7, hi = j & 1;
    const uint32_t (&w)[8] = raw.w;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t x = hi ? (w[i] >> 4) : w[i];
        const uint32_t e0 = x & 0x000F000Fu, e1 = (x >> 8) & 0x000F000Fu;   // bytes (0, 2) and (1, 3), all at p = 0
        qf[4 * i + 0] = h_lo(e0); qf[4 * i + 2] = h_hi(e0);
        qf[4 * i + 1] = h_lo(e1); qf[4 * i + 3] = h_hi(e1);
    }
    const uint32_t hd = __ldg(reinterpret_cast<const uint32_t *>(blk));
    const float d = h_lo(hd), dmin = h_hi(hd);
    const uint32_t s0 = __ldg(reinterpret_cast<const uint32_t *>(blk + 4)), s1 = __ldg(reinterpret_cast<const uint32_t *>(blk + 8)),
                   s2 = __ldg(reinterpret_cast<const uint32_t *>(blk + 12));
    auto byte_of = [&](int i) -> unsigned { return ((i < 4 ? s0 : i < 8 ? s1 : s2) >> (8 * (i & 3))) & 255u; };
    unsigned sc, mn;
    if (j < 4) {
        sc = byte_of(j) & 63u;
        mn = byte_of(j + 4) & 63u;
    } else {
        sc = (byte_of(j + 4) & 0x0fu) | ((byte_of(j - 4) >> 6) << 4);
        mn = (byte_of(j + 4) >> 4) | ((byte_of(j) >> 6) << 4);
    }
    s = d * (float)sc;
    b = -(dmin * (float)mn);
}

// GGUF Q6_K: 210-byte block of 256 values = ql[128] (low nibbles), qh[64] (two high bits), int8 scales[16], d (fp16);
// blocks are only 2-byte aligned.  Chunk c = quarter qd of half h of block c / 8: value l (0..31) has its nibble in
// ql[64 h + 32 (qd & 1) + l] (high nibble for qd >= 2), its high bits at 2 qd of qh[32 h + l], q = nibble + 16 * high - 32,
// scale index 8 h + 2 qd + l / 16 (gguf_dequant_row, finchmoe/infer.m:1631-1657).  Eight aligned words plus one, shifted
// by 16 bits where the run starts on an odd half-word.
__device__ __forceinline__ void load8_unaligned(const uint8_t *a, uint32_t *out) {
    const uint32_t *p = reinterpret_cast<const uint32_t *>((uintptr_t)a & ~(uintptr_t)3);
    const bool odd = ((uintptr_t)a & 2) != 0;
    uint32_t t[9];
#pragma unroll
    for (int i = 0; i < 9; i++) t[i] = __ldg(p + i);
#pragma unroll
    for (int i = 0; i < 8; i++) out[i] = odd ? __funnelshift_r(t[i], t[i + 1], 16) : t[i];
}
template <>
__device__ __forceinline__ Raw<11> load_raw<11>(const FSpec &sp, size_t row, int K, int c) {
    const uint8_t *blk = sp.W + (row * (size_t)(K / 256) + (c >> 3)) * 210;
    const int j = c & 7, h = j >> 2, qd = j & 3;
    Raw<11> r;
    load8_unaligned(blk + 64 * h + 32 * (qd & 1), r.w);
    load8_unaligned(blk + 128 + 32 * h, r.w + 8);
    return r;
}
// qf as for the other formats (q in 0..63, without the -32); s_lo / s_hi: d * scale of values 0..15 / 16..31.
__device__ __forceinline__ void decode_chunk6(const FSpec &sp, size_t row, int K, int c, const Raw<11> &raw, float (&qf)[32], float &s_lo, float &s_hi) {
    const uint8_t *blk = sp.W + (row * (size_t)(K / 256) + (c >> 3)) * 210;
    const int j = c & 7, h = j >> 2, qd = j & 3;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t x = qd >= 2 ? (raw.w[i] >> 4) : raw.w[i], y = raw.w[8 + i] >> (2 * qd);
        const uint32_t e0 = x & 0x000F000Fu, e1 = (x >> 8) & 0x000F000Fu, f0 = y & 0x00030003u, f1 = (y >> 8) & 0x00030003u;
        qf[4 * i + 0] = fmaf(h_lo(f0), 16.0f, h_lo(e0)); qf[4 * i + 2] = fmaf(h_hi(f0), 16.0f, h_hi(e0));
        qf[4 * i + 1] = fmaf(h_lo(f1), 16.0f, h_lo(e1)); qf[4 * i + 3] = fmaf(h_hi(f1), 16.0f, h_hi(e1));
    }
    const uint32_t dd = __ldg(reinterpret_cast<const uint16_t *>(blk + 208));
    const uint32_t sc = __ldg(reinterpret_cast<const uint16_t *>(blk + 192 + 8 * h + 2 * qd));
    const float d = h_lo(dd);
    s_lo = d * (float)(int)(signed char)(sc & 255u);
    s_hi = d * (float)(int)(signed char)(sc >> 8);
}

template <int BITS>
__device__ __forceinline__ float prescale_of(int k) {
    if (BITS == 4) return __uint_as_float((uint32_t)(127 + ((k & 1) ? 20 : 24)) << 23);
    if (BITS == 3) return __uint_as_float((uint32_t)(127 + 24 - pos3_of(k & 31)) << 23);
    return __uint_as_float((uint32_t)(127 + 24) << 23);
}

// grid: (CTAs, specs); block 512.  Shared memory: xs[M][Kp] pre-scaled and permuted, sx[M][Kp / 32].
template <int BITS>
struct Depth {
    static constexpr int value = BITS == 11 ? 1 : 3;   // row-pair chunks whose packed words are in flight ahead of the one being computed
};

template <int BITS, int MT>
__global__ void __launch_bounds__(FNT, 1) fast_matvec_kernel(FPack pack, const void *x, int x_dtype, int M, int K) {
    extern __shared__ __align__(16) float fsm[];
    FSpec sp = pack.s[blockIdx.y];
    if (sp.eid) {
        const int e = sp.eid[sp.id_index];
        if (e < 0 || e >= sp.n_ids || (sp.evalid && !sp.evalid[sp.id_index])) return;   // whole CTA: uniform
        sp.W += sp.slab * (size_t)e;
    }
    x = x_dtype == FINCH_BF16 ? (const void *)((const uint16_t *)x + sp.x_off) : (const void *)((const float *)x + sp.x_off);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int Kp = (K + 1023) & ~1023, nchunk = K / 32;
    float *xs = fsm, *sx = fsm + (size_t)M * Kp, *sx16 = sx + (size_t)M * (Kp / 32);   // sums per 32 and per 16 values
    // ---- rows: two per warp and step; the packed words are loaded PD steps ahead, the first ones before the staging ----
    const int ncb = Kp / 1024, warps = FNT / 32;
    const int first_pair = blockIdx.x * warps + warp, pair_step = gridDim.x * warps;
    const int npairs = (sp.out_dim + 1) / 2;
    const int my_pairs = first_pair < npairs ? (npairs - first_pair + pair_step - 1) / pair_step : 0;
    const int nit = my_pairs * ncb;
    auto row_of = [&](int it) { return (first_pair + (it / ncb) * pair_step) * 2; };
    auto chunk_of = [&](int it) { return (it % ncb) * 32 + lane; };
    constexpr int PD = Depth<BITS>::value;
    Raw<BITS> n0[PD], n1[PD];
    auto fetch = [&](int it, Raw<BITS> &a, Raw<BITS> &b) {
        if (it < nit && chunk_of(it) < nchunk) {
            const int rn = row_of(it);
            a = load_raw<BITS>(sp, (size_t)rn, K, chunk_of(it));
            if (rn + 1 < sp.out_dim) b = load_raw<BITS>(sp, (size_t)rn + 1, K, chunk_of(it));
        }
    };
#pragma unroll
    for (int d = 0; d < PD; d++) {
        n0[d] = Raw<BITS>{};
        n1[d] = Raw<BITS>{};
        fetch(d, n0[d], n1[d]);
    }
    // ---- stage the activations: a thread takes eight consecutive values (16-byte loads), four threads a chunk ----
    const int oct_per_row = Kp / 8;
#pragma unroll 4
    for (int idx = tid; idx < M * oct_per_row; idx += FNT) {
        const int m = idx / oct_per_row, k0 = (idx - m * oct_per_row) * 8;
        float v[8];
        if (k0 < K) {
            if (x_dtype == FINCH_BF16) {
                const uint4 r = __ldg(reinterpret_cast<const uint4 *>((const uint16_t *)x + (size_t)m * K + k0));
                const uint32_t u[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    v[2 * i] = __uint_as_float(u[i] << 16);
                    v[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
                }
            } else {
                const float4 a = __ldg(reinterpret_cast<const float4 *>((const float *)x + (size_t)m * K + k0));
                const float4 b = __ldg(reinterpret_cast<const float4 *>((const float *)x + (size_t)m * K + k0 + 4));
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = 0.f;
        }
        const int c = k0 >> 5, j0 = (k0 & 31) >> 2;
        float *dst = xs + (size_t)m * Kp + (c >> 5) * 1024 + (c & 31) * 4;
        *reinterpret_cast<float4 *>(dst + j0 * 128) = make_float4(v[0] * prescale_of<BITS>(k0), v[1] * prescale_of<BITS>(k0 + 1),
                                                                  v[2] * prescale_of<BITS>(k0 + 2), v[3] * prescale_of<BITS>(k0 + 3));
        *reinterpret_cast<float4 *>(dst + (j0 + 1) * 128) = make_float4(v[4] * prescale_of<BITS>(k0 + 4), v[5] * prescale_of<BITS>(k0 + 5),
                                                                        v[6] * prescale_of<BITS>(k0 + 6), v[7] * prescale_of<BITS>(k0 + 7));
        float sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if (BITS == 11 && (tid & 1) == 0) sx16[m * (Kp / 16) + (k0 >> 4)] = sum;
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((tid & 3) == 0) sx[m * (Kp / 32) + c] = sum;
    }
    __syncthreads();
    const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
    float acc[2][MT];
    for (int it0 = 0; it0 < nit; it0 += PD) {
#pragma unroll
        for (int d = 0; d < PD; d++) {
            const int it = it0 + d;
            if (it >= nit) break;
            const int row0 = row_of(it), cb = it % ncb, c = chunk_of(it);
            const bool two = row0 + 1 < sp.out_dim;
            const Raw<BITS> r0 = n0[d], r1 = n1[d];
            fetch(it + PD, n0[d], n1[d]);
            if (cb == 0) {
#pragma unroll
                for (int m = 0; m < MT; m++) acc[0][m] = acc[1][m] = 0.f;
            }
            if (c < nchunk) {
                float q0[32], q1[32], s0, b0 = 0.f, s1 = 0.f, b1 = 0.f, t0 = 0.f, t1 = 0.f;   // t: second half's scale (Q6_K)
                if constexpr (BITS == 11) {
                    decode_chunk6(sp, (size_t)row0, K, c, r0, q0, s0, t0);
                    if (two) decode_chunk6(sp, (size_t)row0 + 1, K, c, r1, q1, s1, t1);
                } else {
                    decode_chunk<BITS>(sp, (size_t)row0, K, c, r0, q0, s0, b0);
                    if (two) decode_chunk<BITS>(sp, (size_t)row0 + 1, K, c, r1, q1, s1, b1);
                }
                if (!two) {
#pragma unroll
                    for (int i = 0; i < 32; i++) q1[i] = 0.f;
                }
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    if (m < M) {
                        float a0 = 0.f, a1 = 0.f, c0 = 0.f, c1 = 0.f;   // a: values 0..15 (all 32 unless Q6_K), c: values 16..31 (Q6_K)
                        const float4 *xp = xs4 + ((size_t)m * Kp + cb * 1024) / 4 + lane;
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const float4 xv = xp[j * 32];
                            float &u0 = (BITS == 11 && j >= 4) ? c0 : a0, &u1 = (BITS == 11 && j >= 4) ? c1 : a1;
                            u0 = fmaf(q0[4 * j], xv.x, u0); u0 = fmaf(q0[4 * j + 1], xv.y, u0);
                            u0 = fmaf(q0[4 * j + 2], xv.z, u0); u0 = fmaf(q0[4 * j + 3], xv.w, u0);
                            u1 = fmaf(q1[4 * j], xv.x, u1); u1 = fmaf(q1[4 * j + 1], xv.y, u1);
                            u1 = fmaf(q1[4 * j + 2], xv.z, u1); u1 = fmaf(q1[4 * j + 3], xv.w, u1);
                        }
                        if constexpr (BITS == 11) {
                            const float x_lo = sx16[m * (Kp / 16) + 2 * c], x_hi = sx16[m * (Kp / 16) + 2 * c + 1];
                            acc[0][m] += fmaf(s0, fmaf(-32.0f, x_lo, a0), t0 * fmaf(-32.0f, x_hi, c0));
                            acc[1][m] += fmaf(s1, fmaf(-32.0f, x_lo, a1), t1 * fmaf(-32.0f, x_hi, c1));
                        } else {
                            const float sxm = sx[m * (Kp / 32) + c];
                            acc[0][m] += fmaf(s0, a0, b0 * sxm);
                            acc[1][m] += fmaf(s1, a1, b1 * sxm);
                        }
                    }
                }
            }
            if (cb == ncb - 1) {
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    if (m < M) {
                        float v0 = acc[0][m], v1 = acc[1][m];
#pragma unroll
                        for (int o = 16; o; o >>= 1) {
                            v0 += __shfl_xor_sync(0xffffffffu, v0, o);
                            v1 += __shfl_xor_sync(0xffffffffu, v1, o);
                        }
                        if (lane == 0) {
                            sp.out[(size_t)m * sp.out_dim + row0] = v0;
                            if (two) sp.out[(size_t)m * sp.out_dim + row0 + 1] = v1;
                        }
                    }
                }
            }
        }
    }
}

template <int BITS>
int launch_fast(finch_ctx *ctx, cudaStream_t st, const FPack &pack, const void *x, int x_dtype, int M, int K, int max_out, int slot) {
    const int Kp = (K + 1023) & ~1023;
    const size_t smem = ((size_t)M * Kp + (size_t)M * (Kp / 32) + (size_t)M * (Kp / 16)) * sizeof(float);
    const int one = M == 1;   // a single position gets its own instantiation (fewer registers, same code)
    {   // the shared-memory opt-in is a per-device attribute of each instantiation
        const int rc = one ? finch_func_attr_once(ctx, (const void *)fast_matvec_kernel<BITS, 1>, 200 * 1024)
                           : finch_func_attr_once(ctx, (const void *)fast_matvec_kernel<BITS, FM>, 200 * 1024);
        if (rc) return rc;
        (void)slot;
    }
    int ctas = (max_out + 31) / 32;   // 16 warps x 2 rows per sweep
    if (ctas > ctx->sm_count) ctas = ctx->sm_count;
    if (one) fast_matvec_kernel<BITS, 1><<<dim3(ctas, pack.n), FNT, smem, st>>>(pack, x, x_dtype, M, K);
    else fast_matvec_kernel<BITS, FM><<<dim3(ctas, pack.n), FNT, smem, st>>>(pack, x, x_dtype, M, K);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    ctx->launches++;
    return FINCH_OK;
}

}  // namespace

// Returns FINCH_OK after launching, or -1 when the call is not one the streaming kernel takes (the caller
// then uses the generic kernel).  More than eight positions run as passes of eight (the tensors of this
// path fit the L2, so the later passes re-read them from there).
int finch_try_fast_matvec(finch_ctx *ctx, cudaStream_t st, const void *x, int x_dtype, const finch_wdesc *specs, float *const *outs, int n, int M) {
    if (M > 16 * FM || n > 8) return -1;
    const int bits = specs[0].bits, K = specs[0].in_dim;
    if (bits != 3 && bits != 4 && bits != 8 && bits != 10 && bits != 11) return -1;
    if (K % 32 || (bits >= 10 && K % 256)) return -1;
    const int Kp = (K + 1023) & ~1023, Mmax = M < FM ? M : FM;
    if (((size_t)Mmax * Kp + (size_t)Mmax * (Kp / 32) + (size_t)Mmax * (Kp / 16)) * sizeof(float) > 200 * 1024) return -1;
    int max_out = 0;
    for (int i = 0; i < n; i++) {
        if (specs[i].bits != bits || specs[i].in_dim != K) return -1;
        max_out = max_out > specs[i].out_dim ? max_out : specs[i].out_dim;
    }
    const size_t xelt = x_dtype == FINCH_BF16 ? 2 : 4;
    for (int m0 = 0; m0 < M; m0 += FM) {
        const int mt = M - m0 < FM ? M - m0 : FM;
        FPack pack;
        pack.n = n;
        for (int i = 0; i < n; i++)
            pack.s[i] = FSpec{(const uint8_t *)specs[i].W, (const uint16_t *)specs[i].scales, (const uint16_t *)specs[i].biases,
                              outs[i] + (size_t)m0 * specs[i].out_dim, specs[i].out_dim, specs[i].scale_dtype, nullptr, nullptr, 0, 0, 0, 0};
        const void *xm = (const char *)x + (size_t)m0 * K * xelt;
        int rc;
        if (bits == 4) rc = launch_fast<4>(ctx, st, pack, xm, x_dtype, mt, K, max_out, 0);
        else if (bits == 3) rc = launch_fast<3>(ctx, st, pack, xm, x_dtype, mt, K, max_out, 1);
        else if (bits == 8) rc = launch_fast<8>(ctx, st, pack, xm, x_dtype, mt, K, max_out, 4);
        else if (bits == 10) rc = launch_fast<10>(ctx, st, pack, xm, x_dtype, mt, K, max_out, 2);
        else rc = launch_fast<11>(ctx, st, pack, xm, x_dtype, mt, K, max_out, 3);
        if (rc) return rc;
    }
    return FINCH_OK;
}

// ---------------------------------------------------------------------------------------------------
// GGUF expert MLP for decode (gpu_gguf_experts_forward, finchmoe/infer.m:3153-3366): the K selected experts
// of a token straight from the stacked ffn_{gate,up,down}_exps slabs -- gate and up of all K experts in one
// launch (they share the token's activations), SiLU(gate) * up, the K down projections in one launch (each
// with its own input), then the reference's combine: moe_out = sum_k w_k * out_k over the experts whose
// output energy is finite and below 1e20, divided by the accepted weight if that is in (0, 0.99)
// (infer.m:3334-3347).
namespace {

__global__ void gguf_swiglu_kernel(const float *g, const float *u, float *act, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float gv = g[i];
        act[i] = (gv / (1.0f + expf(-gv))) * u[i];
    }
}

// one CTA of 256 threads per token
__global__ void __launch_bounds__(256) gguf_combine_kernel(const float *outs, const int32_t *ids, const float *weights, const uint8_t *valid, int K,
                                                           int n_experts, int hidden, const float *h_mid, float *hidden_out) {
    __shared__ float red[8];
    __shared__ float wk[8];
    __shared__ float total;
    const int tid = threadIdx.x;
    if (tid == 0) total = 0.f;
    for (int k = 0; k < K; k++) {
        const int e = ids[k];
        const bool usable = e >= 0 && e < n_experts && (!valid || valid[k]);
        float er = 0.f;
        if (usable)
            for (int j = tid; j < hidden; j += 256) {
                const float v = outs[(size_t)k * hidden + j];
                er += v * v;
            }
#pragma unroll
        for (int o = 16; o; o >>= 1) er += __shfl_xor_sync(0xffffffffu, er, o);
        if ((tid & 31) == 0) red[tid >> 5] = er;
        __syncthreads();
        if (tid == 0) {
            float s = 0.f;
            for (int w = 0; w < 8; w++) s += red[w];
            const bool ok = usable && isfinite(s) && s < 1e20f;
            wk[k] = ok ? weights[k] : 0.f;
            if (ok) total += weights[k];
        }
        __syncthreads();
    }
    const float tw = total, inv = (tw > 0.f && tw < 0.99f) ? 1.0f / tw : 1.0f;
    for (int j = tid; j < hidden; j += 256) {
        float m = 0.f;
        for (int k = 0; k < K; k++)
            if (wk[k] != 0.f) m = fmaf(wk[k], outs[(size_t)k * hidden + j], m);
        hidden_out[j] = (h_mid ? h_mid[j] : 0.f) + m * inv;
    }
}

int launch_gguf(finch_ctx *ctx, cudaStream_t st, int type, const FPack &pack, const void *x, int x_dtype, int K, int max_out) {
    if (type == 10) return launch_fast<10>(ctx, st, pack, x, x_dtype, 1, K, max_out, 2);
    return launch_fast<11>(ctx, st, pack, x, x_dtype, 1, K, max_out, 3);
}

}  // namespace

int finch_gguf_experts_grouped(finch_ctx *ctx, cudaStream_t st, const finch_gguf_experts *ex, const void *h_post, const int32_t *expert_ids, const float *weights,
                               const uint8_t *valid, const float *h_mid, float *hidden_out, int B);

extern "C" int finch_encode_moe_gguf(finch_ctx *ctx, finch_stream stream, const finch_gguf_experts *ex, const void *h_post, const int32_t *expert_ids,
                                     const float *weights, const uint8_t *valid, const float *h_mid, float *hidden_out, int B) {
    if (!ctx || !ex || !h_post || !expert_ids || !weights || !hidden_out || B < 1) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    const int H = c.hidden, I = c.moe_inter, K = c.top_k;
    for (int t : {ex->gate_type, ex->up_type, ex->down_type})
        if (t != 10 && t != 11) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "GGUF expert tensors must be Q4_K (10) or Q6_K (11)");
    if (H % 256 || I % 256 || K > 8) return finch_fail(ctx, FINCH_E_ARG, "GGUF experts: hidden and inter must be whole 256-value blocks, top_k <= 8");
    if (!ex->gate || !ex->up || !ex->down) return finch_fail(ctx, FINCH_E_ARG, "GGUF experts: null slab");
    cudaSetDevice(c.device);
    cudaStream_t st = finch_pick_stream(ctx, stream);
    if (B >= 9) {   // a prefill chunk: pairs grouped by expert, every selected expert's rows read once (matvec_gguf_mma.cu)
        const int rc = finch_gguf_experts_grouped(ctx, st, ex, h_post, expert_ids, weights, valid, h_mid, hidden_out, B);
        if (rc >= 0) return rc;
    }
    const size_t need = (size_t)K * (3 * I + H) * sizeof(float);
    if (ctx->gguf_ws_bytes < need) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(st, &cap);
        if (cap != cudaStreamCaptureStatusNone) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "first GGUF call must be outside stream capture");
        if (ctx->gguf_ws) cudaFree(ctx->gguf_ws);
        ctx->gguf_ws = nullptr;
        ctx->gguf_ws_bytes = 0;
        if (cudaMalloc(&ctx->gguf_ws, need) != cudaSuccess) {
            cudaGetLastError();
            return finch_fail(ctx, FINCH_E_NOMEM, "GGUF expert scratch (%zu bytes)", need);
        }
        ctx->gguf_ws_bytes = need;
    }
    float *g = (float *)ctx->gguf_ws, *u = g + (size_t)K * I, *act = u + (size_t)K * I, *outs = act + (size_t)K * I;
    const int x_dtype = c.act_dtype;
    for (int b = 0; b < B; b++) {
        const int32_t *ids = expert_ids + (size_t)b * K;
        const uint8_t *vb = valid ? valid + (size_t)b * K : nullptr;
        const void *xb = x_dtype == FINCH_BF16 ? (const void *)((const uint16_t *)h_post + (size_t)b * H) : (const void *)((const float *)h_post + (size_t)b * H);
        // a masked or absent expert leaves its rows untouched: clear them so the combine's energy test reads zeros, not stale data
        FINCH_CUDA_OK(ctx, cudaMemsetAsync(outs, 0, (size_t)K * H * sizeof(float), st));
        FINCH_CUDA_OK(ctx, cudaMemsetAsync(g, 0, (size_t)2 * K * I * sizeof(float), st));
        int rc;
        if (ex->gate_type == ex->up_type) {
            FPack p;
            p.n = 2 * K;
            for (int k = 0; k < K; k++) {
                p.s[k] = FSpec{(const uint8_t *)ex->gate, nullptr, nullptr, g + (size_t)k * I, I, FINCH_FP16, ids, vb, k, c.n_experts, ex->gate_slab, 0};
                p.s[K + k] = FSpec{(const uint8_t *)ex->up, nullptr, nullptr, u + (size_t)k * I, I, FINCH_FP16, ids, vb, k, c.n_experts, ex->up_slab, 0};
            }
            if ((rc = launch_gguf(ctx, st, ex->gate_type, p, xb, x_dtype, H, I))) return rc;
        } else {
            for (int which = 0; which < 2; which++) {
                FPack p;
                p.n = K;
                for (int k = 0; k < K; k++)
                    p.s[k] = FSpec{(const uint8_t *)(which ? ex->up : ex->gate), nullptr, nullptr, (which ? u : g) + (size_t)k * I, I, FINCH_FP16, ids, vb, k,
                                   c.n_experts, which ? ex->up_slab : ex->gate_slab, 0};
                if ((rc = launch_gguf(ctx, st, which ? ex->up_type : ex->gate_type, p, xb, x_dtype, H, I))) return rc;
            }
        }
        gguf_swiglu_kernel<<<(K * I + 255) / 256, 256, 0, st>>>(g, u, act, K * I);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        {
            FPack p;
            p.n = K;
            for (int k = 0; k < K; k++)
                p.s[k] = FSpec{(const uint8_t *)ex->down, nullptr, nullptr, outs + (size_t)k * H, H, FINCH_FP16, ids, vb, k, c.n_experts, ex->down_slab,
                               (size_t)k * I};
            if ((rc = launch_gguf(ctx, st, ex->down_type, p, act, FINCH_F32, I, H))) return rc;
        }
        gguf_combine_kernel<<<1, 256, 0, st>>>(outs, ids, weights + (size_t)b * K, vb, K, c.n_experts, H, h_mid ? h_mid + (size_t)b * H : nullptr,
                                               hidden_out + (size_t)b * H);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        ctx->launches += 2;
    }
    return FINCH_OK;
}
