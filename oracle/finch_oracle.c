/*
 * finch_oracle.c -- CPU restatement of FinchMoE's quantized-expert MoE path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA library is
 * compared against (and the timed "reference CPU arm" of the benchmark).  It
 * is never linked into, imported by or called from the product library.
 *
 * Every function restates (does not copy) the arithmetic of the reference's
 * own CPU path; the reference location it follows is cited above it as
 * <file within the reference project>:<lines>.
 *
 * Parity pin: the affine 3-/4-/8-bit unpack + dequant are checked against the
 * reference's importable Python packers/dequantizers, and the Q4_K / Q6_K
 * block decoders against the gguf-py package's numpy dequantizers (both via
 * committed golden vectors).  The reference ships no golden vectors of its own
 * for this path ("the CPU is the oracle", finchTool/README.md:150), and its
 * Objective-C translation unit cannot be compiled without Apple frameworks, so
 * the matvec / SwiGLU / routing / combine restatements are pinned by
 * construction against finchmoe/infer.m's text, not against an executed build.
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared -pthread (see Makefile).
 * -O2 is the reference's level (finchmoe/Makefile:17); contraction is off so
 * that "q*s + b" is two roundings, matching numpy (quant_audit.py:245).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define FO_API __attribute__((visibility("default")))

enum { FO_SCALE_BF16 = 0, FO_SCALE_FP16 = 1 };
enum { FO_ACC_F32 = 0, FO_ACC_F64 = 1 };

/* ------------------------------------------------------------------ */
/* 16-bit float widening                                               */
/* ------------------------------------------------------------------ */

/* finchmoe/infer.m:690-695 -- bf16 is the top half of an fp32. */
FO_API float fo_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return f;
}

/* finchmoe/infer.m:1579-1593 -- IEEE half to float including subnormals.
 * Restated from the format definition (sign | 5-bit exponent | 10-bit
 * mantissa) rather than from the reference's magic-number form; the two agree
 * on all 65536 inputs for finite values (verified in tests). */
FO_API float fo_fp16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const int e = (h >> 10) & 0x1f;
    const uint32_t m = h & 0x3ffu;
    uint32_t u;
    if (e == 0) {
        if (m == 0) {
            u = sign;
        } else {
            /* subnormal: value = m * 2^-24 */
            float v = (float)m * 0x1.0p-24f;
            memcpy(&u, &v, 4);
            u |= sign;
        }
    } else if (e == 31) {
        u = sign | 0x7f800000u | (m << 13);
    } else {
        u = sign | ((uint32_t)(e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float widen16(uint16_t h, int scale_dtype) {
    return scale_dtype == FO_SCALE_FP16 ? fo_fp16_to_f32(h) : fo_bf16_to_f32(h);
}

/* ------------------------------------------------------------------ */
/* Affine tiers: unpack + dequant                                      */
/* ------------------------------------------------------------------ */

/* Code of element (row, i).
 * 3-bit: finchmoe/infer.m:1716-1727, finchmoe/repack_experts.py:242-257 --
 *   eight codes per little-endian 24-bit triplet, code j at bits 3j..3j+2.
 * 4-/8-bit: finchmoe/infer.m:1734-1758, finchmoe/quantize_non_experts.py:57-65
 *   -- 32/bits codes per little-endian u32, least significant first. */
static inline unsigned code_at(const uint8_t *row, int i, int bits) {
    if (bits == 3) {
        const uint8_t *t = row + (i >> 3) * 3;
        uint32_t pk = (uint32_t)t[0] | ((uint32_t)t[1] << 8) | ((uint32_t)t[2] << 16);
        return (pk >> (3 * (i & 7))) & 7u;
    }
    const int vpw = 32 / bits;
    uint32_t w;
    memcpy(&w, row + (size_t)(i / vpw) * 4, 4);
    return (w >> ((i % vpw) * bits)) & ((1u << bits) - 1u);
}

static inline size_t affine_row_bytes(int in_dim, int bits) {
    return (size_t)in_dim * bits / 8;
}

FO_API int fo_unpack_codes(const void *W, int out_dim, int in_dim, int bits, uint8_t *codes) {
    if (bits != 3 && bits != 4 && bits != 8) return -1;
    const size_t rb = affine_row_bytes(in_dim, bits);
    for (int r = 0; r < out_dim; r++) {
        const uint8_t *row = (const uint8_t *)W + r * rb;
        for (int i = 0; i < in_dim; i++) codes[(size_t)r * in_dim + i] = (uint8_t)code_at(row, i, bits);
    }
    return 0;
}

/* Dequantized weight, defined as fl32(fl32(float(q) * s) + b) with s, b
 * widened exactly from their 16-bit storage: the numpy form of
 * finchTool/tools/quant_audit.py:245 ("vals * S_exp + B_exp"), which is also
 * the C form of finchmoe/infer.m:1725 when the compiler does not contract. */
FO_API int fo_dequant_affine(const void *W, const uint16_t *S, const uint16_t *B, int scale_dtype,
                             int out_dim, int in_dim, int group, int bits, float *w_out) {
    if (bits != 3 && bits != 4 && bits != 8) return -1;
    const size_t rb = affine_row_bytes(in_dim, bits);
    const int ng = in_dim / group;
    for (int r = 0; r < out_dim; r++) {
        const uint8_t *row = (const uint8_t *)W + r * rb;
        for (int i = 0; i < in_dim; i++) {
            const float s = widen16(S[(size_t)r * ng + i / group], scale_dtype);
            const float b = widen16(B[(size_t)r * ng + i / group], scale_dtype);
            volatile float prod = (float)code_at(row, i, bits) * s;
            w_out[(size_t)r * in_dim + i] = prod + b;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* GGUF tiers                                                          */
/* ------------------------------------------------------------------ */

/* finchmoe/infer.m:1595-1603 -- 6-bit (scale, min) pair j of a Q4_K block. */
static inline void q4k_scale_min(int j, const uint8_t *sc12, unsigned *sc, unsigned *mn) {
    if (j < 4) {
        *sc = sc12[j] & 63u;
        *mn = sc12[j + 4] & 63u;
    } else {
        *sc = (sc12[j + 4] & 0x0fu) | ((unsigned)(sc12[j - 4] >> 6) << 4);
        *mn = (sc12[j + 4] >> 4) | ((unsigned)(sc12[j] >> 6) << 4);
    }
}

#define FO_Q4K_BLOCK 144
#define FO_Q6K_BLOCK 210

FO_API size_t fo_gguf_row_bytes(int in_dim, int ggml_type) {
    return (size_t)(in_dim / 256) * (ggml_type == 12 ? FO_Q4K_BLOCK : FO_Q6K_BLOCK);
}

/* finchmoe/infer.m:1604-1657 -- one row of Q4_K (type 12) or Q6_K (type 14)
 * blocks to float.  Evaluation order kept: Q4_K "d*sc" then "*nib - dmin*m";
 * Q6_K "d * sc * q" left to right. */
FO_API int fo_gguf_dequant_row(const void *row, float *y, int n, int ggml_type) {
    const uint8_t *p = (const uint8_t *)row;
    if (ggml_type == 12) {
        for (int blk = 0; blk < n / 256; blk++, p += FO_Q4K_BLOCK, y += 256) {
            uint16_t hd, hm;
            memcpy(&hd, p, 2);
            memcpy(&hm, p + 2, 2);
            const float d = fo_fp16_to_f32(hd), dmin = fo_fp16_to_f32(hm);
            const uint8_t *qs = p + 16;
            for (int c = 0; c < 4; c++) {
                unsigned s0, m0, s1, m1;
                q4k_scale_min(2 * c, p + 4, &s0, &m0);
                q4k_scale_min(2 * c + 1, p + 4, &s1, &m1);
                const float d0 = d * (float)s0, o0 = dmin * (float)m0;
                const float d1 = d * (float)s1, o1 = dmin * (float)m1;
                for (int l = 0; l < 32; l++) {
                    y[64 * c + l] = d0 * (float)(qs[32 * c + l] & 0x0f) - o0;
                    y[64 * c + 32 + l] = d1 * (float)(qs[32 * c + l] >> 4) - o1;
                }
            }
        }
        return 0;
    }
    if (ggml_type == 14) {
        for (int blk = 0; blk < n / 256; blk++, p += FO_Q6K_BLOCK, y += 256) {
            uint16_t hd;
            memcpy(&hd, p + 208, 2);
            const float d = fo_fp16_to_f32(hd);
            for (int h = 0; h < 2; h++) {
                const uint8_t *ql = p + 64 * h, *qh = p + 128 + 32 * h;
                const int8_t *sc = (const int8_t *)(p + 192) + 8 * h;
                float *yy = y + 128 * h;
                for (int l = 0; l < 32; l++) {
                    const int is = l / 16;
                    const int q1 = (int)((ql[l] & 0x0f) | (((qh[l] >> 0) & 3) << 4)) - 32;
                    const int q2 = (int)((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    yy[l] = d * (float)sc[is] * (float)q1;
                    yy[l + 32] = d * (float)sc[is + 2] * (float)q2;
                    yy[l + 64] = d * (float)sc[is + 4] * (float)q3;
                    yy[l + 96] = d * (float)sc[is + 6] * (float)q4;
                }
            }
        }
        return 0;
    }
    return -1;
}

FO_API int fo_dequant_gguf(const void *W, int out_dim, int in_dim, int ggml_type, float *w_out) {
    const size_t rb = fo_gguf_row_bytes(in_dim, ggml_type);
    for (int r = 0; r < out_dim; r++)
        if (fo_gguf_dequant_row((const uint8_t *)W + r * rb, w_out + (size_t)r * in_dim, in_dim, ggml_type))
            return -1;
    return 0;
}

/* Q6_K 6-bit codes (0..63) and Q4_K nibbles (0..15), in value order. */
FO_API int fo_gguf_unpack_codes(const void *W, int out_dim, int in_dim, int ggml_type, uint8_t *codes) {
    const size_t rb = fo_gguf_row_bytes(in_dim, ggml_type);
    for (int r = 0; r < out_dim; r++) {
        const uint8_t *p = (const uint8_t *)W + r * rb;
        uint8_t *c = codes + (size_t)r * in_dim;
        for (int blk = 0; blk < in_dim / 256; blk++, c += 256) {
            if (ggml_type == 12) {
                const uint8_t *qs = p + 16;
                for (int ch = 0; ch < 4; ch++)
                    for (int l = 0; l < 32; l++) {
                        c[64 * ch + l] = qs[32 * ch + l] & 0x0f;
                        c[64 * ch + 32 + l] = qs[32 * ch + l] >> 4;
                    }
                p += FO_Q4K_BLOCK;
            } else if (ggml_type == 14) {
                for (int h = 0; h < 2; h++) {
                    const uint8_t *ql = p + 64 * h, *qh = p + 128 + 32 * h;
                    for (int l = 0; l < 32; l++) {
                        c[128 * h + l] = (ql[l] & 0x0f) | (((qh[l] >> 0) & 3) << 4);
                        c[128 * h + l + 32] = (ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4);
                        c[128 * h + l + 64] = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4);
                        c[128 * h + l + 96] = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4);
                    }
                }
                p += FO_Q6K_BLOCK;
            } else {
                return -1;
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Matvec                                                              */
/* ------------------------------------------------------------------ */

/* One output row, reference order.
 * Affine: finchmoe/infer.m:1711-1729 (3-bit), 1739-1762 (4-/8-bit):
 *   acc += (float(q)*s + b) * x[i], i ascending, fp32.
 * GGUF (bits 10 = Q4_K, 11 = Q6_K): finchmoe/infer.m:1660-1674: dequantize
 *   the row, then acc += y[i]*x[i].
 * accum == FO_ACC_F64 evaluates the same products with a double accumulator
 * (the form finchmoe/test_engine_path.m:28-44 uses as its yardstick) from the
 * fp32 dequantized weight. */
static void matvec_rows(const void *W, const uint16_t *S, const uint16_t *B, int scale_dtype,
                        const float *x, float *out, int r0, int r1, int in_dim, int group,
                        int bits, int accum, float *scratch /* in_dim floats */) {
    if (bits == 10 || bits == 11) {
        const int ty = bits == 10 ? 12 : 14;
        const size_t rb = fo_gguf_row_bytes(in_dim, ty);
        for (int r = r0; r < r1; r++) {
            fo_gguf_dequant_row((const uint8_t *)W + r * rb, scratch, in_dim, ty);
            if (accum == FO_ACC_F64) {
                double acc = 0.0;
                for (int i = 0; i < in_dim; i++) acc += (double)scratch[i] * (double)x[i];
                out[r] = (float)acc;
            } else {
                float acc = 0.0f;
                for (int i = 0; i < in_dim; i++) acc += scratch[i] * x[i];
                out[r] = acc;
            }
        }
        return;
    }
    if (bits == 0 || !S || !B) { /* raw BF16 weights: finchmoe/infer.m:1689-1700 */
        const uint16_t *Wb = (const uint16_t *)W;
        for (int r = r0; r < r1; r++) {
            double accd = 0.0;
            float acc = 0.0f;
            for (int i = 0; i < in_dim; i++) {
                const float w = fo_bf16_to_f32(Wb[(size_t)r * in_dim + i]);
                if (accum == FO_ACC_F64) accd += (double)w * (double)x[i];
                else acc += w * x[i];
            }
            out[r] = accum == FO_ACC_F64 ? (float)accd : acc;
        }
        return;
    }
    const size_t rb = affine_row_bytes(in_dim, bits);
    const int ng = in_dim / group;
    for (int r = r0; r < r1; r++) {
        const uint8_t *row = (const uint8_t *)W + r * rb;
        const uint16_t *sr = S + (size_t)r * ng, *br = B + (size_t)r * ng;
        double accd = 0.0;
        float acc = 0.0f;
        for (int g = 0; g < ng; g++) {
            const float s = widen16(sr[g], scale_dtype), b = widen16(br[g], scale_dtype);
            for (int i = g * group; i < (g + 1) * group; i++) {
                const float w = (float)code_at(row, i, bits) * s + b;
                if (accum == FO_ACC_F64) accd += (double)w * (double)x[i];
                else acc += w * x[i];
            }
        }
        out[r] = accum == FO_ACC_F64 ? (float)accd : acc;
    }
}

/* finchmoe/infer.m:1676-1763 (cpu_dequant_matvec); bits convention
 * 3/4/8 affine, 10 = Q4_K, 11 = Q6_K, 0 = raw BF16 (infer.m:1681-1701). */
FO_API int fo_matvec(const void *W, const uint16_t *S, const uint16_t *B, int scale_dtype,
                     const float *x, float *out, int out_dim, int in_dim, int group, int bits,
                     int accum) {
    if (!(bits == 0 || bits == 3 || bits == 4 || bits == 8 || bits == 10 || bits == 11)) return -1;
    float *scratch = (float *)malloc(sizeof(float) * (size_t)in_dim);
    if (!scratch) return -2;
    matvec_rows(W, S, B, scale_dtype, x, out, 0, out_dim, in_dim, group, bits, accum, scratch);
    free(scratch);
    return 0;
}

/* ------------------------------------------------------------------ */
/* SwiGLU, routing, combine                                            */
/* ------------------------------------------------------------------ */

/* finchmoe/infer.m:1780-1786 */
FO_API void fo_swiglu(const float *gate, const float *up, float *out, int n) {
    for (int i = 0; i < n; i++) {
        const float g = gate[i];
        out[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}

/* finchmoe/infer.m:1794-1808 */
FO_API void fo_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) mx = x[i] > mx ? x[i] : mx;
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        x[i] = expf(x[i] - mx);
        sum += x[i];
    }
    const float inv = 1.0f / sum;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* finchmoe/infer.m:1811-1830 -- K slots start at -1e30 / index 0; each score
 * replaces the slot currently holding the smallest value (lowest slot on
 * ties) when it is strictly greater.  Output stays in slot order. */
FO_API void fo_topk(const float *scores, int n, int K, int *idx, float *val) {
    for (int k = 0; k < K; k++) {
        val[k] = -1e30f;
        idx[k] = 0;
    }
    for (int i = 0; i < n; i++) {
        int lo = 0;
        for (int k = 1; k < K; k++)
            if (val[k] < val[lo]) lo = k;
        if (scores[i] > val[lo]) {
            val[lo] = scores[i];
            idx[lo] = i;
        }
    }
}

/* finchmoe/infer.m:1833-1840 */
FO_API void fo_normalize(float *w, int K) {
    float sum = 0.0f;
    for (int k = 0; k < K; k++) sum += w[k];
    if (sum > 0.0f) {
        const float inv = 1.0f / sum;
        for (int k = 0; k < K; k++) w[k] *= inv;
    }
}

/* Router tail as the engine runs it (finchmoe/infer.m:9285-9289):
 * softmax over all experts, top-K, renormalise.  logits is not modified. */
FO_API void fo_route(const float *logits, int n_experts, int K, int *idx, float *w) {
    float *p = (float *)malloc(sizeof(float) * (size_t)n_experts);
    memcpy(p, logits, sizeof(float) * (size_t)n_experts);
    fo_softmax(p, n_experts);
    fo_topk(p, n_experts, K, idx, w);
    fo_normalize(w, K);
    free(p);
}

static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

/* Combine.
 * guard == 0: the native GPU form, finchmoe/shaders.metal:2196-2231 and its
 *   CPU twin finchmoe/infer.m:7390-7412: moe = sum_{k ascending, valid}
 *   w_k*out_k; hidden = h_mid + moe + sigmoid(score)*shared_out.
 * guard == 1: the CPU-path form, finchmoe/infer.m:3334-3347 / 10190-10204:
 *   experts whose sum of squares is non-finite or >= 1e20 are dropped and the
 *   sum is divided by the kept weight when 0 < kept < 0.99.
 * Any of h_mid / shared_out may be NULL (term omitted).  valid may be NULL. */
FO_API void fo_combine(const float *h_mid, const float *expert_out /*[K][dim]*/, const float *w,
                       const uint8_t *valid, const float *shared_out, float shared_gate_score,
                       int dim, int K, int guard, float *hidden) {
    float *moe = (float *)calloc((size_t)dim, sizeof(float));
    float kept = 0.0f;
    for (int k = 0; k < K; k++) {
        if (valid && !valid[k]) continue;
        const float *o = expert_out + (size_t)k * dim;
        if (guard) {
            float e = 0.0f;
            for (int j = 0; j < dim; j++) e += o[j] * o[j];
            if (!(isfinite(e) && e < 1e20f)) continue;
        }
        for (int j = 0; j < dim; j++) moe[j] += w[k] * o[j];
        kept += w[k];
    }
    if (guard && kept > 0.0f && kept < 0.99f) {
        const float inv = 1.0f / kept;
        for (int j = 0; j < dim; j++) moe[j] *= inv;
    }
    const float sg = shared_out ? sigmoidf_(shared_gate_score) : 0.0f;
    for (int j = 0; j < dim; j++) {
        float h = h_mid ? h_mid[j] : 0.0f;
        h = h + moe[j];
        if (shared_out) h = h + sg * shared_out[j];
        hidden[j] = h;
    }
    free(moe);
}

/* ------------------------------------------------------------------ */
/* Expert MLPs and the whole layer                                     */
/* ------------------------------------------------------------------ */

typedef struct {
    size_t gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b, size;
} fo_layout;

/* Packed expert block: [gate W|S|B | up W|S|B | down W|S|B].
 * finchmoe/infer.m:223-234 (3-bit), 175-184 (4-bit), 187-196 (8-bit);
 * finchmoe/repack_experts.py:137-151.  For hidden 2048 / inter 512 / group 64
 * this reproduces the reference offsets exactly (checked in tests). */
FO_API void fo_expert_layout(int hidden, int inter, int group, int bits, fo_layout *L) {
    const size_t gw = (size_t)inter * hidden * bits / 8, gs = (size_t)inter * (hidden / group) * 2;
    const size_t dw = (size_t)hidden * inter * bits / 8, ds = (size_t)hidden * (inter / group) * 2;
    L->gate_w = 0;
    L->gate_s = gw;
    L->gate_b = gw + gs;
    L->up_w = gw + 2 * gs;
    L->up_s = L->up_w + gw;
    L->up_b = L->up_s + gs;
    L->down_w = L->up_b + gs;
    L->down_s = L->down_w + dw;
    L->down_b = L->down_s + ds;
    L->size = L->down_b + ds;
}

/* One routed expert: gate, up, SwiGLU, down -- the unfused composition of
 * finchmoe/infer.m:4336-4378 (GPU encode order) = infer.m:10169-10186 (CPU).
 * In FO_ACC_F64 mode gate/up/down use double accumulators and SwiGLU is
 * evaluated in double; intermediate vectors are rounded to fp32 between
 * stages exactly where the reference stores them (fp32 buffers). */
FO_API void fo_expert_forward(const uint8_t *block, int bits, int scale_dtype, int hidden,
                              int inter, int group, const float *x, float *out, int accum) {
    fo_layout L;
    fo_expert_layout(hidden, inter, group, bits, &L);
    float *g = (float *)malloc(sizeof(float) * 3 * (size_t)inter + sizeof(float) * (size_t)hidden);
    float *u = g + inter, *a = u + inter, *scratch = a + inter;
    matvec_rows(block + L.gate_w, (const uint16_t *)(block + L.gate_s),
                (const uint16_t *)(block + L.gate_b), scale_dtype, x, g, 0, inter, hidden, group,
                bits, accum, scratch);
    matvec_rows(block + L.up_w, (const uint16_t *)(block + L.up_s),
                (const uint16_t *)(block + L.up_b), scale_dtype, x, u, 0, inter, hidden, group,
                bits, accum, scratch);
    if (accum == FO_ACC_F64) {
        for (int i = 0; i < inter; i++) {
            const double gd = g[i];
            a[i] = (float)(gd / (1.0 + exp(-gd)) * (double)u[i]);
        }
    } else {
        fo_swiglu(g, u, a, inter);
    }
    matvec_rows(block + L.down_w, (const uint16_t *)(block + L.down_s),
                (const uint16_t *)(block + L.down_b), scale_dtype, a, out, 0, hidden, inter, group,
                bits, accum, scratch);
    free(g);
}

/* Shared expert (separate tensors, any supported bits): finchmoe/infer.m:
 * 9608-9629 (swiglu + down) with gate/up from the routing batch (9061-9098). */
typedef struct {
    const void *W;
    const uint16_t *S, *B;
    int out_dim, in_dim, group, bits, scale_dtype;
} fo_wdesc;

FO_API void fo_shared_forward(const fo_wdesc *gate, const fo_wdesc *up, const fo_wdesc *down,
                              const float *x, float *out, int accum) {
    const int inter = gate->out_dim;
    float *g = (float *)malloc(sizeof(float) * (3 * (size_t)inter + (size_t)gate->in_dim));
    float *u = g + inter, *a = u + inter, *scratch = a + inter;
    matvec_rows(gate->W, gate->S, gate->B, gate->scale_dtype, x, g, 0, inter, gate->in_dim,
                gate->group, gate->bits, accum, scratch);
    matvec_rows(up->W, up->S, up->B, up->scale_dtype, x, u, 0, inter, up->in_dim, up->group,
                up->bits, accum, scratch);
    if (accum == FO_ACC_F64) {
        for (int i = 0; i < inter; i++) {
            const double gd = g[i];
            a[i] = (float)(gd / (1.0 + exp(-gd)) * (double)u[i]);
        }
    } else {
        fo_swiglu(g, u, a, inter);
    }
    matvec_rows(down->W, down->S, down->B, down->scale_dtype, a, out, 0, down->out_dim,
                down->in_dim, down->group, down->bits, accum, scratch);
    free(g);
}

typedef struct {
    const uint8_t *block;
    int bits, scale_dtype, hidden, inter, group, accum;
    const float *x;
    float *out;
} expert_job;

static void *expert_thread(void *arg) {
    expert_job *j = (expert_job *)arg;
    fo_expert_forward(j->block, j->bits, j->scale_dtype, j->hidden, j->inter, j->group, j->x, j->out,
                      j->accum);
    return NULL;
}

/* One token through one MoE layer: K routed experts (serial like the
 * reference's --cpu-experts loop, finchmoe/infer.m:10109-10204, or one
 * pthread per expert when nthreads > 1), optional shared expert, combine.
 * blocks[k] may be NULL when valid[k] == 0. */
FO_API void fo_moe_layer(const uint8_t *const *blocks, const float *w, const uint8_t *valid, int K,
                         int bits, int scale_dtype, int hidden, int inter, int group,
                         const float *x, const float *h_mid, const fo_wdesc *sh_gate,
                         const fo_wdesc *sh_up, const fo_wdesc *sh_down, float shared_gate_score,
                         int guard, int accum, int nthreads, float *hidden_out) {
    float *eo = (float *)calloc((size_t)K * hidden + (size_t)hidden, sizeof(float));
    float *so = eo + (size_t)K * hidden;
    expert_job *jobs = (expert_job *)malloc(sizeof(expert_job) * (size_t)K);
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)K);
    for (int k = 0; k < K; k++) {
        jobs[k] = (expert_job){blocks[k], bits, scale_dtype, hidden, inter, group, accum, x,
                               eo + (size_t)k * hidden};
        th[k] = 0;
    }
    for (int k = 0; k < K; k++) {
        if (valid && !valid[k]) continue;
        if (nthreads > 1) pthread_create(&th[k], NULL, expert_thread, &jobs[k]);
        else expert_thread(&jobs[k]);
    }
    if (nthreads > 1)
        for (int k = 0; k < K; k++)
            if (!(valid && !valid[k])) pthread_join(th[k], NULL);
    const int has_shared = sh_gate && sh_up && sh_down;
    if (has_shared) fo_shared_forward(sh_gate, sh_up, sh_down, x, so, accum);
    fo_combine(h_mid, eo, w, valid, has_shared ? so : NULL, shared_gate_score, hidden, K, guard,
               hidden_out);
    free(th);
    free(jobs);
    free(eo);
}

/* Exhaustive self-check helper: the reference's magic-number fp16 widening
 * (finchmoe/infer.m:1579-1593) restated with explicit steps, so the test can
 * confirm the field-based fo_fp16_to_f32 above agrees on all 65536 inputs. */
/* Residual add + RMS norm (residual_norm_fused, finchmoe/shaders.metal:1232-1263; cpu_rms_norm,
 * finchmoe/infer.m:1766-1777): h = resid + oproj (oproj may be NULL), h_mid_out = h (may be NULL),
 * h_post_out = h * (1 / sqrt(mean(h^2) + eps)) * bf16(w), fp32, sequential sum like the CPU form. */
FO_API void fo_residual_norm(const float *resid, const float *oproj, const uint16_t *norm_w, int dim, float eps,
                             float *h_mid_out, float *h_post_out) {
    float sum_sq = 0.0f;
    for (int i = 0; i < dim; i++) {
        const float h = oproj ? resid[i] + oproj[i] : resid[i];
        if (h_mid_out) h_mid_out[i] = h;
        sum_sq += h * h;
    }
    const float inv_rms = 1.0f / sqrtf(sum_sq / (float)dim + eps);
    for (int i = 0; i < dim; i++) {
        const float h = oproj ? resid[i] + oproj[i] : resid[i];
        h_post_out[i] = h * inv_rms * fo_bf16_to_f32(norm_w[i]);
    }
}

FO_API float fo_fp16_to_f32_magic(uint16_t h) {
    const uint32_t w = (uint32_t)h << 16, sign = w & 0x80000000u, two_w = w + w;
    uint32_t nb = (two_w >> 4) + (0xE0u << 23), db = (two_w >> 17) | (126u << 23), rb;
    float nf, df;
    memcpy(&nf, &nb, 4);
    memcpy(&df, &db, 4);
    nf *= 0x1.0p-112f;
    df -= 0.5f;
    if (two_w < (1u << 27)) memcpy(&rb, &df, 4);
    else memcpy(&rb, &nf, 4);
    rb |= sign;
    float r;
    memcpy(&r, &rb, 4);
    return r;
}
