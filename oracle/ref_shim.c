/* Exports the reference's own CPU math for the parity tests.
 *
 * TEST INFRASTRUCTURE ONLY.  This file holds no reference code: `make ref`
 * extracts the pure-C region of the reference's engine source (the bf16 helpers,
 * finchmoe/infer.m:690-702, and the fp16 / GGUF / affine matvec / SwiGLU /
 * softmax / top-K / normalise / vector helpers, finchmoe/infer.m:1575-1868) from
 * a reference checkout into oracle/_ref/infer_cpu_extract.inc (git-ignored) and
 * compiles this shim around it with the reference's optimisation level
 * (finchmoe/Makefile:17).  The functions there are `static`; the wrappers below
 * give them external names.  Only tests/ (and bench.py's reference arm) load the
 * resulting oracle/_ref/libfinch_ref.so; the product never does. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "_ref/infer_cpu_extract.inc"

#define REF_API __attribute__((visibility("default")))

REF_API float ref_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }
REF_API uint16_t ref_f32_to_bf16(float f) { return f32_to_bf16(f); }
REF_API float ref_fp16_to_f32(uint16_t h) { return fp16_to_f32(h); }
REF_API void ref_gguf_dequant_row(const void *row, float *y, int n, int ggml_type) { gguf_dequant_row(row, y, n, ggml_type); }
REF_API void ref_cpu_dequant_matvec(const uint32_t *W, const uint16_t *scales, const uint16_t *biases, const float *x, float *out,
                                    int out_dim, int in_dim, int group_size, int bits) {
    cpu_dequant_matvec(W, scales, biases, x, out, out_dim, in_dim, group_size, bits);
}
REF_API void ref_cpu_rms_norm(const float *x, const uint16_t *w_bf16, float *out, int dim, float eps) { cpu_rms_norm(x, w_bf16, out, dim, eps); }
REF_API void ref_cpu_swiglu(const float *gate, const float *up, float *out, int dim) { cpu_swiglu(gate, up, out, dim); }
REF_API float ref_cpu_sigmoid(float x) { return cpu_sigmoid(x); }
REF_API void ref_cpu_softmax(float *x, int dim) { cpu_softmax(x, dim); }
REF_API void ref_cpu_topk(const float *scores, int dim, int K, int *indices, float *values) { cpu_topk(scores, dim, K, indices, values); }
REF_API void ref_cpu_normalize_weights(float *weights, int K) { cpu_normalize_weights(weights, K); }
REF_API void ref_cpu_vec_madd(float *dst, const float *src, float scale, int dim) { cpu_vec_madd(dst, src, scale, dim); }
