// MoE decode path: routed 3-bit experts (gate, up, SiLU, down), the 4-bit
// shared expert and the router-weighted combine.
//
//   prep      (only when the call has >= PREP_MIN_TOKENS tokens) groups the
//             (token, k) pairs by expert and turns every token's activations
//             into tensor-core operand fragments once, instead of once per CTA
//   kernel A  gate/up/SiLU : one CTA per (expert group, 16 gate rows + the 16
//             matching up rows); writes act[pair][inter]; the last CTA of a
//             group turns the finished activations into fragments for kernel B
//   kernel B  down + combine: one CTA per (expert group, 64 down rows); writes
//             per-pair down outputs to scratch; the last CTA to arrive for a
//             row chunk sums them in k order with the residual and the gated
//             shared expert (the arithmetic of moe_combine_residual,
//             finchmoe/shaders.metal:2196-2231).
//
// "Expert group" = the (token, k) pairs of this call that selected the same
// expert: its weights are read from HBM once for all of them.
//
// How a matvec is evaluated.  The packed codes never become floats on the
// CUDA cores.  A 3-bit code sitting at bits [p, p+3) of a 16-bit half-word,
// p <= 7, is -- after a single AND -- the fp16 *subnormal* q * 2^(p-24); that
// register goes straight into the A operand of mma.sync.m16n8k16 (f16 inputs,
// fp32 accumulate).  The B operand holds the activations, pre-scaled per
// k-slot by 2^(7-p) / norm (norm = power of two > max|x|) and split into an
// fp16 "hi" and a "lo * 2^11" column so that no mantissa bit of an fp32 x is
// lost.  Every product is exact in fp32; the per-group scale and bias are
// applied to the fp32 group sums:  out = sum_g s_g * (sum_i q_i x_i) + b_g *
// (sum_i x_i).  A 96-bit period (32 codes) needs 18 ANDs + 3 shifts.  Lane t
// of a quad owns period t of a 48-byte unit (128 codes = two groups); the two
// groups of a unit are kept apart by giving them different B columns.
#include "finch_internal.cuh"

namespace {

constexpr int A_THREADS = 256;
constexpr int A_WARPS = 8;
constexpr int A_ROWS = 16;  // gate rows (and up rows) per CTA in the 3-bit path: two MMA tiles
constexpr int S_ROWS = 8;   // gate rows (and up rows) per CTA in the 4-bit shared path: one MMA tile
constexpr int B_THREADS = 128;
constexpr int B_ROWS = 64;  // down rows per CTA: one MMA tile per warp
constexpr int PREP_MIN_TOKENS = 3;
constexpr int FRAG_PAD = 64;  // bytes between per-token fragment regions (keeps them on different banks)

struct WRef {  // affine tensor in device memory
    const uint8_t *W;
    const uint16_t *S, *B;
    int out_dim, in_dim;
};

struct MoeArgs {
    const uint8_t *pool_base;
    size_t slot_bytes;
    const int32_t *slot_row;  // slot table row of this layer: [n_experts]
    int n_experts;
    const void *h_post;
    int act_dtype;
    const int32_t *ids;
    const float *weights;
    const uint8_t *valid;
    int P, K, B;
    int hidden, inter;
    size_t gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b;
    int scale_dtype;
    float *act;        // [P][inter]
    float *partial;    // [P + B][hidden]
    unsigned *counters;  // [hidden / 64] row-chunk arrivals of kernel B, then [P + 1] group arrivals of kernel A
    unsigned *cnt_a;
    int *status;
    int has_shared;
    WRef sh_gate, sh_up, sh_down;
    int sh_scale_dtype, sh_inter;
    float *shared_act;  // [B][sh_inter]
    const float *gate_score;
    const float *h_mid;
    float *hidden_out;
    // operand fragments in global scratch
    int use_prep;
    uint2 *xfrag3;  // [B][hidden/128 * 72]   (prep)
    uint2 *xfrag4;  // [B][hidden/64 * 32]    (prep, shared expert)
    float *xXg;     // [B][128]
    int *xE;        // [B]
    int2 *grp;      // [P] {m, slot}: m = 0 unless pair p is the first of its group
    uint8_t *grp_pairs;  // [P][64]
    int *n_groups;
    uint2 *afrag3;  // [P][inter/128 * 72]    (written by kernel A)
    float *aXg;     // [P][128]
    int *aE;        // [P]
    uint2 *sfrag4;  // [B][sh_inter/64 * 32]
    float *sXg;     // [B][128]
    int *sE;        // [B]
};

// slot-in-register tables of the 3-bit extraction: entry [2*e + half] for
// extraction e (0..17) = code index inside the 32-code period (-1: empty) and
// the bit position p of the code inside its half-word.
__constant__ int8_t c_idx3[36] = {0, 6, 1, 7, 2, -1, 3, 8, 4, 9, 5, 10, 11, 16, 12, 17, 13, 18,
                                  14, 19, 15, 20, -1, 21, 22, 27, 23, 28, -1, 29, 24, 30, 25, 31, 26, -1};
__constant__ int8_t c_pos3[36] = {0, 2, 3, 5, 6, 0, 1, 0, 4, 3, 7, 6, 1, 0, 4, 3, 7, 6,
                                  2, 1, 5, 4, 0, 7, 2, 1, 5, 4, 0, 7, 0, 2, 3, 5, 6, 0};

__device__ __forceinline__ void extract3(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t (&e)[18]) {
    const uint32_t v1 = __funnelshift_r(w0, w1, 8), v3 = __funnelshift_r(w1, w2, 8), v5 = w2 >> 8;
    e[0] = w0 & 0x001C0007u;  e[1] = w0 & 0x00E00038u;  e[2] = w0 & 0x000001C0u;
    e[3] = v1 & 0x0007000Eu;  e[4] = v1 & 0x00380070u;  e[5] = v1 & 0x01C00380u;
    e[6] = w1 & 0x0007000Eu;  e[7] = w1 & 0x00380070u;  e[8] = w1 & 0x01C00380u;
    e[9] = v3 & 0x000E001Cu;  e[10] = v3 & 0x007000E0u; e[11] = v3 & 0x03800000u;
    e[12] = w2 & 0x000E001Cu; e[13] = w2 & 0x007000E0u; e[14] = w2 & 0x03800000u;
    e[15] = v5 & 0x001C0007u; e[16] = v5 & 0x00E00038u; e[17] = v5 & 0x000001C0u;
}

// One u32 of eight nibbles -> four registers: (0,4) (1,5) at p = 0 / 4 of the
// word itself, (2,6) (3,7) at p = 0 / 4 of the word shifted right by 8.
__device__ __forceinline__ void extract4(uint32_t w, uint32_t (&e)[4]) {
    const uint32_t v = w >> 8;
    e[0] = w & 0x000F000Fu; e[1] = w & 0x00F000F0u;
    e[2] = v & 0x000F000Fu; e[3] = v & 0x00F000F0u;
}

__device__ __forceinline__ float pow2_biased(int e) { return __uint_as_float((uint32_t)e << 23); }

// Loads one activation row into xs (fp32 shared memory) and produces the group
// sums Xg[0..K/64) and E, the biased exponent of a power of two > max|x|
// (clamped so that every derived scale factor is a normal float).  All NT
// threads of the CTA take part; ends with a barrier.
template <int NT>
__device__ void load_x(const void *src, int dtype, int K, float *xs, float *Xg, float *warp_max, int *E_out) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float amax = 0.f;
    for (int base0 = 0; base0 < K; base0 += NT * 8) {
        const int base = base0 + tid * 8;
        float v[8];
        if (base < K) {
            if (dtype == FINCH_BF16) {
                const uint4 r = __ldcg(reinterpret_cast<const uint4 *>((const uint16_t *)src + base));
                const uint32_t u[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    v[2 * j] = __uint_as_float(u[j] << 16);
                    v[2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
                }
            } else {
                const float4 a = __ldcg(reinterpret_cast<const float4 *>((const float *)src + base));
                const float4 b = __ldcg(reinterpret_cast<const float4 *>((const float *)src + base + 4));
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = 0.f;
        }
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            s += v[j];
            amax = fmaxf(amax, fabsf(v[j]));
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        if (base < K) {
            *reinterpret_cast<float4 *>(xs + base) = make_float4(v[0], v[1], v[2], v[3]);
            *reinterpret_cast<float4 *>(xs + base + 4) = make_float4(v[4], v[5], v[6], v[7]);
            if ((lane & 7) == 0) Xg[base >> 6] = s;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) warp_max[warp] = amax;
    __syncthreads();
    if (tid == 0) {
        float m = 0.f;
        for (int w = 0; w < NT / 32; w++) m = fmaxf(m, warp_max[w]);
        int E = (int)(__float_as_uint(m) >> 23) + 1;
        E = E < 30 ? 30 : (E > 230 ? 230 : E);
        *E_out = E;
    }
    __syncthreads();
}

// hi / lo fp16 split of four pre-scaled activations -> the two B-fragment entries of one lane.
__device__ __forceinline__ void split4(const float (&xv)[4], uint2 &hi, uint2 &lo) {
    float h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __half hh = __float2half_rn(xv[i]);
        h[i] = __half2float(hh);
        l[i] = (xv[i] - h[i]) * 2048.0f;
    }
    hi = make_uint2(finch_pack_h2(h[0], h[1]), finch_pack_h2(h[2], h[3]));
    lo = make_uint2(finch_pack_h2(l[0], l[1]), finch_pack_h2(l[2], l[3]));
}

// B fragments of one token, 3-bit layout: frag[((u * 9 + j) * 2 + term) * 4 + t]
// (K/128 * 72 entries of 8 bytes).  frag may be shared or global memory.
template <int NT>
__device__ void build_frag3(const float *xs, int K, int E, uint2 *frag) {
    const int entries = (K / 128) * 36;
    for (int e = threadIdx.x; e < entries; e += NT) {
        const int u = e / 36, r = e - u * 36, j = r >> 2, t = r & 3;
        float xv[4];
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int ti = (2 * j + (s >> 1)) * 2 + (s & 1);
            const int idx = c_idx3[ti];
            xv[s] = idx < 0 ? 0.f : xs[u * 128 + t * 32 + idx] * pow2_biased(261 - E - c_pos3[ti]);
        }
        uint2 hi, lo;
        split4(xv, hi, lo);
        const int o = (u * 9 + j) * 8 + t;
        frag[o] = hi;
        frag[o + 4] = lo;
    }
}

// B fragments of one token, 4-bit layout: frag[((gamma * 4 + j) * 2 + term) * 4 + t]
// (K/64 * 32 entries).
template <int NT>
__device__ void build_frag4(const float *xs, int K, int E, uint2 *frag) {
    const int entries = (K / 64) * 16;
    for (int e = threadIdx.x; e < entries; e += NT) {
        const int gamma = e >> 4, j = (e >> 2) & 3, t = e & 3;
        const int wbase = gamma * 64 + (2 * t + (j >> 1)) * 8 + ((j & 1) ? 2 : 0);
        // slots: (code, p) = (0,0) (4,0) (1,4) (5,4) for even j; (2,0) (6,0) (3,4) (7,4) for odd j
        float xv[4];
        xv[0] = xs[wbase + 0] * pow2_biased(261 - E);
        xv[1] = xs[wbase + 4] * pow2_biased(261 - E);
        xv[2] = xs[wbase + 1] * pow2_biased(257 - E);
        xv[3] = xs[wbase + 5] * pow2_biased(257 - E);
        uint2 hi, lo;
        split4(xv, hi, lo);
        const int o = (gamma * 4 + j) * 8 + t;
        frag[o] = hi;
        frag[o + 4] = lo;
    }
}

// ---- inner loops ---------------------------------------------------------
// 3-bit.  NTILE MMA tiles share the B fragments of each unit.  Tile i has
// fragment rows g -> packed row rowA[i], g + 8 -> rowB[i] (shared memory), with
// scale rows sA[i], sB[i] (one u32 = the two groups of a unit).  Units u0,
// u0 + ustep, ... are accumulated.  On return lane (g, t) holds in runA/runB
// the raw sums of accumulator columns (token slot t>>1, term t&1).
template <int NTILE>
__device__ __forceinline__ void gemv3_units(const uint32_t *const (&rowA)[NTILE], const uint32_t *const (&rowB)[NTILE],
                                            const uint32_t *const (&sA)[NTILE], const uint32_t *const (&sB)[NTILE],
                                            int scale_dtype, const uint2 *frag0, const uint2 *frag1, int ntok, int units,
                                            int u0, int ustep, float (&runA)[NTILE], float (&runB)[NTILE]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tokslot = g >> 2, term = (g >> 1) & 1;
    const bool bact = ((g & 1) == (t >> 1)) && tokslot < ntok;
    const uint2 *fb = (tokslot ? frag1 : frag0) + term * 4 + t;
#pragma unroll
    for (int i = 0; i < NTILE; i++) runA[i] = runB[i] = 0.f;
    for (int u = u0; u < units; u += ustep) {
        uint2 b[9];
#pragma unroll
        for (int j = 0; j < 9; j++) b[j] = bact ? fb[(u * 9 + j) * 8] : make_uint2(0u, 0u);
#pragma unroll
        for (int i = 0; i < NTILE; i++) {
            const uint32_t *pa = rowA[i] + u * 12 + t * 3, *pb = rowB[i] + u * 12 + t * 3;
            uint32_t ea[18], eb[18];
            extract3(pa[0], pa[1], pa[2], ea);
            extract3(pb[0], pb[1], pb[2], eb);
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 9; j++) finch_mma16816(acc, ea[2 * j], eb[2 * j], ea[2 * j + 1], eb[2 * j + 1], b[j].x, b[j].y);
            float s0, s1;
            finch_widen16x2(sA[i][u], scale_dtype, s0, s1);
            runA[i] = fmaf(s0, acc[0], runA[i]);
            runA[i] = fmaf(s1, acc[1], runA[i]);
            finch_widen16x2(sB[i][u], scale_dtype, s0, s1);
            runB[i] = fmaf(s0, acc[2], runB[i]);
            runB[i] = fmaf(s1, acc[3], runB[i]);
        }
    }
}

// hi (even t) + lo (odd t) columns of a 3-bit result -> value, valid in even-t lanes
__device__ __forceinline__ float combine_hilo(float run, float fac) {
    const float o = __shfl_xor_sync(0xffffffffu, run, 1);
    return (run + o * (1.0f / 2048.0f)) * fac;
}

// 4-bit: one MMA tile (rows rowA / rowB), groups g0, g0 + gstep, ...; two
// tokens per pass (columns 0..3 = token 0 hi/lo, token 1 hi/lo).  Lane (g, t)
// with t < 2 returns the scaled sums (bias not included) of its rows for token t.
__device__ __forceinline__ void gemv4_groups(const uint32_t *rowA, const uint32_t *rowB, const uint16_t *sA, const uint16_t *sB,
                                             int scale_dtype, const uint2 *frag0, const uint2 *frag1, int ntok, int groups,
                                             int g0, int gstep, float &resA, float &resB) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tok = g >> 1, term = g & 1;
    const bool bact = tok < ntok;  // tok >= 2 never is
    const uint2 *fb = ((tok & 1) ? frag1 : frag0) + term * 4 + t;
    float runA = 0.f, runB = 0.f;
    for (int gm = g0; gm < groups; gm += gstep) {
        const uint2 wa = *reinterpret_cast<const uint2 *>(rowA + gm * 8 + t * 2);
        const uint2 wb = *reinterpret_cast<const uint2 *>(rowB + gm * 8 + t * 2);
        uint32_t ea[8], eb[8];
        {
            uint32_t x[4];
            extract4(wa.x, x); ea[0] = x[0]; ea[1] = x[1]; ea[2] = x[2]; ea[3] = x[3];
            extract4(wa.y, x); ea[4] = x[0]; ea[5] = x[1]; ea[6] = x[2]; ea[7] = x[3];
            extract4(wb.x, x); eb[0] = x[0]; eb[1] = x[1]; eb[2] = x[2]; eb[3] = x[3];
            extract4(wb.y, x); eb[4] = x[0]; eb[5] = x[1]; eb[6] = x[2]; eb[7] = x[3];
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint2 b = bact ? fb[(gm * 4 + j) * 8] : make_uint2(0u, 0u);
            finch_mma16816(acc, ea[2 * j], eb[2 * j], ea[2 * j + 1], eb[2 * j + 1], b.x, b.y);
        }
        // accumulator columns 2t, 2t+1 = (token t, hi), (token t, lo)
        runA = fmaf(finch_widen16(sA[gm], scale_dtype), acc[0] + acc[1] * (1.0f / 2048.0f), runA);
        runB = fmaf(finch_widen16(sB[gm], scale_dtype), acc[2] + acc[3] * (1.0f / 2048.0f), runB);
    }
    resA = runA;
    resB = runB;
}

// ---- expert groups -------------------------------------------------------
__device__ __forceinline__ bool pair_ok(const MoeArgs &a, int p) {
    if (a.valid && !a.valid[p]) return false;
    const int e = a.ids[p];
    if (e < 0 || e >= a.n_experts) return false;
    return a.slot_row[e] >= 0;
}

// Finds the pairs that share pair s's expert (no-prep path).  Returns false
// when s is not the first pair of its group.  sm_pairs[0..m) lists the group's
// pairs in ascending order.  Needs >= 64 threads.
__device__ bool find_group(const MoeArgs &a, int s, int *sm_pairs, unsigned *sm_ballot, int &m) {
    const int tid = threadIdx.x;
    if (tid < 64) {
        const bool same = tid < a.P && pair_ok(a, tid) && a.ids[tid] == a.ids[s];
        const unsigned bal = __ballot_sync(0xffffffffu, same);
        if ((tid & 31) == 0) sm_ballot[tid >> 5] = bal;
    }
    __syncthreads();
    const unsigned long long mask = (unsigned long long)sm_ballot[0] | ((unsigned long long)sm_ballot[1] << 32);
    if (!((mask >> s) & 1ull) || (__ffsll((long long)mask) - 1) != s) return false;
    m = __popcll(mask);
    if (tid < 64 && ((mask >> tid) & 1ull)) sm_pairs[__popcll(mask & ((1ull << tid) - 1ull))] = tid;
    __syncthreads();
    return true;
}

// Group of pair s from the prep table or by scanning the ids.  Uniform result.
__device__ bool get_group(const MoeArgs &a, int s, int *sm_pairs, unsigned *sm_ballot, int &m, int &slot) {
    if (a.use_prep) {
        const int2 gi = __ldg(&a.grp[s]);
        m = gi.x;
        slot = gi.y;
        if (m == 0) return false;
        if ((int)threadIdx.x < m) sm_pairs[threadIdx.x] = a.grp_pairs[s * 64 + threadIdx.x];
        __syncthreads();
        return true;
    }
    if (!find_group(a, s, sm_pairs, sm_ballot, m)) return false;
    slot = a.slot_row[a.ids[s]];
    return true;
}

// sm_ids[p] = expert id of pair p, or -1 when the pair is skipped; returns the number of groups.
__device__ int scan_pairs(const MoeArgs &a, int *sm_ids, unsigned *sm_ballot) {
    const int tid = threadIdx.x;
    if (tid < 64) sm_ids[tid] = (tid < a.P && pair_ok(a, tid)) ? a.ids[tid] : -1;
    __syncthreads();
    if (tid < 64) {
        bool first = sm_ids[tid] >= 0;
        for (int j = 0; j < tid && first; j++) first = sm_ids[j] != sm_ids[tid];
        const unsigned bal = __ballot_sync(0xffffffffu, first);
        if ((tid & 31) == 0) sm_ballot[tid >> 5] = bal;
    }
    __syncthreads();
    return __popc(sm_ballot[0]) + __popc(sm_ballot[1]);
}

__host__ __device__ inline int sc_stride_words(int groups) { return groups / 2 + (((groups / 2) % 8 == 0) ? 4 : 0); }
__host__ __device__ inline int frag3_entries(int K) { return (K / 128) * 72; }
__host__ __device__ inline int frag4_entries(int K) { return (K / 64) * 32; }

struct SmemA {  // byte offsets inside kernel A's dynamic shared memory
    int wg, wu, sc, xs, xg, frag, fstride, red, misc, total;
};
__host__ __device__ inline SmemA smem_a_layout(int hidden) {
    const int groups = hidden / 64;
    const int row3 = hidden * 3 / 8 + 16, row4 = hidden / 2 + 16;
    const int w3 = A_ROWS * row3, w4 = S_ROWS * row4;
    const int wbytes = w3 > w4 ? w3 : w4;
    const int sc3 = 4 * A_ROWS * sc_stride_words(groups) * 4, sc4 = 4 * S_ROWS * groups * 2;
    const int f3 = frag3_entries(hidden) * 8, f4 = frag4_entries(hidden) * 8;
    SmemA L;
    L.wg = 0;
    L.wu = wbytes;
    L.sc = 2 * wbytes;
    L.xs = L.sc + (sc3 > sc4 ? sc3 : sc4);
    L.xg = L.xs + hidden * 4;
    L.frag = L.xg + 2 * 128 * 4;
    L.fstride = (f3 > f4 ? f3 : f4) + FRAG_PAD;
    L.red = L.frag + 2 * L.fstride;
    L.misc = L.red + A_WARPS * 2 * 2 * 2 * 8 * 4;
    L.total = L.misc + 512;
    return L;
}

// group sums + E of one token / pair from global scratch into shared memory
__device__ __forceinline__ void fetch_xg(const float *gXg, const int *gE, int idx, int groups, float *Xg, int *sm_E) {
    for (int i = threadIdx.x; i < groups; i += blockDim.x) Xg[i] = __ldcg(gXg + (size_t)idx * 128 + i);
    if (threadIdx.x == 0) *sm_E = __ldcg(gE + idx);
}

// ============================ prep ========================================
// grid: B + 1 CTAs of 256 threads.  CTA b < B: fragments of token b.  CTA B: groups.
__global__ void __launch_bounds__(A_THREADS) moe_prep_kernel(const MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    float *xs = reinterpret_cast<float *>(smem);
    float *Xg = xs + a.hidden;
    float *warp_max = Xg + 128;
    int *sm_E = reinterpret_cast<int *>(warp_max + 8);
    int *sm_ids = sm_E + 4;
    unsigned *sm_ballot = reinterpret_cast<unsigned *>(sm_ids + 64);
    const int b = blockIdx.x, tid = threadIdx.x, K = a.hidden;
    if (b < a.B) {
        const void *src = a.act_dtype == FINCH_BF16 ? (const void *)((const uint16_t *)a.h_post + (size_t)b * K)
                                                     : (const void *)((const float *)a.h_post + (size_t)b * K);
        load_x<A_THREADS>(src, a.act_dtype, K, xs, Xg, warp_max, sm_E);
        const int E = *sm_E;
        build_frag3<A_THREADS>(xs, K, E, a.xfrag3 + (size_t)b * frag3_entries(K));
        if (a.has_shared) build_frag4<A_THREADS>(xs, K, E, a.xfrag4 + (size_t)b * frag4_entries(K));
        for (int i = tid; i < K / 64; i += A_THREADS) a.xXg[(size_t)b * 128 + i] = Xg[i];
        if (tid == 0) a.xE[b] = E;
        return;
    }
    const int ng = scan_pairs(a, sm_ids, sm_ballot);
    if (tid == 0) *a.n_groups = ng;
    if (tid < a.P) {
        const int id = sm_ids[tid];
        bool first = id >= 0;
        for (int j = 0; j < tid && first; j++) first = sm_ids[j] != id;
        int m = 0;
        if (first)
            for (int j = tid; j < a.P; j++)
                if (sm_ids[j] == id) a.grp_pairs[tid * 64 + m++] = (uint8_t)j;
        a.grp[tid] = make_int2(m, first ? a.slot_row[id] : -1);
    }
}

// ============================ kernel A ====================================
// grid: x = row chunk (inter / 16), y = pair slot 0..P-1, then two rows of
// CTAs for the shared expert's gate/up (8 + 8 rows each).
__global__ void __launch_bounds__(A_THREADS) moe_gateup_kernel(const MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const SmemA L = smem_a_layout(a.hidden);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    float *xs = reinterpret_cast<float *>(smem + L.xs);
    float *Xg = reinterpret_cast<float *>(smem + L.xg);
    uint2 *frag0 = reinterpret_cast<uint2 *>(smem + L.frag);
    uint2 *frag1 = reinterpret_cast<uint2 *>(smem + L.frag + L.fstride);
    float *red = reinterpret_cast<float *>(smem + L.red);
    int *sm_pairs = reinterpret_cast<int *>(smem + L.misc);                    // [64]
    unsigned *sm_ballot = reinterpret_cast<unsigned *>(smem + L.misc + 256);   // [2]
    float *warp_max = reinterpret_cast<float *>(smem + L.misc + 272);          // [8]
    int *sm_E = reinterpret_cast<int *>(smem + L.misc + 304);                  // [2]
    int *sm_last = reinterpret_cast<int *>(smem + L.misc + 312);
    uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + L.misc + 320);
    const int s = blockIdx.y, K = a.hidden, groups = K / 64;

    if (s < a.P) {
        // ---------------- routed expert, 3-bit ----------------
        int m = 0, slot = -1;
        if (!get_group(a, s, sm_pairs, sm_ballot, m, slot)) return;
        const int r0 = blockIdx.x * A_ROWS;
        const uint8_t *blk = a.pool_base + (size_t)slot * a.slot_bytes;
        const int rowb = K * 3 / 8, rowp = rowb + 16;  // global / padded shared row pitch
        const unsigned fbytes = (unsigned)frag3_entries(K) * 8u;
        if (tid == 0) finch_mbar_init(mbar, 1);
        __syncthreads();
        if (warp == 0) {
            if (lane == 0) finch_mbar_expect_tx(mbar, 2u * A_ROWS * rowb + (a.use_prep ? (unsigned)min(2, m) * fbytes : 0u));
            __syncwarp();
            const int r = lane & 15;
            const uint8_t *src = blk + (lane < 16 ? a.gate_w : a.up_w) + (size_t)(r0 + r) * rowb;
            finch_bulk_g2s(smem + (lane < 16 ? L.wg : L.wu) + r * rowp, src, rowb, mbar);
            if (a.use_prep && lane < min(2, m))
                finch_bulk_g2s(lane ? frag1 : frag0, a.xfrag3 + (size_t)(sm_pairs[lane] / a.K) * frag3_entries(K), fbytes, mbar);
        }
        // scales and biases: plain loads into padded rows
        const int scw = sc_stride_words(groups), rw = groups / 2;
        uint32_t *sc = reinterpret_cast<uint32_t *>(smem + L.sc);
        for (int i = tid; i < 4 * A_ROWS * rw; i += A_THREADS) {
            const int arr = i / (A_ROWS * rw), rem = i - arr * (A_ROWS * rw), r = rem / rw, c = rem - r * rw;
            const size_t off = arr == 0 ? a.gate_s : arr == 1 ? a.gate_b : arr == 2 ? a.up_s : a.up_b;
            sc[(arr * A_ROWS + r) * scw + c] = __ldg(reinterpret_cast<const uint32_t *>(blk + off + (size_t)(r0 + r) * groups * 2) + c);
        }
        const int npass = (m + 1) / 2;
        for (int ps = 0; ps < npass; ps++) {
            const int ntok = min(2, m - 2 * ps);
            if (a.use_prep) {
                if (ps > 0 && warp == 0) {  // fragments of this pass's tokens (the previous pass is done with the buffers)
                    if (lane == 0) finch_mbar_expect_tx(mbar, (unsigned)ntok * fbytes);
                    __syncwarp();
                    if (lane < ntok)
                        finch_bulk_g2s(lane ? frag1 : frag0, a.xfrag3 + (size_t)(sm_pairs[2 * ps + lane] / a.K) * frag3_entries(K),
                                       fbytes, mbar);
                }
                for (int ts = 0; ts < ntok; ts++) fetch_xg(a.xXg, a.xE, sm_pairs[2 * ps + ts] / a.K, groups, Xg + ts * 128, sm_E + ts);
                __syncthreads();
            } else {
                for (int ts = 0; ts < ntok; ts++) {
                    const int tok = sm_pairs[2 * ps + ts] / a.K;
                    const void *src = a.act_dtype == FINCH_BF16 ? (const void *)((const uint16_t *)a.h_post + (size_t)tok * K)
                                                                 : (const void *)((const float *)a.h_post + (size_t)tok * K);
                    load_x<A_THREADS>(src, a.act_dtype, K, xs, Xg + ts * 128, warp_max, sm_E + ts);
                    build_frag3<A_THREADS>(xs, K, sm_E[ts], ts ? frag1 : frag0);
                    __syncthreads();
                }
            }
            if (a.use_prep || ps == 0) {
                if (!finch_mbar_wait(mbar, ps & 1)) {
                    if (tid == 0) atomicExch(a.status, FINCH_E_TIMEOUT);
                    return;
                }
            }
            const uint32_t *rA[2], *rB[2], *sA[2], *sB[2];
#pragma unroll
            for (int tile = 0; tile < 2; tile++) {
                const int row = tile * 8 + g;
                rA[tile] = reinterpret_cast<const uint32_t *>(smem + L.wg + row * rowp);
                rB[tile] = reinterpret_cast<const uint32_t *>(smem + L.wu + row * rowp);
                sA[tile] = sc + (0 * A_ROWS + row) * scw;
                sB[tile] = sc + (2 * A_ROWS + row) * scw;
            }
            float runG[2], runU[2];
            gemv3_units<2>(rA, rB, sA, sB, a.scale_dtype, frag0, frag1, ntok, K / 128, warp, A_WARPS, runG, runU);
            const float fac = pow2_biased(sm_E[t >> 1] + 17);
#pragma unroll
            for (int tile = 0; tile < 2; tile++) {
                const float vg = combine_hilo(runG[tile], fac), vu = combine_hilo(runU[tile], fac);
                if ((t & 1) == 0) {
                    float *o = red + (((warp * 2 + tile) * 2 + (t >> 1)) * 2) * 8 + g;
                    o[0] = vg;
                    o[8] = vu;
                }
            }
            __syncthreads();
            if (tid < 64) {
                // thread = (tile, token slot, row g, gate|up): cross-warp sum in fixed order + bias . group sums
                const int up = tid & 1, gg = (tid >> 1) & 7, ts = (tid >> 4) & 1, tile = tid >> 5;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < A_WARPS; w++) v += red[(((w * 2 + tile) * 2 + ts) * 2 + up) * 8 + gg];
                const uint32_t *brow = sc + ((up ? 3 : 1) * A_ROWS + tile * 8 + gg) * scw;
                const float *xg = Xg + ts * 128;
                for (int c = 0; c < rw; c++) {
                    float b0, b1;
                    finch_widen16x2(brow[c], a.scale_dtype, b0, b1);
                    v = fmaf(b0, xg[2 * c], v);
                    v = fmaf(b1, xg[2 * c + 1], v);
                }
                const float other = __shfl_xor_sync(0xffffffffu, v, 1);  // gate <-> up of the same row
                if (!up && ts < ntok) {
                    const int pair = sm_pairs[2 * ps + ts];
                    a.act[(size_t)pair * a.inter + r0 + tile * 8 + gg] = (v / (1.0f + expf(-v))) * other;
                }
            }
            __syncthreads();
        }
        // ---- the last CTA of the group turns the finished activations into fragments for kernel B ----
        __threadfence();
        __syncthreads();
        if (tid == 0) *sm_last = atomicAdd(&a.cnt_a[s], 1u) == (unsigned)(gridDim.x - 1);
        __syncthreads();
        if (!*sm_last) return;
        __threadfence();
        for (int i = 0; i < m; i++) {
            const int pair = sm_pairs[i];
            load_x<A_THREADS>(a.act + (size_t)pair * a.inter, FINCH_F32, a.inter, xs, Xg, warp_max, sm_E);
            build_frag3<A_THREADS>(xs, a.inter, *sm_E, a.afrag3 + (size_t)pair * frag3_entries(a.inter));
            for (int c = tid; c < a.inter / 64; c += A_THREADS) a.aXg[(size_t)pair * 128 + c] = Xg[c];
            if (tid == 0) a.aE[pair] = *sm_E;
            __syncthreads();
        }
        if (tid == 0) a.cnt_a[s] = 0u;
        return;
    }

    // ---------------- shared expert gate/up, 4-bit ----------------
    const int I = a.sh_inter;
    const int r0 = ((s - a.P) * gridDim.x + blockIdx.x) * S_ROWS;
    if (r0 >= I) return;
    const int n_ctas = I / S_ROWS;
    const int rowb = K / 2, rowp = rowb + 16;
    const unsigned fbytes = (unsigned)frag4_entries(K) * 8u;
    if (tid == 0) finch_mbar_init(mbar, 1);
    __syncthreads();
    if (warp == 0) {
        if (lane == 0) finch_mbar_expect_tx(mbar, 2u * S_ROWS * rowb + (a.use_prep ? (unsigned)min(2, a.B) * fbytes : 0u));
        __syncwarp();
        if (lane < 2 * S_ROWS) {
            const int r = lane & (S_ROWS - 1);
            const uint8_t *src = (lane < S_ROWS ? a.sh_gate.W : a.sh_up.W) + (size_t)(r0 + r) * rowb;
            finch_bulk_g2s(smem + (lane < S_ROWS ? L.wg : L.wu) + r * rowp, src, rowb, mbar);
        }
        if (a.use_prep && lane < min(2, a.B)) finch_bulk_g2s(lane ? frag1 : frag0, a.xfrag4 + (size_t)lane * frag4_entries(K), fbytes, mbar);
    }
    uint16_t *sc = reinterpret_cast<uint16_t *>(smem + L.sc);  // [4][S_ROWS][groups]: gate S, gate B, up S, up B
    for (int i = tid; i < 4 * S_ROWS * groups; i += A_THREADS) {
        const int arr = i / (S_ROWS * groups), rem = i - arr * (S_ROWS * groups);
        const uint16_t *src = arr == 0 ? a.sh_gate.S : arr == 1 ? a.sh_gate.B : arr == 2 ? a.sh_up.S : a.sh_up.B;
        sc[i] = src[(size_t)r0 * groups + rem];
    }
    const int npass = (a.B + 1) / 2;
    for (int ps = 0; ps < npass; ps++) {
        const int ntok = min(2, a.B - 2 * ps);
        if (a.use_prep) {
            if (ps > 0 && warp == 0) {
                if (lane == 0) finch_mbar_expect_tx(mbar, (unsigned)ntok * fbytes);
                __syncwarp();
                if (lane < ntok) finch_bulk_g2s(lane ? frag1 : frag0, a.xfrag4 + (size_t)(2 * ps + lane) * frag4_entries(K), fbytes, mbar);
            }
            for (int ts = 0; ts < ntok; ts++) fetch_xg(a.xXg, a.xE, 2 * ps + ts, groups, Xg + ts * 128, sm_E + ts);
            __syncthreads();
        } else {
            for (int ts = 0; ts < ntok; ts++) {
                const int tok = 2 * ps + ts;
                const void *src = a.act_dtype == FINCH_BF16 ? (const void *)((const uint16_t *)a.h_post + (size_t)tok * K)
                                                             : (const void *)((const float *)a.h_post + (size_t)tok * K);
                load_x<A_THREADS>(src, a.act_dtype, K, xs, Xg + ts * 128, warp_max, sm_E + ts);
                build_frag4<A_THREADS>(xs, K, sm_E[ts], ts ? frag1 : frag0);
                __syncthreads();
            }
        }
        if (a.use_prep || ps == 0) {
            if (!finch_mbar_wait(mbar, ps & 1)) {
                if (tid == 0) atomicExch(a.status, FINCH_E_TIMEOUT);
                return;
            }
        }
        float rg, ru;
        gemv4_groups(reinterpret_cast<const uint32_t *>(smem + L.wg + g * rowp), reinterpret_cast<const uint32_t *>(smem + L.wu + g * rowp),
                     sc + (0 * S_ROWS + g) * groups, sc + (2 * S_ROWS + g) * groups, a.sh_scale_dtype, frag0, frag1, ntok, groups, warp,
                     A_WARPS, rg, ru);
        if (t < 2) {
            const float fac = pow2_biased(sm_E[t] + 17);
            red[((warp * 2 + t) * 2 + 0) * 8 + g] = rg * fac;
            red[((warp * 2 + t) * 2 + 1) * 8 + g] = ru * fac;
        }
        __syncthreads();
        if (tid < 32) {
            const int up = tid & 1, gg = (tid >> 1) & 7, ts = tid >> 4;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < A_WARPS; w++) v += red[((w * 2 + ts) * 2 + up) * 8 + gg];
            const uint16_t *brow = sc + ((up ? 3 : 1) * S_ROWS + gg) * groups;
            const float *xg = Xg + ts * 128;
            for (int c = 0; c < groups; c++) v = fmaf(finch_widen16(brow[c], a.sh_scale_dtype), xg[c], v);
            const float other = __shfl_xor_sync(0xffffffffu, v, 1);
            if (!up && ts < ntok) a.shared_act[(size_t)(2 * ps + ts) * I + r0 + gg] = (v / (1.0f + expf(-v))) * other;
        }
        __syncthreads();
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) *sm_last = atomicAdd(&a.cnt_a[a.P], 1u) == (unsigned)(n_ctas - 1);
    __syncthreads();
    if (!*sm_last) return;
    __threadfence();
    for (int b = 0; b < a.B; b++) {
        load_x<A_THREADS>(a.shared_act + (size_t)b * I, FINCH_F32, I, xs, Xg, warp_max, sm_E);
        build_frag4<A_THREADS>(xs, I, *sm_E, a.sfrag4 + (size_t)b * frag4_entries(I));
        for (int c = tid; c < I / 64; c += A_THREADS) a.sXg[(size_t)b * 128 + c] = Xg[c];
        if (tid == 0) a.sE[b] = *sm_E;
        __syncthreads();
    }
    if (tid == 0) a.cnt_a[a.P] = 0u;
}

struct SmemB {
    int w, sc, xg, frag, fstride, misc, total;
};
__host__ __device__ inline SmemB smem_b_layout(int inter, int sh_inter) {
    const int row3 = inter * 3 / 8 + 16, row4 = sh_inter / 2 + 16;
    const int wb = B_ROWS * (row3 > row4 ? row3 : row4);
    const int sc3 = 2 * B_ROWS * sc_stride_words(inter / 64) * 4, sc4 = 2 * B_ROWS * (sh_inter / 64) * 2;
    const int f3 = frag3_entries(inter) * 8, f4 = frag4_entries(sh_inter) * 8;
    SmemB L;
    L.w = 0;
    L.sc = wb;
    L.xg = L.sc + (sc3 > sc4 ? sc3 : sc4);
    L.frag = L.xg + 2 * 128 * 4;
    L.fstride = (f3 > f4 ? f3 : f4) + FRAG_PAD;
    L.misc = L.frag + 2 * L.fstride;
    L.total = L.misc + 1024;
    return L;
}

// ============================ kernel B ====================================
// grid: x = row chunk of 64 down rows, y = pair slot (0..P-1 routed; P = shared / finisher)
__global__ void __launch_bounds__(B_THREADS) moe_down_combine_kernel(const MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const SmemB L = smem_b_layout(a.inter, a.sh_inter);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    float *Xg = reinterpret_cast<float *>(smem + L.xg);
    uint2 *frag0 = reinterpret_cast<uint2 *>(smem + L.frag);
    uint2 *frag1 = reinterpret_cast<uint2 *>(smem + L.frag + L.fstride);
    int *sm_pairs = reinterpret_cast<int *>(smem + L.misc);                   // [64]
    int *sm_ids = reinterpret_cast<int *>(smem + L.misc + 256);               // [64]
    unsigned *sm_ballot = reinterpret_cast<unsigned *>(smem + L.misc + 512);  // [2]
    int *sm_E = reinterpret_cast<int *>(smem + L.misc + 528);                 // [2]
    int *sm_last = reinterpret_cast<int *>(smem + L.misc + 540);
    uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + L.misc + 576);
    const int s = blockIdx.y, r0 = blockIdx.x * B_ROWS;
    const int ra = warp * 16 + g, rb = ra + 8;

    if (s < a.P) {
        int m = 0, slot = -1;
        if (!get_group(a, s, sm_pairs, sm_ballot, m, slot)) return;
        const int K = a.inter, groups = K / 64;
        const uint8_t *blk = a.pool_base + (size_t)slot * a.slot_bytes;
        const int rowb = K * 3 / 8, rowp = rowb + 16;
        const unsigned fbytes = (unsigned)frag3_entries(K) * 8u;
        if (tid == 0) finch_mbar_init(mbar, 1);
        __syncthreads();
        if (warp == 0) {
            if (lane == 0) finch_mbar_expect_tx(mbar, (unsigned)B_ROWS * rowb + (unsigned)min(2, m) * fbytes);
            __syncwarp();
            for (int r = lane; r < B_ROWS; r += 32)
                finch_bulk_g2s(smem + L.w + r * rowp, blk + a.down_w + (size_t)(r0 + r) * rowb, rowb, mbar);
            if (lane < min(2, m)) finch_bulk_g2s(lane ? frag1 : frag0, a.afrag3 + (size_t)sm_pairs[lane] * frag3_entries(K), fbytes, mbar);
        }
        const int scw = sc_stride_words(groups), rw = groups / 2;
        uint32_t *sc = reinterpret_cast<uint32_t *>(smem + L.sc);
        for (int i = tid; i < 2 * B_ROWS * rw; i += B_THREADS) {
            const int arr = i / (B_ROWS * rw), rem = i - arr * (B_ROWS * rw), r = rem / rw, c = rem - r * rw;
            sc[(arr * B_ROWS + r) * scw + c] =
                __ldg(reinterpret_cast<const uint32_t *>(blk + (arr ? a.down_b : a.down_s) + (size_t)(r0 + r) * groups * 2) + c);
        }
        const int npass = (m + 1) / 2;
        for (int ps = 0; ps < npass; ps++) {
            const int ntok = min(2, m - 2 * ps);
            if (ps > 0 && warp == 0) {
                if (lane == 0) finch_mbar_expect_tx(mbar, (unsigned)ntok * fbytes);
                __syncwarp();
                if (lane < ntok) finch_bulk_g2s(lane ? frag1 : frag0, a.afrag3 + (size_t)sm_pairs[2 * ps + lane] * frag3_entries(K), fbytes, mbar);
            }
            for (int ts = 0; ts < ntok; ts++) fetch_xg(a.aXg, a.aE, sm_pairs[2 * ps + ts], groups, Xg + ts * 128, sm_E + ts);
            __syncthreads();
            if (!finch_mbar_wait(mbar, ps & 1)) {
                if (tid == 0) atomicExch(a.status, FINCH_E_TIMEOUT);
                return;
            }
            const uint32_t *rA[1] = {reinterpret_cast<const uint32_t *>(smem + L.w + ra * rowp)};
            const uint32_t *rB[1] = {reinterpret_cast<const uint32_t *>(smem + L.w + rb * rowp)};
            const uint32_t *sA[1] = {sc + ra * scw}, *sB[1] = {sc + rb * scw};
            float runA[1], runB[1];
            gemv3_units<1>(rA, rB, sA, sB, a.scale_dtype, frag0, frag1, ntok, K / 128, 0, 1, runA, runB);
            const float fac = pow2_biased(sm_E[t >> 1] + 17);
            float va = combine_hilo(runA[0], fac), vb = combine_hilo(runB[0], fac);
            if ((t & 1) == 0 && (t >> 1) < ntok) {
                const float *xg = Xg + (t >> 1) * 128;
                const uint32_t *ba = sc + (B_ROWS + ra) * scw, *bb = sc + (B_ROWS + rb) * scw;
                for (int c = 0; c < rw; c++) {
                    float b0, b1;
                    finch_widen16x2(ba[c], a.scale_dtype, b0, b1);
                    va = fmaf(b0, xg[2 * c], va);
                    va = fmaf(b1, xg[2 * c + 1], va);
                    finch_widen16x2(bb[c], a.scale_dtype, b0, b1);
                    vb = fmaf(b0, xg[2 * c], vb);
                    vb = fmaf(b1, xg[2 * c + 1], vb);
                }
                const int pair = sm_pairs[2 * ps + (t >> 1)];
                a.partial[(size_t)pair * a.hidden + r0 + ra] = va;
                a.partial[(size_t)pair * a.hidden + r0 + rb] = vb;
            }
            __syncthreads();
        }
    } else if (a.has_shared) {
        // shared expert down projection, 4-bit, all B tokens, two per pass
        const int K = a.sh_inter, groups = K / 64;
        const int rowb = K / 2, rowp = rowb + 16;
        const unsigned fbytes = (unsigned)frag4_entries(K) * 8u;
        if (tid == 0) finch_mbar_init(mbar, 1);
        __syncthreads();
        if (warp == 0) {
            if (lane == 0) finch_mbar_expect_tx(mbar, (unsigned)B_ROWS * rowb + (unsigned)min(2, a.B) * fbytes);
            __syncwarp();
            for (int r = lane; r < B_ROWS; r += 32) finch_bulk_g2s(smem + L.w + r * rowp, a.sh_down.W + (size_t)(r0 + r) * rowb, rowb, mbar);
            if (lane < min(2, a.B)) finch_bulk_g2s(lane ? frag1 : frag0, a.sfrag4 + (size_t)lane * frag4_entries(K), fbytes, mbar);
        }
        uint16_t *sc = reinterpret_cast<uint16_t *>(smem + L.sc);  // [2][B_ROWS][groups]
        for (int i = tid; i < 2 * B_ROWS * groups; i += B_THREADS) {
            const int arr = i / (B_ROWS * groups), rem = i - arr * (B_ROWS * groups);
            sc[i] = (arr ? a.sh_down.B : a.sh_down.S)[(size_t)r0 * groups + rem];
        }
        const int npass = (a.B + 1) / 2;
        for (int ps = 0; ps < npass; ps++) {
            const int ntok = min(2, a.B - 2 * ps);
            if (ps > 0 && warp == 0) {
                if (lane == 0) finch_mbar_expect_tx(mbar, (unsigned)ntok * fbytes);
                __syncwarp();
                if (lane < ntok) finch_bulk_g2s(lane ? frag1 : frag0, a.sfrag4 + (size_t)(2 * ps + lane) * frag4_entries(K), fbytes, mbar);
            }
            for (int ts = 0; ts < ntok; ts++) fetch_xg(a.sXg, a.sE, 2 * ps + ts, groups, Xg + ts * 128, sm_E + ts);
            __syncthreads();
            if (!finch_mbar_wait(mbar, ps & 1)) {
                if (tid == 0) atomicExch(a.status, FINCH_E_TIMEOUT);
                return;
            }
            float va, vb;
            gemv4_groups(reinterpret_cast<const uint32_t *>(smem + L.w + ra * rowp), reinterpret_cast<const uint32_t *>(smem + L.w + rb * rowp),
                         sc + ra * groups, sc + rb * groups, a.sh_scale_dtype, frag0, frag1, ntok, groups, 0, 1, va, vb);
            if (t < ntok) {
                const float fac = pow2_biased(sm_E[t] + 17);
                va *= fac;
                vb *= fac;
                const float *xg = Xg + t * 128;
                const uint16_t *ba = sc + (B_ROWS + ra) * groups, *bb = sc + (B_ROWS + rb) * groups;
                for (int c = 0; c < groups; c++) {
                    va = fmaf(finch_widen16(ba[c], a.sh_scale_dtype), xg[c], va);
                    vb = fmaf(finch_widen16(bb[c], a.sh_scale_dtype), xg[c], vb);
                }
                float *o = a.partial + (size_t)(a.P + 2 * ps + t) * a.hidden + r0;
                o[ra] = va;
                o[rb] = vb;
            }
            __syncthreads();
        }
    }
    // (with no shared expert the y == P CTA only arrives, so that the combine always runs)

    // ---- arrival + combine by the last CTA of this row chunk ----
    int expected;
    if (a.use_prep) {
        expected = __ldcg(a.n_groups) + 1;
    } else {
        expected = scan_pairs(a, sm_ids, sm_ballot) + 1;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) *sm_last = atomicAdd(&a.counters[blockIdx.x], 1u) == (unsigned)(expected - 1);
    __syncthreads();
    if (!*sm_last) return;
    __threadfence();
    if (a.use_prep) scan_pairs(a, sm_ids, sm_ballot);
    for (int i = tid; i < a.B * B_ROWS; i += B_THREADS) {
        const int b = i / B_ROWS, row = r0 + (i % B_ROWS);
        float moe = 0.f;
        for (int k = 0; k < a.K; k++) {
            const int p = b * a.K + k;
            if (sm_ids[p] >= 0) moe = fmaf(a.weights[p], __ldcg(&a.partial[(size_t)p * a.hidden + row]), moe);
        }
        float h = a.h_mid ? a.h_mid[(size_t)b * a.hidden + row] : 0.f;
        h += moe;
        if (a.has_shared) {
            const float sg = 1.0f / (1.0f + expf(-a.gate_score[b]));
            h = fmaf(sg, __ldcg(&a.partial[(size_t)(a.P + b) * a.hidden + row]), h);
        }
        a.hidden_out[(size_t)b * a.hidden + row] = h;
    }
    if (tid == 0) a.counters[blockIdx.x] = 0u;
}

bool g_attr_set = false;

int check_shared(finch_ctx *ctx, const finch_shared *sh) {
    const finch_wdesc *w[3] = {&sh->gate, &sh->up, &sh->down};
    for (int i = 0; i < 3; i++) {
        int rc = finch_validate_wdesc(ctx, w[i], "shared expert");
        if (rc) return rc;
        if (w[i]->bits != 4) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "shared expert tensors must be 4-bit affine");
        if (w[i]->scale_dtype != sh->gate.scale_dtype) return finch_fail(ctx, FINCH_E_ARG, "shared expert: mixed scale dtypes");
    }
    const int H = ctx->cfg.hidden, I = sh->gate.out_dim;
    if (sh->gate.in_dim != H || sh->up.in_dim != H || sh->up.out_dim != I || sh->down.in_dim != I || sh->down.out_dim != H ||
        I % 64 || I < 64 || I > 8192)
        return finch_fail(ctx, FINCH_E_ARG, "shared expert: dims do not form %d -> I -> %d", H, H);
    if (I > (ctx->cfg.shared_inter > 0 ? ctx->cfg.shared_inter : 64))
        return finch_fail(ctx, FINCH_E_ARG, "shared expert: inter %d exceeds the context's shared_inter %d", I, ctx->cfg.shared_inter);
    if (!sh->gate_score) return finch_fail(ctx, FINCH_E_ARG, "shared expert: gate_score is NULL");
    return FINCH_OK;
}

}  // namespace

// Bytes of fragment / group scratch a context needs (allocated in finch_ctx_create).
size_t finch_decode_scratch_bytes(const finch_config &c) {
    const size_t P = (size_t)c.max_tokens * c.top_k, B = c.max_tokens;
    const int shi = c.shared_inter > 0 ? c.shared_inter : 64;
    size_t n = 0;
    n += B * frag3_entries(c.hidden) * 8 + B * frag4_entries(c.hidden) * 8 + B * 128 * 4 + B * 4;
    n += P * 8 + P * 64 + 256;
    n += P * frag3_entries(c.moe_inter) * 8 + P * 128 * 4 + P * 4;
    n += B * frag4_entries(shi) * 8 + B * 128 * 4 + B * 4;
    return n + 16 * 256;
}

extern "C" int finch_encode_moe_decode(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, const void *h_post,
                                       const int32_t *expert_ids, const float *weights, const uint8_t *valid,
                                       const finch_shared *shared, const float *h_mid, float *hidden_out, int B) {
    if (!ctx || !pool || !h_post || !expert_ids || !weights || !hidden_out) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    if (pool->ctx != ctx) return finch_fail(ctx, FINCH_E_ARG, "pool belongs to another context");
    if (layer < 0 || layer >= pool->n_layers) return finch_fail(ctx, FINCH_E_ARG, "layer %d out of range", layer);
    if (B < 1 || B > c.max_tokens) return finch_fail(ctx, FINCH_E_ARG, "B=%d outside 1..max_tokens=%d", B, c.max_tokens);
    if (B * c.top_k > FINCH_MAX_PAIRS)
        return finch_fail(ctx, FINCH_E_UNSUPPORTED, "decode path takes at most %d (token, expert) pairs; use finch_encode_moe_prefill",
                          FINCH_MAX_PAIRS);
    if (pool->n_experts != c.n_experts) return finch_fail(ctx, FINCH_E_ARG, "pool / context expert count mismatch");
    if (shared) {
        int rc = check_shared(ctx, shared);
        if (rc) return rc;
    }
    cudaSetDevice(c.device);
    MoeArgs a{};
    a.pool_base = pool->base;
    a.slot_bytes = pool->slot_bytes;
    a.slot_row = pool->slot_table_dev + (size_t)layer * pool->n_experts;
    a.n_experts = c.n_experts;
    a.h_post = h_post;
    a.act_dtype = c.act_dtype;
    a.ids = expert_ids;
    a.weights = weights;
    a.valid = valid;
    a.P = B * c.top_k;
    a.K = c.top_k;
    a.B = B;
    a.hidden = c.hidden;
    a.inter = c.moe_inter;
    a.gate_w = ctx->lay.gate_w; a.gate_s = ctx->lay.gate_s; a.gate_b = ctx->lay.gate_b;
    a.up_w = ctx->lay.up_w; a.up_s = ctx->lay.up_s; a.up_b = ctx->lay.up_b;
    a.down_w = ctx->lay.down_w; a.down_s = ctx->lay.down_s; a.down_b = ctx->lay.down_b;
    a.scale_dtype = c.scale_dtype;
    a.act = ctx->act;
    a.partial = ctx->partial;
    a.counters = ctx->counters;
    a.cnt_a = ctx->counters + c.hidden / 64;
    a.status = ctx->dev_status;
    a.h_mid = h_mid;
    a.hidden_out = hidden_out;
    a.sh_inter = 64;
    if (shared) {
        a.has_shared = 1;
        a.sh_gate = WRef{(const uint8_t *)shared->gate.W, (const uint16_t *)shared->gate.scales, (const uint16_t *)shared->gate.biases,
                         shared->gate.out_dim, shared->gate.in_dim};
        a.sh_up = WRef{(const uint8_t *)shared->up.W, (const uint16_t *)shared->up.scales, (const uint16_t *)shared->up.biases,
                       shared->up.out_dim, shared->up.in_dim};
        a.sh_down = WRef{(const uint8_t *)shared->down.W, (const uint16_t *)shared->down.scales, (const uint16_t *)shared->down.biases,
                         shared->down.out_dim, shared->down.in_dim};
        a.sh_scale_dtype = shared->gate.scale_dtype;
        a.shared_act = ctx->shared_act;
        a.gate_score = shared->gate_score;
        a.sh_inter = shared->gate.out_dim;
    }
    // carve the fragment scratch (same order as finch_decode_scratch_bytes)
    {
        const size_t Pm = (size_t)c.max_tokens * c.top_k, Bm = c.max_tokens;
        const int shi = c.shared_inter > 0 ? c.shared_inter : 64;
        char *p = (char *)ctx->frag_scratch;
        auto take = [&](size_t bytes) {
            char *r = p;
            p += (bytes + 255) & ~(size_t)255;
            return r;
        };
        a.xfrag3 = (uint2 *)take(Bm * frag3_entries(c.hidden) * 8);
        a.xfrag4 = (uint2 *)take(Bm * frag4_entries(c.hidden) * 8);
        a.xXg = (float *)take(Bm * 128 * 4);
        a.xE = (int *)take(Bm * 4);
        a.grp = (int2 *)take(Pm * 8);
        a.grp_pairs = (uint8_t *)take(Pm * 64);
        a.n_groups = (int *)take(256);
        a.afrag3 = (uint2 *)take(Pm * frag3_entries(c.moe_inter) * 8);
        a.aXg = (float *)take(Pm * 128 * 4);
        a.aE = (int *)take(Pm * 4);
        a.sfrag4 = (uint2 *)take(Bm * frag4_entries(shi) * 8);
        a.sXg = (float *)take(Bm * 128 * 4);
        a.sE = (int *)take(Bm * 4);
    }
    a.use_prep = ctx->force_prep >= 0 ? ctx->force_prep : (B >= PREP_MIN_TOKENS ? 1 : 0);
    const SmemA LA = smem_a_layout(c.hidden);
    const SmemB LB = smem_b_layout(c.moe_inter, a.sh_inter);
    const int prep_smem = c.hidden * 4 + 128 * 4 + 64 + 64 * 4 + 64;
    if (LA.total > 227 * 1024 || LB.total > 227 * 1024) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "dims need too much shared memory");
    if (!g_attr_set) {
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_down_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
        g_attr_set = true;
    }
    cudaStream_t st = finch_pick_stream(ctx, stream);
    cudaEvent_t *pe = nullptr;
    if (ctx->profile) {
        while (ctx->prof_events.size() < ctx->prof_used + 3) {
            cudaEvent_t e;
            FINCH_CUDA_OK(ctx, cudaEventCreate(&e));
            ctx->prof_events.push_back(e);
        }
        pe = &ctx->prof_events[ctx->prof_used];
        ctx->prof_used += 3;
    }
    if (a.use_prep) {
        moe_prep_kernel<<<B + 1, A_THREADS, prep_smem, st>>>(a);
        FINCH_CUDA_OK(ctx, cudaGetLastError());
        ctx->launches++;
    }
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[0], st));
    const int chunks_r = c.moe_inter / A_ROWS;
    const int sh_rows_of_ctas = shared ? (a.sh_inter / S_ROWS + chunks_r - 1) / chunks_r : 0;
    dim3 ga(chunks_r, a.P + sh_rows_of_ctas);
    moe_gateup_kernel<<<ga, A_THREADS, LA.total, st>>>(a);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[1], st));
    dim3 gb(c.hidden / B_ROWS, a.P + 1);
    moe_down_combine_kernel<<<gb, B_THREADS, LB.total, st>>>(a);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[2], st));
    ctx->launches += 2;
    return FINCH_OK;
}

extern "C" int finch_profile_enable(finch_ctx *ctx, int on) {
    if (!ctx) return FINCH_E_ARG;
    ctx->profile = on != 0;
    ctx->prof_used = 0;
    return FINCH_OK;
}

extern "C" int finch_profile_read(finch_ctx *ctx, float *ms_gateup, float *ms_down_combine, int *n_calls) {
    if (!ctx || !ms_gateup || !ms_down_combine || !n_calls) return FINCH_E_ARG;
    cudaSetDevice(ctx->cfg.device);
    FINCH_CUDA_OK(ctx, cudaDeviceSynchronize());
    float a = 0.f, b = 0.f;
    for (size_t i = 0; i + 2 < ctx->prof_used; i += 3) {
        float t0 = 0.f, t1 = 0.f;
        FINCH_CUDA_OK(ctx, cudaEventElapsedTime(&t0, ctx->prof_events[i], ctx->prof_events[i + 1]));
        FINCH_CUDA_OK(ctx, cudaEventElapsedTime(&t1, ctx->prof_events[i + 1], ctx->prof_events[i + 2]));
        a += t0;
        b += t1;
    }
    *ms_gateup = a;
    *ms_down_combine = b;
    *n_calls = (int)(ctx->prof_used / 3);
    ctx->prof_used = 0;
    return FINCH_OK;
}

// Test hook: -1 = choose by batch size, 0 = never run the prep kernel, 1 = always.
extern "C" int finch_debug_force_prep(finch_ctx *ctx, int mode) {
    if (!ctx || mode < -1 || mode > 1) return FINCH_E_ARG;
    ctx->force_prep = mode;
    return FINCH_OK;
}
