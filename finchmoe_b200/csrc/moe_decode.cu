// MoE decode path: routed 3-bit experts (gate, up, SiLU, down), the 4-bit
// shared expert and the router-weighted combine, in four launches per layer chained
// with programmatic dependent launch.
//
//   prep      groups the (token, k) pairs by expert, turns every token's
//             activations into tensor-core operand records, and cuts the job
//             lists of the two streaming kernels into one contiguous,
//             cost-balanced range per CTA (the shared expert's jobs get CTAs
//             of their own when they take several passes)
//   gate/up   (moe_gateup_kernel) gate, up and SiLU.  One persistent CTA per SM: a
//             producer warp streams tiles (8 gate rows + the 8 matching up rows of
//             one expert = one contiguous 14 KB piece of the tiled pool) through a
//             ring of shared-memory stages with bulk async copies; six teams of
//             four consumer warps take whole tiles, the warps of a team split K and
//             whichever finishes last adds the partial sums.  Writes act[pair][inter].
//   down      (moe_down_combine_kernel) same structure with tiles of 16 down rows
//             and sixteen independent consumer warps; the tiles are small, so one
//             producer lane per stage issues the copies.  Every CTA first turns the
//             activations of the (few) expert groups in its range into operand
//             records in its own shared memory.  Writes one fp32 row per pair.
//   combine   (moe_combine_kernel) sums the rows of a token in k order with the
//             residual and the gated shared expert (the arithmetic of
//             moe_combine_residual, finchmoe/shaders.metal:2196-2231).
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
#include "tile_layout.h"

namespace {

constexpr int TEAM_A = 4;                   // warps that split the K dimension of one gate/up tile
constexpr int NTEAM_A = 6;
constexpr int CW_A = TEAM_A * NTEAM_A;      // consumer warps of kernel A
constexpr int NT_A = (CW_A + 1) * 32;       // + one producer warp
constexpr int CW_B = 16;
constexpr int NT_B = (CW_B + 1) * 32;
constexpr int MAXP = FINCH_MAX_PAIRS;
constexpr int MAXM = 8;                     // pairs per expert group (<= tokens per call)
constexpr int MAXG = 160;                   // CTAs per streaming kernel (range table size)
constexpr int REC_CAP = 24;                 // act records a CTA of kernel B can hold

struct GroupTab {  // expert groups of one call + the job ranges of the CTAs
    int ng;
    int slot[MAXP];             // pool slot of the group's expert
    unsigned char m[MAXP];      // pairs in the group
    unsigned char pairs[MAXP][MAXM];
    int range_a[MAXG + 1];      // CTA b of kernel A runs jobs [range_a[b], range_a[b+1])
    int range_b[MAXG + 1];
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
    int scale_dtype;
    float *act;          // [P][inter]
    float *partial;      // [P + B][hidden]
    int *status;
    int has_shared;
    const uint8_t *sh_tiles;  // prepared (tiled) copy of the shared expert
    int sh_scale_dtype, sh_inter;
    float *shared_act;   // [B][sh_inter]
    const float *gate_score;
    const float *h_mid;
    float *hidden_out;
    GroupTab *gtab;      // written by prep
    uint8_t *xrec3;      // [B] records: 3-bit-layout operands of h_post + header
    uint8_t *xrec4;      // [B] 4-bit-layout operand fragments of h_post (shared expert)
    int grid_a, grid_b, stages_a, stages_b;
    long long *dbg;      // optional per-CTA cycle counters (finch_debug_timing), or NULL
};

// ---- operand records -------------------------------------------------------
// record = fragments (8-byte entries) followed by a header of floats:
// hdr[0..groups) = sum of x over each group of 64, hdr[groups] = E (int bits).
__host__ __device__ inline int frag3_bytes(int K) { return (K / 128) * 72 * 8; }
__host__ __device__ inline int frag4_bytes(int K) { return (K / 64) * 32 * 8; }
__host__ __device__ inline int hdr_bytes(int K) { return ((K / 64 + 1 + 15) / 16) * 64; }
__host__ __device__ inline int rec3_bytes(int K) { return frag3_bytes(K) + hdr_bytes(K); }
__host__ __device__ inline int rec4_bytes(int K) { return frag4_bytes(K) + hdr_bytes(K); }

// Slot tables of the 3-bit extraction.  Extraction e (0..17, see extract3) yields a register with one
// code in each 16-bit half; MMA j uses extractions 2j and 2j+1, i.e. four slots 4j..4j+3.  Slot s holds
// code number idx (0..31) of the 32-code period at bit position pos of its half, or is empty:
//   idx: 0 6 1 7 | 2 - 3 8 | 4 9 5 10 | 11 16 12 17 | 13 18 14 19 | 15 20 - 21 | 22 27 23 28 | - 29 24 30 | 25 31 26 -
//   pos: 0 2 3 5 | 6 0 1 0 | 4 3 7 6  | 1 0 4 3     | 7 6 2 1     | 5 4 0 7   | 2 1 5 4     | 0 7 0 2   | 3 5 6 0
// They are packed into immediates (one byte idx | pos << 5 per slot, empty slots flagged in a bit mask) so
// that a thread gets the four slots of its MMA without touching memory.
__device__ __forceinline__ uint32_t slots3_of(int j) {
    const unsigned long long w = j < 2 ? 0x082300c2a7614600ull : j < 4 ? 0x718c102bcae56984ull : j < 6 ? 0xf50094af334ed2edull
                               : j < 8 ? 0x5e18fd009cb73b56ull : 0x0000000000dabf79ull;
    return (uint32_t)(w >> (32 * (j & 1)));
}
__device__ __forceinline__ uint32_t empty3_of(int j) { return (uint32_t)(0x810400020ull >> (4 * j)) & 15u; }

__device__ __forceinline__ void extract3(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t (&e)[18]) {
    const uint32_t v1 = __funnelshift_r(w0, w1, 8), v3 = __funnelshift_r(w1, w2, 8), v5 = w2 >> 8;
    e[0] = w0 & 0x001C0007u;  e[1] = w0 & 0x00E00038u;  e[2] = w0 & 0x000001C0u;
    e[3] = v1 & 0x0007000Eu;  e[4] = v1 & 0x00380070u;  e[5] = v1 & 0x01C00380u;
    e[6] = w1 & 0x0007000Eu;  e[7] = w1 & 0x00380070u;  e[8] = w1 & 0x01C00380u;
    e[9] = v3 & 0x000E001Cu;  e[10] = v3 & 0x007000E0u; e[11] = v3 & 0x03800000u;
    e[12] = w2 & 0x000E001Cu; e[13] = w2 & 0x007000E0u; e[14] = w2 & 0x03800000u;
    e[15] = v5 & 0x001C0007u; e[16] = v5 & 0x00E00038u; e[17] = v5 & 0x000001C0u;
}

// The same extraction, one register at a time (k = 0..17, compile-time): lets the matvec loop form the four A
// registers of an MMA right before issuing it, which keeps few of them alive at once.
template <int k>
__device__ __forceinline__ uint32_t extract3_one(uint32_t w0, uint32_t v1, uint32_t w1, uint32_t v3, uint32_t w2, uint32_t v5) {
    constexpr uint32_t M0[3] = {0x001C0007u, 0x00E00038u, 0x000001C0u}, M1[3] = {0x0007000Eu, 0x00380070u, 0x01C00380u},
                       M2[3] = {0x000E001Cu, 0x007000E0u, 0x03800000u};
    constexpr int grp = k / 3, i = k % 3;
    return grp == 0 ? (w0 & M0[i]) : grp == 1 ? (v1 & M1[i]) : grp == 2 ? (w1 & M1[i]) : grp == 3 ? (v3 & M2[i]) : grp == 4 ? (w2 & M2[i]) : (v5 & M0[i]);
}

// One u32 of eight nibbles -> four registers: (0,4) (1,5) at p = 0 / 4 of the
// word itself, (2,6) (3,7) at p = 0 / 4 of the word shifted right by 8.
__device__ __forceinline__ void extract4(uint32_t w, uint32_t (&e)[4]) {
    const uint32_t v = w >> 8;
    e[0] = w & 0x000F000Fu; e[1] = w & 0x00F000F0u;
    e[2] = v & 0x000F000Fu; e[3] = v & 0x00F000F0u;
}

// Programmatic dependent launch: the kernels of a call are launched so that each may start while
// its predecessor drains; nothing written by the predecessor may be read before this returns.
__device__ __forceinline__ long long gtime() {
    long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the chain be scheduled as soon as SMs free up instead of when this grid has
// drained: its CTAs run their prologue (and whatever does not depend on this grid's output) and then
// block in griddepcontrol.wait until this grid has completed and its writes are visible.
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float pow2_biased(int e) { return __uint_as_float((uint32_t)e << 23); }
__device__ __forceinline__ void bar_sync(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(finch_smem_u32(bar)) : "memory");
}

// Loads one activation row into xs (fp32 shared memory) and writes the group
// sums hdr[0..K/64) and hdr[K/64] = E, the biased exponent of a power of two
// > max|x| (clamped so every derived scale factor is a normal float).  Run by
// the NT threads tid = 0..NT-1 that share named barrier `bar`; ends with it.
template <int NT>
__device__ void load_x(const void *src, int dtype, int K, float *xs, float *hdr, float *warp_max, int bar) {
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
            if ((lane & 7) == 0) hdr[base >> 6] = s;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) warp_max[warp] = amax;
    bar_sync(bar, NT);
    if (tid == 0) {
        float m = 0.f;
        for (int w = 0; w < NT / 32; w++) m = fmaxf(m, warp_max[w]);
        int E = (int)(__float_as_uint(m) >> 23) + 1;
        E = E < 30 ? 30 : (E > 230 ? 230 : E);
        hdr[K / 64] = __int_as_float(E);
    }
    bar_sync(bar, NT);
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

// B fragments of one token, 3-bit layout: frag[((u * 9 + j) * 2 + term) * 4 + t].
// frag may be shared or global memory.  Thread `first` of `stride` (stride >= 32) cooperating threads.
// A thread keeps one (j, t) position of the 9 x 4 entries of a unit and walks the units, so the slots
// are decoded once per thread, not once per entry.
__device__ __forceinline__ void build_frag3_range(const float *xs, int K, int E, uint2 *frag, int first, int stride) {
    const int units = K / 128;
    const int ulanes = stride >= 36 ? stride / 36 : 1;       // threads side by side along the units
    const int rounds = stride >= 36 ? 1 : 2;                 // a single warp covers the 36 positions in two rounds
    for (int rd = 0; rd < rounds; rd++) {
        const int jt = stride >= 36 ? first % 36 : first + 32 * rd;
        const int u0 = stride >= 36 ? first / 36 : 0;
        if (jt >= 36 || u0 >= ulanes) continue;
        const int j = jt >> 2, t = jt & 3;
        int idx[4];
        float mul[4];
        const uint32_t slots = slots3_of(j), hole = empty3_of(j);
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const uint32_t b = (slots >> (8 * s)) & 255u;
            idx[s] = (int)(b & 31u);
            mul[s] = ((hole >> s) & 1u) ? 0.f : pow2_biased(261 - E - (int)(b >> 5));
        }
#pragma unroll 4
        for (int u = u0; u < units; u += ulanes) {
            float xv[4];
#pragma unroll
            for (int s = 0; s < 4; s++) xv[s] = mul[s] == 0.f ? 0.f : xs[u * 128 + t * 32 + idx[s]] * mul[s];
            uint2 hi, lo;
            split4(xv, hi, lo);
            const int o = (u * 9 + j) * 8 + t;
            frag[o] = hi;
            frag[o + 4] = lo;
        }
    }
}

template <int NT>
__device__ __forceinline__ void build_frag3(const float *xs, int K, int E, uint2 *frag) {
    build_frag3_range(xs, K, E, frag, threadIdx.x, NT);
}

// B fragments of one token, 4-bit layout: frag[((gamma * 4 + j) * 2 + term) * 4 + t].
__device__ __forceinline__ void build_frag4_range(const float *xs, int K, int E, uint2 *frag, int first, int stride) {
    const int entries = (K / 64) * 16;
    for (int e = first; e < entries; e += stride) {
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
template <int NT>
__device__ __forceinline__ void build_frag4(const float *xs, int K, int E, uint2 *frag) {
    build_frag4_range(xs, K, E, frag, threadIdx.x, NT);
}

// One warp turns K fp32 values at src (global memory written by an earlier
// launch) into an operand record (shared or global memory).  BITS selects the layout.
// stage: K floats of shared memory private to the warp, or NULL; with it the scattered reads of the
// second pass come from shared memory instead of paying an L2 round trip each.
template <int BITS>
__device__ void warp_make_record(const float *src, int K, uint8_t *rec, float *stage = nullptr) {
    const int lane = threadIdx.x & 31;
    float *hdr = reinterpret_cast<float *>(rec + (BITS == 3 ? frag3_bytes(K) : frag4_bytes(K)));
    float amax = 0.f;
#pragma unroll 4
    for (int base = lane * 8; base < K; base += 256) {  // K is a multiple of 64, so a warp never splits a group
        const float4 a = __ldcg(reinterpret_cast<const float4 *>(src + base));
        const float4 b = __ldcg(reinterpret_cast<const float4 *>(src + base + 4));
        float s = ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
        amax = fmaxf(amax, fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))),
                                 fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w)))));
        // the eight lanes of a group are active together (K % 64 == 0)
        const unsigned mask = __activemask();
        s += __shfl_xor_sync(mask, s, 1);
        s += __shfl_xor_sync(mask, s, 2);
        s += __shfl_xor_sync(mask, s, 4);
        if ((lane & 7) == 0) hdr[base >> 6] = s;
        if (stage) {
            *reinterpret_cast<float4 *>(stage + base) = a;
            *reinterpret_cast<float4 *>(stage + base + 4) = b;
        }
    }
    __syncwarp();
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    int E = (int)(__float_as_uint(amax) >> 23) + 1;
    E = E < 30 ? 30 : (E > 230 ? 230 : E);
    if (lane == 0) hdr[K / 64] = __int_as_float(E);
    __syncwarp();
    const float *xs = stage ? stage : src;
    if (BITS == 3) build_frag3_range(xs, K, E, reinterpret_cast<uint2 *>(rec), lane, 32);
    else build_frag4_range(xs, K, E, reinterpret_cast<uint2 *>(rec), lane, 32);
    __syncwarp();
}

// ---- inner loops ---------------------------------------------------------
// First MMA of a chain: C = 0 comes from the zero register, no accumulator initialisation needed.
__device__ __forceinline__ void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Shared-memory loads with a 32-bit address and an immediate offset: the inner loops keep a few running
// addresses and spend no instructions on address arithmetic per load.
template <int OFF>
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(addr), "n"(OFF));
    return v;
}
template <int OFF>
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4+%5];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr), "n"(OFF));
    return v;
}
__device__ __forceinline__ float lds32f(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}
constexpr int ZERO3_BYTES = 640;   // zeroed shared memory a lane with a structurally zero B column reads instead of a record

// 3-bit tile (tile_layout.h) against up to two tokens.  Everything is in shared memory: the tile, the
// operand records of the two tokens (frag0 / frag1 with their headers h0 / h1 = group sums, E) and
// `zero`, ZERO3_BYTES of zeros.  On return lane (g, t), t even, holds for token slot t>>1 the dot
// products resA (fragment row g) and resB (row g + 8), bias included, over units u0, u0 + ustep, ...
__device__ __forceinline__ void gemv3_tile(const uint8_t *tile, int units, int u0, int ustep, int scale_dtype, const uint2 *frag0,
                                           const uint2 *frag1, const float *h0, const float *h1, const void *zero, int ntok,
                                           float &resA, float &resB) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tokslot = g >> 2, term = (g >> 1) & 1;
    const bool bact = ((g & 1) == (t >> 1)) && tokslot < ntok;
    // lanes whose B column is structurally zero walk a block of zeros with unit stride 0: no select, no moves
    uint32_t pb = (bact ? finch_smem_u32(tokslot ? frag1 : frag0) + (uint32_t)u0 * 576u : finch_smem_u32(zero)) + (uint32_t)(term * 4 + t) * 8u;
    const uint32_t sb_step = bact ? (uint32_t)ustep * 576u : 0u;
    const uint32_t h32 = finch_smem_u32((t >> 1) ? h1 : h0);  // token whose result this lane's accumulator columns hold
    const uint32_t tile32 = finch_smem_u32(tile);
    uint32_t pw = tile32 + (uint32_t)(u0 * 32 + lane) * 24u, ps = tile32 + (uint32_t)units * 768u + (uint32_t)(u0 * 8 + g) * 16u;
    uint32_t ph = h32 + (uint32_t)u0 * 8u;
    float runA = 0.f, runB = 0.f, biasA = 0.f, biasB = 0.f;
    for (int u = u0; u < units; u += ustep) {
        uint2 b[9];
        b[0] = lds64<0>(pb);   b[1] = lds64<64>(pb);  b[2] = lds64<128>(pb);
        b[3] = lds64<192>(pb); b[4] = lds64<256>(pb); b[5] = lds64<320>(pb);
        b[6] = lds64<384>(pb); b[7] = lds64<448>(pb); b[8] = lds64<512>(pb);
        const uint2 q0 = lds64<0>(pw), q1 = lds64<8>(pw), q2 = lds64<16>(pw);
        const uint4 s = lds128<0>(ps);
        const uint2 xgb = lds64<0>(ph);
        const float2 xg = make_float2(__uint_as_float(xgb.x), __uint_as_float(xgb.y));
        pb += sb_step;
        pw += (uint32_t)ustep * 768u;
        ps += (uint32_t)ustep * 128u;
        ph += (uint32_t)ustep * 8u;
        // row A words q0.x q0.y q1.x, row B words q1.y q2.x q2.y; the shifted views of extract3
        const uint32_t av1 = __funnelshift_r(q0.x, q0.y, 8), av3 = __funnelshift_r(q0.y, q1.x, 8), av5 = q1.x >> 8;
        const uint32_t bv1 = __funnelshift_r(q1.y, q2.x, 8), bv3 = __funnelshift_r(q2.x, q2.y, 8), bv5 = q2.y >> 8;
        float acc[2][4];  // two independent accumulator chains
#define FINCH_MMA3(j)                                                                                                     \
    {                                                                                                                     \
        const uint32_t a0 = extract3_one<2 * (j)>(q0.x, av1, q0.y, av3, q1.x, av5);                                       \
        const uint32_t a1 = extract3_one<2 * (j)>(q1.y, bv1, q2.x, bv3, q2.y, bv5);                                       \
        const uint32_t a2 = extract3_one<2 * (j) + 1>(q0.x, av1, q0.y, av3, q1.x, av5);                                   \
        const uint32_t a3 = extract3_one<2 * (j) + 1>(q1.y, bv1, q2.x, bv3, q2.y, bv5);                                   \
        if ((j) < 2) mma16816_z(acc[(j) & 1], a0, a1, a2, a3, b[j].x, b[j].y);                                            \
        else finch_mma16816(acc[(j) & 1], a0, a1, a2, a3, b[j].x, b[j].y);                                                \
    }
        FINCH_MMA3(0) FINCH_MMA3(1) FINCH_MMA3(2) FINCH_MMA3(3) FINCH_MMA3(4) FINCH_MMA3(5) FINCH_MMA3(6) FINCH_MMA3(7) FINCH_MMA3(8)
#undef FINCH_MMA3
        float s0, s1;
        finch_widen16x2(s.x, scale_dtype, s0, s1);
        runA = fmaf(s0, acc[0][0] + acc[1][0], runA);
        runA = fmaf(s1, acc[0][1] + acc[1][1], runA);
        finch_widen16x2(s.y, scale_dtype, s0, s1);
        runB = fmaf(s0, acc[0][2] + acc[1][2], runB);
        runB = fmaf(s1, acc[0][3] + acc[1][3], runB);
        finch_widen16x2(s.z, scale_dtype, s0, s1);
        biasA = fmaf(s0, xg.x, biasA);
        biasA = fmaf(s1, xg.y, biasA);
        finch_widen16x2(s.w, scale_dtype, s0, s1);
        biasB = fmaf(s0, xg.x, biasB);
        biasB = fmaf(s1, xg.y, biasB);
    }
    // accumulator columns of lane t: token slot t>>1, term t&1 -> hi in even t, lo in odd t
    const float fac = pow2_biased(__float_as_int(lds32f(h32 + (uint32_t)units * 8u)) + 17);
    const float oA = __shfl_xor_sync(0xffffffffu, runA, 1), oB = __shfl_xor_sync(0xffffffffu, runB, 1);
    resA = fmaf(runA + oA * (1.0f / 2048.0f), fac, biasA);
    resB = fmaf(runB + oB * (1.0f / 2048.0f), fac, biasB);
}

// 4-bit tile of the prepared shared expert (tile_layout.h) against up to two tokens (columns 0..3 =
// token 0 hi/lo, token 1 hi/lo).  chunk: index of this lane's 16-byte operand chunk inside a group
// (lane for a 16-row tile, (g&3)*4+t for a 4+4-row tile), per_group: chunks per group (32 / 16),
// sidx / s_per_group: the same for the 8-byte scale/bias entries.  Lane (g, t) with t < 2 returns
// the finished dot products of its two fragment rows for token t.
__device__ __forceinline__ void gemv4_tile(const uint8_t *tile, int groups, int g0, int gstep, int chunk, int per_group, int sidx, int s_per_group,
                                           int scale_dtype, const uint2 *frag0, const uint2 *frag1, const float *h0, const float *h1,
                                           const uint2 *zero, int ntok, float &resA, float &resB) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int tok = g >> 1, term = g & 1;
    const bool bact = tok < ntok;  // ntok <= 2
    const uint2 *fb = bact ? (tok ? frag1 : frag0) + term * 4 + t : zero;
    const int fstride = bact ? 8 : 0;
    const float *h = (t & 1) ? h1 : h0;
    const uint8_t *sb = tile + (size_t)groups * per_group * 16;
    float runA = 0.f, runB = 0.f, biasA = 0.f, biasB = 0.f;
    for (int gm = g0; gm < groups; gm += gstep) {
        uint2 b[4];
#pragma unroll
        for (int j = 0; j < 4; j++) b[j] = fb[(gm * 4 + j) * fstride];
        const uint4 w = *reinterpret_cast<const uint4 *>(tile + (size_t)(gm * per_group + chunk) * 16);
        const uint2 s = *reinterpret_cast<const uint2 *>(sb + (size_t)(gm * s_per_group + sidx) * 8);
        const float xg = h[gm];
        uint32_t ea[8], eb[8];
        {
            uint32_t x[4];
            extract4(w.x, x); ea[0] = x[0]; ea[1] = x[1]; ea[2] = x[2]; ea[3] = x[3];
            extract4(w.y, x); ea[4] = x[0]; ea[5] = x[1]; ea[6] = x[2]; ea[7] = x[3];
            extract4(w.z, x); eb[0] = x[0]; eb[1] = x[1]; eb[2] = x[2]; eb[3] = x[3];
            extract4(w.w, x); eb[4] = x[0]; eb[5] = x[1]; eb[6] = x[2]; eb[7] = x[3];
        }
        float acc[2][4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (j < 2) mma16816_z(acc[j], ea[2 * j], eb[2 * j], ea[2 * j + 1], eb[2 * j + 1], b[j].x, b[j].y);
            else finch_mma16816(acc[j & 1], ea[2 * j], eb[2 * j], ea[2 * j + 1], eb[2 * j + 1], b[j].x, b[j].y);
        }
        // accumulator columns 2t, 2t+1 = (token t, hi), (token t, lo)
        float s0, s1, b0, b1;
        finch_widen16x2(s.x, scale_dtype, s0, s1);  // scale of row A, of row B
        finch_widen16x2(s.y, scale_dtype, b0, b1);  // bias of row A, of row B
        runA = fmaf(s0, (acc[0][0] + acc[1][0]) + (acc[0][1] + acc[1][1]) * (1.0f / 2048.0f), runA);
        runB = fmaf(s1, (acc[0][2] + acc[1][2]) + (acc[0][3] + acc[1][3]) * (1.0f / 2048.0f), runB);
        biasA = fmaf(b0, xg, biasA);
        biasB = fmaf(b1, xg, biasB);
    }
    const float fac = pow2_biased(__float_as_int(h[groups]) + 17);
    resA = fmaf(runA, fac, biasA);
    resB = fmaf(runB, fac, biasB);
}

// ---- expert groups -------------------------------------------------------
__device__ __forceinline__ bool pair_ok(const MoeArgs &a, int p) {
    if (a.valid && !a.valid[p]) return false;
    const int e = a.ids[p];
    if (e < 0 || e >= a.n_experts) return false;
    return a.slot_row[e] >= 0;
}

// Builds the group table in shared memory.  Run by threads 0..nthreads-1 (nthreads >= 64, whole
// warps) sharing named barrier `bar`; the first two warps hold one pair per lane.  Groups are
// numbered by their first pair; pairs inside a group ascend.  sm_ids: MAXP + 2 ints.
__device__ void build_groups(const MoeArgs &a, GroupTab *T, int *sm_ids, unsigned char *sm_rank, int bar, int nthreads) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int id = -1, slot = -1;
    if (tid < a.P) {
        // mask and id are loaded side by side (one memory round trip instead of two on the layer's critical path)
        const int e = a.ids[tid];
        const bool on = !a.valid || a.valid[tid];
        if (on && e >= 0 && e < a.n_experts) {
            slot = a.slot_row[e];
            if (slot >= 0) id = e;
        }
    }
    if (tid < MAXP) sm_ids[tid] = id;
    bar_sync(bar, nthreads);
    unsigned same = 0, other = 0, fb = 0;
    bool first = false;
    if (tid < MAXP) {
        same = __match_any_sync(0xffffffffu, id);                 // lanes of my warp with my expert
        const int *o = sm_ids + 32 * (warp ^ 1);
        for (int j = 0; j < 32; j++) other |= (unsigned)(o[j] == id) << j;   // lanes of the other warp
        const unsigned lt = (1u << lane) - 1u;
        first = id >= 0 && !(same & lt) && (warp == 0 || other == 0);
        fb = __ballot_sync(0xffffffffu, first);
        if (lane == 0) sm_ids[MAXP + warp] = (int)fb;
    }
    bar_sync(bar, nthreads);
    if (tid < MAXP) {
        const unsigned lt = (1u << lane) - 1u;
        const int before = warp == 1 ? __popc((unsigned)sm_ids[MAXP]) : 0;
        if (first) sm_rank[tid] = (unsigned char)(before + __popc(fb & lt));
        if (tid == 0) T->ng = __popc((unsigned)sm_ids[MAXP]) + __popc((unsigned)sm_ids[MAXP + 1]);
    }
    bar_sync(bar, nthreads);
    if (tid < MAXP && id >= 0) {
        const unsigned lt = (1u << lane) - 1u;
        const int fp = (warp == 1 && other) ? __ffs(other) - 1 : 32 * warp + __ffs(same) - 1;   // first pair of my group
        const int gi = sm_rank[fp];
        const int pos = (warp == 1 ? __popc(other) : 0) + __popc(same & lt);
        if (pos < MAXM) T->pairs[gi][pos] = (unsigned char)tid;
        if (first) {
            const int m = __popc(same) + __popc(other);
            T->m[gi] = (unsigned char)(m < MAXM ? m : MAXM);
            T->slot[gi] = slot;
        }
    }
    bar_sync(bar, nthreads);
}

// ---- work distribution ---------------------------------------------------
// Jobs (one tile against the tokens of its group) are laid out group-major:
// job = gi * per_group + tile for the routed experts, then the shared-expert
// tiles.  Every CTA takes one contiguous range, balanced by cost (a job of a
// group with m pairs costs ceil(m/2) passes).  Contiguous ranges keep the
// groups a CTA touches few: few act records to prepare.
__device__ __forceinline__ int npass_of(const GroupTab *tab, int gi) { return (tab->m[gi] + 1) >> 1; }

// pre[gi] = passes of the groups before gi (32-bit: at most 64 groups x 4 passes).  The job whose
// cost interval starts at or after `target` (cost units: tile-passes).
__device__ int job_at(const int *pre, int ng, int per_group, int n_sh, int nps, int target) {
    const int routed_cost = pre[ng] * per_group;
    if (target >= routed_cost) {
        if (n_sh > 0 && target < routed_cost + n_sh * nps) return ng * per_group + (target - routed_cost + nps - 1) / nps;
        return ng * per_group + n_sh;
    }
    int lo = 0, hi = ng - 1;   // last group whose first job starts at or before target
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] * per_group <= target) lo = mid;
        else hi = mid - 1;
    }
    const int gi = lo, np = pre[gi + 1] - pre[gi];
    return gi * per_group + (target - pre[gi] * per_group + np - 1) / np;
}

// How many CTAs at the end of the grid take the shared expert's jobs (`units` jobs each).  A CTA whose range
// crosses from routed to shared-expert jobs would finish last: its consumer units (teams or warps, `units` of
// them, one job at a time each) are dealt its jobs round robin, and a shared-expert job - every token, so
// several passes - lands on a unit that already has its share of routed ones.  So with three tokens or more
// (two passes per shared job) the boundary is put on a CTA boundary and every shared CTA gets one job per
// unit.  Returns -1 where that does not apply (no shared expert, one pass per job, a grid too small to split):
// ranges are proportional to cost then.
__device__ __forceinline__ int shared_ctas(int grid, int units, int n_sh, int nps) {
    if (n_sh == 0 || nps < 2) return -1;
    const int gs = (n_sh + units - 1) / units;
    return gs < grid ? gs : -1;
}

// start of CTA i's range under that split
__device__ int range_start(const int *pre, int ng, int per_group, int n_sh, int nps, int grid, int gs, int per, int i) {
    const int routed_cost = pre[ng] * per_group, n_routed = ng * per_group;
    if (gs < 0) return job_at(pre, ng, per_group, n_sh, nps, (int)((long long)(routed_cost + n_sh * nps) * i / grid));
    const int gr = grid - gs;
    if (i <= gr) return job_at(pre, ng, per_group, 0, 1, (int)((long long)routed_cost * i / gr));
    const int j = (i - gr) * per;
    return n_routed + (j < n_sh ? j : n_sh);
}

// ============================ prep ========================================
// grid: B + 1 CTAs of 256 threads.  CTA b < B: operand records of token b.  CTA B: groups and ranges.
__global__ void __launch_bounds__(256) moe_prep_kernel(const MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    float *xs = reinterpret_cast<float *>(smem);
    float *hdr = xs + a.hidden;              // [hidden/64 + 1]
    float *warp_max = hdr + 144;
    int *sm_ids = reinterpret_cast<int *>(warp_max + 8);
    unsigned char *sm_first = reinterpret_cast<unsigned char *>(sm_ids + MAXP + 2);
    GroupTab *T = reinterpret_cast<GroupTab *>(sm_first + MAXP + 8);
    const int b = blockIdx.x, tid = threadIdx.x, K = a.hidden;
    const long long gt0 = gtime();
    grid_dep_launch();
    grid_dep_wait();
    if (a.dbg && tid == 0) a.dbg[(size_t)(1300 + b) * 8] = gt0, a.dbg[(size_t)(1300 + b) * 8 + 1] = gtime();
    if (b < a.B) {
        const void *src = a.act_dtype == FINCH_BF16 ? (const void *)((const uint16_t *)a.h_post + (size_t)b * K)
                                                     : (const void *)((const float *)a.h_post + (size_t)b * K);
        load_x<256>(src, a.act_dtype, K, xs, hdr, warp_max, 0);
        const int E = __float_as_int(hdr[K / 64]);
        uint8_t *rec = a.xrec3 + (size_t)b * rec3_bytes(K);
        build_frag3<256>(xs, K, E, reinterpret_cast<uint2 *>(rec));
        if (a.has_shared) build_frag4<256>(xs, K, E, reinterpret_cast<uint2 *>(a.xrec4 + (size_t)b * frag4_bytes(K)));
        float *gh = reinterpret_cast<float *>(rec + frag3_bytes(K));
        for (int i = tid; i <= K / 64; i += 256) gh[i] = hdr[i];
        if (a.dbg && tid == 0) a.dbg[(size_t)(1300 + b) * 8 + 2] = gtime();
        return;
    }
    build_groups(a, T, sm_ids, sm_first, 0, 256);
    // job ranges of the two streaming kernels (thread i computes the start of CTA i)
    const FinchTile L3 = finch_tile(a.hidden, a.inter);
    const int nps = (a.B + 1) / 2;
    const int n_sh_a = a.has_shared ? a.sh_inter / 4 : 0, n_sh_b = a.has_shared ? L3.nTB : 0;
    int *pre = sm_ids;  // the pair ids are no longer needed: reuse as prefix sums of the groups' passes
    const int ng = T->ng;
    if (tid < 64) {   // exclusive scan of the per-group pass counts over two warps
        const int lane = tid & 31, np = tid < ng ? npass_of(T, tid) : 0;
        int inc = np;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += v;
        }
        if (tid == 31) pre[MAXP + 1] = inc;   // total of the first warp
        __syncwarp();
        pre[tid] = inc - np;
        if (tid == 63) pre[MAXP] = inc;
    }
    __syncthreads();
    if (tid >= 32 && tid < 65) pre[tid] += pre[MAXP + 1];   // tid 64 fixes up the grand total in pre[MAXP]
    __syncthreads();
    const int gs_a = shared_ctas(a.grid_a, NTEAM_A, n_sh_a, nps), gs_b = shared_ctas(a.grid_b, CW_B, n_sh_b, nps);
    for (int i = tid; i <= a.grid_a; i += 256) T->range_a[i] = range_start(pre, ng, L3.nTA, n_sh_a, nps, a.grid_a, gs_a, NTEAM_A, i);
    for (int i = tid; i <= a.grid_b; i += 256) T->range_b[i] = range_start(pre, ng, L3.nTB, n_sh_b, nps, a.grid_b, gs_b, CW_B, i);
    __syncthreads();
    const int *s = reinterpret_cast<const int *>(T);
    int *d = reinterpret_cast<int *>(a.gtab);
    for (int i = tid; i < (int)(sizeof(GroupTab) / 4); i += 256) d[i] = s[i];
    if (a.dbg && tid == 0) a.dbg[(size_t)(1300 + b) * 8 + 2] = gtime();
}

// Re-tiles a shared expert from the reference tensor layout into FinchTile4 tiles (run once per
// expert).  One thread per 16-byte operand chunk or 8-byte scale/bias entry.
struct SharedSrc {
    const uint32_t *gw, *uw, *dw;   // packed rows: in_dim / 8 words each
    const uint16_t *gs, *gb, *us, *ub, *ds, *db;
};
__global__ void shared_retile_kernel(SharedSrc S, int hidden, int inter, uint8_t *out) {
    const FinchTile4 T = finch_tile4(hidden, inter);
    const size_t nA = (size_t)T.nTA * T.groupsA * 20, nB = (size_t)T.nTB * T.groupsD * 40;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < nA + nB; i += (size_t)gridDim.x * blockDim.x) {
        if (i < nA) {
            const int ta = (int)(i / (T.groupsA * 20)), r = (int)(i % (T.groupsA * 20)), gm = r / 20, e = r % 20;
            uint8_t *tile = out + (size_t)ta * T.tileA;
            if (e < 16) {  // operand chunk of lane (g4, t)
                const int g4 = e >> 2, t = e & 3;
                const size_t row = (size_t)4 * ta + g4, wpr = hidden / 8;
                const uint32_t *ga = S.gw + row * wpr + gm * 8 + 2 * t, *ua = S.uw + row * wpr + gm * 8 + 2 * t;
                *reinterpret_cast<uint4 *>(tile + (size_t)(gm * 16 + e) * 16) = make_uint4(ga[0], ga[1], ua[0], ua[1]);
            } else {
                const int g4 = e - 16;
                const size_t o = ((size_t)4 * ta + g4) * T.groupsA + gm;
                *reinterpret_cast<uint2 *>(tile + T.sbA + (size_t)(gm * 4 + g4) * 8) =
                    make_uint2((uint32_t)S.gs[o] | ((uint32_t)S.us[o] << 16), (uint32_t)S.gb[o] | ((uint32_t)S.ub[o] << 16));
            }
        } else {
            const size_t k = i - nA;
            const int tb = (int)(k / (T.groupsD * 40)), r = (int)(k % (T.groupsD * 40)), gm = r / 40, e = r % 40;
            uint8_t *tile = out + T.b_base + (size_t)tb * T.tileB;
            if (e < 32) {
                const int g = e >> 2, t = e & 3;
                const size_t r0 = (size_t)16 * tb + g, r1 = r0 + 8, wpr = inter / 8;
                const uint32_t *pa = S.dw + r0 * wpr + gm * 8 + 2 * t, *pb = S.dw + r1 * wpr + gm * 8 + 2 * t;
                *reinterpret_cast<uint4 *>(tile + (size_t)(gm * 32 + e) * 16) = make_uint4(pa[0], pa[1], pb[0], pb[1]);
            } else {
                const int g = e - 32;
                const size_t o0 = ((size_t)16 * tb + g) * T.groupsD + gm, o1 = o0 + (size_t)8 * T.groupsD;
                *reinterpret_cast<uint2 *>(tile + T.sbB + (size_t)(gm * 8 + g) * 8) =
                    make_uint2((uint32_t)S.ds[o0] | ((uint32_t)S.ds[o1] << 16), (uint32_t)S.db[o0] | ((uint32_t)S.db[o1] << 16));
            }
        }
    }
}

// ============================ kernel A ====================================
__host__ __device__ inline int up128(int x) { return (x + 127) & ~127; }
// Stage s of a ring is used by whichever consumer the job order assigns, and the producer lanes of different
// stages run independently, so a consumer can be ready for the n-th fill of a stage while the job of its
// (n-1)-th fill is still in progress (or that fill has not even been issued).  An mbarrier cannot tell these
// apart: a barrier one phase behind reports the awaited phase's parity as complete.  So every stage carries a
// count of the jobs consumed from it, and a consumer waits for the barrier only once that count says the
// previous fill has been used up.  Bounded like every other wait here.
__device__ __forceinline__ bool wait_consumed(const int *cnt, int want) {
    const volatile int *c = cnt;
    for (unsigned i = 0; i < (1u << 22); ++i) {
        if (*c >= want) return true;
        __nanosleep(40);
    }
    return false;
}

struct SmemA {
    int stage, stg, rec, rx3, rec4, f4s, n4, red, qcnt, tab, zero, bar, total;
};
__host__ __device__ inline SmemA smem_a_layout(int hidden, int inter, int sh_inter, int B, int has_shared, int stages) {
    const FinchTile T = finch_tile(hidden, inter);
    const FinchTile4 T4 = finch_tile4(hidden, sh_inter);
    SmemA L;
    L.stage = 0;
    L.stg = up128(has_shared && T4.tileA > T.tileA ? T4.tileA : T.tileA);
    L.rec = L.stage + stages * L.stg;         // operand records of all tokens (3-bit layout)
    L.rx3 = rec3_bytes(hidden);
    L.rec4 = up128(L.rec + B * L.rx3);        // 4-bit-layout fragments of the first n4 tokens (the rest stay in global memory)
    L.f4s = frag4_bytes(hidden) + 64;
    L.n4 = has_shared ? (B < 2 ? B : 2) : 0;
    L.red = up128(L.rec4 + L.n4 * L.f4s);
    L.qcnt = L.red + stages * (MAXM / 2) * TEAM_A * 32 * 4;   // per stage: [pass][warp][32] partial sums
    L.tab = L.qcnt + 64 * 4;                                  // + jobs consumed per stage
    L.zero = up128(L.tab + (int)sizeof(GroupTab));
    L.bar = L.zero + ZERO3_BYTES;
    L.total = L.bar + 2 * 32 * 8 + 16 + 16;
    return L;
}

// grid: one CTA per SM (persistent); block: NTEAM_A teams of TEAM_A consumer warps + 1 producer warp.
// A team takes whole tiles; its warps split the K dimension and one of them adds the partial sums.
__global__ void __launch_bounds__(NT_A, 1) moe_gateup_kernel(const MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const long long tk0 = clock64(), gt0 = gtime();
    const int Smax = a.stages_a;
    const SmemA L = smem_a_layout(a.hidden, a.inter, a.sh_inter, a.B, a.has_shared, Smax);
    const FinchTile T = finch_tile(a.hidden, a.inter);
    const FinchTile4 T4 = finch_tile4(a.hidden, a.sh_inter);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    GroupTab *tab = reinterpret_cast<GroupTab *>(smem + L.tab);
    float *red = reinterpret_cast<float *>(smem + L.red);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar), *empty = full + 32;
    const uint2 *zero8 = reinterpret_cast<const uint2 *>(empty + 32);
    uint64_t *xbar = empty + 34, *xbar2 = empty + 35;
    const int K = a.hidden, groups = K / 64, I = a.sh_inter;
    const int f4b = frag4_bytes(K);

    if (tid < 64) reinterpret_cast<int *>(smem + L.qcnt)[tid] = 0;
    if (tid < ZERO3_BYTES / 4) reinterpret_cast<int *>(smem + L.zero)[tid] = 0;
    if (tid == 0) {
        empty[32] = 0ull;
        for (int s = 0; s < Smax; s++) {
            finch_mbar_init(full + s, 1);
            finch_mbar_init(empty + s, TEAM_A);
        }
        finch_mbar_init(xbar, 1);
        finch_mbar_init(xbar2, 1);
    }
    grid_dep_wait();  // everything above overlaps the tail of the preparation kernel
    // only now may the down kernel be scheduled: it reads the preparation kernel's tables before its own wait,
    // and every CTA of this grid gets here only after the preparation kernel has completed
    grid_dep_launch();
    if (tid == 0) {
        // operand records of the tokens: one bulk copy each, under way while the group table is read
        finch_mbar_expect_tx(xbar, (unsigned)(a.B * L.rx3 + L.n4 * f4b));
        for (int b = 0; b < a.B; b++) finch_bulk_g2s(smem + L.rec + b * L.rx3, a.xrec3 + (size_t)b * L.rx3, L.rx3, xbar);
        for (int b = 0; b < L.n4; b++) finch_bulk_g2s(smem + L.rec4 + b * L.f4s, a.xrec4 + (size_t)b * f4b, f4b, xbar);
    }
    {
        const int *s = reinterpret_cast<const int *>(a.gtab);
        int *d = reinterpret_cast<int *>(tab);
        for (int i = tid; i < (int)(sizeof(GroupTab) / 4); i += NT_A) d[i] = __ldcg(s + i);
    }
    // A CTA whose range reaches into the shared-expert jobs keeps the 4-bit-layout fragments of every
    // token in shared memory too: it gives up the last stages of its ring for them.
    const int n_routed = __ldcg(&a.gtab->ng) * T.nTA;
    const int job0 = __ldcg(&a.gtab->range_a[blockIdx.x]), job1 = __ldcg(&a.gtab->range_a[blockIdx.x + 1]);
    const int n4x = (a.has_shared && job1 > n_routed && job1 > job0) ? a.B - L.n4 : 0;   // tokens beyond the fixed area
    const int tail_off = L.stage + Smax * L.stg - n4x * L.f4s;
    const int S = (Smax * L.stg - n4x * L.f4s) / L.stg;
    if (tid == 0 && n4x > 0) {
        // the other tokens' 4-bit-layout fragments, only in CTAs with shared-expert jobs
        finch_mbar_expect_tx(xbar2, (unsigned)(n4x * f4b));
        for (int b = 0; b < n4x; b++) finch_bulk_g2s(smem + tail_off + b * L.f4s, a.xrec4 + (size_t)(L.n4 + b) * f4b, f4b, xbar2);
    }
    __syncthreads();
    const long long tk1 = clock64();

    if (warp == CW_A) {
        // ---------------- producer warp: one bulk copy per job, issued in job order ----------------
        if (lane == 0) {
            for (int job = job0, it = 0; job < job1; ++job, ++it) {
                const int st = it % S, use = it / S;
                if (use > 0 && !finch_mbar_wait(empty + st, (use - 1) & 1)) {
                    atomicExch(a.status, FINCH_E_TIMEOUT);
                    return;
                }
                uint8_t *dst = smem + L.stage + st * L.stg;
                if (job < n_routed) {
                    const int gi = job / T.nTA, ta = job - gi * T.nTA;
                    finch_mbar_expect_tx(full + st, (unsigned)T.tileA);
                    finch_bulk_g2s(dst, a.pool_base + (size_t)tab->slot[gi] * a.slot_bytes + (size_t)ta * T.tileA, T.tileA, full + st);
                } else {
                    finch_mbar_expect_tx(full + st, (unsigned)T4.tileA);
                    finch_bulk_g2s(dst, a.sh_tiles + (size_t)(job - n_routed) * T4.tileA, T4.tileA, full + st);
                }
            }
        }
        return;
    }

    // ---------------- consumer warps ----------------
    // Warp w works on the K-quarter kw = w % 4 of the CTA's jobs w / 4, w / 4 + 4, ...  The four
    // warps of a job never wait for each other: each leaves its partial sums in the job's slot and
    // bumps the slot's counter; whoever comes last adds the four partials in fixed order.
    const int team = warp / TEAM_A, kw = warp % TEAM_A;
    int *qcnt = reinterpret_cast<int *>(smem + L.qcnt);
    if (!finch_mbar_wait(xbar, 0) || (n4x > 0 && !finch_mbar_wait(xbar2, 0))) {
        if (lane == 0) atomicExch(a.status, FINCH_E_TIMEOUT);
        return;
    }
    const long long tk2 = clock64();
    long long wait_acc = 0;
    int njobs = 0;
    // a CTA with fewer stages than teams lets its surplus teams sit out
    const int nteam = NTEAM_A < S ? NTEAM_A : S;
    int *cons = qcnt + 32;
    for (int it = team; team < nteam && job0 + it < job1; it += nteam, ++njobs) {
        const int job = job0 + it, st = it % S, use = it / S;
        const long long w0 = clock64();
        if (!wait_consumed(cons + st, use) || !finch_mbar_wait(full + st, use & 1)) {
            if (lane == 0) atomicExch(a.status, FINCH_E_TIMEOUT);
            return;
        }
        wait_acc += clock64() - w0;
        const uint8_t *tile = smem + L.stage + st * L.stg;
        float *slot = red + st * (MAXM / 2) * TEAM_A * 32;   // [pass][warp of the job][32]
        const bool routed = job < n_routed;
        const int gi = routed ? job / T.nTA : 0, ta = routed ? job - gi * T.nTA : job - n_routed;
        const int m = routed ? tab->m[gi] : a.B, npass = (m + 1) / 2;
        for (int ps = 0; ps < npass; ps++) {
            const int ntok = min(2, m - 2 * ps);
            float vA, vB;
            float *mine = slot + (ps * TEAM_A + kw) * 32;   // [token slot][row g][A|B]
            if (routed) {
                const int tok0 = tab->pairs[gi][2 * ps] / a.K, tok1 = tab->pairs[gi][2 * ps + (ntok > 1)] / a.K;
                const uint8_t *rec0 = smem + L.rec + tok0 * L.rx3, *rec1 = smem + L.rec + tok1 * L.rx3;
                gemv3_tile(tile, T.unitsA, kw, TEAM_A, a.scale_dtype, reinterpret_cast<const uint2 *>(rec0), reinterpret_cast<const uint2 *>(rec1),
                           reinterpret_cast<const float *>(rec0 + frag3_bytes(K)), reinterpret_cast<const float *>(rec1 + frag3_bytes(K)),
                           smem + L.zero, ntok, vA, vB);
                if ((t & 1) == 0) {
                    mine[(t >> 1) * 16 + g * 2] = vA;
                    mine[(t >> 1) * 16 + g * 2 + 1] = vB;
                }
            } else {
                // shared expert gate/up tile: 4 gate rows + 4 up rows, every token, two per pass
                const int tok0 = 2 * ps, tok1 = 2 * ps + (ntok > 1);
                const uint2 *f0 = reinterpret_cast<const uint2 *>(smem + (tok0 < L.n4 ? L.rec4 + tok0 * L.f4s : tail_off + (tok0 - L.n4) * L.f4s));
                const uint2 *f1 = reinterpret_cast<const uint2 *>(smem + (tok1 < L.n4 ? L.rec4 + tok1 * L.f4s : tail_off + (tok1 - L.n4) * L.f4s));
                gemv4_tile(tile, groups, kw, TEAM_A, (g & 3) * 4 + t, 16, g & 3, 4, a.sh_scale_dtype, f0, f1,
                           reinterpret_cast<const float *>(smem + L.rec + tok0 * L.rx3 + frag3_bytes(K)),
                           reinterpret_cast<const float *>(smem + L.rec + tok1 * L.rx3 + frag3_bytes(K)), zero8, ntok, vA, vB);
                if (t < 2) {
                    mine[t * 16 + g * 2] = vA;      // rows g >= 4 duplicate rows g - 4 and are never stored
                    mine[t * 16 + g * 2 + 1] = vB;
                }
            }
        }
        __threadfence_block();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(&qcnt[st], 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == TEAM_A - 1) {
            // last of the four: lane = (token slot, row g, gate|up); sum in fixed order, then SiLU(gate) * up
            __threadfence_block();
            for (int ps = 0; ps < npass; ps++) {
                const int ntok = min(2, m - 2 * ps);
                const float *src = slot + ps * TEAM_A * 32 + lane;
                float v = 0.f;
#pragma unroll
                for (int k = 0; k < TEAM_A; k++) v += src[k * 32];
                const float other = __shfl_xor_sync(0xffffffffu, v, 1);
                const int ts = lane >> 4, gg = (lane >> 1) & 7;
                if (!(lane & 1) && ts < ntok) {
                    const float r = (v / (1.0f + expf(-v))) * other;
                    if (routed) a.act[(size_t)tab->pairs[gi][2 * ps + ts] * a.inter + 8 * ta + gg] = r;
                    else if (gg < 4) a.shared_act[(size_t)(2 * ps + ts) * I + 4 * ta + gg] = r;
                }
            }
            if (lane == 0) {
                qcnt[st] = 0;
                __threadfence_block();
                *reinterpret_cast<volatile int *>(cons + st) = use + 1;
            }
            __syncwarp();
        }
        if (lane == 0) mbar_arrive(empty + st);
    }
    if (a.dbg && lane == 0) atomicMax(reinterpret_cast<unsigned long long *>(a.dbg + (size_t)blockIdx.x * 8 + 5), (unsigned long long)gtime());
    if (a.dbg && tid == 0) {
        long long *d = a.dbg + (size_t)blockIdx.x * 8;
        d[0] = tk1 - tk0;           // table + barriers
        d[1] = tk2 - tk1;           // waiting for the token records
        d[2] = clock64() - tk2;     // job loop of team 0
        d[3] = wait_acc;            // ... of which waiting for a full stage
        d[4] = gt0;
        d[6] = njobs;
        d[7] = job1 - job0;
    }
}

// ============================ kernel B ====================================
struct SmemB {
    int stage, stg, rec, srec, xstage, umax, tab, zero, bar, total;
};
__host__ __device__ inline SmemB smem_b_layout(int hidden, int inter, int sh_inter, int B, int has_shared, int stages) {
    const FinchTile T = finch_tile(hidden, inter);
    const FinchTile4 T4 = finch_tile4(hidden, sh_inter);
    SmemB L;
    L.stage = 0;
    L.stg = up128(has_shared && T4.tileB > T.tileB ? T4.tileB : T.tileB);
    L.rec = L.stage + stages * L.stg;                        // act records of the groups in this CTA's range
    L.srec = up128(L.rec + REC_CAP * rec3_bytes(inter));     // shared_act records
    L.xstage = up128(L.srec + (has_shared ? B * rec4_bytes(sh_inter) : 0));   // the act rows behind the records, staged as fp32
    L.umax = up128(L.xstage + REC_CAP * 4 * inter);                            // max |act| per (record, 128-value unit)
    L.tab = up128(L.umax + REC_CAP * (inter / 128) * 4);
    L.zero = up128(L.tab + (int)sizeof(GroupTab));
    L.bar = L.zero + ZERO3_BYTES;
    L.total = L.bar + 2 * 32 * 8 + 16 + 32 * 4;              // barriers, 16 zero bytes, jobs consumed per stage
    return L;
}

// grid: one CTA per SM (persistent); block: CW_B consumer warps + 1 producer warp.
__global__ void __launch_bounds__(NT_B, 1) moe_down_combine_kernel(const MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const long long tk0 = clock64(), gt0 = gtime();
    const int S = a.stages_b;
    const SmemB L = smem_b_layout(a.hidden, a.inter, a.sh_inter, a.B, a.has_shared, S);
    const FinchTile T = finch_tile(a.hidden, a.inter);
    const FinchTile4 T4 = finch_tile4(a.hidden, a.sh_inter);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    GroupTab *tab = reinterpret_cast<GroupTab *>(smem + L.tab);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar), *empty = full + 32;
    const uint2 *zero8 = reinterpret_cast<const uint2 *>(empty + 32);
    const int K = a.inter, Ks = a.sh_inter;
    const int r3b = rec3_bytes(K), r4b = rec4_bytes(Ks);

    if (tid == 0) {
        empty[32] = 0ull;
        for (int s = 0; s < S; s++) {
            finch_mbar_init(full + s, 1);
            finch_mbar_init(empty + s, 1);
        }
    }
    if (tid < ZERO3_BYTES / 4) reinterpret_cast<int *>(smem + L.zero)[tid] = 0;
    int *cons = reinterpret_cast<int *>(smem + L.bar + 2 * 32 * 8 + 16);
    if (tid < 32) cons[tid] = 0;
    grid_dep_launch();
    // The group table and the job ranges are the preparation kernel's output: that grid completed before the
    // gate/up kernel started, so they can be read, and the weight tiles streamed, while the gate/up kernel
    // is still finishing on other SMs.  Only the activations (its output) have to wait.
    {
        const int *s = reinterpret_cast<const int *>(a.gtab);
        int *d = reinterpret_cast<int *>(tab);
        for (int i = tid; i < (int)(sizeof(GroupTab) / 4); i += NT_B) d[i] = __ldcg(s + i);
    }
    __syncthreads();
    const long long tk1 = clock64();
    const int ng = tab->ng, n_routed = ng * T.nTB;
    const int job0 = tab->range_b[blockIdx.x], job1 = tab->range_b[blockIdx.x + 1];

    if (warp == CW_B) {
        // Producer warp: lane s owns stage s and issues that stage's fills in order (a single thread cannot issue
        // a 3.5 KB tile as fast as sixteen consumer warps use them up).  Per stage the order of fills and waits is
        // the serial one, so the producer's waits never see a barrier more than one phase behind.
        if (lane < S) {
            const int st = lane;
            for (int it = lane, use = 0; job0 + it < job1; it += S, ++use) {
                const int job = job0 + it;
                if (use > 0 && !finch_mbar_wait(empty + st, (use - 1) & 1)) {
                    atomicExch(a.status, FINCH_E_TIMEOUT);
                    return;
                }
                uint8_t *dst = smem + L.stage + st * L.stg;
                if (job < n_routed) {
                    const int gi = job / T.nTB, tb = job - gi * T.nTB;
                    finch_mbar_expect_tx(full + st, (unsigned)T.tileB);
                    finch_bulk_g2s(dst, a.pool_base + (size_t)tab->slot[gi] * a.slot_bytes + T.b_base + (size_t)tb * T.tileB, T.tileB, full + st);
                } else {
                    finch_mbar_expect_tx(full + st, (unsigned)T4.tileB);
                    finch_bulk_g2s(dst, a.sh_tiles + T4.b_base + (size_t)(job - n_routed) * T4.tileB, T4.tileB, full + st);
                }
            }
        }
        return;
    }

    // ---------------- consumer warps ----------------
    grid_dep_wait();   // the gate/up kernel has completed: act / shared_act are final
    const long long tkw = clock64();
    // operand records of the activations this CTA needs: the pairs of the groups in its job range
    // (and every token's shared activations if it has shared-expert jobs)
    const int g_lo = job0 < n_routed ? job0 / T.nTB : ng;
    const int g_hi = job1 > job0 ? min(ng - 1, (job1 - 1) / T.nTB) : -1;   // inclusive
    {
        // One warp per (record, 128-value unit): first the unit's values are staged, its two group sums written and its
        // largest magnitude noted; after a barrier every unit knows its record's exponent and builds its fragments.
        float *xstage = reinterpret_cast<float *>(smem + L.xstage), *umax = reinterpret_cast<float *>(smem + L.umax);
        const int units = K / 128;
        int nrec = 0;
        for (int gi = g_lo; gi <= g_hi; gi++) nrec += tab->m[gi];
        if (nrec > REC_CAP) {
            if (tid == 0) atomicExch(a.status, FINCH_E_UNSUPPORTED);
            nrec = REC_CAP;
        }
        auto pair_of = [&](int q) {   // q-th record of the CTA -> its (token, k) pair
            int gi = g_lo;
            while (q >= tab->m[gi]) q -= tab->m[gi++];
            return (int)tab->pairs[gi][q];
        };
        for (int it = warp; it < nrec * units; it += CW_B) {
            const int q = it / units, u = it - q * units;
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(a.act + (size_t)pair_of(q) * K + u * 128) + lane);
            *reinterpret_cast<float4 *>(xstage + q * K + u * 128 + lane * 4) = v;
            float sum = (v.x + v.y) + (v.z + v.w), mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            float *hdr = reinterpret_cast<float *>(smem + L.rec + q * r3b + frag3_bytes(K));
            if ((lane & 15) == 0) hdr[2 * u + (lane >> 4)] = sum;
            if (lane == 0) umax[it] = mx;
        }
        // the shared expert's records, from the last warp down (the first warps have the routed records), before the
        // barrier so that they overlap the loads above
        if (a.has_shared && job1 > n_routed && job1 > job0)
            for (int b = CW_B - 1 - warp; b >= 0 && b < a.B; b += CW_B) {
                // staged in the rows of the staging area that the routed records leave free, when there are enough
                float *stg = (Ks <= K && nrec + a.B <= REC_CAP) ? xstage + (size_t)(REC_CAP - 1 - b) * K : nullptr;
                warp_make_record<4>(a.shared_act + (size_t)b * Ks, Ks, smem + L.srec + b * r4b, stg);
            }
        bar_sync(1, CW_B * 32);
        for (int it = warp; it < nrec * units; it += CW_B) {
            const int q = it / units, u = it - q * units;
            float m = 0.f;
            for (int j = 0; j < units; j++) m = fmaxf(m, umax[q * units + j]);
            int E = (int)(__float_as_uint(m) >> 23) + 1;
            E = E < 30 ? 30 : (E > 230 ? 230 : E);
            uint8_t *rec = smem + L.rec + q * r3b;
            if (u == 0 && lane == 0) reinterpret_cast<float *>(rec + frag3_bytes(K))[K / 64] = __int_as_float(E);
            build_frag3_range(xstage + q * K + u * 128, 128, E, reinterpret_cast<uint2 *>(rec) + u * 72, lane, 32);
        }
    }
    bar_sync(1, CW_B * 32);
    const long long tk2 = clock64();

    long long wait_acc = 0;
    int njobs = 0;
    for (int it = warp; job0 + it < job1; it += CW_B, ++njobs) {
        const int job = job0 + it, st = it % S, use = it / S;
        const long long w0 = clock64();
        if (!wait_consumed(cons + st, use) || !finch_mbar_wait(full + st, use & 1)) {
            if (lane == 0) atomicExch(a.status, FINCH_E_TIMEOUT);
            break;
        }
        wait_acc += clock64() - w0;
        const uint8_t *tile = smem + L.stage + st * L.stg;
        int tb;
        if (job < n_routed) {
            const int gi = job / T.nTB, m = tab->m[gi], npass = (m + 1) / 2;
            tb = job - gi * T.nTB;
            int slot0 = 0;  // first record of this group in the CTA's record area
            for (int j = g_lo; j < gi; j++) slot0 += tab->m[j];
            for (int ps = 0; ps < npass; ps++) {
                const int ntok = min(2, m - 2 * ps);
                const uint8_t *rec0 = smem + L.rec + (slot0 + 2 * ps) * r3b, *rec1 = smem + L.rec + (slot0 + 2 * ps + (ntok > 1)) * r3b;
                float va, vb;
                gemv3_tile(tile, T.unitsD, 0, 1, a.scale_dtype, reinterpret_cast<const uint2 *>(rec0), reinterpret_cast<const uint2 *>(rec1),
                           reinterpret_cast<const float *>(rec0 + frag3_bytes(K)), reinterpret_cast<const float *>(rec1 + frag3_bytes(K)),
                           smem + L.zero, ntok, va, vb);
                if ((t & 1) == 0 && (t >> 1) < ntok) {
                    float *o = a.partial + (size_t)tab->pairs[gi][2 * ps + (t >> 1)] * a.hidden + 16 * tb + g;
                    o[0] = va;
                    o[8] = vb;
                }
            }
        } else {
            tb = job - n_routed;
            const int npass = (a.B + 1) / 2;
            for (int ps = 0; ps < npass; ps++) {
                const int ntok = min(2, a.B - 2 * ps);
                const uint8_t *rec0 = smem + L.srec + (2 * ps) * r4b, *rec1 = smem + L.srec + (2 * ps + (ntok > 1)) * r4b;
                float va, vb;
                gemv4_tile(tile, Ks / 64, 0, 1, lane, 32, g, 8, a.sh_scale_dtype, reinterpret_cast<const uint2 *>(rec0),
                           reinterpret_cast<const uint2 *>(rec1), reinterpret_cast<const float *>(rec0 + frag4_bytes(Ks)),
                           reinterpret_cast<const float *>(rec1 + frag4_bytes(Ks)), zero8, ntok, va, vb);
                if (t < ntok) {
                    float *o = a.partial + (size_t)(a.P + 2 * ps + t) * a.hidden + 16 * tb + g;
                    o[0] = va;
                    o[8] = vb;
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            *reinterpret_cast<volatile int *>(cons + st) = use + 1;
            mbar_arrive(empty + st);
        }
        (void)tb;
    }

    const long long tk3 = clock64();
    if (a.dbg && lane == 0) atomicMax(reinterpret_cast<unsigned long long *>(a.dbg + (size_t)(1024 + blockIdx.x) * 8 + 5), (unsigned long long)gtime());
    if (a.dbg && tid == 0) {
        long long *d = a.dbg + (size_t)(1024 + blockIdx.x) * 8;
        d[0] = tk1 - tk0;   // table + barriers
        d[1] = tk2 - tkw;   // act records
        d[2] = tk3 - tk2;   // job loop of warp 0
        d[3] = wait_acc;    // ... of which waiting for a full stage
        d[4] = gt0;
        d[6] = tkw - tk1;   // waiting for the gate/up kernel
        d[7] = job1 - job0;
    }
}

// ============================ combine =====================================
// hidden = h_mid + sum_{k ascending, usable} w_k * out_k + sigmoid(score) * shared_out, the arithmetic of
// moe_combine_residual (finchmoe/shaders.metal:2196-2231).  grid: (hidden / 256, B); block 256.
__global__ void __launch_bounds__(256) moe_combine_kernel(const MoeArgs a) {
    __shared__ int ok[8];
    __shared__ float wk[8];
    const int b = blockIdx.y, row = blockIdx.x * 256 + threadIdx.x;
    const long long gt0 = gtime();
    grid_dep_launch();
    // Routing, router weights, gate scores and h_mid are inputs of the whole call: final since the preparation
    // kernel (the first of the chain) passed its own wait, and this kernel only starts once the down kernel has,
    // which started after the gate/up kernel's wait, i.e. after the preparation kernel completed.  Only the
    // partial rows (the down kernel's output) have to wait; the dependent loads of the routing (mask -> id ->
    // slot) are out of the way by then.
    if (threadIdx.x < a.K) {
        ok[threadIdx.x] = pair_ok(a, b * a.K + threadIdx.x);
        wk[threadIdx.x] = a.weights[b * a.K + threadIdx.x];
    }
    const bool live = row < a.hidden;
    float h = live && a.h_mid ? a.h_mid[(size_t)b * a.hidden + row] : 0.f;
    const float sg = a.has_shared ? 1.0f / (1.0f + expf(-a.gate_score[b])) : 0.f;
    __syncthreads();
    grid_dep_wait();
    if (!live) return;
    float moe = 0.f;
    for (int k = 0; k < a.K; k++)
        if (ok[k]) moe = fmaf(wk[k], a.partial[(size_t)(b * a.K + k) * a.hidden + row], moe);
    h += moe;
    if (a.has_shared) h = fmaf(sg, a.partial[(size_t)(a.P + b) * a.hidden + row], h);
    a.hidden_out[(size_t)b * a.hidden + row] = h;
    if (a.dbg && threadIdx.x == 0) {
        long long *d = a.dbg + (size_t)(1400 + blockIdx.y * gridDim.x + blockIdx.x) * 8;
        d[0] = gt0;
        d[1] = gtime();
    }
}

constexpr int SMEM_MAX = 227 * 1024;
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

// Tiled copy of a shared expert, made the first time the expert is seen (keyed by its three weight
// pointers) and kept for the life of the context.
int prepared_shared(finch_ctx *ctx, const finch_shared *sh, cudaStream_t st, const uint8_t **out) {
    for (auto &e : ctx->shared_cache)
        if (e.key[0] == sh->gate.W && e.key[1] == sh->up.W && e.key[2] == sh->down.W) {
            *out = (const uint8_t *)e.tiles;
            return FINCH_OK;
        }
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cap);
    if (cap != cudaStreamCaptureStatusNone)
        return finch_fail(ctx, FINCH_E_UNSUPPORTED, "a shared expert must be used once outside stream capture before it is captured");
    const FinchTile4 T4 = finch_tile4(ctx->cfg.hidden, sh->gate.out_dim);
    void *buf = nullptr;
    if (cudaMalloc(&buf, T4.total) != cudaSuccess) {
        cudaGetLastError();
        return finch_fail(ctx, FINCH_E_NOMEM, "tiled copy of the shared expert (%zu bytes)", T4.total);
    }
    SharedSrc S{(const uint32_t *)sh->gate.W,      (const uint32_t *)sh->up.W,        (const uint32_t *)sh->down.W,
                (const uint16_t *)sh->gate.scales, (const uint16_t *)sh->gate.biases, (const uint16_t *)sh->up.scales,
                (const uint16_t *)sh->up.biases,   (const uint16_t *)sh->down.scales, (const uint16_t *)sh->down.biases};
    shared_retile_kernel<<<256, 256, 0, st>>>(S, ctx->cfg.hidden, sh->gate.out_dim, (uint8_t *)buf);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        cudaFree(buf);
        return finch_fail(ctx, FINCH_E_CUDA, "shared_retile_kernel: %s", cudaGetErrorString(e));
    }
    ctx->launches++;
    ctx->shared_cache.push_back({{sh->gate.W, sh->up.W, sh->down.W}, buf});
    *out = (const uint8_t *)buf;
    return FINCH_OK;
}

inline size_t up256z(size_t n) { return (n + 255) & ~(size_t)255; }

}  // namespace

// Bytes of operand-record / group-table scratch a context needs (allocated in finch_ctx_create).
size_t finch_decode_scratch_bytes(const finch_config &c) {
    const size_t B = c.max_tokens;
    return up256z(sizeof(GroupTab)) + up256z(B * rec3_bytes(c.hidden)) + up256z(B * frag4_bytes(c.hidden)) + 1024;
}

extern "C" int finch_encode_moe_decode(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, const void *h_post,
                                       const int32_t *expert_ids, const float *weights, const uint8_t *valid,
                                       const finch_shared *shared, const float *h_mid, float *hidden_out, int B) {
    if (!ctx || !pool || !h_post || !expert_ids || !weights || !hidden_out) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    if (pool->ctx != ctx) return finch_fail(ctx, FINCH_E_ARG, "pool belongs to another context");
    if (layer < 0 || layer >= pool->n_layers) return finch_fail(ctx, FINCH_E_ARG, "layer %d out of range", layer);
    if (B < 1 || B > c.max_tokens) return finch_fail(ctx, FINCH_E_ARG, "B=%d outside 1..max_tokens=%d", B, c.max_tokens);
    if (B * c.top_k > FINCH_MAX_PAIRS || B > MAXM)
        return finch_fail(ctx, FINCH_E_UNSUPPORTED, "decode path takes at most %d tokens / %d (token, expert) pairs; use finch_encode_moe_prefill",
                          MAXM, FINCH_MAX_PAIRS);
    if (pool->n_experts != c.n_experts) return finch_fail(ctx, FINCH_E_ARG, "pool / context expert count mismatch");
    cudaSetDevice(c.device);
    cudaStream_t st = finch_pick_stream(ctx, stream);
    MoeArgs a{};
    a.sh_inter = 64;
    if (shared) {
        int rc = check_shared(ctx, shared);
        if (rc) return rc;
        if ((rc = prepared_shared(ctx, shared, st, &a.sh_tiles))) return rc;
        a.has_shared = 1;
        a.sh_scale_dtype = shared->gate.scale_dtype;
        a.shared_act = ctx->shared_act;
        a.gate_score = shared->gate_score;
        a.sh_inter = shared->gate.out_dim;
    }
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
    a.scale_dtype = c.scale_dtype;
    a.act = ctx->act;
    a.partial = ctx->partial;
    a.status = ctx->dev_status;
    a.h_mid = h_mid;
    a.hidden_out = hidden_out;
    a.dbg = (long long *)ctx->dbg;
    {  // carve the scratch (same order as finch_decode_scratch_bytes)
        const size_t Bm = c.max_tokens;
        char *p = (char *)ctx->frag_scratch;
        auto take = [&](size_t bytes) {
            char *r = p;
            p += up256z(bytes);
            return r;
        };
        a.gtab = (GroupTab *)take(sizeof(GroupTab));
        a.xrec3 = (uint8_t *)take(Bm * rec3_bytes(c.hidden));
        a.xrec4 = (uint8_t *)take(Bm * frag4_bytes(c.hidden));
    }
    const int grid = ctx->sm_count < MAXG ? ctx->sm_count : MAXG;
    a.grid_a = a.grid_b = grid;
    // pipeline depth: as many stages as fit
    const SmemA A0 = smem_a_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, 0);
    const SmemB B0 = smem_b_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, 0);
    int sa = (SMEM_MAX - A0.total) / (A0.stg + (MAXM / 2) * TEAM_A * 32 * 4), sb = (SMEM_MAX - B0.total) / B0.stg;
    sa = sa > 32 ? 32 : sa;
    sb = sb > 32 ? 32 : sb;
    {  // CTAs that also run shared-expert jobs give some stages up for the 4-bit-layout fragments of the tokens
        const int extra = a.has_shared ? (B - A0.n4) * A0.f4s : 0;
        if (sa >= 2 && (sa * A0.stg - extra) / A0.stg < 2) sa = 0;
    }
    if (sa < 2 || sb < CW_B) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "dims need too much shared memory");
    a.stages_a = sa;
    a.stages_b = sb;
    const SmemA LA = smem_a_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, sa);
    const SmemB LB = smem_b_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, sb);
    const int prep_smem = c.hidden * 4 + 144 * 4 + 32 + (MAXP + 2) * 4 + MAXP + 8 + (int)sizeof(GroupTab) + 64;
    if (!g_attr_set) {
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_down_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024));
        // one shared-memory carve-out for all four kernels: an SM that has to change its L1 / shared split
        // between consecutive launches drains first
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_prep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_gateup_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_down_combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        g_attr_set = true;
    }
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
    // Launched with programmatic stream serialization: a kernel may be scheduled while its predecessor
    // drains and runs its prologue up to griddepcontrol.wait, which hides most of the launch latency.
    auto launch = [&](const void *fn, dim3 g, int threads, size_t smem_bytes) -> cudaError_t {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = g;
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = smem_bytes;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = ctx->no_pdl ? 0 : 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        void *args[] = {(void *)&a};
        return cudaLaunchKernelExC(&cfg, fn, args);
    };
    FINCH_CUDA_OK(ctx, launch((const void *)moe_prep_kernel, dim3(B + 1), 256, prep_smem));
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[0], st));
    FINCH_CUDA_OK(ctx, launch((const void *)moe_gateup_kernel, dim3(grid), NT_A, LA.total));
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[1], st));
    FINCH_CUDA_OK(ctx, launch((const void *)moe_down_combine_kernel, dim3(grid), NT_B, LB.total));
    FINCH_CUDA_OK(ctx, launch((const void *)moe_combine_kernel, dim3((c.hidden + 255) / 256, B), 256, 0));
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[2], st));
    ctx->launches += 4;
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

// Kept for binary compatibility of the test hook: the preparation kernel now always runs.
extern "C" int finch_debug_timing(finch_ctx *ctx, void *buf) {
    if (!ctx) return FINCH_E_ARG;
    ctx->dbg = buf;
    return FINCH_OK;
}
