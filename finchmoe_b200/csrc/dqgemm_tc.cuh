// Dequant-GEMM on the 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
//   D[128 weight rows, TN tokens] += Wdq[128, K] * X[TN, K]^T        (bf16 x bf16 -> fp32)
//
// One CTA owns one 128-row weight tile and up to tn_max tokens.  Per K block of 64 values (one scale group) its
// eight dequantising warps turn packed codes (EXPERT_*: brought into a ring of shared-memory slots by bulk copies;
// DENSE4: loaded from global memory one block ahead) into the weight fl32(fl32(q*s)+b) -- the value the
// reference's dequantised weight has (quant_audit.py:245 semantics) -- and write it as TWO bf16 planes, the
// value rounded to bf16 and the bf16-rounded remainder (16 significant bits together), into shared memory in
// the 128-byte-swizzled K-major layout the tensor core reads; the tokens' activations arrive by cp.async
// (one bf16 plane, or two when the caller passes the remainder plane of fp32 activations).  Lane 0 of a ninth,
// control warp issues the block's tcgen05.mma (K = 16 each, both weight planes into the same accumulator)
// and commits them to an mbarrier.  Two weight stages and three activation stages: the warps dequantise block
// i+1 while the tensor core works on block i, and the activations of block i+1 are requested before block i is
// dequantised, so no block waits for a load it has just issued.  Two CTAs fit an SM.  The epilogue reads the
// accumulator with tcgen05.ld, one lane (= weight row) per thread.
//
// Shared by moe_prefill.cu (grouped 3-bit expert GEMMs over the pool's tiled layout) and the dense
// 4-bit projections.  Every wait is bounded; on a time-out the CTA reports through `status`, frees
// its tensor memory and returns.
#pragma once
#include "finch_internal.cuh"
#include "tile_layout.h"

namespace dqgemm {

constexpr int GM = 128;       // weight rows per CTA = UMMA M
constexpr int BK = 64;        // K values per stage = one 64-value swizzle atom = one scale group
constexpr int NS = 2;         // weight stages
constexpr int NB = 3;         // activation stages
constexpr int NT = 256;       // dequantising threads per CTA: two per weight row, one for each 32-value half of a K block
constexpr int NTB = NT + 32;  // + one control warp: its lane 0 issues the MMAs and the bulk copies of the packed blocks
constexpr int A_ATOM = GM * 128;   // bytes of one 64-value atom of the weight tile
constexpr int RD = 3;         // depth of the ring of packed expert blocks (EXPERT_* modes)
constexpr int RAW_STAGE = 8 * 768 + 8 * 128;   // one 128-value unit (two K blocks) of eight 16-row pool tiles: operand words, then scale/bias entries

enum Mode { EXPERT_GATEUP = 0, EXPERT_DOWN = 1, DENSE4 = 2 };

struct Args {
    int mode;
    int K;                    // reduction length (multiple of 128)
    int tn_max;               // token-tile capacity of a CTA: 16..256, multiple of 16
    int scale_dtype;
    // EXPERT_*: weights come from the pool (tiled layout, tile_layout.h)
    const uint8_t *pool_base;
    size_t slot_bytes;
    const int32_t *slot_row;  // [n_experts] slot of each expert of this layer, < 0: absent
    int hidden, inter;
    const int *seg;           // [n_experts + 1] ranges of `order`
    const int *order;         // pair ids sorted by expert
    const int2 *items;        // (expert, first pair of the tile inside the expert's range), one per blockIdx.y
    const int *n_items;
    int top_k;
    // DENSE4: reference tensor layout (u32 words, 16-bit scales and biases per group of 64)
    const uint32_t *W;
    const uint16_t *S, *B;
    int rows;                 // output rows
    int n_tokens;
    // activations: bf16 rows of K values; row index = token (GATEUP, DENSE4) or pair (DOWN).  X2, when
    // not NULL, is a second plane added to the first (value = X + X2): the low-order part of an
    // activation kept to about 16 bits, multiplied by the same weight tile into the same accumulator.
    const uint16_t *X, *X2;
    // outputs
    uint16_t *act_out;        // GATEUP: bf16 [pairs][inter] = SiLU(gate) * up, rounded to bf16 ...
    uint16_t *act_out_lo;     // ... and bf16(value - that), or NULL
    float *out;               // DOWN: fp32 [pairs][hidden]; DENSE4: fp32 [tokens][rows]
    int *status;
};

__host__ __device__ inline int smem_bytes(int tn_max, int planes, int expert) {
    return 1024 + NS * 2 * A_ATOM + NB * planes * tn_max * 128 + (expert ? RD * RAW_STAGE : 0) + 256 + tn_max * 4;
}

__host__ __device__ inline int tmem_cols(int tn_max) { return tn_max <= 32 ? 32 : tn_max <= 64 ? 64 : tn_max <= 128 ? 128 : 256; }

// ---- tcgen05 wrappers ----------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t smem_dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_dst), "r"(cols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(finch_smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 16 consecutive fp32 columns of this thread's lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
          "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: bf16 x bf16 -> fp32, both operands K-major, M = 128, N = tn.
__device__ __forceinline__ uint32_t instr_desc(int tn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(tn >> 3) << 17) | ((uint32_t)(GM >> 4) << 24);
}

// Byte offset of 16-byte chunk c (0..7) of row r inside a 64-value atom.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
// two fp32 values -> their bf16 images (packed) and the bf16 images of the remainders
__device__ __forceinline__ void bf16x2_split(float lo, float hi, uint32_t &h, uint32_t &r) {
    h = bf16x2_rn(lo, hi);
    r = bf16x2_rn(lo - __uint_as_float(h << 16), hi - __uint_as_float(h & 0xffff0000u));
}
__device__ __forceinline__ void st_shared16(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// 16-byte asynchronous copy global -> shared (lands while the warps dequantise)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Dequantisation without integer-to-float conversions: a code isolated by one AND at bits [p, p+4) of a
// 16-bit half is the fp16 subnormal q * 2^(p-24); widening it to fp32 is exact, and
//   fma(q * 2^(p-24), s * 2^(24-p), b)  =  round_fp32(q * s + b)  =  fl32(fl32(q * s) + b)
// because q * s is exact in fp32 (3- or 4-bit q, at most 11-bit s): the value the reference's
// dequantised weight has (quant_audit.py:245), written to the tile as a bf16 value and a bf16 remainder.
struct GroupScale {
    float sp[8];   // s * 2^(24-p), p = 0..7
    float b;
};
__device__ __forceinline__ GroupScale group_scale(float s, float b) {
    GroupScale g;
#pragma unroll
    for (int p = 0; p < 8; p++) g.sp[p] = s * __uint_as_float((uint32_t)(127 + 24 - p) << 23);
    g.b = b;
    return g;
}
__device__ __forceinline__ float half_lo(uint32_t r) { return __low2float(*reinterpret_cast<const __half2 *>(&r)); }
__device__ __forceinline__ float half_hi(uint32_t r) { return __high2float(*reinterpret_cast<const __half2 *>(&r)); }

// 32 three-bit codes in three words (a little-endian bit stream) -> four chunks of 8 bf16 (value plane o, remainder plane ol).
// 18 masked registers hold two codes each; IDX / POS say which code and at which bit of its half.
__device__ __forceinline__ void dq3_piece(uint32_t w0, uint32_t w1, uint32_t w2, const GroupScale &gs, uint32_t (&o)[16], uint32_t (&ol)[16]) {
    constexpr int IDX[36] = {0, 6, 1, 7, 2, -1, 3, 8, 4, 9, 5, 10, 11, 16, 12, 17, 13, 18,
                             14, 19, 15, 20, -1, 21, 22, 27, 23, 28, -1, 29, 24, 30, 25, 31, 26, -1};
    constexpr int POS[36] = {0, 2, 3, 5, 6, 0, 1, 0, 4, 3, 7, 6, 1, 0, 4, 3, 7, 6,
                             2, 1, 5, 4, 0, 7, 2, 1, 5, 4, 0, 7, 0, 2, 3, 5, 6, 0};
    const uint32_t v1 = __funnelshift_r(w0, w1, 8), v3 = __funnelshift_r(w1, w2, 8), v5 = w2 >> 8;
    uint32_t e[18];
    e[0] = w0 & 0x001C0007u;  e[1] = w0 & 0x00E00038u;  e[2] = w0 & 0x000001C0u;
    e[3] = v1 & 0x0007000Eu;  e[4] = v1 & 0x00380070u;  e[5] = v1 & 0x01C00380u;
    e[6] = w1 & 0x0007000Eu;  e[7] = w1 & 0x00380070u;  e[8] = w1 & 0x01C00380u;
    e[9] = v3 & 0x000E001Cu;  e[10] = v3 & 0x007000E0u; e[11] = v3 & 0x03800000u;
    e[12] = w2 & 0x000E001Cu; e[13] = w2 & 0x007000E0u; e[14] = w2 & 0x03800000u;
    e[15] = v5 & 0x001C0007u; e[16] = v5 & 0x00E00038u; e[17] = v5 & 0x000001C0u;
    float v[32];
#pragma unroll
    for (int k = 0; k < 36; k++) {
        if (IDX[k] < 0) continue;
        const float q = (k & 1) ? half_hi(e[k >> 1]) : half_lo(e[k >> 1]);
        v[IDX[k]] = fmaf(q, gs.sp[POS[k]], gs.b);
    }
#pragma unroll
    for (int i = 0; i < 16; i++) bf16x2_split(v[2 * i], v[2 * i + 1], o[i], ol[i]);
}
// 8 four-bit codes in one word -> one chunk of 8 bf16 (value plane and remainder plane).
__device__ __forceinline__ void dq4_word(uint32_t w, const GroupScale &gs, uint32_t (&o)[4], uint32_t (&ol)[4]) {
    const uint32_t x = w >> 8;
    const uint32_t e0 = w & 0x000F000Fu, e1 = w & 0x00F000F0u, e2 = x & 0x000F000Fu, e3 = x & 0x00F000F0u;   // codes (0,4) (1,5) (2,6) (3,7)
    float v[8];
    v[0] = fmaf(half_lo(e0), gs.sp[0], gs.b); v[4] = fmaf(half_hi(e0), gs.sp[0], gs.b);
    v[1] = fmaf(half_lo(e1), gs.sp[4], gs.b); v[5] = fmaf(half_hi(e1), gs.sp[4], gs.b);
    v[2] = fmaf(half_lo(e2), gs.sp[0], gs.b); v[6] = fmaf(half_hi(e2), gs.sp[0], gs.b);
    v[3] = fmaf(half_lo(e3), gs.sp[4], gs.b); v[7] = fmaf(half_hi(e3), gs.sp[4], gs.b);
#pragma unroll
    for (int i = 0; i < 4; i++) bf16x2_split(v[2 * i], v[2 * i + 1], o[i], ol[i]);
}

// grid: x = 128-row weight tile; EXPERT_*: y = (expert, token tile) item; DENSE4: z = token tile.  block: 288 threads.
//
// No CTA-wide barrier inside the K loop.  Each of the eight dequantising warps writes its share of block
// kb into weight stage kb % NS and arrives on a_full[stage]; lane 0 of the ninth (control) warp then issues the
// block's MMAs and commits them to done[stage], which frees the stage (and the activation stage of the same
// block), while the other warps already work on block kb + 1; the same thread keeps the ring of packed units
// filled, refilling a slot once raw_empty[slot] says that every dequantising warp has read both of its groups.
__global__ void __launch_bounds__(NTB, 2) dqgemm_tc_kernel(const Args a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tn_max = a.tn_max;
    // ---- which tokens ----
    int m_total, first, t0, expert_id = 0;
    const int *rows_of = nullptr;   // EXPERT_*: pair ids of this expert
    if (a.mode == DENSE4) {
        m_total = a.n_tokens;
        first = 0;
        t0 = blockIdx.z * tn_max;
    } else {
        if ((int)blockIdx.y >= *a.n_items) return;
        const int2 it = a.items[blockIdx.y];
        expert_id = it.x;
        t0 = it.y;
        first = a.seg[expert_id];
        m_total = a.seg[expert_id + 1] - first;
        rows_of = a.order + first;
    }
    if (t0 >= m_total) return;
    const int m = min(tn_max, m_total - t0);        // tokens of this CTA
    const int tn = (m + 15) & ~15;                   // token columns of the accumulator (per plane)

    const uint32_t base = (finch_smem_u32(smem_raw) + 1023u) & ~1023u;
    // The two activation planes sit side by side along N: rows [0, tn) of an atom are plane 0, rows
    // [tn, 2 tn) plane 1, one MMA covers both and the epilogue adds the two halves of the accumulator.
    const int planes = a.X2 ? 2 : 1, b_atom = planes * tn_max * 128;
    const int a_stage = 2 * A_ATOM;                    // weights of one K block: value plane, remainder plane
    const bool expert = a.mode != DENSE4;
    const uint32_t bbase = base + NS * a_stage;        // NB activation stages of b_atom bytes
    const uint32_t raw = bbase + NB * b_atom;          // EXPERT_*: ring of packed units, filled by bulk copies
    const uint32_t ctl = raw + (expert ? RD * RAW_STAGE : 0);   // barriers, tensor-memory address, row list
    uint8_t *ctl_p = smem_raw + (ctl - finch_smem_u32(smem_raw));
    uint8_t *raw_p = smem_raw + (raw - finch_smem_u32(smem_raw));
    uint64_t *done = reinterpret_cast<uint64_t *>(ctl_p);   // [NS]  MMAs of the block in this weight stage finished
    uint64_t *a_full = done + NS;                            // [NS]  all warps wrote their share of the stage
    uint64_t *raw_full = a_full + NS;                        // [RD]  packed unit landed
    uint64_t *raw_empty = raw_full + RD;                     // [RD]  all warps read the packed unit
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(ctl_p + 128);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(ctl_p + 132);   // set by whoever gives up on a wait
    int *src_rows = reinterpret_cast<int *>(ctl_p + 256);   // [tn_max] activation row of each token of the tile
    constexpr int NW = NT / 32;   // dequantising warps
    const bool control = warp == NW;

    // zero the activation stages once: rows >= m are never written and must read as 0
    for (int i = tid; i < NB * b_atom / 16 && !control; i += NT) st_shared16(bbase + i * 16, 0u, 0u, 0u, 0u);
    for (int j = tid; j < m && !control; j += NT) {
        int row = t0 + j;
        if (a.mode != DENSE4) {
            const int pair = rows_of[t0 + j];
            row = a.mode == EXPERT_GATEUP ? pair / a.top_k : pair;
        }
        src_rows[j] = row;
    }
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < NS; s++) {
            finch_mbar_init(done + s, 1);
            finch_mbar_init(a_full + s, NW);
        }
        for (int s = 0; s < RD; s++) {
            finch_mbar_init(raw_full + s, 1);
            finch_mbar_init(raw_empty + s, NW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    const uint32_t ncols = (uint32_t)tmem_cols(planes * tn_max);
    if (warp == 0) {
        tmem_alloc(finch_smem_u32(tmem_slot), ncols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;

    // ---- this thread's weight row ----
    const int r = tid & (GM - 1), kh = tid >> 7;   // row of the tile (= tensor-memory lane) and 32-value half of a K block
    const uint32_t *w4 = nullptr;      // DENSE4: packed row
    const uint16_t *s4 = nullptr, *b4 = nullptr;
    uint32_t raw_w = 0, raw_s = 0;     // EXPERT_*: this thread's words / scale inside a ring slot (first group of the unit)
    const uint8_t *tile0 = nullptr;    // EXPERT_*: first of the CTA's eight pool tiles
    int tile_stride = 0, sb_off = 0;
    if (a.mode == DENSE4) {
        const size_t row = (size_t)blockIdx.x * GM + r;
        w4 = a.W + row * (a.K / 8);
        s4 = a.S + row * (a.K / 64);
        b4 = a.B + row * (a.K / 64);
    } else {
        const FinchTile T = finch_tile(a.hidden, a.inter);
        const int fr = r & 15, g = fr & 7, half = fr >> 3;
        const uint8_t *blk = a.pool_base + (size_t)a.slot_row[expert_id] * a.slot_bytes;
        raw_w = (uint32_t)((r >> 4) * 768 + (g * 4 + kh) * 24 + half * 12);   // period kh of the unit's first group; the second group is 48 bytes on
        raw_s = (uint32_t)(8 * 768 + (r >> 4) * 128 + g * 16 + half * 4);     // + 2 for the second group, + 8 for the bias
        tile0 = a.mode == EXPERT_GATEUP ? blk + (size_t)blockIdx.x * 8 * T.tileA : blk + T.b_base + (size_t)blockIdx.x * 8 * T.tileB;
        tile_stride = a.mode == EXPERT_GATEUP ? T.tileA : T.tileB;
        sb_off = a.mode == EXPERT_GATEUP ? T.sbA : T.sbB;
    }

    const int nkb = a.K / BK, nunits = a.K / 128;
    const uint32_t idesc = instr_desc(planes * tn);
    bool failed = false;
    uint32_t wreg[4];
    uint32_t sreg = 0, breg = 0;   // low 16 bits: scale / bias of this thread's group
    auto load_block = [&](int kb) {   // DENSE4: straight from global memory, one block ahead
        const uint4 v0 = __ldg(reinterpret_cast<const uint4 *>(w4 + kb * 8 + kh * 4));
        wreg[0] = v0.x; wreg[1] = v0.y; wreg[2] = v0.z; wreg[3] = v0.w;
        sreg = __ldg(s4 + kb);
        breg = __ldg(b4 + kb);
    };
    // EXPERT_*: one thread keeps up to RD units of packed bytes in flight (16 bulk copies per unit)
    auto issue_raw = [&](int u) {
        const int slot = u % RD;
        uint8_t *dst = raw_p + slot * RAW_STAGE;
        finch_mbar_expect_tx(raw_full + slot, (unsigned)RAW_STAGE);
        for (int d = 0; d < 8; d++) {
            const uint8_t *t = tile0 + (size_t)d * tile_stride;
            finch_bulk_g2s(dst + d * 768, t + (size_t)u * 768, 768, raw_full + slot);
            finch_bulk_g2s(dst + 8 * 768 + d * 128, t + sb_off + (size_t)u * 128, 128, raw_full + slot);
        }
    };
    // descriptors of the stages; a K step of 16 values advances the start address by 32 bytes (2 units)
    auto issue_mma = [&](int kb) {
        const uint32_t ast = base + (kb % NS) * a_stage, bst = bbase + (kb % NB) * b_atom;
        const uint64_t ad = smem_desc(ast), bd = smem_desc(bst);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint64_t off = (uint64_t)((k * 32) >> 4);
            tc_mma_bf16(tmem_d, ad + off, bd + off, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            tc_mma_bf16(tmem_d, ad + off + (uint64_t)(A_ATOM >> 4), bd + off, idesc, 1u);   // the remainder plane of the weights
        }
        tc_commit(done + kb % NS);
    };
    // the activations of block kb: m rows of 64 values, copied asynchronously into activation stage kb % NB
    auto issue_acts = [&](int kb) {
        const uint32_t bst = bbase + (kb % NB) * b_atom;
        for (int i = tid; i < m * 8; i += NT) {
            const int j = i >> 3, c = i & 7;
            const size_t src = (size_t)src_rows[j] * a.K + (size_t)kb * BK + c * 8;
            cp_async16(bst + swz(j, c), a.X + src);
            if (a.X2) cp_async16(bst + swz(tn + j, c), a.X2 + src);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (expert) {
        if (control && lane == 0)
            for (int u = 0; u < RD && u < nunits; u++) issue_raw(u);
    } else if (!control) {
        load_block(0);
    }

    if (control) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; kb++) {
                const int st = kb % NS, use = kb / NS;
                if (*abort_flag || !finch_mbar_wait(a_full + st, use & 1)) {
                    *abort_flag = 1;
                    break;
                }
                issue_mma(kb);
                // every dequantising warp read the unit's ring slot before it arrived on a_full for its second block: refill it
                if (expert && (kb & 1) && (kb >> 1) + RD < nunits) {
                    const int u = kb >> 1;
                    if (finch_mbar_wait(raw_empty + u % RD, (u / RD) & 1)) issue_raw(u + RD);
                    else *abort_flag = 1;
                }
            }
        }
    } else {
        issue_acts(0);
        for (int kb = 0; kb < nkb; kb++) {
            const int st = kb % NS, u = kb >> 1, slot = u % RD;
            const uint32_t ast = base + st * a_stage;
            // Block kb - 2 used this weight stage and the activation stage block kb + 1 goes into: the tensor core must be
            // done with it.  The packed unit must have landed.  (The decision to give up is taken per warp, so that no
            // lane leaves its warp behind.)
            bool ok = !*abort_flag;
            if (ok && kb >= NS) ok = finch_mbar_wait(done + st, ((kb - NS) / NS) & 1);
            if (ok && expert && !(kb & 1)) ok = finch_mbar_wait(raw_full + slot, (u / RD) & 1);
            if (!__all_sync(0xffffffffu, ok)) {
                *abort_flag = 1;
                failed = true;
                break;
            }
            if (kb + 1 < nkb) issue_acts(kb + 1);   // lands while this block is dequantised
            // ---- weights: 32 values of row r, group kb ----
            uint32_t cur[4];
            if (expert) {
                const uint32_t rs = raw + slot * RAW_STAGE, wo = rs + raw_w + (uint32_t)((kb & 1) * 48), so = rs + raw_s + (uint32_t)((kb & 1) * 2);
                asm volatile("ld.shared.u32 %0, [%1];" : "=r"(cur[0]) : "r"(wo));
                asm volatile("ld.shared.u32 %0, [%1+4];" : "=r"(cur[1]) : "r"(wo));
                asm volatile("ld.shared.u32 %0, [%1+8];" : "=r"(cur[2]) : "r"(wo));
                asm volatile("ld.shared.u16 %0, [%1];" : "=r"(sreg) : "r"(so));
                asm volatile("ld.shared.u16 %0, [%1+8];" : "=r"(breg) : "r"(so));
                cur[3] = 0;
                __syncwarp();
                if ((kb & 1) && lane == 0) {   // this warp is done with the ring slot
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(finch_smem_u32(raw_empty + slot)) : "memory");
                }
            } else {
#pragma unroll
                for (int i = 0; i < 4; i++) cur[i] = wreg[i];
            }
            float s0, b0, unused;
            finch_widen16x2(sreg, a.scale_dtype, s0, unused);
            finch_widen16x2(breg, a.scale_dtype, b0, unused);
            const GroupScale gs = group_scale(s0, b0);
            if (!expert && kb + 1 < nkb) load_block(kb + 1);   // in flight while this block is dequantised
            // row r of the atom: chunk c sits at (c ^ (r & 7)) * 16 inside the row; this thread owns chunks 4 kh .. 4 kh + 3
            const uint32_t arow = ast + (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
            const uint32_t rx = (uint32_t)(r & 7);
            if (a.mode == DENSE4) {
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    uint32_t o[4], ol[4];
                    dq4_word(cur[c], gs, o, ol);
                    st_shared16(arow + (((kh * 4 + c) ^ rx) << 4), o[0], o[1], o[2], o[3]);
                    st_shared16(arow + A_ATOM + (((kh * 4 + c) ^ rx) << 4), ol[0], ol[1], ol[2], ol[3]);
                }
            } else {
                uint32_t o[16], ol[16];
                dq3_piece(cur[0], cur[1], cur[2], gs, o, ol);
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    st_shared16(arow + (((kh * 4 + c) ^ rx) << 4), o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                    st_shared16(arow + A_ATOM + (((kh * 4 + c) ^ rx) << 4), ol[4 * c], ol[4 * c + 1], ol[4 * c + 2], ol[4 * c + 3]);
                }
            }
            // the activations of this block have landed (those of the next one may still be on their way)
            if (kb + 1 < nkb) asm volatile("cp.async.wait_group 1;" ::: "memory");
            else asm volatile("cp.async.wait_group 0;" ::: "memory");
            proxy_fence();          // generic-proxy writes -> visible to the tensor core (async proxy)
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(finch_smem_u32(a_full + st)) : "memory");
        }
    }

    // ---- epilogue ----
    {
        const int last = nkb - 1;
        __syncthreads();   // thread 0 has issued the last commit (or given up) before it gets here
        bool ok = !failed && !*abort_flag;
        if (ok) ok = finch_mbar_wait(done + last % NS, (last / NS) & 1);
        if (__syncthreads_or(!ok)) failed = true;
    }
    if (!failed && !control) {
        tc_fence_after();
        // warps w and w + 4 read the same 32 lanes and take alternate 16-column chunks
        const uint32_t trow = tmem_d + ((uint32_t)((warp & 3) * 32) << 16);
        for (int c0 = (warp >> 2) * 16; c0 < tn; c0 += 32) {
            float v[16];
            tmem_ld16(trow + (uint32_t)c0, v);
            if (planes == 2) {
                float v2[16];
                tmem_ld16(trow + (uint32_t)(tn + c0), v2);
#pragma unroll
                for (int j = 0; j < 16; j++) v[j] += v2[j];
            }
            if (a.mode == EXPERT_GATEUP) {
                // lanes l and l ^ 8 hold the gate and the up row of the same index
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float other = __shfl_xor_sync(0xffffffffu, v[j], 8);
                    if (!(lane & 8) && c0 + j < m) {
                        const float gv = v[j], act = (gv / (1.0f + expf(-gv))) * other;
                        const int pair = rows_of[t0 + c0 + j];
                        const int idx = (blockIdx.x * 8 + (r >> 4)) * 8 + (r & 7);
                        const uint32_t hi = bf16x2_rn(act, 0.f) & 0xffffu;
                        a.act_out[(size_t)pair * a.inter + idx] = (uint16_t)hi;
                        if (a.act_out_lo)
                            a.act_out_lo[(size_t)pair * a.inter + idx] = (uint16_t)(bf16x2_rn(act - __uint_as_float(hi << 16), 0.f) & 0xffffu);
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (c0 + j < m) {
                        if (a.mode == EXPERT_DOWN) a.out[(size_t)rows_of[t0 + c0 + j] * a.hidden + (size_t)blockIdx.x * GM + r] = v[j];
                        else a.out[(size_t)(t0 + c0 + j) * a.rows + (size_t)blockIdx.x * GM + r] = v[j];
                    }
                }
            }
        }
    } else if (failed && tid == 0) {
        atomicExch(a.status, FINCH_E_TIMEOUT);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem_d, ncols);
}

}  // namespace dqgemm
