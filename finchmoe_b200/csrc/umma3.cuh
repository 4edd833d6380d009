// Grouped 3-bit expert GEMMs with the PACKED CODES as the tensor core's own operand (tcgen05, accumulators in
// tensor memory): nothing is dequantised.
//
// A 3-bit code isolated by one AND at bits [p, p+3) of a 16-bit half-word, p <= 7, is the fp16 subnormal
// q * 2^(p-24).  Eighteen ANDs (and three funnel shifts) turn the 96 bits of 32 codes into eighteen registers
// of two such half-words each; written to shared memory as they are, they form the A operand of
// tcgen05.mma kind::f16.  The B operand holds the tokens' activations in the same slot order, each pre-scaled
// by 2^(7-p) / norm (norm: a power of two above the row's largest magnitude), as fp16 -- and, for fp32
// activations, a second column with the remainder * 2^11, so that no mantissa bit is lost.  Every product is
// exact in fp32.  One scale group (64 codes) takes 72 of 80 k-slots = five K = 16 steps into its own
// accumulator D_g[128 rows, tokens]; the eight warps that unpack group g + 1 read D_g back (tcgen05.ld) and
// add  s_g * D_g + b_g * sum_g(x)  to their fp32 accumulators in registers, which is the arithmetic of
// dequant_matvec_3bit (finchmoe/shaders.metal:544-612) with the sums taken in another order.
//
// Per group and 128-row tile the CUDA cores issue about 35 instructions per (row, half group) to unpack and
// about 4 per (row, token) to fold the accumulator, against 6.5 per WEIGHT for a dequantising GEMM.
//
// One CTA: one 128-row tile of one expert (eight 16-row pool tiles) and up to 64 of the expert's tokens (32 when a
// token takes two columns).
// The packed bytes arrive by bulk copies in a ring of units, the activation records by cp.async.  Two
// weight stages, four activation stages, two accumulator buffers; every wait is bounded.
#pragma once
#include "dqgemm_tc.cuh"

namespace umma3 {

using namespace dqgemm;

constexpr int SLOTS = 80;              // k-slots of one group in shared memory: 72 used + 8 that stay zero
constexpr int REC = 144;               // bytes of one (row, group, plane) activation record in global memory (72 slots)
constexpr int A_ST = GM * SLOTS * 2;   // bytes of one weight stage (20,480)
constexpr int NCOL = 64;               // accumulator columns of a CTA: 64 tokens with one activation column each, 32 with two
constexpr int NBS = 4;                 // activation stages: the records of group g + 2 are requested while group g is unpacked
constexpr int TM_BUF = NCOL;             // tensor-memory columns of one accumulator buffer

struct Args {
    int down;                 // 0: gate/up tiles (8 gate + 8 up rows per pool tile), K = hidden; 1: down tiles, K = inter
    int K;
    int planes;               // 1: one fp16 column per token; 2: hi and lo columns
    int scale_dtype;
    const uint8_t *pool_base;
    size_t slot_bytes;
    const int32_t *slot_row;
    int hidden, inter;
    const int *seg, *order;
    const int2 *items;
    const int *n_items;
    int top_k;
    const uint8_t *recs;      // [rows][K / 64][planes][REC]
    const float *xsum;        // [rows][K / 64]   sum of the 64 activations of each group, divided by fac
    const float *fac;         // [rows]           2^(E - 110): undoes the pre-scaling
    float *act_out;           // gate/up: fp32 [pairs][inter] = SiLU(gate) * up
    float *out;               // down: fp32 [pairs][hidden]
    int *status;
};

__host__ __device__ inline int tokens_per_cta(int planes) { return NCOL / planes; }
__host__ __device__ inline int smem_bytes(int K, int planes) {
    return 1024 + 2 * A_ST + NBS * NCOL * SLOTS * 2 + (K / 64) * tokens_per_cta(planes) * 4 + RD * RAW_STAGE + 512;
}

// no swizzle, K-major: 16-byte chunk c of row r sits at c * lbo + (r / 8) * 128 + (r % 8) * 16
__device__ __forceinline__ uint64_t desc_plain(uint32_t addr, uint32_t lbo) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(128u >> 4) << 32) | (1ull << 46);
}
// fp16 x fp16 -> fp32, both operands K-major, M = 128, N = n
__device__ __forceinline__ uint32_t idesc_f16(int n) { return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(GM >> 4) << 24); }

// 16 consecutive fp32 columns of this thread's lane, without waiting for them: several loads go out before one tmem_ld_wait
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
                   "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
// The loaded values are operands of the wait, so that nothing that uses them can be scheduled ahead of it.
__device__ __forceinline__ void tmem_ld_wait(float (&a)[16], float (&b)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+f"(a[0]), "+f"(a[1]), "+f"(a[2]), "+f"(a[3]), "+f"(a[4]), "+f"(a[5]), "+f"(a[6]), "+f"(a[7]), "+f"(a[8]), "+f"(a[9]), "+f"(a[10]),
                   "+f"(a[11]), "+f"(a[12]), "+f"(a[13]), "+f"(a[14]), "+f"(a[15]), "+f"(b[0]), "+f"(b[1]), "+f"(b[2]), "+f"(b[3]), "+f"(b[4]), "+f"(b[5]),
                   "+f"(b[6]), "+f"(b[7]), "+f"(b[8]), "+f"(b[9]), "+f"(b[10]), "+f"(b[11]), "+f"(b[12]), "+f"(b[13]), "+f"(b[14]), "+f"(b[15])
                 :
                 : "memory");
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

// Slot k (0..35) of a 32-code period: code IDX[k] at bit POS[k] of its half-word (-1: the slot is empty).
// Slots 2i and 2i + 1 are the low and the high half of masked register i below.
#define UMMA3_IDX {0, 6, 1, 7, 2, -1, 3, 8, 4, 9, 5, 10, 11, 16, 12, 17, 13, 18, 14, 19, 15, 20, -1, 21, 22, 27, 23, 28, -1, 29, 24, 30, 25, 31, 26, -1}
#define UMMA3_POS {0, 2, 3, 5, 6, 0, 1, 0, 4, 3, 7, 6, 1, 0, 4, 3, 7, 6, 2, 1, 5, 4, 0, 7, 2, 1, 5, 4, 0, 7, 0, 2, 3, 5, 6, 0}

// ---- activation records ---------------------------------------------------
// One warp per row: lane = 32-code period (strided).  src: [rows][K] bf16 or fp32.
template <bool SRC_BF16, bool HILO>
__global__ void __launch_bounds__(256) records_kernel(const void *src, int rows, int K, uint8_t *recs, float *xsum, float *fac) {
    constexpr int IDX[36] = UMMA3_IDX;
    constexpr int POS[36] = UMMA3_POS;
    const int lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
    const int ng = K / 64, np = K / 32, planes = HILO ? 2 : 1;
    for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < rows; row += gridDim.x * wpb) {
        const uint8_t *xr = (const uint8_t *)src + (size_t)row * K * (SRC_BF16 ? 2 : 4);
        auto load32 = [&](int p, float (&x)[32]) {
            if (SRC_BF16) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint4 r = __ldg(reinterpret_cast<const uint4 *>(xr + (size_t)(p * 32 + 8 * i) * 2));
                    const uint32_t u[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        x[8 * i + 2 * j] = __uint_as_float(u[j] << 16);
                        x[8 * i + 2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float4 r = __ldg(reinterpret_cast<const float4 *>(xr + (size_t)(p * 32 + 4 * i) * 4));
                    x[4 * i] = r.x; x[4 * i + 1] = r.y; x[4 * i + 2] = r.z; x[4 * i + 3] = r.w;
                }
            }
        };
        float amax = 0.f;
        for (int p = lane; p < np; p += 32) {
            float x[32];
            load32(p, x);
#pragma unroll
            for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        int E = (int)(__float_as_uint(amax) >> 23) + 1;
        E = E < 30 ? 30 : (E > 230 ? 230 : E);
        if (lane == 0) fac[row] = __uint_as_float((uint32_t)(E + 17) << 23);
        const float inv_fac = __uint_as_float((uint32_t)(237 - E) << 23);   // 2^(110 - E), exact
        float c[8];
#pragma unroll
        for (int q = 0; q < 8; q++) c[q] = __uint_as_float((uint32_t)(261 - E - q) << 23);
        for (int p0 = 0; p0 < np; p0 += 32) {   // whole warp: the shuffle below needs both periods of a group
            const int p = p0 + lane;
            const bool live = p < np;
            float x[32];
            if (live) load32(p, x);
            else {
#pragma unroll
                for (int i = 0; i < 32; i++) x[i] = 0.f;
            }
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 32; i += 8) s += ((x[i] + x[i + 1]) + (x[i + 2] + x[i + 3])) + ((x[i + 4] + x[i + 5]) + (x[i + 6] + x[i + 7]));
            const float so = __shfl_xor_sync(0xffffffffu, s, 1);
            if (live && !(p & 1)) xsum[(size_t)row * ng + (p >> 1)] = (s + so) * inv_fac;
            if (!live) continue;
            uint32_t hi[18], lo[18];
#pragma unroll
            for (int i = 0; i < 18; i++) {
                float v[2];
#pragma unroll
                for (int h = 0; h < 2; h++) v[h] = IDX[2 * i + h] < 0 ? 0.f : x[IDX[2 * i + h] < 0 ? 0 : IDX[2 * i + h]] * c[POS[2 * i + h]];
                const __half2 hh = __floats2half2_rn(v[0], v[1]);
                hi[i] = *reinterpret_cast<const uint32_t *>(&hh);
                if (HILO) {
                    const float2 hf = __half22float2(hh);
                    lo[i] = finch_pack_h2((v[0] - hf.x) * 2048.0f, (v[1] - hf.y) * 2048.0f);
                }
            }
            uint8_t *o = recs + ((size_t)row * ng + (p >> 1)) * planes * REC;
            const int kh = p & 1;
#pragma unroll
            for (int i = 0; i < 4; i++) *reinterpret_cast<uint4 *>(o + kh * 64 + i * 16) = make_uint4(hi[4 * i], hi[4 * i + 1], hi[4 * i + 2], hi[4 * i + 3]);
            *reinterpret_cast<uint2 *>(o + 128 + kh * 8) = make_uint2(hi[16], hi[17]);
            if (HILO) {
#pragma unroll
                for (int i = 0; i < 4; i++)
                    *reinterpret_cast<uint4 *>(o + REC + kh * 64 + i * 16) = make_uint4(lo[4 * i], lo[4 * i + 1], lo[4 * i + 2], lo[4 * i + 3]);
                *reinterpret_cast<uint2 *>(o + REC + 128 + kh * 8) = make_uint2(lo[16], lo[17]);
            }
        }
    }
}

// ---- the GEMM ---------------------------------------------------------------
// grid: x = 128-row tile of the expert's gate/up (inter / 64 tiles) or down (hidden / 128 tiles) rows, y = (expert, token tile) item.
// block: 288 threads = eight unpacking warps (thread = row r of the tile and half kh of the group; warps w and
// w + 4 share the tensor-memory lanes of rows 32 (w % 4) ..) + one control warp whose lane 0 issues the MMAs and the bulk copies.
__global__ void __launch_bounds__(NTB, 2) gemm_kernel(const Args a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if ((int)blockIdx.y >= *a.n_items) return;
    const int2 it = a.items[blockIdx.y];
    const int expert_id = it.x, t0 = it.y, first = a.seg[expert_id], m_total = a.seg[expert_id + 1] - first;
    if (t0 >= m_total) return;
    const int *rows_of = a.order + first;
    const int planes = a.planes, TN = tokens_per_cta(planes);
    const int m = min(TN, m_total - t0), tn = (m + 15) & ~15, ncol = planes * tn;
    const int ng = a.K / 64, nunits = a.K / 128;

    const uint32_t base = (finch_smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t b_stage = (uint32_t)(NCOL * SLOTS * 2);
    const uint32_t bbase = base + 2 * A_ST, xs32 = bbase + NBS * b_stage, raw = xs32 + (uint32_t)(ng * TN * 4), ctl = raw + RD * RAW_STAGE;
    uint8_t *base_p = smem_raw + (base - finch_smem_u32(smem_raw));
    uint8_t *ctl_p = base_p + (ctl - base), *raw_p = base_p + (raw - base);
    const float *xs_p = reinterpret_cast<const float *>(base_p + (xs32 - base));
    uint64_t *done = reinterpret_cast<uint64_t *>(ctl_p);   // [2] MMAs of the group in this weight stage / accumulator buffer finished
    uint64_t *a_full = done + 2;                             // [2] all warps wrote their share of the stage
    uint64_t *tm_empty = a_full + 2;                         // [2] all warps read the accumulator buffer
    uint64_t *raw_full = tm_empty + 2;                       // [RD]
    uint64_t *raw_empty = raw_full + RD;                     // [RD]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(ctl_p + 128);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(ctl_p + 132);
    int *src_rows = reinterpret_cast<int *>(ctl_p + 256);   // [64]
    constexpr int NW = NT / 32;
    const bool control = warp == NW;

    // zero the weight stages (their last chunk stays zero) and the activation stages (rows >= m, last chunk)
    for (int i = tid; i < (int)(2 * A_ST + NBS * b_stage) / 16 && !control; i += NT) st_shared16(base + i * 16, 0u, 0u, 0u, 0u);
    if (tid < m) {
        const int pair = rows_of[t0 + tid];
        src_rows[tid] = a.down ? pair : pair / a.top_k;
    }
    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < 2; s++) {
            finch_mbar_init(done + s, 1);
            finch_mbar_init(a_full + s, NW);
            finch_mbar_init(tm_empty + s, NW);
        }
        for (int s = 0; s < RD; s++) {
            finch_mbar_init(raw_full + s, 1);
            finch_mbar_init(raw_empty + s, NW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    constexpr uint32_t NCOLS = 2 * TM_BUF;
    if (warp == 0) {
        tmem_alloc(finch_smem_u32(tmem_slot), NCOLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;

    const int r = tid & (GM - 1), kh = (tid >> 7) & 1;
    const FinchTile T = finch_tile(a.hidden, a.inter);
    const uint8_t *blk = a.pool_base + (size_t)a.slot_row[expert_id] * a.slot_bytes;
    const uint8_t *tile0 = a.down ? blk + T.b_base + (size_t)blockIdx.x * 8 * T.tileB : blk + (size_t)blockIdx.x * 8 * T.tileA;
    const int tile_stride = a.down ? T.tileB : T.tileA, sb_off = a.down ? T.sbB : T.sbA;
    const int fr = r & 15, g8 = fr & 7, half = fr >> 3;
    const uint32_t raw_w = (uint32_t)((r >> 4) * 768 + (g8 * 4 + kh) * 24 + half * 12);
    const uint32_t raw_s = (uint32_t)(8 * 768 + (r >> 4) * 128 + g8 * 16 + half * 4);
    const uint32_t a_row = (uint32_t)((r >> 3) * 128 + (r & 7) * 16);
    const uint32_t idesc = idesc_f16(ncol);
    const uint32_t lbo_b = (uint32_t)ncol * 16u;

    // one packed unit of the CTA's eight pool tiles: sixteen bulk copies, one per lane of the control warp (a single
    // thread issuing all of them holds up the MMAs it has to issue next)
    auto issue_raw = [&](int u) {
        const int slot = u % RD;
        uint8_t *dst = raw_p + slot * RAW_STAGE;
        if (lane == 0) finch_mbar_expect_tx(raw_full + slot, (unsigned)RAW_STAGE);
        __syncwarp();
        if (lane < 16) {
            const int d = lane & 7;
            const uint8_t *t = tile0 + (size_t)d * tile_stride;
            if (lane < 8) finch_bulk_g2s(dst + d * 768, t + (size_t)u * 768, 768, raw_full + slot);
            else finch_bulk_g2s(dst + 8 * 768 + d * 128, t + sb_off + (size_t)u * 128, 128, raw_full + slot);
        }
    };
    auto issue_mma = [&](int g) {
        const uint32_t ast = base + (g & 1) * A_ST, bst = bbase + (g % NBS) * b_stage, td = tmem_d + (uint32_t)((g & 1) * TM_BUF);
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < SLOTS / 16; k++)
            tc_mma_bf16(td, desc_plain(ast + k * 2 * (GM * 16), GM * 16), desc_plain(bst + k * 2 * lbo_b, lbo_b), idesc, k > 0 ? 1u : 0u);
        tc_commit(done + (g & 1));
    };
    // records of group g of the CTA's tokens: nine 16-byte chunks per (token, plane), at most three chunks per thread;
    // where they come from and where they go is worked out once (only the group moves)
    uint32_t act_dst[3];
    const uint8_t *act_src[3];
#pragma unroll
    for (int n = 0; n < 3; n++) {
        const int i = tid + n * NT;
        act_src[n] = nullptr;
        act_dst[n] = 0;
        if (!control && i < m * planes * 9) {
            const int c = i % 9, jp = i / 9, pl = jp % planes, j = jp / planes, row = pl * tn + j;
            act_dst[n] = c * lbo_b + (uint32_t)((row >> 3) * 128 + (row & 7) * 16);
            act_src[n] = a.recs + ((size_t)src_rows[j] * ng * planes + pl) * REC + c * 16;
        }
    }
    const size_t act_step = (size_t)planes * REC;
    auto issue_acts = [&](int g) {
        const uint32_t bst = bbase + (g % NBS) * b_stage;
#pragma unroll
        for (int n = 0; n < 3; n++)
            if (act_src[n]) cp_async16(bst + act_dst[n], act_src[n] + (size_t)g * act_step);
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    bool failed = false;
    // acc = sum_g s_g * D_g + b_g * (sum_g(x) / fac); the row's output is acc * fac.  A thread folds the 16-column
    // chunks ch and ch + 2 of its row (warps w and w + 4 share the rows 32 (w % 4) ..).
    float acc[2][16];
#pragma unroll
    for (int q = 0; q < 2; q++)
#pragma unroll
        for (int j = 0; j < 16; j++) acc[q][j] = 0.f;
    const int ch = warp >> 2;
    const uint32_t trow = tmem_d + ((uint32_t)((warp & 3) * 32) << 16);
    auto fold = [&](int g, float s, float b) -> bool {
        bool ok = !*abort_flag && finch_mbar_wait(done + (g & 1), (g >> 1) & 1);
        if (!__all_sync(0xffffffffu, ok)) return false;
        tc_fence_after();
        // the loads of the iteration go out together: with two columns per token the hi and the lo chunk (the thread's
        // second chunk lies beyond 32 tokens then), with one column the thread's two chunks
        const uint32_t tb = trow + (uint32_t)((g & 1) * TM_BUF);
        const int c0 = ch * 16, c1 = planes == 2 ? tn + c0 : c0 + 32;
        const bool use0 = c0 < tn, use1 = use0 && (planes == 2 || c1 < tn);
        float v0[16], v1[16];
#pragma unroll
        for (int j = 0; j < 16; j++) v0[j] = v1[j] = 0.f;
        if (use0) tmem_ld16_issue(tb + (uint32_t)c0, v0);
        if (use1) tmem_ld16_issue(tb + (uint32_t)c1, v1);
        if (use0) tmem_ld_wait(v0, v1);
        auto add = [&](float (&ac)[16], const float (&v)[16], int col0) {
            const float4 *xq = reinterpret_cast<const float4 *>(xs_p + g * TN + col0);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float4 x4 = xq[k];
                ac[4 * k] = fmaf(b, x4.x, fmaf(s, v[4 * k], ac[4 * k]));
                ac[4 * k + 1] = fmaf(b, x4.y, fmaf(s, v[4 * k + 1], ac[4 * k + 1]));
                ac[4 * k + 2] = fmaf(b, x4.z, fmaf(s, v[4 * k + 2], ac[4 * k + 2]));
                ac[4 * k + 3] = fmaf(b, x4.w, fmaf(s, v[4 * k + 3], ac[4 * k + 3]));
            }
        };
        if (use0) {
            if (planes == 2) {
#pragma unroll
                for (int j = 0; j < 16; j++) v0[j] = fmaf(v1[j], 1.0f / 2048.0f, v0[j]);
            }
            add(acc[0], v0, c0);
        }
        if (use1 && planes == 1) add(acc[1], v1, c1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(finch_smem_u32(tm_empty + (g & 1))) : "memory");
        return true;
    };

    if (control) {
        for (int u = 0; u < RD && u < nunits; u++) issue_raw(u);
        for (int g = 0; g < ng; g++) {
            bool ok = !*abort_flag && finch_mbar_wait(a_full + (g & 1), (g >> 1) & 1);
            if (ok && g >= 2) ok = finch_mbar_wait(tm_empty + (g & 1), ((g - 2) >> 1) & 1);
            if (ok && (g & 1) && (g >> 1) + RD < nunits) ok = finch_mbar_wait(raw_empty + (g >> 1) % RD, ((g >> 1) / RD) & 1);   // complete before a_full
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0) *abort_flag = 1;
                break;
            }
            if (lane == 0) issue_mma(g);
            __syncwarp();
            if ((g & 1) && (g >> 1) + RD < nunits) issue_raw((g >> 1) + RD);
        }
    } else {
        // the group sums of the CTA's tokens, all groups at once
        for (int i = tid; i < ng * m; i += NT) {
            const int g = i / m, j = i - g * m;
            cp_async4(xs32 + (uint32_t)((g * TN + j) * 4), a.xsum + (size_t)src_rows[j] * ng + g);
        }
        issue_acts(0);
        if (ng > 1) issue_acts(1);
        float s_prev = 0.f, b_prev = 0.f;
        for (int g = 0; g < ng; g++) {
            const int st = g & 1, u = g >> 1, slot = u % RD;
            bool ok = !*abort_flag;
            if (ok && !(g & 1)) ok = finch_mbar_wait(raw_full + slot, (u / RD) & 1);
            if (!__all_sync(0xffffffffu, ok)) {
                *abort_flag = 1;
                failed = true;
                break;
            }
            // stage (g + 2) % 4 held group g - 2, whose MMAs this thread saw finished when it folded that group
            if (g + 2 < ng) issue_acts(g + 2);
            // ---- the 32 codes of row r, half kh of group g ----
            const uint32_t rs = raw + slot * RAW_STAGE, wo = rs + raw_w + (uint32_t)((g & 1) * 48), so = rs + raw_s + (uint32_t)((g & 1) * 2);
            uint32_t w0, w1, w2, sreg, breg;
            asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w0) : "r"(wo));
            asm volatile("ld.shared.u32 %0, [%1+4];" : "=r"(w1) : "r"(wo));
            asm volatile("ld.shared.u32 %0, [%1+8];" : "=r"(w2) : "r"(wo));
            asm volatile("ld.shared.u16 %0, [%1];" : "=r"(sreg) : "r"(so));
            asm volatile("ld.shared.u16 %0, [%1+8];" : "=r"(breg) : "r"(so));
            __syncwarp();
            if ((g & 1) && lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(finch_smem_u32(raw_empty + slot)) : "memory");
            const uint32_t v1 = __funnelshift_r(w0, w1, 8), v3 = __funnelshift_r(w1, w2, 8), v5 = w2 >> 8;
            const uint32_t ast = base + st * A_ST + a_row + (uint32_t)(kh * 4) * (GM * 16);
            st_shared16(ast, w0 & 0x001C0007u, w0 & 0x00E00038u, w0 & 0x000001C0u, v1 & 0x0007000Eu);
            st_shared16(ast + GM * 16, v1 & 0x00380070u, v1 & 0x01C00380u, w1 & 0x0007000Eu, w1 & 0x00380070u);
            st_shared16(ast + 2 * GM * 16, w1 & 0x01C00380u, v3 & 0x000E001Cu, v3 & 0x007000E0u, v3 & 0x03800000u);
            st_shared16(ast + 3 * GM * 16, w2 & 0x000E001Cu, w2 & 0x007000E0u, w2 & 0x03800000u, v5 & 0x001C0007u);
            asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(base + st * A_ST + a_row + 8u * (GM * 16) + (uint32_t)(kh * 8)), "r"(v5 & 0x00E00038u),
                         "r"(v5 & 0x000001C0u)
                         : "memory");
            float s_cur, b_cur, unused;
            finch_widen16x2(sreg, a.scale_dtype, s_cur, unused);
            finch_widen16x2(breg, a.scale_dtype, b_cur, unused);
            if (g + 2 < ng) asm volatile("cp.async.wait_group 2;" ::: "memory");
            else if (g + 1 < ng) asm volatile("cp.async.wait_group 1;" ::: "memory");
            else asm volatile("cp.async.wait_group 0;" ::: "memory");
            proxy_fence();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(finch_smem_u32(a_full + st)) : "memory");
            // ---- the accumulator of the group before, while the tensor core works on this one ----
            if (g >= 1 && !fold(g - 1, s_prev, b_prev)) {
                *abort_flag = 1;
                failed = true;
                break;
            }
            s_prev = s_cur;
            b_prev = b_cur;
        }
        if (!failed && !fold(ng - 1, s_prev, b_prev)) {
            *abort_flag = 1;
            failed = true;
        }
    }
    if (__syncthreads_or(failed || *abort_flag)) failed = true;

    if (!failed && !control) {
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const int c0 = (ch + 2 * q) * 16;
            if (c0 >= tn) continue;   // the same for every lane of the warp
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int col = c0 + j;
                const float val = acc[q][j] * (col < m ? a.fac[src_rows[col]] : 0.f);
                if (!a.down) {
                    // lanes l and l ^ 8 hold the gate and the up row of the same index
                    const float other = __shfl_xor_sync(0xffffffffu, val, 8);
                    if (!(lane & 8) && col < m) {
                        const int pair = rows_of[t0 + col];
                        const int idx = (blockIdx.x * 8 + (r >> 4)) * 8 + (r & 7);
                        a.act_out[(size_t)pair * a.inter + idx] = (val / (1.0f + expf(-val))) * other;
                    }
                } else if (col < m) {
                    a.out[(size_t)rows_of[t0 + col] * a.hidden + (size_t)blockIdx.x * GM + r] = val;
                }
            }
        }
    } else if (failed && tid == 0) {
        atomicExch(a.status, FINCH_E_TIMEOUT);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem_d, NCOLS);
}

}  // namespace umma3
