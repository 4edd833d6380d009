// MoE decode path: routed 3-bit experts (gate, up, SiLU, down), the 4-bit
// shared expert and the router-weighted combine, in three launches per layer
// chained with programmatic dependent launch.
//
//   gate/up   (moe_gateup_kernel) gate, up and SiLU.  One persistent CTA per SM.  Every CTA
//             prepares for itself (no preparation launch): two warps group the (token, k)
//             pairs of the call by expert while the others turn the tokens' activations
//             (brought in by bulk copies, a few tens of KB from L2) into tensor-core operand
//             records in shared memory.  The work is cut into tiles (8 gate rows + the 8
//             matching up rows of one expert); a team of four warps takes a contiguous,
//             cost-balanced range of tiles, each warp one quarter of K: it fetches its own
//             piece (3.5 KB of the tiled pool) with bulk async copies into two private
//             stages, so there is no producer warp, no ring shared between warps and no
//             empty-barrier traffic.  The team adds its four partial sums in fixed order
//             behind a named barrier, applies SiLU(gate) * up and writes act[pair][inter].
//   down      (moe_down_kernel) same structure with tiles of 16 down rows = one piece, one
//             warp per tile.  A CTA takes a contiguous, cost-balanced range of the
//             group-major job list, so it needs the activations of one or two expert groups
//             only; it turns those into operand records after its dependency wait (its first
//             weight pieces are already on their way by then).  Writes one fp32 row per pair.
//   combine   (moe_combine_kernel) sums the rows of a token in k order with the
//             residual and the gated shared expert (the arithmetic of
//             moe_combine_residual, finchmoe/shaders.metal:2196-2231).
//
// The shared expert's tiles go to CTAs of their own at the end of each grid (their number
// follows the expected share of the work), which keep the 4-bit-layout records instead.
//
// "Expert group" = the (token, k) pairs of this call that selected the same
// expert: its weights are read from HBM once for all of them.
//
// How a matvec is evaluated.  The packed codes never become floats on the
// CUDA cores.  A 3-bit code sitting at bits [p, p+3) of a 16-bit half-word,
// p <= 7, is -- after a single AND -- the fp16 *subnormal* q * 2^(p-24); that
// register goes straight into the A operand of mma.sync.m16n8k16 (f16 inputs,
// fp32 accumulate).  The B operand holds the activations, pre-scaled per
// k-slot by 2^(7-p) / norm (norm = power of two > max|x|).  An fp32 activation is
// split into an fp16 "hi" and a "lo * 2^11" column so that none of its mantissa bits
// is lost; a bf16 activation (8 significant bits) is its own "hi" and needs no second
// column: it is exact unless it lies below 2^-17 of the row's largest magnitude, where
// it is rounded to a multiple of 2^-24 * norm (a change of less than 2^-25 * norm in
// one term, below the rounding noise of the fp32 accumulation).  Every product is exact
// in fp32; the per-group scale and bias are applied to the fp32 group sums:
// out = sum_g s_g * (sum_i q_i x_i) + b_g * (sum_i x_i).  A 96-bit period (32 codes)
// needs 18 ANDs + 3 shifts.  Lane t of a quad owns period t of a 48-byte unit
// (128 codes = two groups); the two groups of a unit are kept apart by giving them
// different B columns, so the eight columns of an MMA are four "virtual columns"
// (token, or token x {hi, lo}) times two groups: one pass over a tile serves four
// bf16 tokens or two fp32 tokens.
#include <algorithm>

#include "finch_internal.cuh"
#include "tile_layout.h"

namespace {

constexpr int TEAM = 4;                     // warps that split the K dimension of one gate/up tile
constexpr int MAXP = FINCH_MAX_PAIRS;
constexpr int MAXM = 8;                     // pairs per expert group (<= tokens per call)
constexpr int NW_MAX = 24;                  // consumer warps per CTA
constexpr int MAX_CALLS = 16;               // batches of one multi-batch launch (one per expert-parallel rank)
constexpr int REC_CAP = 24;                 // act records a CTA of the down kernel can hold
constexpr int UB = 288;                     // bytes of one 128-value unit in one section of a 3-bit operand record
constexpr int GB4 = 128;                    // bytes of one 64-value group in one section of a 4-bit operand record
constexpr int MMA_A3 = 9, MMA_A4 = 4;       // MMAs per 3-bit unit / per 4-bit group (cost model of the work split)

struct GroupTab {  // expert groups of one call
    int ng;
    int slot[MAXP];             // pool slot of the group's expert
    unsigned char m[MAXP];      // pairs in the group
    unsigned char pairs[MAXP][MAXM];
    int pre[MAXP + 2];          // pre[gi] = passes of the groups before gi; pre[ng] = total
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
    float *act;          // [P][inter]
    float *partial;      // [P + B][hidden]
    int *status;
    int has_shared;
    const uint8_t *sh_tiles;  // prepared (tiled) copy of the shared expert
    int sh_inter, sh_fp16;    // shared expert: intermediate size, scales / biases are fp16 (else bf16)
    float *shared_act;   // [B][sh_inter]
    const float *gate_score;
    const float *h_mid;
    float *hidden_out;
    int gs_a, gs_b;      // CTAs at the end of the gate/up / down grid that take the shared expert's tiles
    int fault;           // finch_debug_fault: 1 = one warp of the gate/up kernel withholds its first fetch
    // Several independent batches of B tokens in one launch sequence (n_calls > 1): batch c owns rows
    // [c * B, (c + 1) * B) of h_post / ids / weights / valid and the CTAs [cta0[c], cta0[c + 1]) of the two big
    // grids.  Only batch own_call has h_mid, the shared expert and hidden_out; the others write their routed
    // sums to rows_out[c * B + t].
    int n_calls, own_call;
    int cta0[MAX_CALLS + 1];
    float *rows_out;
    // host-pointer path: when host_done is set, the last CTA of the combine kernel copies the status word to
    // host_status and then writes the word at done_seq_src (device memory, staged with the call's inputs, so that the
    // launch sequence can be replayed from a graph) to host_done (both mapped pinned memory): the host waits on that word
    unsigned *done_ticket, *host_done;
    int *host_status;
    const unsigned *done_seq_src;
    // expert-parallel layer: the other batches' rows go to their ranks' receive areas (ret.epoch != NULL), see finch_ret_info
    finch_ret_info ret;
};

// The view of batch c of a multi-batch launch: pointers moved to its rows, the shared expert and the residual
// only for the caller's own batch.  vb / vg: the CTA's index and the CTA count inside the batch.
__device__ __forceinline__ void select_call(MoeArgs &a, int c) {
    const size_t P = (size_t)a.P, B = (size_t)a.B;
    a.h_post = reinterpret_cast<const char *>(a.h_post) + c * B * a.hidden * (a.act_dtype == FINCH_BF16 ? 2 : 4);
    a.ids += c * P;
    a.weights += c * P;
    if (a.valid) a.valid += c * P;
    a.act += c * P * a.inter;
    a.partial += c * (P + B) * a.hidden;
    if (c != a.own_call) {
        a.has_shared = 0;
        a.gs_a = a.gs_b = 0;
        a.h_mid = nullptr;
        a.hidden_out = a.rows_out + c * B * a.hidden;
    }
}
// a0: the kernel parameter (its table is indexed at run time, which a copy in registers could not be)
__device__ __forceinline__ void pick_call(const MoeArgs &a0, MoeArgs &a, int &vb, int &vg) {
    vb = blockIdx.x;
    vg = gridDim.x;
    if (a0.n_calls > 1) {
        int c = 0;
        while (c + 1 < a0.n_calls && (int)blockIdx.x >= a0.cta0[c + 1]) ++c;
        vb = blockIdx.x - a0.cta0[c];
        vg = a0.cta0[c + 1] - a0.cta0[c];
        select_call(a, c);
    }
}

// ---- operand records -------------------------------------------------------
// record = one or two sections of B fragments (hi; hi + lo) followed by a header of floats:
// hdr[0..groups) = sum of x over each group of 64, hdr[groups] = E (int bits).
// 3-bit section: per unit UB bytes = MMA pairs (0,1) (2,3) (4,5) (6,7) as [pair][t][16 B], then MMA 8 as [t][8 B].
// 4-bit section: per group GB4 bytes = MMA pairs (0,1) (2,3) as [pair][t][16 B].
__host__ __device__ inline int up128(int x) { return (x + 127) & ~127; }
__host__ __device__ inline int sec3_bytes(int K) { return (K / 128) * UB; }
__host__ __device__ inline int sec4_bytes(int K) { return (K / 64) * GB4; }
__host__ __device__ inline int hdr_bytes(int K) { return ((K / 64 + 1 + 15) / 16) * 64; }
__host__ __device__ inline int rec3_bytes(int K, int hilo) { return up128(sec3_bytes(K) * (1 + hilo) + hdr_bytes(K)); }
__host__ __device__ inline int rec4_bytes(int K, int hilo) { return up128(sec4_bytes(K) * (1 + hilo) + hdr_bytes(K)); }

// Extraction k (0..17, compile-time) of a 96-bit period given as its words w0 w1 w2 and the views shifted by a byte.
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
// its predecessor drains; nothing written by the predecessor may be read before the wait returns.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the chain be scheduled as soon as SMs free up instead of when this grid has
// drained: its CTAs run their prologue (and whatever does not depend on this grid's output) and then
// block in griddepcontrol.wait until this grid has completed and its writes are visible.
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float pow2_biased(int e) { return __uint_as_float((uint32_t)e << 23); }

__device__ __forceinline__ bool mbar_wait_lim(uint64_t *bar, unsigned parity, unsigned tries) {
    const uint32_t a = finch_smem_u32(bar);
    for (unsigned it = 0; it < tries; ++it) {
        unsigned done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity), "r"(20000u)
            : "memory");
        if (done) return true;
    }
    return false;
}

// A warp that gives up records the timeout and, before it returns, lets the one fetch it may still have in
// flight land (a CTA's shared memory must not be released under a copy).
__device__ __forceinline__ void give_up(int *status, uint64_t *pending, unsigned parity) {
    if ((threadIdx.x & 31) == 0) atomicExch(status, FINCH_E_TIMEOUT);
    if (pending) mbar_wait_lim(pending, parity, 1u << 13);
}

// Orders this thread's earlier generic-proxy accesses to shared memory before later async-proxy (bulk copy) ones.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Pulls the 128-byte lines of [p, p + bytes) into L2 (no data is consumed: allowed ahead of the dependency wait).
__device__ __forceinline__ void prefetch_l2(const void *p, int bytes, int first, int stride) {
    for (int o = first * 128; o < bytes; o += stride * 128) asm volatile("prefetch.global.L2 [%0];" ::"l"((const char *)p + o));
}
// Release / acquire on shared-memory words (CTA scope): a team's hand-over of its partial sums.
__device__ __forceinline__ int atom_add_acq_rel(int *p, int v) {
    int old;
    asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(finch_smem_u32(p)), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void st_release(int *p, int v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(finch_smem_u32(p)), "r"(v) : "memory");
}
// Bounded wait for a shared-memory word to reach a value (a teammate publishes it).
__device__ __forceinline__ bool wait_ge(const int *p, int want, unsigned limit) {
    const uint32_t a = finch_smem_u32(p);
    for (unsigned i = 0; i < limit; ++i) {
        int v;
        asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
        if (v >= want) return true;
        __nanosleep(32);
    }
    return false;
}

// Named barrier `id` (1..15; 0 is __syncthreads) over `threads` threads.
__device__ __forceinline__ void named_sync(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }
constexpr int BAR_GROUPS = 7, BAR_RECORDS = 8;   // ids 1..6 belong to the teams of the gate/up kernel

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

// B fragments of `units` 128-value units of one row, 3-bit layout.  xs: the unit's values (fp32, shared memory);
// sec: first byte of the hi section at unit 0; lo_off: distance of the lo section (HILO only).  Thread `first`
// of `stride` (stride >= 32) cooperating threads.  A thread keeps one (j, t) position of the 9 x 4 entries
// of a unit and walks the units, so the slots are decoded once per thread, not once per entry.
// Values base .. base + N - 1 of a staged row (bf16 or fp32 in shared memory, 16-byte aligned) as floats.
template <bool SRC_BF16, int N>
__device__ __forceinline__ void row_vals(const uint8_t *row, int base, float (&x)[N]) {
    if (SRC_BF16) {
#pragma unroll
        for (int i = 0; i < N / 8; i++) {
            const uint4 r = *reinterpret_cast<const uint4 *>(row + (size_t)(base + 8 * i) * 2);
            const uint32_t u[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                x[8 * i + 2 * j] = __uint_as_float(u[j] << 16);
                x[8 * i + 2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < N / 4; i++) {
            const float4 r = *reinterpret_cast<const float4 *>(row + (size_t)(base + 4 * i) * 4);
            x[4 * i] = r.x; x[4 * i + 1] = r.y; x[4 * i + 2] = r.z; x[4 * i + 3] = r.w;
        }
    }
}

// Eight pre-scaled values = the entries of two consecutive MMAs of one lane -> 16 bytes of the hi section (and of the lo one).
template <bool HILO>
__device__ __forceinline__ void store_pair(const float (&v)[8], uint8_t *o, int lo_off) {
    if (HILO) {
        const float a[4] = {v[0], v[1], v[2], v[3]}, b[4] = {v[4], v[5], v[6], v[7]};
        uint2 h0, l0, h1, l1;
        split4(a, h0, l0);
        split4(b, h1, l1);
        *reinterpret_cast<uint4 *>(o) = make_uint4(h0.x, h0.y, h1.x, h1.y);
        *reinterpret_cast<uint4 *>(o + lo_off) = make_uint4(l0.x, l0.y, l1.x, l1.y);
    } else {
        *reinterpret_cast<uint4 *>(o) = make_uint4(finch_pack_h2(v[0], v[1]), finch_pack_h2(v[2], v[3]), finch_pack_h2(v[4], v[5]), finch_pack_h2(v[6], v[7]));
    }
}

// B entries of period t of unit u of one row, 3-bit layout: the period's 32 values against the slot table
// (code number and bit position of every k-slot of the nine MMAs; -1 = empty slot), which follows from the
// masks of extract3_one.  sec: the hi section of the row's record; lo_off: distance of the lo section.
template <bool HILO, bool SRC_BF16>
__device__ __forceinline__ void build_frag3_item(const uint8_t *row, int u, int t, int E, uint8_t *sec, int lo_off) {
    constexpr int IDX[36] = {0, 6, 1, 7, 2, -1, 3, 8, 4, 9, 5, 10, 11, 16, 12, 17, 13, 18, 14, 19, 15, 20, -1, 21, 22, 27, 23, 28, -1, 29, 24, 30, 25, 31, 26, -1};
    constexpr int POS[36] = {0, 2, 3, 5, 6, 0, 1, 0, 4, 3, 7, 6, 1, 0, 4, 3, 7, 6, 2, 1, 5, 4, 0, 7, 2, 1, 5, 4, 0, 7, 0, 2, 3, 5, 6, 0};
    float x[32], c[8];
    row_vals<SRC_BF16, 32>(row, u * 128 + t * 32, x);
#pragma unroll
    for (int p = 0; p < 8; p++) c[p] = pow2_biased(261 - E - p);
    uint8_t *o = sec + u * UB + t * 16;
#pragma unroll
    for (int jp = 0; jp < 4; jp++) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = IDX[jp * 8 + k] < 0 ? 0.f : x[IDX[jp * 8 + k] < 0 ? 0 : IDX[jp * 8 + k]] * c[POS[jp * 8 + k]];
        store_pair<HILO>(v, o + jp * 64, lo_off);
    }
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = IDX[32 + k] < 0 ? 0.f : x[IDX[32 + k] < 0 ? 0 : IDX[32 + k]] * c[POS[32 + k]];
    uint8_t *o8 = sec + u * UB + 256 + t * 8;
    if (HILO) {
        uint2 hi, lo;
        split4(v, hi, lo);
        *reinterpret_cast<uint2 *>(o8) = hi;
        *reinterpret_cast<uint2 *>(o8 + lo_off) = lo;
    } else {
        *reinterpret_cast<uint2 *>(o8) = make_uint2(finch_pack_h2(v[0], v[1]), finch_pack_h2(v[2], v[3]));
    }
}

// B entries of quad lane t of group gamma of one row, 4-bit layout: words 2t, 2t + 1 of the group (16 values).
// MMA j takes codes (0,4,1,5) of word 2t (j = 0), (2,6,3,7) (j = 1), then the same of word 2t + 1; codes in the low
// half of a byte sit at p = 0, in the high half at p = 4.
template <bool HILO, bool SRC_BF16>
__device__ __forceinline__ void build_frag4_item(const uint8_t *row, int gamma, int t, int E, uint8_t *sec, int lo_off) {
    float x[16];
    row_vals<SRC_BF16, 16>(row, gamma * 64 + t * 16, x);
    const float c0 = pow2_biased(261 - E), c4 = pow2_biased(257 - E);
    uint8_t *o = sec + gamma * GB4 + t * 16;
#pragma unroll
    for (int jp = 0; jp < 2; jp++) {
        const int b = jp * 8;
        const float v[8] = {x[b] * c0, x[b + 4] * c0, x[b + 1] * c4, x[b + 5] * c4, x[b + 2] * c0, x[b + 6] * c0, x[b + 3] * c4, x[b + 7] * c4};
        store_pair<HILO>(v, o + jp * 64, lo_off);
    }
}

// Phase stamps for working out where a launch spends its time: compiled in with -DFINCH_STAMPS only.
#ifdef FINCH_STAMPS
__device__ long long g_stamps[2 * 160 * 32 * 16];
__device__ __forceinline__ long long gtime() {
    long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
#define STAMP(i) do { if ((threadIdx.x & 31) == 0) g_stamps[((size_t)blockIdx.x * 32 + (threadIdx.x >> 5)) * 16 + (i)] = gtime(); } while (0)
#define STAMP_ADD(i, v) do { if ((threadIdx.x & 31) == 0) g_stamps[((size_t)blockIdx.x * 32 + (threadIdx.x >> 5)) * 16 + (i)] += (v); } while (0)
#define STAMPB(i) do { if ((threadIdx.x & 31) == 0) g_stamps[(160 * 32 + (size_t)blockIdx.x * 32 + (threadIdx.x >> 5)) * 16 + (i)] = gtime(); } while (0)
#define STAMP_CLK() clock64()
#else
#define STAMPB(i) do {} while (0)
#define STAMP(i) do {} while (0)
#define STAMP_ADD(i, v) do {} while (0)
#define STAMP_CLK() 0ll
#endif

// Operand records are built from rows staged in shared memory in two steps, by the nthr threads tid0 .. tid0 + nthr - 1
// of the CTA (whole warps).  BITS selects the layout.  rows: nb staged rows of K values (bf16 or fp32), records
// r0 .. r0 + nb - 1.  umax: one float per (staged row, 256-value slab).
// Step 1: the group sums of every row into its header, the largest magnitude of every slab into umax.
template <int BITS, bool HILO, bool SRC_BF16>
__device__ void records_sums(int nb, int r0, int K, uint8_t *recs, int rec_stride, const uint8_t *xs, float *umax, int tid0, int nthr) {
    const int tid = threadIdx.x - tid0, lane = tid & 31, warp = tid >> 5, nwarp = nthr >> 5;
    const int rowb = K * (SRC_BF16 ? 2 : 4), nsl = (K + 255) / 256;
    const int hdr_off = (BITS == 3 ? sec3_bytes(K) : sec4_bytes(K)) * (HILO ? 2 : 1);
    for (int it = warp; it < nb * nsl; it += nwarp) {
        const int bl = it / nsl, sl = it - bl * nsl, base = sl * 256 + lane * 8;
        float v[8];
        const bool live = base < K;
        if (live) row_vals<SRC_BF16, 8>(xs + (size_t)bl * rowb, base, v);
        else {
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = 0.f;
        }
        float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7])), amax = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(v[j]));
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (live && (lane & 7) == 0) reinterpret_cast<float *>(recs + (size_t)(r0 + bl) * rec_stride + hdr_off)[base >> 6] = s;
        if (lane == 0) umax[it] = amax;
    }
}
// Step 2 (after a barrier): the B fragments; one (row, unit, period) or (row, group, quad lane) item per thread and turn.
template <int BITS, bool HILO, bool SRC_BF16>
__device__ void records_frags(int nb, int r0, int K, uint8_t *recs, int rec_stride, const uint8_t *xs, const float *umax, int tid0, int nthr) {
    const int tid = threadIdx.x - tid0;
    const int rowb = K * (SRC_BF16 ? 2 : 4), nsl = (K + 255) / 256;
    const int secb = BITS == 3 ? sec3_bytes(K) : sec4_bytes(K), hdr_off = secb * (HILO ? 2 : 1);
    const int per_row = BITS == 3 ? (K / 128) * 4 : (K / 64) * 4;
    for (int it = tid; it < nb * per_row; it += nthr) {
        const int bl = it / per_row, q = it - bl * per_row;
        float m = 0.f;
        for (int j = 0; j < nsl; j++) m = fmaxf(m, umax[bl * nsl + j]);
        int E = (int)(__float_as_uint(m) >> 23) + 1;
        E = E < 30 ? 30 : (E > 230 ? 230 : E);
        uint8_t *rec = recs + (size_t)(r0 + bl) * rec_stride;
        if (q == 0) reinterpret_cast<float *>(rec + hdr_off)[K / 64] = __int_as_float(E);
        if (BITS == 3) build_frag3_item<HILO, SRC_BF16>(xs + (size_t)bl * rowb, q >> 2, q & 3, E, rec, secb);
        else build_frag4_item<HILO, SRC_BF16>(xs + (size_t)bl * rowb, q >> 2, q & 3, E, rec, secb);
    }
}
// Brings rows r0 .. r0 + nb - 1 into the staging area: one bulk copy each, issued by the calling thread and
// signalled on xbar (an mbarrier of count 1 that nothing else uses).  row_ptr(r): global address of row r (16-byte aligned).
template <class RowPtr>
__device__ __forceinline__ void records_fetch_rows(int nb, int r0, int rowb, uint8_t *xs, uint64_t *xbar, RowPtr row_ptr) {
    fence_async_smem();
    finch_mbar_expect_tx(xbar, (unsigned)(nb * rowb));
    for (int i = 0; i < nb; i++) finch_bulk_g2s(xs + (size_t)i * rowb, row_ptr(r0 + i), (unsigned)rowb, xbar);
}

// Turns `nrec` rows of K values into operand records in shared memory, xs_rows rows at a time.  Run by the nthr threads
// tid0 .. tid0 + nthr - 1, which share named barrier `bar`; the first of them brings the rows in.  xs_rows * nsl must
// not exceed the floats of umax.
template <int BITS, bool HILO, bool SRC_BF16, class RowPtr>
__device__ void build_records(int nrec, int K, uint8_t *recs, int rec_stride, uint8_t *xs, int xs_rows, float *umax, uint64_t *xbar, int tid0,
                              int nthr, int bar, unsigned tries, int *status, RowPtr row_ptr) {
    const int tid = threadIdx.x - tid0;
    const int rowb = K * (SRC_BF16 ? 2 : 4);
    int round = 0;
    for (int r0 = 0; r0 < nrec; r0 += xs_rows, ++round) {
        const int nb = min(xs_rows, nrec - r0);
        if (tid == 0) records_fetch_rows(nb, r0, rowb, xs, xbar, row_ptr);
        if (!mbar_wait_lim(xbar, round & 1, tries) && (tid & 31) == 0) atomicExch(status, FINCH_E_TIMEOUT);
        records_sums<BITS, HILO, SRC_BF16>(nb, r0, K, recs, rec_stride, xs, umax, tid0, nthr);
        named_sync(bar, nthr);
        records_frags<BITS, HILO, SRC_BF16>(nb, r0, K, recs, rec_stride, xs, umax, tid0, nthr);
        named_sync(bar, nthr);
    }
}

// ---- inner loops ---------------------------------------------------------
// D = A(16x16, f16, row) * B(16x8, f16, col) + C.  Not volatile: a pure function of its operands.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// First MMA of a chain: C = 0 comes from the zero register, no accumulator initialisation needed.
__device__ __forceinline__ void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Shared-memory loads by 32-bit address.  Volatile: they must stay behind the barrier wait that makes the stage
// readable; constant offsets added by the caller are folded into the instruction's immediate.
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts64f(uint32_t addr, float x, float y) {
    asm volatile("st.shared.v2.f32 [%0], {%1,%2};" ::"r"(addr), "f"(x), "f"(y) : "memory");
}
// global -> shared bulk copy to a 32-bit shared address; src, dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void finch_bulk_g2s_a(uint32_t dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src), "r"(bytes),
                 "r"(finch_smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ float lds32f(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

template <bool FP16S>
__device__ __forceinline__ void widen2(uint32_t w, float &lo, float &hi) {
    if (FP16S) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w));
        lo = f.x;
        hi = f.y;
    } else {
        lo = __uint_as_float(w << 16);
        hi = __uint_as_float(w & 0xffff0000u);
    }
}

// One 128-code unit of a 3-bit piece against the four virtual columns of a pass.
//   pw   this lane's 24 bytes of the unit's weights (3 words of fragment row g, 3 of row g + 8)
//   ps   the 16-byte scale / bias entry of rows g, g + 8
//   pb   this lane's B entries: the unit's section of the record of virtual column g >> 1 (or of the zero
//        record when the lane's k-slots belong to the other group or the column is unused), + t * 16
//   pb8  the same + 256 + t * 8 (the ninth MMA's entry)
//   ph   the two group sums of the unit in the header of the token whose result this lane's accumulator
//        columns (virtual column t) hold
// run / bias accumulate sum_g s_g * (sum q x') and sum_g b_g * (sum x) for rows g (A) and g + 8 (B).
template <bool FP16S>
__device__ __forceinline__ void gemv3_unit(uint32_t pw, uint32_t ps, uint32_t pb, uint32_t pb8, uint32_t ph, float &runA, float &runB,
                                           float &biasA, float &biasB) {
    const uint4 b01 = lds128(pb), b23 = lds128(pb + 64), b45 = lds128(pb + 128), b67 = lds128(pb + 192);
    const uint2 b8 = lds64(pb8);
    const uint2 q0 = lds64(pw), q1 = lds64(pw + 8), q2 = lds64(pw + 16);
    const uint4 s = lds128(ps);
    const uint2 xgb = lds64(ph);
    // row A words q0.x q0.y q1.x, row B words q1.y q2.x q2.y; the shifted views of the extraction
    const uint32_t av1 = __funnelshift_r(q0.x, q0.y, 8), av3 = __funnelshift_r(q0.y, q1.x, 8), av5 = q1.x >> 8;
    const uint32_t bv1 = __funnelshift_r(q1.y, q2.x, 8), bv3 = __funnelshift_r(q2.x, q2.y, 8), bv5 = q2.y >> 8;
    float acc[4];
#define FINCH_MMA3(j, B0, B1)                                                                                             \
    {                                                                                                                     \
        const uint32_t a0 = extract3_one<2 * (j)>(q0.x, av1, q0.y, av3, q1.x, av5);                                       \
        const uint32_t a1 = extract3_one<2 * (j)>(q1.y, bv1, q2.x, bv3, q2.y, bv5);                                       \
        const uint32_t a2 = extract3_one<2 * (j) + 1>(q0.x, av1, q0.y, av3, q1.x, av5);                                   \
        const uint32_t a3 = extract3_one<2 * (j) + 1>(q1.y, bv1, q2.x, bv3, q2.y, bv5);                                   \
        if ((j) == 0) mma16816_z(acc, a0, a1, a2, a3, B0, B1);                                                            \
        else mma16816(acc, a0, a1, a2, a3, B0, B1);                                                                       \
    }
    FINCH_MMA3(0, b01.x, b01.y) FINCH_MMA3(1, b01.z, b01.w) FINCH_MMA3(2, b23.x, b23.y) FINCH_MMA3(3, b23.z, b23.w)
    FINCH_MMA3(4, b45.x, b45.y) FINCH_MMA3(5, b45.z, b45.w) FINCH_MMA3(6, b67.x, b67.y) FINCH_MMA3(7, b67.z, b67.w)
    FINCH_MMA3(8, b8.x, b8.y)
#undef FINCH_MMA3
    const float x0 = __uint_as_float(xgb.x), x1 = __uint_as_float(xgb.y);
    float s0, s1;
    widen2<FP16S>(s.x, s0, s1);
    runA = fmaf(s0, acc[0], runA);
    runA = fmaf(s1, acc[1], runA);
    widen2<FP16S>(s.y, s0, s1);
    runB = fmaf(s0, acc[2], runB);
    runB = fmaf(s1, acc[3], runB);
    widen2<FP16S>(s.z, s0, s1);
    biasA = fmaf(s0, x0, biasA);
    biasA = fmaf(s1, x1, biasA);
    widen2<FP16S>(s.w, s0, s1);
    biasB = fmaf(s0, x0, biasB);
    biasB = fmaf(s1, x1, biasB);
}

// nu consecutive units of a piece: weights [nu][32][24 B], scale / bias entries [nu][8][16 B].  pw, ps: this lane's
// words of the first unit (+ lane * 24, + g * 16); pb: the section of its B column at the first unit.
template <bool FP16S>
__device__ __forceinline__ void gemv3_piece(uint32_t pw, uint32_t ps, int nu, uint32_t pb, uint32_t ph, float &runA, float &runB, float &biasA,
                                            float &biasB) {
    const int t = threadIdx.x & 3;
    const uint32_t pb16 = pb + t * 16, pb8 = pb + 256 + t * 8;
    runA = runB = biasA = biasB = 0.f;
#ifndef FINCH_ROLLED_UNITS
    if (nu == 4) {
#pragma unroll
        for (int u = 0; u < 4; u++) gemv3_unit<FP16S>(pw + u * 768, ps + u * 128, pb16 + u * UB, pb8 + u * UB, ph + u * 8, runA, runB, biasA, biasB);
        return;
    }
#endif
#pragma unroll 1
    for (int u = 0; u < nu; u++) gemv3_unit<FP16S>(pw + u * 768, ps + u * 128, pb16 + u * UB, pb8 + u * UB, ph + u * 8, runA, runB, biasA, biasB);
}

// ngr 64-code groups of a 4-bit piece against the eight columns of a pass.
//   pw / wstep   this lane's 16-byte chunk of the first group, bytes per group
//   ps / sstep   the 8-byte scale / bias entry (scale row A, scale row B, bias row A, bias row B as u16)
//   pb / bstep   this lane's B entries (record section of column g, + t * 16), bytes per group (0 for the zero block)
//   ph0, ph1     the group sums in the headers of the tokens of accumulator columns 2t and 2t + 1
// r[0..3] / bias[0..3]: (row A, col 2t) (row A, col 2t+1) (row B, col 2t) (row B, col 2t+1).
template <bool FP16S>
__device__ __forceinline__ void gemv4_piece(uint32_t pw, int wstep, uint32_t ps, int sstep, int ngr, uint32_t pb, int bstep, uint32_t ph0,
                                            uint32_t ph1, float (&r)[4], float (&bias)[4]) {
#pragma unroll
    for (int i = 0; i < 4; i++) r[i] = bias[i] = 0.f;
    for (int gm = 0; gm < ngr; gm++) {
        const uint4 b01 = lds128(pb), b23 = lds128(pb + 64);
        const uint4 w = lds128(pw);
        const uint2 s = lds64(ps);
        const float x0 = lds32f(ph0), x1 = lds32f(ph1);
        pb += bstep;
        pw += wstep;
        ps += sstep;
        ph0 += 4;
        ph1 += 4;
        uint32_t ea[8], eb[8];
        {
            uint32_t x[4];
            extract4(w.x, x); ea[0] = x[0]; ea[1] = x[1]; ea[2] = x[2]; ea[3] = x[3];
            extract4(w.y, x); ea[4] = x[0]; ea[5] = x[1]; ea[6] = x[2]; ea[7] = x[3];
            extract4(w.z, x); eb[0] = x[0]; eb[1] = x[1]; eb[2] = x[2]; eb[3] = x[3];
            extract4(w.w, x); eb[4] = x[0]; eb[5] = x[1]; eb[6] = x[2]; eb[7] = x[3];
        }
        float acc[4];
        mma16816_z(acc, ea[0], eb[0], ea[1], eb[1], b01.x, b01.y);
        mma16816(acc, ea[2], eb[2], ea[3], eb[3], b01.z, b01.w);
        mma16816(acc, ea[4], eb[4], ea[5], eb[5], b23.x, b23.y);
        mma16816(acc, ea[6], eb[6], ea[7], eb[7], b23.z, b23.w);
        float s0, s1, b0, b1;
        widen2<FP16S>(s.x, s0, s1);  // scale of row A, of row B
        widen2<FP16S>(s.y, b0, b1);  // bias of row A, of row B
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

// ---- expert groups -------------------------------------------------------
__device__ __forceinline__ bool pair_ok(const MoeArgs &a, int p) {
    if (a.valid && !a.valid[p]) return false;
    const int e = a.ids[p];
    if (e < 0 || e >= a.n_experts) return false;
    return a.slot_row[e] >= 0;
}

// Jobs of the down kernel are laid out group-major: job = gi * per_group + tile.  Every routed CTA takes one
// contiguous range, balanced by cost (a job of a group costs its pass count).  The job whose cost interval
// starts at or after `target`.
__device__ int job_at(const int *pre, int ng, int per_group, int target) {
    if (target >= pre[ng] * per_group) return ng * per_group;
    int lo = 0, hi = ng - 1;   // last group whose first job starts at or before target
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] * per_group <= target) lo = mid;
        else hi = mid - 1;
    }
    const int gi = lo, np = pre[gi + 1] - pre[gi];
    return gi * per_group + (target - pre[gi] * per_group + np - 1) / np;
}

// Builds the group table in shared memory.  Run by the first two warps of the CTA (one pair per lane), which
// share named barrier BAR_GROUPS.  Groups are numbered by their first pair; pairs inside a group ascend.
// per_pass: pairs a pass serves (2 or 4); T->pre gets the prefix sums of the groups' pass counts.
// col (optional, [MAXP][MAXM]): shared address of the operand record of the token of every (group, pair of
// the group), rec32 + token * rstride, or 0 where the group has no such pair.
// sm_ids: MAXP + 2 ints, sm_rank: MAXP bytes of scratch.
// bound (optional, nbound + 1 ints): boundaries of nbound cost-balanced contiguous ranges of the group-major tile list
// (per_group tiles per group) for the teams first_team .. first_team + nbound - 1 of n_teams.
template <bool ONE = false>   // ONE: the call has a single token (compiled into kernels of their own, the others carry none of it)
__device__ void build_groups(const MoeArgs &a, GroupTab *T, int *sm_ids, unsigned char *sm_rank, int per_pass, uint32_t *col, uint32_t rec32,
                             int rstride, int *bound = nullptr, int nbound = 0, int first_team = 0, int n_teams = 1, int per_group = 1) {
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
    if (ONE) {
        // One token: every usable pair is its own group (a token's experts are distinct; should two coincide, the expert
        // is simply read twice).  No matching across the two warps, one barrier.
        if (col)
            for (int i = tid; i < MAXP * MAXM; i += 64) col[i] = 0u;
        const unsigned fb1 = __ballot_sync(0xffffffffu, id >= 0);   // P <= 8: all pairs sit in warp 0
        const int ng1 = __popc(fb1);
        if (warp == 0) {
            if (id >= 0) {
                const int gi = __popc(fb1 & ((1u << lane) - 1u));
                T->pairs[gi][0] = (unsigned char)tid;
                T->m[gi] = 1;
                T->slot[gi] = slot;
            }
            T->pre[lane] = lane < ng1 ? lane : ng1;      // one pass per group
            T->pre[lane + 32] = ng1;
            if (lane == 0) {
                T->ng = ng1;
                T->pre[64] = ng1;
            }
        }
        named_sync(BAR_GROUPS, 64);
        if (col && warp == 0 && id >= 0) col[__popc(fb1 & ((1u << lane) - 1u)) * MAXM] = rec32;   // after the zeroing above
        if (bound && tid <= nbound) {
            const int ng = T->ng;
            const unsigned total = (unsigned)(T->pre[ng] * per_group);
            bound[tid] = job_at(T->pre, ng, per_group, (int)(total * (unsigned)(first_team + tid) / (unsigned)n_teams));
        }
        return;
    }
    sm_ids[tid] = id;
    if (col)
        for (int i = tid; i < MAXP * MAXM; i += 64) col[i] = 0u;
    named_sync(BAR_GROUPS, 64);
    unsigned same = 0, other = 0, fb = 0;
    bool first = false;
    same = __match_any_sync(0xffffffffu, id);                 // lanes of my warp with my expert
    const int *o = sm_ids + 32 * (warp ^ 1);
    for (int j = 0; j < 32; j++) other |= (unsigned)(o[j] == id) << j;   // lanes of the other warp
    const unsigned lt = (1u << lane) - 1u;
    first = id >= 0 && !(same & lt) && (warp == 0 || other == 0);
    fb = __ballot_sync(0xffffffffu, first);
    if (lane == 0) sm_ids[MAXP + warp] = (int)fb;
    named_sync(BAR_GROUPS, 64);
    const int before = warp == 1 ? __popc((unsigned)sm_ids[MAXP]) : 0;
    if (first) sm_rank[tid] = (unsigned char)(before + __popc(fb & lt));
    const int ng = __popc((unsigned)sm_ids[MAXP]) + __popc((unsigned)sm_ids[MAXP + 1]);
    if (tid == 0) T->ng = ng;
    named_sync(BAR_GROUPS, 64);
    int np = 0;   // passes of group `tid`
    if (id >= 0) {
        const int fp = (warp == 1 && other) ? __ffs(other) - 1 : 32 * warp + __ffs(same) - 1;   // first pair of my group
        const int gi = sm_rank[fp];
        const int pos = (warp == 1 ? __popc(other) : 0) + __popc(same & lt);
        if (pos < MAXM) {
            T->pairs[gi][pos] = (unsigned char)tid;
            if (col) col[gi * MAXM + pos] = rec32 + (uint32_t)((tid / a.K) * rstride);
        }
        if (first) {
            const int m = __popc(same) + __popc(other);
            T->m[gi] = (unsigned char)(m < MAXM ? m : MAXM);
            T->slot[gi] = slot;
        }
    }
    named_sync(BAR_GROUPS, 64);
    // exclusive scan of the per-group pass counts over the two warps
    np = tid < ng ? (T->m[tid] + per_pass - 1) / per_pass : 0;
    int inc = np;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += v;
    }
    if (tid == 31) sm_ids[0] = inc;   // total of the first warp
    named_sync(BAR_GROUPS, 64);
    const int add = warp == 1 ? sm_ids[0] : 0;
    T->pre[tid] = inc - np + add;
    if (tid == 63) T->pre[64] = inc + add;
    named_sync(BAR_GROUPS, 64);
    if (bound && tid <= nbound) {
        // total <= 64 groups * 4 passes * tiles per group and the team count is a few thousand: the products fit 32 bits
        const unsigned total = (unsigned)(T->pre[ng] * per_group);
        bound[tid] = job_at(T->pre, ng, per_group, (int)(total * (unsigned)(first_team + tid) / (unsigned)n_teams));
    }
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

// ============================ gate / up ===================================
// Shared memory of a gate/up CTA.  stage: [2][warps][stg]; while the records are built the second half
// (every warp's stage 1) is the staging area of the rows.
struct SmemA {
    int stage, stg, rec, rstride, zero, red, umax, tab, col, ids, rank, sync, bar, total;
};
__host__ __device__ inline SmemA smem_a_layout(int hidden, int inter, int sh_inter, int B, int has_shared, int hilo, int nwarps) {
    const FinchTile T = finch_tile(hidden, inter);
    const int upq = (T.unitsA + TEAM - 1) / TEAM, gq = (hidden / 64 + TEAM - 1) / TEAM;
    (void)sh_inter;
    SmemA L;
    L.stage = 0;
    L.stg = up128(upq * 896 > (has_shared ? gq * 288 : 0) ? upq * 896 : gq * 288);
    L.rec = L.stage + 2 * nwarps * L.stg;
    const int r3 = rec3_bytes(hidden, hilo), r4 = has_shared ? rec4_bytes(hidden, hilo) : 0;
    L.rstride = r3 > r4 ? r3 : r4;
    // the zero record sits 64 bytes off the records' 128-byte grid: a lane reading zeros and a lane reading the
    // same offset of a record then never share a bank
    L.zero = L.rec + B * L.rstride + 64;
    L.red = L.zero + sec3_bytes(hidden) + 64;
    L.umax = L.red + (nwarps / TEAM) * TEAM * MAXM * 64;      // per team: [4 K-quarters][8 tokens][8 g][gate | up] floats
    L.tab = L.umax + 8 * ((hidden + 255) / 256) * 4;
    L.col = L.tab + (((int)sizeof(GroupTab) + 15) & ~15);     // [group][pair of the group]: shared address of the token's record, or 0
    L.ids = L.col + MAXP * MAXM * 4;
    L.rank = L.ids + (MAXP + 2) * 4;
    L.sync = (L.rank + MAXP + 7) & ~7;                        // per team: partial sums written, reductions done
    L.bar = L.sync + 4 * (NW_MAX / TEAM) * 4;                 // + the boundaries of the teams' tile ranges
    L.total = L.bar + (2 * NW_MAX + 1) * 8;
    return L;
}

// What a warp of the gate/up kernel works on: its K-quarter of every tile of its team's range.
struct WarpJobA {
    int u0, nu, nkw;   // first unit / units of the quarter (groups for the shared expert), quarters that exist
    int j0, j1, step;  // tiles j0, j0 + step, ... < j1
};
// bound: the routed teams' range boundaries left by build_groups.
__device__ __forceinline__ WarpJobA warp_job_a(bool routed, int units, int n_tiles_shared, int cta, int Gr, int gs, int nteam, int w, const int *bound) {
    WarpJobA J;
    const int team = w / TEAM, kw = w % TEAM, upq = (units + TEAM - 1) / TEAM;
    J.u0 = kw * upq;
    J.nu = min(upq, units - J.u0);
    J.nkw = (units + upq - 1) / upq;
    if (routed) {
        J.j0 = bound[team];
        J.j1 = bound[team + 1];
        J.step = 1;
    } else {
        J.j0 = (cta - Gr) * nteam + team;
        J.j1 = n_tiles_shared;
        J.step = gs * nteam;
    }
    return J;
}

// grid: one CTA per SM (persistent); block: nteam teams of TEAM warps.
template <bool HILO, bool FP16S, bool ONE = false>
__global__ void __launch_bounds__(NW_MAX * 32, 1) moe_gateup_kernel(const MoeArgs a0) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int nwarps = blockDim.x >> 5, nteam = nwarps / TEAM;
    const SmemA L = smem_a_layout(a0.hidden, a0.inter, a0.sh_inter, a0.B, a0.has_shared, HILO, nwarps);
    MoeArgs a = a0;
    int vb, vg;
    pick_call(a0, a, vb, vg);
    const FinchTile T = finch_tile(a.hidden, a.inter);
    const FinchTile4 T4 = finch_tile4(a.hidden, a.sh_inter);
    GroupTab *tab = reinterpret_cast<GroupTab *>(smem + L.tab);
    int *sm_ids = reinterpret_cast<int *>(smem + L.ids);
    unsigned char *sm_rank = smem + L.rank;
    uint32_t *col = reinterpret_cast<uint32_t *>(smem + L.col);
    int *arrived = reinterpret_cast<int *>(smem + L.sync), *reduced = arrived + NW_MAX / TEAM, *trange = reduced + NW_MAX / TEAM;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar);
    uint64_t *full = bars + 2 * warp;   // this warp's two stages
    uint64_t *xbar = bars + 2 * NW_MAX;
    const int K = a.hidden;
    const unsigned tries = a.fault ? 4u : (1u << 13);
    const unsigned spins = a.fault ? 64u : (1u << 22);
    constexpr int PER_PASS = HILO ? 2 : 4;
    const int Gr = vg - a.gs_a;
    const bool routed = vb < Gr;
    const uint32_t rec32 = finch_smem_u32(smem + L.rec), zero32 = finch_smem_u32(smem + L.zero), col32 = finch_smem_u32(col);
    const uint32_t stage32 = finch_smem_u32(smem + L.stage), stdelta = (uint32_t)(nwarps * L.stg);   // stage s of warp w at stage32 + w * stg + s * stdelta
    const int rowb = K * (HILO ? 4 : 2);

    if (lane == 0) {
        finch_mbar_init(full, 1);
        finch_mbar_init(full + 1, 1);
        if (warp == 0) finch_mbar_init(xbar, 1);
    }
    if (tid < 4 * (NW_MAX / TEAM)) arrived[tid] = 0;
    for (int i = tid; i < sec3_bytes(K) / 4; i += blockDim.x) reinterpret_cast<int *>(smem + L.zero)[i] = 0;
    // the call's inputs on their way into L2 while the previous kernel of the stream drains
    if (warp == 0) {
        prefetch_l2(a.ids, a.P * 4, lane, 32);
        prefetch_l2(a.slot_row, a.n_experts * 4, lane, 32);
        if (a.valid) prefetch_l2(a.valid, a.P, lane, 32);
    } else {
        prefetch_l2(a.h_post, a.B * rowb, tid - 32, blockDim.x - 32);
    }
    __syncthreads();
    STAMP(0);
    grid_dep_wait();  // everything above overlaps the tail of the previous kernel in the stream
    STAMP(1);
    // only now may the down kernel be scheduled: it reads this call's inputs before its own wait, and every
    // CTA of this grid gets here only after whatever produced those inputs has completed
    grid_dep_launch();
    const int units = routed ? T.unitsA : T4.groupsA, unit_w = routed ? 768 : 256, unit_s = routed ? 128 : 32;
    // Fetch of tile j of warp job J into shared address dst (lane 0).
    auto fetch = [&](const WarpJobA &J, int j, uint32_t dst, uint64_t *bar) {
        const uint8_t *src;
        int sb;
        if (routed) {
            const int gi = j / T.nTA, ta = j - gi * T.nTA;
            src = a.pool_base + (size_t)tab->slot[gi] * a.slot_bytes + (size_t)ta * T.tileA;
            sb = T.sbA;
        } else {
            src = a.sh_tiles + (size_t)j * T4.tileA;
            sb = T4.sbA;
        }
        finch_mbar_expect_tx(bar, (unsigned)(J.nu * (unit_w + unit_s)));
        finch_bulk_g2s_a(dst, src + (size_t)J.u0 * unit_w, (unsigned)(J.nu * unit_w), bar);
        finch_bulk_g2s_a(dst + J.nu * unit_w, src + sb + (size_t)J.u0 * unit_s, (unsigned)(J.nu * unit_s), bar);
    };
    // Two warps sort out the routing (and the teams' tile ranges) while the others bring the activation rows in
    // and take their group sums.  Once both are done every warp requests its first piece, and the rows are turned
    // into operand records while that piece is on its way.
    uint8_t *xs = smem + L.stage + nwarps * L.stg;
    float *umax = reinterpret_cast<float *>(smem + L.umax);
    int xs_rows = (nwarps * L.stg) / rowb;
    xs_rows = xs_rows > 8 ? 8 : xs_rows;
    auto row_ptr = [&](int b) { return (const void *)((const uint8_t *)a.h_post + (size_t)b * rowb); };
    const bool one_round = a.B <= xs_rows;   // else: the records are built round by round before anything is fetched
    if (warp < 2) {
        build_groups<ONE>(a, tab, sm_ids, sm_rank, PER_PASS, routed ? col : nullptr, rec32, L.rstride, trange, routed ? nteam : 0, vb * nteam, Gr * nteam, T.nTA);
        STAMP(2);
    } else if (one_round) {
        if (tid == 64) records_fetch_rows(a.B, 0, rowb, xs, xbar, row_ptr);
        if (!mbar_wait_lim(xbar, 0, tries) && lane == 0) atomicExch(a.status, FINCH_E_TIMEOUT);
        if (routed) records_sums<3, HILO, !HILO>(a.B, 0, K, smem + L.rec, L.rstride, xs, umax, 64, blockDim.x - 64);
        else records_sums<4, HILO, !HILO>(a.B, 0, K, smem + L.rec, L.rstride, xs, umax, 64, blockDim.x - 64);
        STAMP(12);
    } else {
        xs_rows = xs_rows > nwarps - 2 ? nwarps - 2 : xs_rows;
        if (routed) build_records<3, HILO, !HILO>(a.B, K, smem + L.rec, L.rstride, xs, xs_rows, umax, xbar, 64, blockDim.x - 64, BAR_RECORDS, tries, a.status, row_ptr);
        else build_records<4, HILO, !HILO>(a.B, K, smem + L.rec, L.rstride, xs, xs_rows, umax, xbar, 64, blockDim.x - 64, BAR_RECORDS, tries, a.status, row_ptr);
    }
    __syncthreads();
    STAMP(13);
    const WarpJobA J = warp_job_a(routed, units, T4.nTA, vb, Gr, a.gs_a, nteam, warp, trange);
    const bool withhold = a.fault == 1 && routed && J.j0 == 0 && warp % TEAM == 0;   // the warp that owns the first quarter of tile 0
    if (lane == 0 && J.nu > 0 && J.j0 < J.j1 && !withhold) fetch(J, J.j0, stage32 + (uint32_t)(warp * L.stg), full);
    if (one_round) {
        if (routed) records_frags<3, HILO, !HILO>(a.B, 0, K, smem + L.rec, L.rstride, xs, umax, 0, blockDim.x);
        else records_frags<4, HILO, !HILO>(a.B, 0, K, smem + L.rec, L.rstride, xs, umax, 0, blockDim.x);
        STAMP(3);
        __syncthreads();
    }
    STAMP(7);
#ifdef FINCH_STAMPS
    if (lane == 0)
        for (int i = 8; i < 12; i++) g_stamps[((size_t)blockIdx.x * 32 + warp) * 16 + i] = 0;
#endif
    if (J.nu <= 0) return;
    const int team = warp / TEAM, kw = warp % TEAM, nkw = J.nkw, u0 = J.u0, nu = J.nu;
    const uint32_t st32 = stage32 + (uint32_t)(warp * L.stg);
    float *slot = reinterpret_cast<float *>(smem + L.red) + team * (TEAM * MAXM * 16);   // [kw][ti][g][gate | up]
    const uint32_t slot32 = finch_smem_u32(slot);
    bool dead = false;   // a wait ran out: the warp keeps its team's protocol going and does nothing else
    // second piece (the second stages were the staging area of the rows until the barrier above)
    int fj = J.j0 + J.step;
    if (lane == 0) {
        fence_async_smem();
        if (fj < J.j1) fetch(J, fj, st32 + stdelta, full + 1);
    }
    fj += J.step;

    // One tile's partial sums are in the team's slot: the warp that arrives last adds the K-quarters in fixed
    // order and applies SiLU(gate) * up.  `store(ti, gg, v)` takes the value of (token ti of the tile, row gg).
    auto finish = [&](int n, int nti, auto store) {
        __syncwarp();   // the lanes' partial sums are ordered before lane 0's release
        int old = 0;
        if (lane == 0) old = atom_add_acq_rel(arrived + team, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != nkw * (n + 1) - 1) return;
        __syncwarp();   // ... and lane 0's acquire before the lanes' reads
        for (int item = lane; item < nti * 8; item += 32) {
            const int ti = item >> 3, gg = item & 7;
            float va = 0.f, vb = 0.f;
            for (int k = 0; k < nkw; k++) {
                const float2 v = *reinterpret_cast<const float2 *>(slot + ((k * MAXM + ti) * 8 + gg) * 2);
                va += v.x;
                vb += v.y;
            }
            store(ti, gg, __fdividef(va, 1.0f + __expf(-va)) * vb);
        }
        __syncwarp();
        if (lane == 0) st_release(reduced + team, n + 1);
    };

    if (routed) {
        // ---------------- routed experts: 3-bit tiles ----------------
        const int sec = sec3_bytes(K), hdr_off = sec * (HILO ? 2 : 1);
        const bool mine = (g & 1) == (t >> 1);   // this lane's k-slots belong to the group of its B column
        // lane constants: which pair of a pass this lane's B column / accumulator columns belong to
        const int pos_b = HILO ? (g >> 2) : (g >> 1), pos_o = HILO ? (t >> 1) : t;
        const uint32_t sec_b = HILO ? (uint32_t)(((g >> 1) & 1) * sec) : 0u;
        const uint32_t lane_w = (uint32_t)lane * 24u, lane_s = (uint32_t)(nu * 768 + g * 16), boff = (uint32_t)(u0 * UB);
        const uint32_t my_slot = slot32 + (uint32_t)(((kw * MAXM) * 8 + g) * 8);
        int gi = J.j0 / T.nTA, ta = J.j0 - gi * T.nTA;
        STAMP(14);
        for (int j = J.j0, n = 0; j < J.j1; ++j, ++n) {
            const int st = n & 1;
            const int m = tab->m[gi], npass = (m + PER_PASS - 1) / PER_PASS;
            const long long c0 = STAMP_CLK();
            if (!dead && !mbar_wait_lim(full + st, (n >> 1) & 1, tries)) {
                give_up(a.status, j + 1 < J.j1 ? full + ((n + 1) & 1) : nullptr, ((n + 1) >> 1) & 1);
                dead = true;
            }
            const long long c1 = STAMP_CLK();
            STAMP_ADD(8, c1 - c0);
            if (n == 0) STAMP(4);
            const uint32_t w32 = st32 + (uint32_t)st * stdelta;
            for (int ps = 0; ps < npass && !dead; ps++) {
                const uint32_t cb = lds32(col32 + (uint32_t)((gi * MAXM + ps * PER_PASS + pos_b) * 4));
                const uint32_t co = lds32(col32 + (uint32_t)((gi * MAXM + ps * PER_PASS + pos_o) * 4));
                const uint32_t pb = ((mine && cb) ? cb + sec_b : zero32) + boff;
                const uint32_t ph = (co ? co : rec32) + hdr_off;
                float runA, runB, biasA, biasB;
                gemv3_piece<FP16S>(w32 + lane_w, w32 + lane_s, nu, pb, ph + u0 * 8, runA, runB, biasA, biasB);
                const float fac = pow2_biased(__float_as_int(lds32f(ph + (K / 64) * 4)) + 17);
                if (HILO) {
                    const float oA = __shfl_xor_sync(0xffffffffu, runA, 1), oB = __shfl_xor_sync(0xffffffffu, runB, 1);
                    runA += oA * (1.0f / 2048.0f);
                    runB += oB * (1.0f / 2048.0f);
                }
                if (ps == 0) {
                    if (npass == 1) {   // the stage is free before the hand-over: the next fetch goes out first
                        __syncwarp();
                        if (lane == 0 && fj < J.j1) fetch(J, fj, w32, full + st);
                    }
                    const long long c2 = STAMP_CLK();
                    STAMP_ADD(9, c2 - c1);
                    // the previous tile's partial sums have been read before this tile's overwrite them
                    if (nkw > 1 && n > 0 && !wait_ge(reduced + team, n, spins)) {
                        give_up(a.status, j + 1 < J.j1 ? full + ((n + 1) & 1) : nullptr, ((n + 1) >> 1) & 1);
                        dead = true;
                        break;
                    }
                    STAMP_ADD(10, STAMP_CLK() - c2);
                }
                if (co && (!HILO || !(t & 1))) sts64f(my_slot + (uint32_t)((ps * PER_PASS + pos_o) * 64), fmaf(runA, fac, biasA), fmaf(runB, fac, biasB));
            }
            if (npass > 1 && !dead) {
                __syncwarp();   // every lane is done with the stage
                if (lane == 0 && fj < J.j1) fetch(J, fj, w32, full + st);
            }
            fj += J.step;
            if (n == 0) STAMP(5);
            finish(n, m, [&](int ti, int gg, float v) { a.act[(size_t)tab->pairs[gi][ti] * a.inter + 8 * ta + gg] = v; });
            STAMP_ADD(11, 1);
            if (++ta == T.nTA) ta = 0, ++gi;
        }
        STAMP(6);
    } else {
        // ---------------- shared expert: 4-bit tiles of 4 gate rows + the 4 matching up rows ----------------
        const int g0 = u0, ngr = nu;
        const int nps = HILO ? (a.B + 3) / 4 : (a.B + 7) / 8;   // passes of a tile (every token): four (hi + lo) or eight tokens each
        const int sec = sec4_bytes(K), hdr_off = sec * (HILO ? 2 : 1);
        const int I = a.sh_inter;
        int n = 0;
        for (int tile = J.j0; tile < J.j1; tile += J.step, ++n) {
            const int st = n & 1;
            if (!dead && !mbar_wait_lim(full + st, (n >> 1) & 1, tries)) {
                give_up(a.status, tile + J.step < J.j1 ? full + ((n + 1) & 1) : nullptr, ((n + 1) >> 1) & 1);
                dead = true;
            }
            const uint32_t w32 = st32 + (uint32_t)st * stdelta, s32 = w32 + ngr * 256;
            if (nkw > 1 && n > 0 && !dead && !wait_ge(reduced + team, n, spins)) {
                give_up(a.status, tile + J.step < J.j1 ? full + ((n + 1) & 1) : nullptr, ((n + 1) >> 1) & 1);
                dead = true;
            }
            if (!dead) {
                for (int ps = 0; ps < nps; ps++) {
                    // column g of the pass: HILO: token 4 ps + (g >> 1), term g & 1; else token 8 ps + g
                    const int tokb = HILO ? 4 * ps + (g >> 1) : 8 * ps + g;
                    const int tok0 = HILO ? 4 * ps + t : 8 * ps + 2 * t, tok1 = HILO ? tok0 : tok0 + 1;   // accumulator columns 2t, 2t + 1
                    const bool bact = tokb < a.B;
                    const uint32_t pb = (bact ? rec32 + tokb * L.rstride + (HILO ? (g & 1) * sec : 0) + g0 * GB4 : zero32) + t * 16;
                    const uint32_t ph0 = rec32 + (tok0 < a.B ? tok0 : 0) * L.rstride + hdr_off, ph1 = rec32 + (tok1 < a.B ? tok1 : 0) * L.rstride + hdr_off;
                    float r[4], bias[4];
                    if (a.sh_fp16) gemv4_piece<true>(w32 + ((g & 3) * 4 + t) * 16, 256, s32 + (g & 3) * 8, 32, ngr, pb, bact ? GB4 : 0, ph0 + g0 * 4, ph1 + g0 * 4, r, bias);
                    else gemv4_piece<false>(w32 + ((g & 3) * 4 + t) * 16, 256, s32 + (g & 3) * 8, 32, ngr, pb, bact ? GB4 : 0, ph0 + g0 * 4, ph1 + g0 * 4, r, bias);
                    const float f0 = pow2_biased(__float_as_int(lds32f(ph0 + (K / 64) * 4)) + 17);
                    const float f1 = pow2_biased(__float_as_int(lds32f(ph1 + (K / 64) * 4)) + 17);
                    if (g < 4) {   // rows g >= 4 duplicate rows g - 4
                        if (HILO) {
                            if (tok0 < a.B)
                                *reinterpret_cast<float2 *>(slot + ((kw * MAXM + tok0) * 8 + g) * 2) =
                                    make_float2(fmaf(r[0] + r[1] * (1.0f / 2048.0f), f0, bias[0]), fmaf(r[2] + r[3] * (1.0f / 2048.0f), f0, bias[2]));
                        } else {
                            if (tok0 < a.B)
                                *reinterpret_cast<float2 *>(slot + ((kw * MAXM + tok0) * 8 + g) * 2) = make_float2(fmaf(r[0], f0, bias[0]), fmaf(r[2], f0, bias[2]));
                            if (tok1 < a.B)
                                *reinterpret_cast<float2 *>(slot + ((kw * MAXM + tok1) * 8 + g) * 2) = make_float2(fmaf(r[1], f1, bias[1]), fmaf(r[3], f1, bias[3]));
                        }
                    }
                }
                __syncwarp();
                if (lane == 0 && fj < J.j1) fetch(J, fj, w32, full + st);
            }
            fj += J.step;
            finish(n, a.B, [&](int ti, int gg, float v) {
                if (gg < 4) a.shared_act[(size_t)ti * I + 4 * tile + gg] = v;
            });
            if (n == 0) STAMP(5);
            STAMP_ADD(11, 1);
        }
        STAMP(6);
    }
}

// ============================ down ========================================
// stage: [2][warps][stg] as in the gate/up kernel (the second half doubles as the staging area of the rows).
struct SmemB {
    int stage, stg, rec, rstride, zero, umax, tab, col, ids, rank, bar, total;
};
__host__ __device__ inline SmemB smem_b_layout(int hidden, int inter, int sh_inter, int B, int has_shared, int nwarps) {
    const FinchTile T = finch_tile(hidden, inter);
    const FinchTile4 T4 = finch_tile4(hidden, sh_inter);
    SmemB L;
    L.stage = 0;
    L.stg = up128(has_shared && T4.tileB > T.tileB ? T4.tileB : T.tileB);
    L.rec = L.stage + 2 * nwarps * L.stg;
    L.rstride = rec3_bytes(inter, 1);
    const int routed = REC_CAP * L.rstride, shared = has_shared ? B * rec4_bytes(sh_inter, 1) : 0;
    L.zero = L.rec + (routed > shared ? routed : shared) + 64;
    L.umax = L.zero + sec3_bytes(inter) + 64;
    L.tab = L.umax + REC_CAP * (((inter > sh_inter ? inter : sh_inter) + 255) / 256) * 4;
    L.col = L.tab + (((int)sizeof(GroupTab) + 15) & ~15);
    L.ids = L.col + MAXP * MAXM * 4;
    L.rank = L.ids + (MAXP + 2) * 4;
    L.bar = (L.rank + MAXP + 7) & ~7;
    L.total = L.bar + (2 * NW_MAX + 1) * 8;
    return L;
}

// grid: one CTA per SM (persistent); block: nwarps warps, each takes whole tiles.
template <bool FP16S>
__global__ void __launch_bounds__(NW_MAX * 32, 1) moe_down_kernel(const MoeArgs a0) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int nwarps = blockDim.x >> 5;
    const SmemB L = smem_b_layout(a0.hidden, a0.inter, a0.sh_inter, a0.B, a0.has_shared, nwarps);
    MoeArgs a = a0;
    int vb, vg;
    pick_call(a0, a, vb, vg);
    const FinchTile T = finch_tile(a.hidden, a.inter);
    const FinchTile4 T4 = finch_tile4(a.hidden, a.sh_inter);
    GroupTab *tab = reinterpret_cast<GroupTab *>(smem + L.tab);
    int *sm_ids = reinterpret_cast<int *>(smem + L.ids);
    unsigned char *sm_rank = smem + L.rank;
    uint32_t *col = reinterpret_cast<uint32_t *>(smem + L.col);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar) + 2 * warp;
    uint64_t *xbar = reinterpret_cast<uint64_t *>(smem + L.bar) + 2 * NW_MAX;
    const int K = a.inter, Ks = a.sh_inter;
    const unsigned tries = a.fault ? 4u : (1u << 13);
    const int Gr = vg - a.gs_b;
    const bool routed = vb < Gr;

    if (lane == 0) {
        finch_mbar_init(full, 1);
        finch_mbar_init(full + 1, 1);
        if (warp == 0) finch_mbar_init(xbar, 1);
    }
    for (int i = tid; i < sec3_bytes(K) / 4; i += blockDim.x) reinterpret_cast<int *>(smem + L.zero)[i] = 0;
    STAMPB(0);
    grid_dep_launch();
    // The routing is an input of the whole call, final since the gate/up kernel passed its own wait (this grid
    // is scheduled only after that): groups, ranges and the first weight pieces do not wait for the gate/up
    // kernel to finish.  Only the activations (its output) do.
    // (the two ends of this CTA's job range are worked out by two threads side by side, into sm_ids[0..1])
    if (routed && warp < 2) build_groups(a, tab, sm_ids, sm_rank, 2, nullptr, 0u, 0, sm_ids, 1, vb, Gr, T.nTB);
    __syncthreads();
    STAMPB(1);
    const uint32_t st32 = finch_smem_u32(smem + L.stage + warp * L.stg), stdelta = (uint32_t)(nwarps * L.stg);
    uint8_t *xs = smem + L.stage + nwarps * L.stg;
    float *umax = reinterpret_cast<float *>(smem + L.umax);
    const uint32_t zero32 = finch_smem_u32(smem + L.zero), rec32 = finch_smem_u32(smem + L.rec), col32 = finch_smem_u32(col);

    if (routed) {
        const int ng = tab->ng;
        const int job0 = sm_ids[0], job1 = sm_ids[1];
        auto fetch = [&](int gi, int tb, uint32_t dst, uint64_t *bar) {   // lane 0
            finch_mbar_expect_tx(bar, (unsigned)T.tileB);
            finch_bulk_g2s_a(dst, a.pool_base + (size_t)tab->slot[gi] * a.slot_bytes + T.b_base + (size_t)tb * T.tileB, (unsigned)T.tileB, bar);
        };
        const int dgi = nwarps / T.nTB, dtb = nwarps - dgi * T.nTB;
        auto advance = [&](int &G, int &A) {
            G += dgi;
            A += dtb;
            if (A >= T.nTB) A -= T.nTB, ++G;
        };
        const int first = job0 + warp;
        int gi = first / T.nTB, tb = first - gi * T.nTB, fgi = gi, ftb = tb, fjob = first;
        if (lane == 0 && fjob < job1) fetch(fgi, ftb, st32, full);
        fjob += nwarps;
        advance(fgi, ftb);
        // operand records of the activations this CTA needs: the pairs of the groups in its job range
        const int g_lo = job0 < job1 ? job0 / T.nTB : 0;
        const int g_hi = job0 < job1 ? (job1 - 1) / T.nTB : -1;   // inclusive
        int nrec = 0;
        for (int j = g_lo; j <= g_hi; j++) nrec += tab->m[j];
        for (int i = tid; i < MAXP * MAXM; i += blockDim.x) {
            const int j = i / MAXM, pos = i % MAXM;
            int r0 = 0;   // first record of group j in the CTA's record area
            for (int q = g_lo; q < j && q <= g_hi; q++) r0 += tab->m[q];
            col[i] = (j >= g_lo && j <= g_hi && pos < tab->m[j] && r0 + pos < REC_CAP) ? rec32 + (r0 + pos) * L.rstride : 0u;
        }
        STAMPB(2);
        grid_dep_wait();   // the gate/up kernel has completed: act is final
        STAMPB(3);
        if (nrec > REC_CAP) {   // cannot happen with a grid of a hundred CTAs or more; refuse instead of clipping
            if (tid == 0) atomicExch(a.status, FINCH_E_UNSUPPORTED);
            if (first < job1) mbar_wait_lim(full, 0, 1u << 13);   // the fetch under way
            return;
        }
        int xs_rows = (nwarps * L.stg) / (K * 4);
        xs_rows = xs_rows > nwarps ? nwarps : xs_rows;
        auto row_ptr = [&](int q) {   // q-th record of the CTA -> the activations of its (token, k) pair
            int j = g_lo;
            while (q >= tab->m[j]) q -= tab->m[j++];
            return (const void *)(a.act + (size_t)tab->pairs[j][q] * K);
        };
        build_records<3, true, false>(nrec, K, smem + L.rec, L.rstride, xs, xs_rows, umax, xbar, 0, blockDim.x, BAR_RECORDS, tries, a.status, row_ptr);
        STAMPB(4);
        if (lane == 0) {
            fence_async_smem();
            if (fjob < job1) fetch(fgi, ftb, st32 + stdelta, full + 1);
        }
        fjob += nwarps;
        advance(fgi, ftb);
        const int sec = sec3_bytes(K), hdr_off = 2 * sec;
        const bool mine = (g & 1) == (t >> 1);
        const int pos_b = g >> 2, pos_o = t >> 1;
        const uint32_t sec_b = (uint32_t)(((g >> 1) & 1) * sec);
        const uint32_t lane_w = (uint32_t)lane * 24u, lane_s = (uint32_t)(T.sbB + g * 16);
        int n = 0;
        for (int job = first; job < job1; job += nwarps, ++n, advance(gi, tb)) {
            const int st = n & 1;
            if (!mbar_wait_lim(full + st, (n >> 1) & 1, tries)) {
                give_up(a.status, job + nwarps < job1 ? full + ((n + 1) & 1) : nullptr, ((n + 1) >> 1) & 1);
                return;
            }
            const int m = tab->m[gi], npass = (m + 1) / 2;
            const uint32_t w32 = st32 + (uint32_t)st * stdelta;
            if (n == 0) STAMPB(5);
            for (int ps = 0; ps < npass; ps++) {
                const uint32_t cb = lds32(col32 + (uint32_t)((gi * MAXM + 2 * ps + pos_b) * 4));
                const uint32_t co = lds32(col32 + (uint32_t)((gi * MAXM + 2 * ps + pos_o) * 4));
                const uint32_t pb = (mine && cb) ? cb + sec_b : zero32;
                const uint32_t ph = (co ? co : rec32) + hdr_off;
                float runA, runB, biasA, biasB;
                gemv3_piece<FP16S>(w32 + lane_w, w32 + lane_s, T.unitsD, pb, ph, runA, runB, biasA, biasB);
                const float fac = pow2_biased(__float_as_int(lds32f(ph + (K / 64) * 4)) + 17);
                const float oA = __shfl_xor_sync(0xffffffffu, runA, 1), oB = __shfl_xor_sync(0xffffffffu, runB, 1);
                if (!(t & 1) && co) {
                    float *o = a.partial + (size_t)tab->pairs[gi][2 * ps + pos_o] * a.hidden + 16 * tb + g;
                    o[0] = fmaf(runA + oA * (1.0f / 2048.0f), fac, biasA);
                    o[8] = fmaf(runB + oB * (1.0f / 2048.0f), fac, biasB);
                }
            }
            __syncwarp();
            if (lane == 0 && fjob < job1) fetch(fgi, ftb, w32, full + st);
            fjob += nwarps;
            advance(fgi, ftb);
            if (n == 0) STAMPB(6);
        }
        STAMPB(7);
    } else {
        // ---------------- shared expert: 4-bit tiles of 16 down rows ----------------
        const int nps = (a.B + 3) / 4;   // passes of a tile: four tokens (hi + lo columns) each
        const int n_tiles = T4.nTB, stride = a.gs_b * nwarps;
        const int tile0 = (vb - Gr) * nwarps + warp;
        auto fetch = [&](int tile, uint32_t dst, uint64_t *bar) {   // lane 0
            finch_mbar_expect_tx(bar, (unsigned)T4.tileB);
            finch_bulk_g2s_a(dst, a.sh_tiles + T4.b_base + (size_t)tile * T4.tileB, (unsigned)T4.tileB, bar);
        };
        if (lane == 0 && tile0 < n_tiles) fetch(tile0, st32, full);
        grid_dep_wait();   // shared_act is final
        int xs_rows = (nwarps * L.stg) / (Ks * 4);
        xs_rows = xs_rows > 8 ? 8 : xs_rows;
        const int r4 = rec4_bytes(Ks, 1);
        auto row_ptr = [&](int b) { return (const void *)(a.shared_act + (size_t)b * Ks); };
        build_records<4, true, false>(a.B, Ks, smem + L.rec, r4, xs, xs_rows, umax, xbar, 0, blockDim.x, BAR_RECORDS, tries, a.status, row_ptr);
        if (lane == 0) {
            fence_async_smem();
            if (tile0 + stride < n_tiles) fetch(tile0 + stride, st32 + stdelta, full + 1);
        }
        const int sec = sec4_bytes(Ks), hdr_off = 2 * sec;
        int n = 0;
        for (int tile = tile0; tile < n_tiles; tile += stride, ++n) {
            const int st = n & 1;
            if (!mbar_wait_lim(full + st, (n >> 1) & 1, tries)) {
                give_up(a.status, tile + stride < n_tiles ? full + ((n + 1) & 1) : nullptr, ((n + 1) >> 1) & 1);
                return;
            }
            const uint32_t w32 = st32 + (uint32_t)st * stdelta, s32 = w32 + T4.sbB;
            for (int ps = 0; ps < nps; ps++) {
                const int tokb = 4 * ps + (g >> 1), tok = 4 * ps + t;   // column g: (token, term g & 1); accumulator columns 2t, 2t + 1: token t, hi | lo
                const bool bact = tokb < a.B;
                const uint32_t pb = (bact ? rec32 + tokb * r4 + (g & 1) * sec : zero32) + t * 16;
                const uint32_t ph = rec32 + (tok < a.B ? tok : 0) * r4 + hdr_off;
                float r[4], bias[4];
                if (a.sh_fp16) gemv4_piece<true>(w32 + lane * 16, 512, s32 + g * 8, 64, T4.groupsD, pb, bact ? GB4 : 0, ph, ph, r, bias);
                else gemv4_piece<false>(w32 + lane * 16, 512, s32 + g * 8, 64, T4.groupsD, pb, bact ? GB4 : 0, ph, ph, r, bias);
                const float fac = pow2_biased(__float_as_int(lds32f(ph + (Ks / 64) * 4)) + 17);
                if (tok < a.B) {
                    float *o = a.partial + (size_t)(a.P + tok) * a.hidden + 16 * tile + g;
                    o[0] = fmaf(r[0] + r[1] * (1.0f / 2048.0f), fac, bias[0]);
                    o[8] = fmaf(r[2] + r[3] * (1.0f / 2048.0f), fac, bias[2]);
                }
            }
            __syncwarp();
            if (lane == 0 && tile + 2 * stride < n_tiles) fetch(tile + 2 * stride, w32, full + st);
        }
    }
}

// ============================ combine =====================================
// hidden = h_mid + sum_{k ascending, usable} w_k * out_k + sigmoid(score) * shared_out, the arithmetic of
// moe_combine_residual (finchmoe/shaders.metal:2196-2231).  grid: (hidden / 256, B); block 256.
__global__ void __launch_bounds__(256) moe_combine_kernel(const MoeArgs a0) {
    __shared__ int ok[8];
    __shared__ float wk[8];
    MoeArgs a = a0;
    const int b = blockIdx.y % a0.B, c = blockIdx.y / a0.B, row = blockIdx.x * 256 + threadIdx.x;   // grid.y = B * n_calls
    if (a0.n_calls > 1) select_call(a, c);
    grid_dep_launch();
    // Routing, router weights, gate scores and h_mid are inputs of the whole call: final since the gate/up
    // kernel (the first of the chain) passed its own wait, and this kernel only starts once the down kernel has
    // started, which was after that.  Only the partial rows (the down kernel's output) have to wait; the
    // dependent loads of the routing (mask -> id -> slot) are out of the way by then.
    if (threadIdx.x < a.K) {
        ok[threadIdx.x] = pair_ok(a, b * a.K + threadIdx.x);
        wk[threadIdx.x] = a.weights[b * a.K + threadIdx.x];
    }
    const bool live = row < a.hidden;
    float h = live && a.h_mid ? a.h_mid[(size_t)b * a.hidden + row] : 0.f;
    const float sg = a.has_shared ? 1.0f / (1.0f + expf(-a.gate_score[b])) : 0.f;
    const bool away = a0.ret.epoch && c != a0.own_call;   // this batch's rows belong to another rank
    const uint32_t e = away ? *reinterpret_cast<const volatile uint32_t *>(a0.ret.epoch) : 0u;
    __syncthreads();
    grid_dep_wait();
    if (live) {
        float moe = 0.f;
        for (int k = 0; k < a.K; k++)
            if (ok[k]) moe = fmaf(wk[k], __ldcg(a.partial + (size_t)(b * a.K + k) * a.hidden + row), moe);
        h += moe;
        if (a.has_shared) h = fmaf(sg, __ldcg(a.partial + (size_t)(a.P + b) * a.hidden + row), h);
    }
    if (away) {
        // {h[row], epoch, h[row + 1], epoch} into slot [my rank][b] of rank c's area: the receiver takes a pair once it
        // carries the epoch it expects (the word pairs of ep_peer.cu)
        const float hn = __shfl_down_sync(0xffffffffu, h, 1);
        if (live && !(row & 1)) {
            uint4 *dst = reinterpret_cast<uint4 *>(a0.ret.area[c] + a0.ret.off_back) + (size_t)(a0.ret.rank * a0.ret.T + b) * (a.hidden / 2) + (row >> 1);
            asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(dst), "r"(__float_as_uint(h)), "r"(e), "r"(__float_as_uint(hn)), "r"(e)
                         : "memory");
        }
    } else if (live) {
        a.hidden_out[(size_t)b * a.hidden + row] = h;
    }
    if (a0.host_done) {   // launch-uniform
        __threadfence_system();          // this thread's output is on its way to the host before the CTA reports
        __syncthreads();
        if (threadIdx.x == 0 && atomicAdd(a0.done_ticket, 1u) == gridDim.x * gridDim.y - 1) {
            *a0.done_ticket = 0u;
            *a0.host_status = *reinterpret_cast<volatile int *>(a0.status);
            __threadfence_system();
            *reinterpret_cast<volatile unsigned *>(a0.host_done) = *reinterpret_cast<const volatile unsigned *>(a0.done_seq_src);
        }
    }
}

constexpr int SMEM_MAX = 227 * 1024;

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

// The kernels' opt-in to 227 KB of shared memory is a per-device function attribute: set once per device.
int set_attrs_once(finch_ctx *ctx) {
    static std::mutex mu;
    static std::vector<int> done;
    std::lock_guard<std::mutex> lk(mu);
    const int dev = ctx->cfg.device;
    for (int d : done)
        if (d == dev) return FINCH_OK;
    const void *big[] = {(const void *)moe_gateup_kernel<false, false>, (const void *)moe_gateup_kernel<false, true>,
                         (const void *)moe_gateup_kernel<true, false>,  (const void *)moe_gateup_kernel<true, true>,
                         (const void *)moe_gateup_kernel<false, false, true>, (const void *)moe_gateup_kernel<false, true, true>,
                         (const void *)moe_gateup_kernel<true, false, true>,  (const void *)moe_gateup_kernel<true, true, true>,
                         (const void *)moe_down_kernel<false>,          (const void *)moe_down_kernel<true>};
    for (const void *f : big) {
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
        // one shared-memory carve-out for all kernels of the chain: an SM that has to change its L1 / shared
        // split between consecutive launches drains first
        FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    }
    FINCH_CUDA_OK(ctx, cudaFuncSetAttribute(moe_combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    done.push_back(dev);
    return FINCH_OK;
}


// =============== grouped 3-bit expert passes for prefill chunks (mma.sync) ================
// The pairs of a chunk sorted by expert; an expert's tokens are served up to 16 (8 with two activation planes) at a
// time by the unit loop of the decode kernels, with ONE unpack of a unit's codes for all its passes: 21 logic
// operations per 32 codes whatever the number of tokens, against a dequantisation into shared-memory tiles that a
// tensor-memory GEMM needs.  At the few tokens per expert of a prefill chunk (about 16 at 512 tokens, top-8 of 256)
// this is the cheaper form; the tcgen05 GEMM takes over when experts see many tokens (expert-parallel ranks).
struct G3Args {
    const uint8_t *pool_base;
    size_t slot_bytes;
    const int32_t *slot_row;   // the layer's slot table [n_experts]
    int hidden, inter;
    const uint8_t *recs;       // operand records (global memory): record rec_of[position], or record `position` when rec_of is NULL
    const int *rec_of;
    int rstride;
    const int4 *items;         // (expert, first position, tokens, -)
    const int *n_items;
    const int *order;          // position -> pair index t * K + k
    float *out;                // gate/up: act [position][inter]; down: [pair][hidden]
    int *status;
};

// One CTA: positions = the usable pairs sorted by expert.  order[pos] = pair, src_tok[pos] = token.  Item lists for
// the gate/up passes (ppa tokens per pass) and the down passes (ppb): an expert with at most pp / 2 pp tokens is one
// item of list 0 / 1, a larger one chunks of 4 pp in list 2.  counts = {nA0, nA1, nA2, nB0, nB1, nB2, positions}.
__global__ void __launch_bounds__(1024) g3_sort_kernel(const int32_t *ids, const uint8_t *valid, const int32_t *slot_row, int n_experts, int P, int Kx,
                                                       int ppa, int ppb, int *order, int *src_tok, int4 *la0, int4 *la1, int4 *la2, int4 *lb0, int4 *lb1,
                                                       int4 *lb2, int *counts) {
    extern __shared__ int g3s[];
    __shared__ int wsum[7][32];
    int *cnt = g3s, *cur = g3s + n_experts;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    for (int e = tid; e < n_experts; e += 1024) cnt[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += 1024) {
        const int e = ids[p];
        if ((valid && !valid[p]) || e < 0 || e >= n_experts || slot_row[e] < 0) continue;
        atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    // Exclusive scans over the experts, 1024 at a time (carry between rounds): positions, and the number of items every
    // expert adds to each of the six lists.
    int carry[7] = {0, 0, 0, 0, 0, 0, 0};
    for (int e0 = 0; e0 < n_experts; e0 += 1024) {
        const int e = e0 + tid, c = e < n_experts ? cnt[e] : 0;
        int v[7], inc[7];
        v[0] = c;
#pragma unroll
        for (int side = 0; side < 2; side++) {
            const int pp = side ? ppb : ppa;
            v[1 + 3 * side] = c > 0 && c <= pp;
            v[2 + 3 * side] = c > pp && c <= 2 * pp;
            v[3 + 3 * side] = c > 2 * pp ? (c + 4 * pp - 1) / (4 * pp) : 0;
        }
#pragma unroll
        for (int q = 0; q < 7; q++) {
            inc[q] = v[q];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, inc[q], o);
                if (lane >= o) inc[q] += u;
            }
            if (lane == 31) wsum[q][wid] = inc[q];
        }
        __syncthreads();
        if (wid == 0) {
#pragma unroll
            for (int q = 0; q < 7; q++) {
                const int w = wsum[q][lane];
                int acc = w;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int u = __shfl_up_sync(0xffffffffu, acc, o);
                    if (lane >= o) acc += u;
                }
                wsum[q][lane] = acc - w;
            }
        }
        __syncthreads();
        int ex[7];
#pragma unroll
        for (int q = 0; q < 7; q++) ex[q] = carry[q] + wsum[q][wid] + inc[q] - v[q];
        if (e < n_experts) {
            cur[e] = ex[0];
            if (c > 0) {
#pragma unroll
                for (int side = 0; side < 2; side++) {
                    const int pp = side ? ppb : ppa;
                    int4 *l0 = side ? lb0 : la0, *l1 = side ? lb1 : la1, *l2 = side ? lb2 : la2;
                    if (c <= pp) l0[ex[1 + 3 * side]] = make_int4(e, ex[0], c, 0);
                    else if (c <= 2 * pp) l1[ex[2 + 3 * side]] = make_int4(e, ex[0], c, 0);
                    else
                        for (int o = 0, i = 0; o < c; o += 4 * pp, i++) l2[ex[3 + 3 * side] + i] = make_int4(e, ex[0] + o, c - o < 4 * pp ? c - o : 4 * pp, 0);
                }
            }
        }
        // totals of this round -> carry (every thread computes the same: last lane of last warp's inclusive value)
        __syncthreads();
        if (tid == 1023) {
#pragma unroll
            for (int q = 0; q < 7; q++) wsum[q][0] = ex[q] + v[q];
        }
        __syncthreads();
#pragma unroll
        for (int q = 0; q < 7; q++) carry[q] = wsum[q][0];
        __syncthreads();
    }
    if (tid == 0) {
        for (int q = 0; q < 6; q++) counts[q] = carry[q + 1];
        counts[6] = carry[0];
    }
    for (int p = tid; p < P; p += 1024) {
        const int e = ids[p];
        if ((valid && !valid[p]) || e < 0 || e >= n_experts || slot_row[e] < 0) continue;
        const int pos = atomicAdd(&cur[e], 1);   // the order inside an expert's range is arbitrary: a pair's row depends on its own input only
        order[pos] = p;
        src_tok[pos] = p / Kx;
    }
}

// One CTA of 128 threads per position: the operand record (B fragments of every unit, group sums, exponent) of row
// src[pos] of x (identity: row pos), written to recs + pos * rstride.
template <bool HILO, bool SRC_BF16>
__global__ void __launch_bounds__(128) g3_records_kernel(const void *x, const int *src, int identity, const int *total, int K, uint8_t *recs, int rstride) {
    extern __shared__ __align__(16) uint8_t g3row[];
    __shared__ float wmax[4];
    const int pos = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (total && pos >= *total) return;      // total == NULL: every CTA of the grid has a row
    const size_t row = identity ? (size_t)pos : (size_t)src[pos];
    const int rowb = K * (SRC_BF16 ? 2 : 4);
    const uint4 *g = reinterpret_cast<const uint4 *>(reinterpret_cast<const uint8_t *>(x) + row * rowb);
    for (int i = tid; i < rowb / 16; i += 128) reinterpret_cast<uint4 *>(g3row)[i] = g[i];
    __syncthreads();
    uint8_t *rec = recs + (size_t)pos * rstride;
    const int secb = sec3_bytes(K), hdr_off = secb * (HILO ? 2 : 1);
    float amax = 0.f;
    for (int grp = warp; grp < K / 64; grp += 4) {       // a warp per group of 64: two values per lane
        float v[2];
        if (SRC_BF16) {
            const uint32_t u = reinterpret_cast<const uint32_t *>(g3row)[grp * 32 + lane];
            v[0] = __uint_as_float(u << 16);
            v[1] = __uint_as_float(u & 0xffff0000u);
        } else {
            const float2 f = reinterpret_cast<const float2 *>(g3row)[grp * 32 + lane];
            v[0] = f.x;
            v[1] = f.y;
        }
        float s = v[0] + v[1];
        amax = fmaxf(amax, fmaxf(fabsf(v[0]), fabsf(v[1])));
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) reinterpret_cast<float *>(rec + hdr_off)[grp] = s;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) wmax[warp] = amax;
    __syncthreads();
    const float m = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
    int E = (int)(__float_as_uint(m) >> 23) + 1;
    E = E < 30 ? 30 : (E > 230 ? 230 : E);
    if (tid == 0) reinterpret_cast<float *>(rec + hdr_off)[K / 64] = __int_as_float(E);
    for (int it = tid; it < (K / 128) * 4; it += 128) build_frag3_item<HILO, SRC_BF16>(g3row, it >> 2, it & 3, E, rec, secb);
}

// grid (tile splits, items), 256 threads = 8 warps, two CTAs per SM.  A warp takes whole tiles (16 fragment rows,
// all of K); the item's records sit in shared memory; the packed units come straight from the pool by coalesced
// loads (768 contiguous bytes per unit), two units ahead.
template <bool HILO, bool FP16S, int NPASS, bool DOWN>
__global__ void __launch_bounds__(256, 2) moe_group3_kernel(const G3Args a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int PP = HILO ? 2 : 4, NTOK = PP * NPASS;
    if ((int)blockIdx.y >= *a.n_items) return;
    const int4 item = a.items[blockIdx.y];
    const int count = item.z;
    const FinchTile T = finch_tile(a.hidden, a.inter);
    const int K = DOWN ? a.inter : a.hidden, units = K / 128;
    const int ntiles = DOWN ? T.nTB : T.nTA, tile_bytes = DOWN ? T.tileB : T.tileA;
    const uint8_t *tiles = a.pool_base + (size_t)a.slot_row[item.x] * a.slot_bytes + (DOWN ? T.b_base : 0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int sec = sec3_bytes(K), hdr_off = sec * (HILO ? 2 : 1);
    // records of the item's tokens
    {
        const int per = a.rstride / 16;
        uint4 *dst = reinterpret_cast<uint4 *>(smem);
        if (a.rec_of) {     // the tokens' records: one per token, shared by all the token's pairs
            for (int q = 0; q < count; q++) {
                const uint4 *src = reinterpret_cast<const uint4 *>(a.recs + (size_t)a.rec_of[item.y + q] * a.rstride);
                for (int i = tid; i < per; i += 256) dst[q * per + i] = __ldg(src + i);
            }
        } else {
            const uint4 *src = reinterpret_cast<const uint4 *>(a.recs + (size_t)item.y * a.rstride);
            for (int i = tid; i < count * per; i += 256) dst[i] = __ldg(src + i);
        }
    }
    __syncthreads();
    const uint32_t rec32 = finch_smem_u32(smem);
    const bool mine = (g & 1) == (t >> 1);
    const int pos_b = HILO ? (g >> 2) : (g >> 1), pos_o = HILO ? (t >> 1) : t;
    const uint32_t sec_b = HILO ? (uint32_t)(((g >> 1) & 1) * sec) : 0u;
    // B operand of this lane per pass: the record section of its column's token, or nothing (zeros in registers) when
    // the lane's k-slots belong to the other group of the unit or the column has no token.  Plain loads from shared
    // memory (the records do not change after the barrier), so the compiler schedules them ahead of the MMAs.
    const uint8_t *pb[NPASS];
    uint32_t ph[NPASS];
    bool live[NPASS], hasb[NPASS];
#pragma unroll
    for (int ps = 0; ps < NPASS; ps++) {
        const int tb = ps * PP + pos_b, to = ps * PP + pos_o;
        hasb[ps] = mine && tb < count;
        pb[ps] = smem + (hasb[ps] ? tb * a.rstride + (int)sec_b : 0) + t * 16;
        live[ps] = to < count;
        ph[ps] = rec32 + (uint32_t)((live[ps] ? to : 0) * a.rstride + hdr_off);
    }
    struct Unit {
        uint2 q0, q1, q2;
        uint4 s;
    };
    for (int tile = blockIdx.x * 8 + warp; tile < ntiles; tile += gridDim.x * 8) {
        const uint8_t *tp = tiles + (size_t)tile * tile_bytes;
        auto load_unit = [&](int u, Unit &o) {
            const uint2 *w = reinterpret_cast<const uint2 *>(tp + (size_t)u * 768 + lane * 24);
            o.q0 = __ldg(w);
            o.q1 = __ldg(w + 1);
            o.q2 = __ldg(w + 2);
            o.s = __ldg(reinterpret_cast<const uint4 *>(tp + (size_t)units * 768 + u * 128 + g * 16));
        };
        float run[NPASS][4];   // runA, runB, biasA, biasB of every pass
#pragma unroll
        for (int ps = 0; ps < NPASS; ps++) run[ps][0] = run[ps][1] = run[ps][2] = run[ps][3] = 0.f;
        // packed units are requested PD units ahead of their use (more where few passes leave registers free)
        constexpr int PD = NPASS == 4 ? 2 : 4;
        Unit nx[PD];
#pragma unroll
        for (int d = 0; d < PD; d++) load_unit(d < units ? d : 0, nx[d]);
#pragma unroll 1
        for (int u = 0; u < units; u += PD) {
#pragma unroll
            for (int h = 0; h < PD; h++) {
                if (u + h >= units) break;
                const Unit cu = nx[h];
                if (u + h + PD < units) load_unit(u + h + PD, nx[h]);
                const uint2 q0 = cu.q0, q1 = cu.q1, q2 = cu.q2;
                const uint32_t av1 = __funnelshift_r(q0.x, q0.y, 8), av3 = __funnelshift_r(q0.y, q1.x, 8), av5 = q1.x >> 8;
                const uint32_t bv1 = __funnelshift_r(q1.y, q2.x, 8), bv3 = __funnelshift_r(q2.x, q2.y, 8), bv5 = q2.y >> 8;
                float sA0, sA1, sB0, sB1, bA0, bA1, bB0, bB1;
                widen2<FP16S>(cu.s.x, sA0, sA1);
                widen2<FP16S>(cu.s.y, sB0, sB1);
                widen2<FP16S>(cu.s.z, bA0, bA1);
                widen2<FP16S>(cu.s.w, bB0, bB1);
                const int uo = (u + h) * UB;
                // The nine MMAs of the unit, two at a time: their A fragments are extracted once and used by every pass,
                // and the passes' accumulators are independent chains that keep the tensor pipe busy between them.
                float acc[NPASS][4];
#define FINCH_A3(j, r)                                                     \
    r[0] = extract3_one<2 * (j)>(q0.x, av1, q0.y, av3, q1.x, av5);         \
    r[1] = extract3_one<2 * (j)>(q1.y, bv1, q2.x, bv3, q2.y, bv5);         \
    r[2] = extract3_one<2 * (j) + 1>(q0.x, av1, q0.y, av3, q1.x, av5);     \
    r[3] = extract3_one<2 * (j) + 1>(q1.y, bv1, q2.x, bv3, q2.y, bv5);
#define FINCH_PAIR3(jp)                                                                                   \
    {                                                                                                     \
        uint32_t A0[4], A1[4];                                                                            \
        FINCH_A3(2 * (jp), A0) FINCH_A3(2 * (jp) + 1, A1)                                                 \
        uint4 bb[NPASS];                                                                                  \
        _Pragma("unroll") for (int ps = 0; ps < NPASS; ps++)                                              \
            bb[ps] = hasb[ps] ? *reinterpret_cast<const uint4 *>(pb[ps] + uo + (jp) * 64) : make_uint4(0u, 0u, 0u, 0u); \
        _Pragma("unroll") for (int ps = 0; ps < NPASS; ps++) {                                            \
            if ((jp) == 0) mma16816_z(acc[ps], A0[0], A0[1], A0[2], A0[3], bb[ps].x, bb[ps].y);           \
            else mma16816(acc[ps], A0[0], A0[1], A0[2], A0[3], bb[ps].x, bb[ps].y);                       \
        }                                                                                                 \
        _Pragma("unroll") for (int ps = 0; ps < NPASS; ps++) mma16816(acc[ps], A1[0], A1[1], A1[2], A1[3], bb[ps].z, bb[ps].w); \
    }
                FINCH_PAIR3(0) FINCH_PAIR3(1) FINCH_PAIR3(2) FINCH_PAIR3(3)
                {
                    uint32_t A8[4];
                    FINCH_A3(8, A8)
                    uint2 b8[NPASS];
#pragma unroll
                    for (int ps = 0; ps < NPASS; ps++)   // section + 256 + t * 8 (pb carries t * 16)
                        b8[ps] = hasb[ps] ? *reinterpret_cast<const uint2 *>(pb[ps] + uo + 256 - t * 8) : make_uint2(0u, 0u);
#pragma unroll
                    for (int ps = 0; ps < NPASS; ps++) mma16816(acc[ps], A8[0], A8[1], A8[2], A8[3], b8[ps].x, b8[ps].y);
                }
#undef FINCH_PAIR3
#undef FINCH_A3
#pragma unroll
                for (int ps = 0; ps < NPASS; ps++) {
                    const uint2 xgb = lds64(ph[ps] + (uint32_t)((u + h) * 8));
                    const float x0 = __uint_as_float(xgb.x), x1 = __uint_as_float(xgb.y);
                    run[ps][0] = fmaf(sA1, acc[ps][1], fmaf(sA0, acc[ps][0], run[ps][0]));
                    run[ps][1] = fmaf(sB1, acc[ps][3], fmaf(sB0, acc[ps][2], run[ps][1]));
                    run[ps][2] = fmaf(bA1, x1, fmaf(bA0, x0, run[ps][2]));
                    run[ps][3] = fmaf(bB1, x1, fmaf(bB0, x0, run[ps][3]));
                }
            }
        }
#pragma unroll
        for (int ps = 0; ps < NPASS; ps++) {
            float runA = run[ps][0], runB = run[ps][1];
            if (HILO) {
                const float oA = __shfl_xor_sync(0xffffffffu, runA, 1), oB = __shfl_xor_sync(0xffffffffu, runB, 1);
                runA += oA * (1.0f / 2048.0f);
                runB += oB * (1.0f / 2048.0f);
            }
            if (live[ps] && (!HILO || !(t & 1))) {
                const float fac = pow2_biased(__float_as_int(lds32f(ph[ps] + (uint32_t)((K / 64) * 4))) + 17);
                const float vA = fmaf(runA, fac, run[ps][2]), vB = fmaf(runB, fac, run[ps][3]);
                const int pos = item.y + ps * PP + pos_o;
                if (DOWN) {
                    float *o = a.out + (size_t)a.order[pos] * a.hidden + 16 * tile + g;
                    o[0] = vA;
                    o[8] = vB;
                } else {
                    a.out[(size_t)pos * a.inter + 8 * tile + g] = __fdividef(vA, 1.0f + __expf(-vA)) * vB;
                }
            }
        }
    }
}

// The three item classes are independent: the two small ones (few tokens per item: little work per unit, bound by
// load latency) run on a second stream beside the large one and join before whatever reads their output.
template <bool HILO, bool FP16S, bool DOWN>
static cudaError_t g3_launch_lists(finch_ctx *ctx, cudaStream_t st, G3Args a, int4 *const lists[3], const int *counts, const int bounds[3], int split,
                                   int rstride, int K) {
    // split: CTAs per item of the largest class; items with fewer tokens do less per tile and get more CTAs each
    constexpr int PP = HILO ? 2 : 4;
    const int sec = sec3_bytes(K);
    cudaError_t e;
    cudaStream_t s2 = ctx->side2;
    if ((e = cudaEventRecord(ctx->ev_fork2, st)) != cudaSuccess) return e;
    if ((e = cudaStreamWaitEvent(s2, ctx->ev_fork2, 0)) != cudaSuccess) return e;
    a.items = lists[0];
    a.n_items = counts;
    moe_group3_kernel<HILO, FP16S, 1, DOWN><<<dim3(4 * split, bounds[0]), 256, PP * 1 * rstride + sec, s2>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    a.items = lists[1];
    a.n_items = counts + 1;
    moe_group3_kernel<HILO, FP16S, 2, DOWN><<<dim3(2 * split, bounds[1]), 256, PP * 2 * rstride + sec, s2>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = cudaEventRecord(ctx->ev_join2, s2)) != cudaSuccess) return e;
    a.items = lists[2];
    a.n_items = counts + 2;
    moe_group3_kernel<HILO, FP16S, 4, DOWN><<<dim3(split, bounds[2]), 256, PP * 4 * rstride + sec, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    return cudaStreamWaitEvent(st, ctx->ev_join2, 0);
}

template <bool HILO, bool FP16S, bool DOWN>
static int g3_attrs(finch_ctx *ctx, int rstride, int K) {
    constexpr int PP = HILO ? 2 : 4;
    const int sec = sec3_bytes(K);
    int rc;
    if ((rc = finch_func_attr_once(ctx, (const void *)moe_group3_kernel<HILO, FP16S, 1, DOWN>, PP * 1 * rstride + sec))) return rc;
    if ((rc = finch_func_attr_once(ctx, (const void *)moe_group3_kernel<HILO, FP16S, 2, DOWN>, PP * 2 * rstride + sec))) return rc;
    return finch_func_attr_once(ctx, (const void *)moe_group3_kernel<HILO, FP16S, 4, DOWN>, PP * 4 * rstride + sec);
}

}  // namespace

// ---- host side of the grouped 3-bit passes (called by finch_encode_moe_prefill) ----
namespace {
struct G3Plan {
    int P, ppa, bound01, bound2a, bound2b, rs_a, rs_b;
    size_t o_order, o_src, o_counts, o_la[3], o_lb[3], o_ra, o_rb, o_act, total;
};
G3Plan g3_plan(const finch_config &c, int T) {
    G3Plan p{};
    p.P = T * c.top_k;
    const int hilo_a = c.act_dtype != FINCH_BF16;
    p.ppa = hilo_a ? 2 : 4;
    p.bound01 = c.n_experts < p.P ? c.n_experts : p.P;
    p.bound2a = p.P / (4 * p.ppa) + p.bound01 + 1;
    p.bound2b = p.P / 8 + p.bound01 + 1;
    p.rs_a = rec3_bytes(c.hidden, hilo_a);
    p.rs_b = rec3_bytes(c.moe_inter, 1);
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t r = off;
        off += (b + 255) & ~(size_t)255;
        return r;
    };
    p.o_order = take((size_t)p.P * 4);
    p.o_src = take((size_t)p.P * 4);
    p.o_counts = take(64);
    p.o_la[0] = take((size_t)p.bound01 * 16);
    p.o_la[1] = take((size_t)p.bound01 * 16);
    p.o_la[2] = take((size_t)p.bound2a * 16);
    p.o_lb[0] = take((size_t)p.bound01 * 16);
    p.o_lb[1] = take((size_t)p.bound01 * 16);
    p.o_lb[2] = take((size_t)p.bound2b * 16);
    p.o_ra = take((size_t)p.P * p.rs_a);
    p.o_rb = take((size_t)p.P * p.rs_b);
    p.o_act = take((size_t)p.P * c.moe_inter * 4);
    p.total = off;
    return p;
}
}  // namespace

size_t finch_group3_ws_bytes(finch_ctx *ctx, int T) { return g3_plan(ctx->cfg, T).total; }

// down_out[pair][hidden] = expert(pair) applied to its token's row, for every usable pair of the chunk (pairs that are
// masked, out of range or not resident are left alone).  ws: finch_group3_ws_bytes(ctx, T) bytes of device memory.
int finch_group3_prefill(finch_ctx *ctx, cudaStream_t st, finch_pool *pool, int layer, const void *x, const int32_t *ids, const uint8_t *valid, int T, void *ws,
                         float *down_out) {
    const finch_config &c = ctx->cfg;
    if (c.n_experts > 4096) return finch_fail(ctx, FINCH_E_UNSUPPORTED, "the grouped prefill passes take at most 4096 experts");
    const G3Plan p = g3_plan(c, T);
    char *w = (char *)ws;
    int *order = (int *)(w + p.o_order), *src_tok = (int *)(w + p.o_src), *counts = (int *)(w + p.o_counts);
    int4 *la[3] = {(int4 *)(w + p.o_la[0]), (int4 *)(w + p.o_la[1]), (int4 *)(w + p.o_la[2])};
    int4 *lb[3] = {(int4 *)(w + p.o_lb[0]), (int4 *)(w + p.o_lb[1]), (int4 *)(w + p.o_lb[2])};
    uint8_t *recs_a = (uint8_t *)(w + p.o_ra), *recs_b = (uint8_t *)(w + p.o_rb);
    float *act = (float *)(w + p.o_act);
    const int32_t *slot_row = pool->slot_table_dev + (size_t)layer * pool->n_experts;
    const bool hilo_a = c.act_dtype != FINCH_BF16, fp16s = c.scale_dtype == FINCH_FP16;
    int rc;
    if (hilo_a) rc = fp16s ? g3_attrs<true, true, false>(ctx, p.rs_a, c.hidden) : g3_attrs<true, false, false>(ctx, p.rs_a, c.hidden);
    else rc = fp16s ? g3_attrs<false, true, false>(ctx, p.rs_a, c.hidden) : g3_attrs<false, false, false>(ctx, p.rs_a, c.hidden);
    if (rc) return rc;
    if ((rc = fp16s ? g3_attrs<true, true, true>(ctx, p.rs_b, c.moe_inter) : g3_attrs<true, false, true>(ctx, p.rs_b, c.moe_inter))) return rc;

    g3_sort_kernel<<<1, 1024, 2 * c.n_experts * sizeof(int), st>>>(ids, valid, slot_row, c.n_experts, p.P, c.top_k, p.ppa, 2, order, src_tok, la[0], la[1], la[2],
                                                                    lb[0], lb[1], lb[2], counts);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    // one operand record per position (a token's pairs each get a copy: the item kernels then read their records as one run)
    if (hilo_a) g3_records_kernel<true, false><<<p.P, 128, c.hidden * 4, st>>>(x, src_tok, 0, counts + 6, c.hidden, recs_a, p.rs_a);
    else g3_records_kernel<false, true><<<p.P, 128, c.hidden * 2, st>>>(x, src_tok, 0, counts + 6, c.hidden, recs_a, p.rs_a);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    G3Args a{};
    a.pool_base = pool->base;
    a.slot_bytes = pool->slot_bytes;
    a.slot_row = slot_row;
    a.hidden = c.hidden;
    a.inter = c.moe_inter;
    a.order = order;
    a.status = ctx->dev_status;
    a.recs = recs_a;
    a.rec_of = nullptr;
    a.rstride = p.rs_a;
    a.out = act;
    const int bounds_a[3] = {p.bound01, p.bound01, p.bound2a}, bounds_b[3] = {p.bound01, p.bound01, p.bound2b};
    cudaError_t e;
    if (hilo_a) e = fp16s ? g3_launch_lists<true, true, false>(ctx, st, a, la, counts, bounds_a, 2, p.rs_a, c.hidden)
                          : g3_launch_lists<true, false, false>(ctx, st, a, la, counts, bounds_a, 2, p.rs_a, c.hidden);
    else e = fp16s ? g3_launch_lists<false, true, false>(ctx, st, a, la, counts, bounds_a, 2, p.rs_a, c.hidden)
                   : g3_launch_lists<false, false, false>(ctx, st, a, la, counts, bounds_a, 2, p.rs_a, c.hidden);
    FINCH_CUDA_OK(ctx, e);
    g3_records_kernel<true, false><<<p.P, 128, c.moe_inter * 4, st>>>(act, src_tok, 1, counts + 6, c.moe_inter, recs_b, p.rs_b);
    FINCH_CUDA_OK(ctx, cudaGetLastError());
    a.recs = recs_b;
    a.rec_of = nullptr;
    a.rstride = p.rs_b;
    a.out = down_out;
    e = fp16s ? g3_launch_lists<true, true, true>(ctx, st, a, lb, counts + 3, bounds_b, 4, p.rs_b, c.moe_inter)
              : g3_launch_lists<true, false, true>(ctx, st, a, lb, counts + 3, bounds_b, 4, p.rs_b, c.moe_inter);
    FINCH_CUDA_OK(ctx, e);
    ctx->launches += 9;
    return FINCH_OK;
}

// n_calls batches of B tokens each (rows [c * B, (c + 1) * B) of the inputs) in one sequence of three launches.
// Batch own_call gets shared / h_mid and writes hidden_out; the others write their routed sums to rows_out.
static int encode_decode_calls(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, const void *h_post, const int32_t *expert_ids,
                               const float *weights, const uint8_t *valid, const finch_shared *shared, const float *h_mid, float *hidden_out, int B,
                               int n_calls, int own_call, float *rows_out, const finch_ret_info *ret = nullptr) {
    if (!ctx || !pool || !h_post || !expert_ids || !weights || !hidden_out) return FINCH_E_ARG;
    const finch_config &c = ctx->cfg;
    if (pool->ctx != ctx) return finch_fail(ctx, FINCH_E_ARG, "pool belongs to another context");
    if (layer < 0 || layer >= pool->n_layers) return finch_fail(ctx, FINCH_E_ARG, "layer %d out of range", layer);
    if (B < 1 || (long long)B * n_calls > c.max_tokens)
        return finch_fail(ctx, FINCH_E_ARG, "%d batch(es) of B=%d outside 1..max_tokens=%d", n_calls, B, c.max_tokens);
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
        a.shared_act = ctx->shared_act;
        a.gate_score = shared->gate_score;
        a.sh_inter = shared->gate.out_dim;
        a.sh_fp16 = shared->gate.scale_dtype == FINCH_FP16;
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
    a.act = ctx->act;
    a.partial = ctx->partial;
    a.status = ctx->dev_status;
    a.h_mid = h_mid;
    a.hidden_out = hidden_out;
    a.fault = ctx->fault;
    a.n_calls = n_calls;
    a.own_call = n_calls > 1 ? own_call : 0;
    a.rows_out = rows_out;
    if (ret) a.ret = *ret;
    if (ctx->hp_done && n_calls == 1) {      // armed by the host-pointer entry point for this one call
        a.done_ticket = ctx->hp_ticket;
        a.host_done = ctx->hp_done;
        a.host_status = ctx->hp_status;
        a.done_seq_src = ctx->hp_seq_src;
    }
    ctx->hp_done = nullptr;
    if ((uintptr_t)h_post & 15) return finch_fail(ctx, FINCH_E_ARG, "h_post must be 16-byte aligned");
    const int hilo = c.act_dtype == FINCH_BF16 ? 0 : 1;
    const bool fp16s = c.scale_dtype == FINCH_FP16;
    int grid = ctx->sm_count;
    const int sm_all = grid;
    if (n_calls > 1) {
        // CTAs per batch: the routed experts of a batch cost about the same everywhere (a token's K experts spread over
        // the ranks); the caller's own batch also carries the shared expert, about three routed experts' worth of MMAs.
        const double routed = std::max(1.0, (double)B * c.top_k / n_calls), own = routed + (shared ? 3.0 : 0.0);
        const double total = routed * (n_calls - 1) + own;
        double acc = 0.0;
        a.cta0[0] = 0;
        for (int q = 0; q < n_calls; q++) {
            acc += q == own_call ? own : routed;
            int e = (int)(sm_all * acc / total + 0.5);
            if (e < a.cta0[q] + 2) e = a.cta0[q] + 2;      // a batch with the shared expert needs a routed and a shared CTA
            a.cta0[q + 1] = e;
        }
        a.cta0[n_calls] = std::max(a.cta0[n_calls], sm_all);   // at most 16 batches: every one gets CTAs of the first wave
        grid = a.cta0[own_call >= 0 && own_call < n_calls ? own_call + 1 : 1] - a.cta0[own_call >= 0 && own_call < n_calls ? own_call : 0];
    }
    if (shared) {
        // CTAs that take the shared expert's tiles: its expected share of the MMAs of each kernel.  The routing is
        // not known on the host: the distinct experts of a call are estimated from the batch (a token's K experts
        // are distinct; tokens overlap more as the batch grows) and so are the passes of a popular expert's tiles.
        const FinchTile T = finch_tile(c.hidden, c.moe_inter);
        const FinchTile4 T4 = finch_tile4(c.hidden, a.sh_inter);
        const double U = n_calls > 1 ? std::max(1.0, (double)a.P / n_calls)
                                     : (B == 1 ? c.top_k : std::max((double)c.top_k, a.P * (1.0 - 0.04 * (B - 1))));
        const int ppa = hilo ? 2 : 4;
        const double fa = 1.0 + (B > ppa ? 0.1 : 0.0) + (hilo && B > 2 ? 0.35 * (B - 2) / 6.0 : 0.0), fb = B > 2 ? 1.0 + 0.45 * (B - 2) / 6.0 : 1.0;
        const int npa = hilo ? (B + 3) / 4 : (B + 7) / 8, npb = (B + 3) / 4;
        auto split = [&](double routed, double sh) {
            int gs = (int)(grid * sh / (routed + sh) + 0.5);
            return gs < 1 ? 1 : (gs > grid / 2 ? grid / 2 : gs);
        };
        // a gate/up tile of the shared expert carries 4 + 4 rows (half of the MMA's rows are duplicates) and its
        // group loop is not unrolled: per MMA it costs about 2.3 times a routed tile's (measured)
        a.gs_a = split(U * T.nTA * T.unitsA * MMA_A3 * fa, 2.3 * npa * T4.nTA * T4.groupsA * MMA_A4);
        a.gs_b = split(U * T.nTB * T.unitsD * MMA_A3 * fb, (double)npb * T4.nTB * T4.groupsD * MMA_A4);
    }
    // as many teams / warps as their stages leave room for
    int nteam = NW_MAX / TEAM;
    while (nteam > 0 && smem_a_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, hilo, nteam * TEAM).total > SMEM_MAX) --nteam;
    int nwb = NW_MAX;
    while (nwb > 0 && smem_b_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, nwb).total > SMEM_MAX) nwb -= 2;
    // the staging area (every warp's second stage) has to hold one row, and a row gets at least a warp
    if (nteam < 2 || nwb < 4 || nteam * TEAM * smem_a_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, hilo, nteam * TEAM).stg < c.hidden * 4 ||
        nwb * smem_b_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, nwb).stg < (c.moe_inter > a.sh_inter ? c.moe_inter : a.sh_inter) * 4)
        return finch_fail(ctx, FINCH_E_UNSUPPORTED, "dims need too much shared memory");
    const SmemA LA = smem_a_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, hilo, nteam * TEAM);
    const SmemB LB = smem_b_layout(c.hidden, c.moe_inter, a.sh_inter, B, a.has_shared, nwb);
    {
        int rc = set_attrs_once(ctx);
        if (rc) return rc;
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
    const void *ka = hilo ? (fp16s ? (const void *)moe_gateup_kernel<true, true> : (const void *)moe_gateup_kernel<true, false>)
                          : (fp16s ? (const void *)moe_gateup_kernel<false, true> : (const void *)moe_gateup_kernel<false, false>);
    if (B == 1)   // one token per batch: the grouping has nothing to match
        ka = hilo ? (fp16s ? (const void *)moe_gateup_kernel<true, true, true> : (const void *)moe_gateup_kernel<true, false, true>)
                  : (fp16s ? (const void *)moe_gateup_kernel<false, true, true> : (const void *)moe_gateup_kernel<false, false, true>);
    const void *kb = fp16s ? (const void *)moe_down_kernel<true> : (const void *)moe_down_kernel<false>;
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[0], st));
    const int grid_all = n_calls > 1 ? a.cta0[n_calls] : grid;
    FINCH_CUDA_OK(ctx, launch(ka, dim3(grid_all), nteam * TEAM * 32, LA.total));
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[1], st));
    FINCH_CUDA_OK(ctx, launch(kb, dim3(grid_all), nwb * 32, LB.total));
    FINCH_CUDA_OK(ctx, launch((const void *)moe_combine_kernel, dim3((c.hidden + 255) / 256, B * n_calls), 256, 0));
    if (pe) FINCH_CUDA_OK(ctx, cudaEventRecord(pe[2], st));
    ctx->launches += 3;
    return FINCH_OK;
}

extern "C" int finch_encode_moe_decode(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, const void *h_post,
                                       const int32_t *expert_ids, const float *weights, const uint8_t *valid,
                                       const finch_shared *shared, const float *h_mid, float *hidden_out, int B) {
    return encode_decode_calls(ctx, stream, pool, layer, h_post, expert_ids, weights, valid, shared, h_mid, hidden_out, B, 1, 0, nullptr);
}

extern "C" int finch_encode_moe_decode_multi(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, int n_batches, int B, const void *h_post,
                                             const int32_t *expert_ids, const float *weights, const uint8_t *valid, int own_batch,
                                             const finch_shared *shared, const float *h_mid, float *hidden_out, float *rows_out) {
    if (n_batches < 1 || n_batches > MAX_CALLS || own_batch < 0 || own_batch >= n_batches || !rows_out) return FINCH_E_ARG;
    return encode_decode_calls(ctx, stream, pool, layer, h_post, expert_ids, weights, valid, shared, h_mid, hidden_out, B, n_batches, own_batch, rows_out);
}

int finch_encode_moe_decode_multi_ret(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, int n_batches, int B, const void *h_post,
                                      const int32_t *expert_ids, const float *weights, const uint8_t *valid, int own_batch,
                                      const finch_shared *shared, const float *h_mid, float *hidden_out, const finch_ret_info *ret) {
    if (n_batches < 1 || n_batches > MAX_CALLS || own_batch < 0 || own_batch >= n_batches || !ret || !ret->epoch || ret->T != B) return FINCH_E_ARG;
    if (ctx && ctx->cfg.hidden % 2) return FINCH_E_ARG;
    return encode_decode_calls(ctx, stream, pool, layer, h_post, expert_ids, weights, valid, shared, h_mid, hidden_out, B, n_batches, own_batch, nullptr, ret);
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

#ifdef FINCH_STAMPS
extern "C" __attribute__((visibility("default"))) int finch_stamps_read(long long *host, int n) {
    return cudaMemcpyFromSymbol(host, g_stamps, (size_t)n * sizeof(long long)) == cudaSuccess ? 0 : 1;
}
#endif

extern "C" int finch_debug_fault(finch_ctx *ctx, int kind) {
    if (!ctx || kind < 0 || kind > 1) return FINCH_E_ARG;
    ctx->fault = kind;
    return FINCH_OK;
}
