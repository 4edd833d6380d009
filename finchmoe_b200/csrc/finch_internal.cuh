// Internal declarations shared by the translation units of libfinchcuda.
// Nothing here is part of the C ABI (see include/finch_cuda.h).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "finch_cuda.h"

#define FINCH_MAX_PAIRS 64  // B * K limit of the decode-shaped kernels

struct finch_ctx {
    finch_config cfg{};
    cudaStream_t stream = nullptr;  // context-owned stream (used when the caller passes NULL)
    cudaStream_t side = nullptr;    // second stream: the shared expert of a prefill chunk runs beside the routed experts
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    cudaStream_t side2 = nullptr;   // third stream: the small item classes of the grouped prefill passes beside the large one
    cudaEvent_t ev_fork2 = nullptr, ev_join2 = nullptr;
    int sm_count = 0;
    // scratch shared by every call on this context (calls that overlap on the GPU race)
    float *act = nullptr;           // [max_pairs][moe_inter]   routed SwiGLU activations
    float *shared_act = nullptr;    // [max_tokens][shared_inter]
    float *partial = nullptr;       // [max_pairs + max_tokens][hidden] per-pair down outputs (+ shared rows)
    int *dev_status = nullptr;      // sticky device status word
    unsigned *hp_ticket = nullptr;  // device word: CTAs of the combine kernel that have finished (host-pointer path)
    unsigned *hp_done = nullptr;    // armed by finch_moe_forward_host for its next decode call: device address of the host's
    int *hp_status = nullptr;       //   completion word and status word (mapped pinned memory), and the value to write
    unsigned hp_seq = 0;
    const unsigned *hp_seq_src = nullptr;   // device word the completion value is read from (staged with the inputs)
    // finch_moe_forward_host: the launch sequence of a decode-sized call (input fetch, gate/up, down, combine), captured
    // once per (pool, layer, T, which optional inputs, shared expert) and replayed with one graph launch.  All addresses
    // in it are the staging blocks'; stage_gen changes when those are reallocated.
    struct HostGraph {
        finch_pool *pool;
        int layer, T;
        bool valid, h_mid, has_shared;
        int fault;                  // finch_debug_fault is part of the kernels' parameters
        finch_shared shared;
        unsigned stage_gen;
        int seen;                   // calls so far; the second one is captured; < 0: capture failed, stay with plain launches
        cudaGraphExec_t exec;
    };
    std::vector<HostGraph> host_graphs;
    unsigned stage_gen = 0;
    int fault = 0;                  // finch_debug_fault: failure injected into the next decode calls
    bool no_pdl = false;            // FINCH_NO_PDL=1 in the environment: plain stream-ordered launches
    struct SharedPrepared {
        const void *key[3];
        void *tiles;
    };
    std::vector<SharedPrepared> shared_cache;  // tiled copies of the shared experts seen so far
    // staging for the host-pointer entry points
    void *stage_dev = nullptr;
    void *stage_host = nullptr;     // pinned
    size_t stage_bytes = 0;
    // prefill workspace (allocated on first use)
    void *pf_ws = nullptr;
    size_t pf_ws_bytes = 0;
    float *logits = nullptr;        // [max_tokens][n_experts] router logits (finch_encode_router, allocated on first use)
    void *gguf_ws = nullptr;        // scratch of finch_encode_moe_gguf (allocated on first use)
    size_t gguf_ws_bytes = 0;
    void *gq_ws = nullptr;          // activation planes of the GGUF many-position matvec (matvec_gguf_mma.cu)
    size_t gq_ws_bytes = 0;
    int prefill_chunk = 0;          // finch_set_prefill_chunk: tokens per tensor-core pass, 0 = 512
    int prefill_mode = 0;           // finch_set_prefill_mode: 0 by chunk length, 1 sub-batches through decode, 2 / 3 / 4 the tensor-core paths
    uint64_t launches = 0;
    // optional per-kernel timing of the MoE decode call (finch_profile_enable)
    bool profile = false;
    std::vector<cudaEvent_t> prof_events;  // triples: before gate/up, between, after down+combine
    size_t prof_used = 0;
    std::string err;
    size_t expert_bytes = 0;
    struct {
        size_t gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b;
    } lay{};
};

struct finch_pool {
    finch_ctx *ctx = nullptr;
    int n_layers = 0, n_experts = 0, slots = 0, used = 0;
    size_t slot_bytes = 0;
    uint8_t *base = nullptr;          // device: slots * slot_bytes
    int32_t *slot_table_dev = nullptr;  // device: [n_layers][n_experts] slot or -1
    std::vector<int32_t> slot_of;     // host mirror
    std::vector<int32_t> owner;       // slot -> layer * n_experts + expert, or -1
    std::vector<uint64_t> last_used;
    uint64_t clock = 0, hits = 0, misses = 0, evictions = 0;
    int cursor = 0;  // next slot to probe when looking for a free one
    std::vector<uint8_t> tmp;  // host staging for the disk <-> tiled permutation
};

struct finch_event {
    finch_ctx *ctx = nullptr;
    cudaEvent_t ev = nullptr;
};

int finch_fail(finch_ctx *ctx, int code, const char *fmt, ...);

#define FINCH_CUDA_OK(ctx, expr)                                                                   \
    do {                                                                                           \
        cudaError_t e__ = (expr);                                                                  \
        if (e__ != cudaSuccess)                                                                    \
            return finch_fail((ctx), FINCH_E_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e__), \
                              __FILE__, __LINE__);                                                 \
    } while (0)

static inline cudaStream_t finch_pick_stream(finch_ctx *ctx, finch_stream s) {
    return s ? (cudaStream_t)s : ctx->stream;
}

// Opt-in to more than 48 KB of dynamic shared memory: a per-device function attribute, set once per (function, device).
int finch_func_attr_once(finch_ctx *ctx, const void *func, int smem_bytes);

// Where the rows of the other batches of a multi-batch decode call go when the batches are the ranks of an
// expert-parallel layer: straight into the partial-row slots of those ranks' receive areas (ep_peer.cu), every
// pair of values beside the sender's epoch, instead of into a local array that a second kernel would send.
struct finch_ret_info {
    uint8_t *area[16];        // every rank's receive area as this process addresses it
    size_t off_back;          // where the partial-row slots begin inside an area
    int rank, T;              // this rank; tokens per rank (slot [rank][t] of the destination's area)
    const uint32_t *epoch;    // this rank's epoch word
};
// finch_encode_moe_decode_multi with the rows of the other batches returned through `ret` (implemented in moe_decode.cu)
int finch_encode_moe_decode_multi_ret(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, int n_batches, int B, const void *h_post,
                                      const int32_t *expert_ids, const float *weights, const uint8_t *valid, int own_batch,
                                      const finch_shared *shared, const float *h_mid, float *hidden_out, const finch_ret_info *ret);

// Implemented in moe_decode.cu / moe_prefill.cu, used by the host-pointer entry point.
int finch_validate_wdesc(finch_ctx *ctx, const finch_wdesc *w, const char *what);

// ------------------------------------------------------------------ device helpers
#ifdef __CUDACC__

__device__ __forceinline__ float finch_widen16(uint16_t h, int scale_dtype) {
    if (scale_dtype == FINCH_FP16) return __half2float(__ushort_as_half(h));
    return __uint_as_float(((uint32_t)h) << 16);
}

// two adjacent 16-bit values packed in one word -> floats (lo = first in memory)
__device__ __forceinline__ void finch_widen16x2(uint32_t w, int scale_dtype, float &lo, float &hi) {
    if (scale_dtype == FINCH_FP16) {
        const __half2 h = *reinterpret_cast<const __half2 *>(&w);
        const float2 f = __half22float2(h);
        lo = f.x;
        hi = f.y;
    } else {
        lo = __uint_as_float(w << 16);
        hi = __uint_as_float(w & 0xffff0000u);
    }
}

__device__ __forceinline__ uint32_t finch_smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier + bulk async copy (TMA, untiled form) ----
__device__ __forceinline__ void finch_mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(finch_smem_u32(bar)), "r"(count));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void finch_mbar_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(finch_smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Bounded wait: returns false when the phase did not complete within the limit.  try_wait is given a
// suspend-time hint, so a waiting thread sleeps in hardware (and is woken when the phase completes)
// instead of spending the SM's issue slots on polling; the hint also bounds one attempt, so the
// attempt count bounds the total wait (about a fifth of a second; legitimate waits are microseconds).
__device__ __forceinline__ bool finch_mbar_wait(uint64_t *bar, unsigned parity) {
    const uint32_t a = finch_smem_u32(bar);
    for (unsigned it = 0; it < (1u << 13); ++it) {
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
// global -> shared bulk copy; src, dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void finch_bulk_g2s(void *dst_smem, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            finch_smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(finch_smem_u32(bar))
        : "memory");
}

// D = A(16x16, f16, row) * B(16x8, f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void finch_mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t finch_pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

#endif  // __CUDACC__
