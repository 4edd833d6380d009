/*
 * finch_cuda.h -- C ABI of libfinchcuda: the quantized-expert MoE hot path of
 * the FinchMoE engine on NVIDIA B200 (sm_100a).
 *
 * The reference engine (finchmoe/infer.m) has no plugin layer: its C host code
 * builds Metal command buffers inline.  Each entry point below replaces one of
 * the seams where that host code stops deciding what to run and starts
 * encoding GPU work; the seam is cited as <reference file>:<lines>.  Conventions
 * kept from the reference: plain C types, caller-owned pointers, per-expert
 * valid[] masks instead of errors for missing experts, one calling thread per
 * context, work made asynchronous by "encode, do not wait" (here: stream order).
 * Changed on purpose: programmer errors return a status instead of abort().
 *
 * "encode" functions take DEVICE pointers and only enqueue work on `stream`;
 * functions without "encode" take HOST pointers, copy in and out, and return
 * when the result is in host memory.
 */
#ifndef FINCH_CUDA_H
#define FINCH_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define FINCH_API
#else
#define FINCH_API __attribute__((visibility("default")))
#endif

/* ---- status codes -------------------------------------------------------
 * FINCH_E_UNSUPPORTED mirrors the reference helpers that return 0 / -1 for
 * "not handled here, caller falls back" (finchmoe/infer.m:3048-3053, 10955). */
enum {
    FINCH_OK = 0,
    FINCH_E_ARG = 1,         /* shape / alignment / range */
    FINCH_E_NOSLOT = 2,      /* expert not resident in the pool */
    FINCH_E_CUDA = 3,
    FINCH_E_NCCL = 4,
    FINCH_E_TIMEOUT = 5,     /* a bounded device- or host-side wait ran out */
    FINCH_E_UNSUPPORTED = 6,
    FINCH_E_NOMEM = 7
};

/* 16-bit storage of scales/biases: the reference's files hold BF16
 * (finchmoe/infer.m:1718-1719); the benchmark's synthetic tensors hold FP16. */
enum { FINCH_BF16 = 0, FINCH_FP16 = 1, FINCH_F32 = 2 };

/* `bits` convention of the reference's matvec seam (finchmoe/infer.m:1681-1701,
 * 1249-1258): 3 / 4 / 8 = affine group-quantized, 10 = GGUF Q4_K,
 * 11 = GGUF Q6_K, 0 = raw BF16 weights. */
enum { FINCH_BITS_BF16 = 0, FINCH_BITS_Q4_K = 10, FINCH_BITS_Q6_K = 11 };

typedef struct finch_ctx finch_ctx;
typedef struct finch_pool finch_pool;
typedef struct finch_event finch_event;
typedef void *finch_stream; /* cudaStream_t; NULL = the context's own stream */

/* Replaces the model #defines (finchmoe/infer.m:144-156) and the tier globals
 * g_use_3bit etc. (infer.m:432-436). */
typedef struct finch_config {
    int device;       /* CUDA ordinal */
    int hidden;       /* 2048; multiple of 128 */
    int n_experts;    /* 256 */
    int top_k;        /* 8 (1..8) */
    int moe_inter;    /* 512; multiple of 128 */
    int shared_inter; /* 512 */
    int group_size;   /* 64 */
    int n_layers;     /* 40 */
    int expert_bits;  /* 3 */
    int scale_dtype;  /* FINCH_BF16 | FINCH_FP16: storage of scales and biases */
    int act_dtype;    /* FINCH_F32 | FINCH_BF16: element type of h_post inputs */
    int max_tokens;   /* largest B / T any encode call will pass (scratch sizing) */
} finch_config;

/* metal_setup() / teardown, finchmoe/infer.m:2388. */
FINCH_API int finch_ctx_create(const finch_config *cfg, finch_ctx **out);
FINCH_API void finch_ctx_destroy(finch_ctx *ctx);
FINCH_API const char *finch_last_error(const finch_ctx *ctx);
FINCH_API const char *finch_status_str(int status);
/* Bytes of one packed routed-expert block for this context
 * ([gate W|S|B|up W|S|B|down W|S|B], finchmoe/infer.m:223-234). */
FINCH_API size_t finch_expert_bytes(const finch_ctx *ctx);

/* metal_set_weights(), finchmoe/infer.m:2813: wraps the non-expert weight file
 * in a GPU buffer; tensors are then addressed as base + offset (2892-2894). */
FINCH_API int finch_weights_upload(finch_ctx *ctx, const void *host, size_t bytes, void **dev);
FINCH_API int finch_buf_alloc(finch_ctx *ctx, size_t bytes, void **dev);
FINCH_API int finch_buf_free(finch_ctx *ctx, void *dev);

/* ---- expert pool --------------------------------------------------------
 * expert_cache_new / _lookup / _insert / _free (finchmoe/infer.m:6179-6291),
 * the positional prefill pool (2596-2631) and the pread targets
 * (6057-6122).  With max_slots == 0 every (layer, expert) owns a slot (all
 * 40 x 256 3-bit experts are 14.09 GB and stay resident in HBM); with fewer
 * slots, put() evicts the least recently used entry as the reference's LRU
 * does (6268-6276).  The (layer, expert) -> slot table also lives on the
 * device, so kernels resolve expert ids without a host round trip; an expert
 * that is not resident behaves as valid[k] = 0. */
FINCH_API int finch_pool_create(finch_ctx *ctx, int n_layers, int n_experts, int max_slots, finch_pool **out);
FINCH_API void finch_pool_destroy(finch_pool *pool);
/* Stores the exact on-disk block of one expert (host memory).  A put that replaces a resident expert or
 * evicts one first waits for the work already queued on the device (a kernel in flight may be reading that
 * slot or the slot table); a put into a free slot does not wait.  The LRU clock is advanced by put() and
 * lookup(), as the reference's access_counter is (finchmoe/infer.m:6216-6276). */
FINCH_API int finch_pool_put(finch_pool *pool, int layer, int expert, const void *packed_block);
/* Reads a resident block back to host memory (diagnostics, parity checks). */
FINCH_API int finch_pool_get(finch_pool *pool, int layer, int expert, void *packed_block_out);
/* slot_out = slot index, dev_ptr_out = device address of the block.
 * Returns FINCH_E_NOSLOT when the expert is not resident. */
FINCH_API int finch_pool_lookup(finch_pool *pool, int layer, int expert, int *slot_out, void **dev_ptr_out);
typedef struct finch_pool_stats {
    uint64_t hits, misses, evictions;
    int slots, used;
    size_t slot_bytes;
} finch_pool_stats;
FINCH_API int finch_pool_get_stats(const finch_pool *pool, finch_pool_stats *out);
/* Benchmark helper: fills layers [layer0, layer1) with seeded synthetic experts
 * on the device (codes uniform, scale = |N(0,0.01)|, bias = -4*scale in the
 * context's scale_dtype) and marks them resident. */
FINCH_API int finch_pool_fill_synthetic(finch_pool *pool, int layer0, int layer1, uint64_t seed);

/* ---- weight descriptor --------------------------------------------------
 * BatchMatvecSpec, finchmoe/infer.m:3401-3411 (W / scales / biases / dims /
 * group_size / bits).  All three pointers are device addresses.  scales and
 * biases are NULL for bits 0, 10 and 11. */
typedef struct finch_wdesc {
    const void *W;
    const void *scales;
    const void *biases;
    int out_dim;
    int in_dim;
    int group_size;
    int bits;
    int scale_dtype;
} finch_wdesc;

/* fast_dequant_matvec / gpu_dequant_matvec (finchmoe/infer.m:3369, 2872) and
 * gpu_gguf_dequant_matvec (3050): out[m][r] = sum_i w[r][i] * x[m][i].
 * x and out are HOST fp32 arrays ([M][in_dim], [M][out_dim]); synchronous. */
FINCH_API int finch_matvec(finch_ctx *ctx, const finch_wdesc *w, const float *x_host, float *out_host, int M);

/* The same matvec for callers that must not allocate device memory: code that
 * runs inside somebody else's memory budget or allocator (an engine that has
 * handed all of HBM to its own pool, a plugin host that forbids cudaMalloc in
 * callbacks, a latency-critical thread where an allocation could block on the
 * driver).  It needs no context.  x and out (HOST fp32, [M][in_dim] and
 * [M][out_dim]) are staged through a fixed 512 KiB buffer that is part of the
 * library image, so M * (in_dim + out_dim) floats must fit in it; larger calls
 * return FINCH_E_UNSUPPORTED.  The weights are device pointers as above and
 * must live on the current device.  The first call made on a device looks up
 * the buffer's device address; make that first call before starting any
 * stream capture.  All calls share the one buffer: calls that overlap on the
 * GPU (different streams or threads) overwrite each other's data.  Nothing in
 * the buffer has to start out zeroed.  Synchronous: returns when out is
 * written.  This entry point has no counterpart in the reference. */
FINCH_API int finch_matvec_noalloc(const finch_wdesc *w, const float *x_host, float *out_host, int M, finch_stream stream);

/* fast_batch_matvec / gpu_encode_batch_matvec / routing_batch_fused and
 * gpu_encode_prefill_matvec (finchmoe/infer.m:4477, 3528, 9061, 3672): n
 * matvecs of mixed bit width sharing one input x[M][in_dim] (device, element
 * type x_dtype), outs[i] = device fp32 [M][specs[i].out_dim]. */
FINCH_API int finch_encode_batch_matvec(finch_ctx *ctx, finch_stream stream, const void *x, int x_dtype,
                                        const finch_wdesc *specs, float *const *outs, int n, int M);

/* cpu_softmax + cpu_topk + cpu_normalize_weights, run on the CPU by the
 * reference after a GPU wait (finchmoe/infer.m:9285-9289, 1794-1840).
 * logits [T][n_experts] -> ids [T][K], weights [T][K] (device).  Same
 * selection and tie rule (earlier index wins); ids are emitted by descending
 * probability instead of the reference's slot order. */
FINCH_API int finch_encode_route_topk(finch_ctx *ctx, finch_stream stream, const float *logits, int n_experts,
                                      int K, int32_t *ids, float *weights, int T);

/* Router front end of a layer without the host round trip the reference pays (finchmoe/infer.m:9061-9105 runs
 * the gate matvecs on the GPU, waits, then cpu_softmax / cpu_topk / cpu_normalize_weights, 9285-9289): logits =
 * gate [n_experts x hidden] * h_post, shared_score = shared_gate [1 x hidden] * h_post (or NULL), then
 * finch_encode_route_topk.  gate / shared_gate are any matvec tier (BF16 rows with the default quantizer,
 * finchmoe/quantize_non_experts.py:103-105).  h_post [T][hidden] in the context's act dtype; all device. */
FINCH_API int finch_encode_router(finch_ctx *ctx, finch_stream stream, const finch_wdesc *gate, const finch_wdesc *shared_gate,
                                  const void *h_post, int32_t *ids, float *weights, float *shared_score, int T);

/* residual_norm_fused (finchmoe/shaders.metal:1232-1263) before the layer, and the RMS norm of the next
 * layer's input after the combine (finchmoe/infer.m:9705-9737) with oproj = NULL: h = resid + oproj,
 * h_mid_out = h (or NULL), h_post_out = h / sqrt(mean(h^2) + eps) * norm_w, written in the context's act dtype.
 * resid / oproj / h_mid_out fp32 [T][hidden], norm_w bf16 [hidden]; device pointers. */
FINCH_API int finch_encode_residual_norm(finch_ctx *ctx, finch_stream stream, const float *resid, const float *oproj,
                                         const uint16_t *norm_w_bf16, float eps, float *h_mid_out, void *h_post_out, int T);

/* Shared expert and its gate: finchmoe/infer.m:9608-9629 and the
 * sigmoid(shared_gate_score) factor of moe_combine_residual
 * (finchmoe/shaders.metal:2196-2231). */
typedef struct finch_shared {
    finch_wdesc gate, up, down;   /* 4-bit affine, group 64 */
    const float *gate_score;      /* device [B]: raw shared_expert_gate score */
} finch_shared;

/* gpu_encode_experts_batched + shared expert + moe_combine_residual
 * (finchmoe/infer.m:4065-4381, 9603-9703): for each of B tokens
 *   hidden_out = h_mid + sum_{k<K, valid} weights[k] * down_k(silu(gate_k x) * up_k x)
 *                + sigmoid(gate_score) * shared(x)
 * with k ascending.  h_post [B][hidden] in the context's act_dtype, expert_ids
 * / weights [B][K], valid [B][K] bytes or NULL, shared or NULL, h_mid fp32
 * [B][hidden] or NULL, hidden_out fp32 [B][hidden]; all device pointers.
 * Experts with valid == 0, an id outside [0, n_experts) or no pool slot are
 * skipped (never multiplied by zero).  B * K <= 64. */
FINCH_API int finch_encode_moe_decode(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer,
                                      const void *h_post, const int32_t *expert_ids, const float *weights,
                                      const uint8_t *valid, const finch_shared *shared, const float *h_mid,
                                      float *hidden_out, int B);

/* prefill_chunk_cmd3 / _batch_general (finchmoe/infer.m:10704-11241): the same
 * result for a chunk of T tokens.  Chunks of 128 tokens and more take the
 * tensor-core path: (token, k) pairs sorted by expert, grouped dequant-GEMMs on
 * bf16 tiles (weights RNE-rounded from the exact dequantised value, activations
 * rounded to bf16, fp32 accumulation), every selected expert read once per 512
 * tokens.  Shorter chunks go through the decode kernels in groups of eight
 * tokens and are bit-identical to finch_encode_moe_decode.  T <= max_tokens on
 * the tensor-core path; its first call sizes a workspace and must be outside
 * stream capture. */
FINCH_API int finch_encode_moe_prefill(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer,
                                       const void *h_post, const int32_t *expert_ids, const float *weights,
                                       const uint8_t *valid, const finch_shared *shared, const float *h_mid,
                                       float *hidden_out, int T);

/* Host-pointer form of the two calls above (copies in, runs, copies out,
 * waits): what a caller holding CPU buffers uses, as the reference's
 * gpu_gguf_experts_forward does (finchmoe/infer.m:3153-3366).  A decode-sized
 * call (T * top_k <= FINCH_MAX_PAIRS) stages the caller's buffers in pinned
 * memory that the kernels read and write in place (no copy operations on the
 * stream); larger calls copy through device memory.  FINCH_HOST_PATH=0 in the
 * environment forces the copies. */
FINCH_API int finch_moe_forward_host(finch_ctx *ctx, finch_pool *pool, int layer, const void *h_post,
                                     const int32_t *expert_ids, const float *weights, const uint8_t *valid,
                                     const finch_shared *shared, const float *shared_gate_score_host,
                                     const float *h_mid, float *hidden_out, int T);

/* [cmd commit] / waitUntilCompleted / complete_deferred_experts
 * (finchmoe/infer.m:9741, 7437-7454). */
FINCH_API int finch_event_create(finch_ctx *ctx, finch_event **out);
FINCH_API int finch_event_record(finch_event *ev, finch_stream stream);
FINCH_API int finch_event_wait(finch_event *ev, int timeout_ms); /* FINCH_E_TIMEOUT if not done in time */
FINCH_API void finch_event_destroy(finch_event *ev);
FINCH_API int finch_sync(finch_ctx *ctx);
/* Sticky device-side status (bounded waits inside kernels); 0 when clean.  Synchronises with the
 * work already queued.  finch_device_status_clear puts it back to 0 after the caller has dealt
 * with a failure (the reference's analogue is discard_deferred_experts, finchmoe/infer.m:7448-7454). */
FINCH_API int finch_device_status(finch_ctx *ctx, int *status_out);
FINCH_API int finch_device_status_clear(finch_ctx *ctx);

/* --compare-experts (finchmoe/infer.m:9766): the bit-exactness probe.  Writes,
 * for a weight tensor, the unpacked integer codes [out][in] (u8), the fp32
 * dequantized weights fl32(fl32(q*s)+b) and their round-to-nearest-even 16-bit
 * image in w16_dtype (FINCH_BF16 / FINCH_FP16).  Outputs are HOST pointers; any
 * may be NULL. */
FINCH_API int finch_debug_dequant(finch_ctx *ctx, const finch_wdesc *w, uint8_t *codes, float *w_f32,
                                  uint16_t *w16, int w16_dtype);

/* --timing / LayerTimingAccum (finchmoe/infer.m:281-299): while enabled, every
 * finch_encode_moe_decode call records CUDA events around its two kernels on
 * the launching stream; read() waits, returns the summed milliseconds of the
 * gate/up/SiLU kernels, of the down+combine kernels and the number of calls,
 * and resets the accumulators. */
FINCH_API int finch_profile_enable(finch_ctx *ctx, int on);
FINCH_API int finch_profile_read(finch_ctx *ctx, float *ms_gateup, float *ms_down_combine, int *n_calls);

/* Path selection of finch_encode_moe_prefill: 0 = by chunk length (default:
 * chunks of 80 tokens and more as mode 3, shorter ones as mode 1), 1 = always the
 * sub-batch path through the decode kernels, 2 = the routed experts as two grouped
 * dequant-GEMMs on tcgen05 (best when experts see 64 tokens and more, e.g. the rows
 * an expert-parallel rank receives), 3 = the routed experts as grouped mma.sync
 * passes that unpack a unit of codes once for up to 16 tokens of its expert (best at
 * the few tokens per expert of an ordinary chunk), 4 = the routed experts as two
 * grouped tcgen05 GEMMs that take the packed codes themselves as the A operand (a
 * masked code is an fp16 subnormal; nothing is dequantised, each scale group is
 * accumulated in tensor memory and folded with its scale and bias by the warps that
 * unpack the next one; measured level with modes 2 and 3, not chosen by mode 0).
 * In modes 2, 3 and 4 the shared expert runs as dense tcgen05 GEMMs.  The reference
 * has one path only (per-position CMD3). */
FINCH_API int finch_set_prefill_mode(finch_ctx *ctx, int mode);

/* Tokens per pass of the tensor-core path of finch_encode_moe_prefill (the
 * reference's chunk length, PREFILL_CHUNK in finchmoe/infer.m:12892-12902, is the
 * caller's T; this bounds how many of them share one sort and one pair of
 * grouped GEMMs).  0 = the default 512; at most max_tokens.  An expert-parallel
 * rank, whose rows each select few local experts, raises it so that a pass
 * still carries a few thousand (token, expert) pairs. */
FINCH_API int finch_set_prefill_chunk(finch_ctx *ctx, int tokens);

/* gpu_encode_prefill_matvec (finchmoe/infer.m:3672) for M >= 16 positions and a
 * 4-bit g64 tensor: out fp32 [M][out_dim] = x * dequant(w)^T on the tensor
 * cores; x is bf16 [M][in_dim] on the device, in_dim and out_dim multiples of
 * 128.  Weights are rounded to bf16 after the exact dequantisation. */
FINCH_API int finch_encode_dense_gemm(finch_ctx *ctx, finch_stream stream, const finch_wdesc *w, const void *x_bf16,
                                      float *out, int M);

/* gpu_gguf_experts_forward (finchmoe/infer.m:3153-3366; GgufExpertInfo 1017-1021): the K selected experts
 * of each of B tokens straight from the stacked GGUF slabs ffn_{gate,up,down}_exps (device copies; expert e of a
 * tensor starts at base + e * slab), types FINCH_BITS_Q4_K / FINCH_BITS_Q6_K.  hidden_out[b] = h_mid[b] (or 0) +
 * sum_k w_k * out_k over the experts whose output energy is finite and < 1e20, renormalised by the accepted
 * weight when that lies in (0, 0.99) -- the reference's guarded combine (infer.m:3334-3347).  No shared expert
 * here: the reference's GGUF path adds it in the caller.  The first call allocates scratch (outside capture).
 * B <= 8 runs token by token; a chunk of B >= 9 tokens (prefill) sorts its (token, expert) pairs by expert and
 * reads every selected expert's rows once for all the tokens that chose it (the reference's pool de-duplication,
 * infer.m:12424-12532; fused_gate_up_swiglu_qk_pool_prefill / dequant_matvec_qk_pool_prefill,
 * finchmoe/shaders.metal:3460-3517, 3641-3712), on the tensor cores. */
typedef struct finch_gguf_experts {
    const void *gate, *up, *down;
    size_t gate_slab, up_slab, down_slab;
    int gate_type, up_type, down_type;
} finch_gguf_experts;
FINCH_API int finch_encode_moe_gguf(finch_ctx *ctx, finch_stream stream, const finch_gguf_experts *experts, const void *h_post,
                                    const int32_t *expert_ids, const float *weights, const uint8_t *valid, const float *h_mid,
                                    float *hidden_out, int B);

/* ---- expert parallelism (no counterpart in the reference, which runs on one
 * device; extends the per-layer CMD3 of finchmoe/infer.m:9597-9741 across GPUs).
 * Rank r of `world` owns experts [r*E/world, (r+1)*E/world) of every layer and
 * keeps only those in its pool; tokens stay with their owner.  The host layer
 * (finchmoe_b200/ep.py) runs, per layer: plan -> pack -> all-to-all (NCCL) ->
 * unpack -> finch_encode_moe_prefill on the received rows (experts that are not
 * in the pool are skipped, so the result is the weighted sum over the local
 * experts) -> all-to-all back -> combine.  All pointers are device pointers. */

/* Bytes of one dispatch record: activation row, K ids, K weights, K mask bytes, padded to 16. */
FINCH_API int finch_ep_record_bytes(const finch_ctx *ctx);
/* counts[world], offs[world + 1] (exclusive prefix), send_tok[<= T * world] (tokens per
 * destination, ascending), slot_of[T][world] (position of token t in destination d's list, or -1).
 * A token goes to a rank once, however many of its experts live there.  Nothing goes to skip_rank
 * (its counts entry is 0, its slot_of column -1): the calling rank's own index when it runs its own
 * experts on its own tokens in place (finch_encode_moe_prefill on its pool), else -1. */
FINCH_API int finch_encode_ep_plan(finch_ctx *ctx, finch_stream stream, const int32_t *expert_ids, const uint8_t *valid,
                                   int T, int world, int skip_rank, int *counts, int *offs, int *send_tok, int *slot_of);
FINCH_API int finch_encode_ep_pack(finch_ctx *ctx, finch_stream stream, const void *h_post, const int32_t *expert_ids,
                                   const float *weights, const uint8_t *valid, int T, int world, const int *offs,
                                   const int *send_tok, void *records);
FINCH_API int finch_encode_ep_unpack(finch_ctx *ctx, finch_stream stream, const void *records, int n, void *h_post,
                                     int32_t *expert_ids, float *weights, uint8_t *valid);
/* hidden_out[t] += sum over destinations d in ascending order of back_rows[offs[d] + slot_of[t][d]]. */
FINCH_API int finch_encode_ep_combine(finch_ctx *ctx, finch_stream stream, float *hidden_out, const float *back_rows,
                                      const int *slot_of, const int *offs, int T, int world);
/* n_batches independent decode-sized batches of B tokens (B <= 8, B * top_k <= FINCH_MAX_PAIRS,
 * n_batches <= 16, n_batches * B <= max_tokens) in one sequence of three launches: rows
 * [c * B, (c + 1) * B) of h_post / expert_ids / weights / valid are batch c, and the SMs are divided
 * among the batches.  Batch own_batch is finch_encode_moe_decode as it stands (h_mid, shared expert,
 * result in hidden_out [B][hidden]); every other batch gets the weighted sum over its usable routed
 * experts only, in rows_out[c * B + t] (row block own_batch of rows_out is not written).  This is the
 * per-layer call of an expert-parallel rank for decode: batch c holds the tokens of rank c, most of
 * whose experts are not in this rank's pool and are skipped. */
FINCH_API int finch_encode_moe_decode_multi(finch_ctx *ctx, finch_stream stream, finch_pool *pool, int layer, int n_batches, int B,
                                            const void *h_post, const int32_t *expert_ids, const float *weights,
                                            const uint8_t *valid, int own_batch, const finch_shared *shared, const float *h_mid,
                                            float *hidden_out, float *rows_out);

/* ---- the fixed-capacity exchange over NVLink peer memory (decode-sized batches: every rank owns
 * tokens_per_rank tokens and sends each to every rank).  The ranks' kernels store records and partial
 * rows into each other's receive areas, every payload word beside the sender's epoch (a per-rank
 * counter that combine advances once per layer), and the receiving kernels read until the words carry
 * the epoch they expect: no fence, no collective call and no host step per layer, so a layer is a
 * fixed sequence of launches that a CUDA graph can hold.  All ranks must issue the per-layer calls in
 * the same order the same number of times (combine included, also with one rank).  Setup, once:
 * every rank creates its area, exports a 64-byte handle, receives the other ranks' handles by whatever
 * channel the host has (the MPI / NCCL bootstrap, a file) and imports them.  Per layer, every rank, in
 * this order: dispatch -> receive -> finch_encode_moe_decode_multi on the world batches of received rows
 * (or: finch_encode_moe_decode on its own tokens, receive with mask_own, finch_encode_moe_prefill on the
 * received rows) -> return -> combine.
 * Every device-side wait is bounded: words that do not arrive record FINCH_E_TIMEOUT in the
 * device status word, the slot counts as empty and later waits no longer spin; the host then calls
 * finch_ep_peer_reset on every rank (after a barrier: it clears the area and restarts the epoch) or
 * falls back to the all-to-all steps above. */
typedef struct finch_ep_peer finch_ep_peer;
FINCH_API int finch_ep_peer_create(finch_ctx *ctx, int rank, int world, int tokens_per_rank, finch_ep_peer **out);
FINCH_API int finch_ep_peer_export(finch_ep_peer *peer, void *handle64);                        /* this rank's area, for the others */
FINCH_API int finch_ep_peer_import(finch_ep_peer *peer, int src_rank, const void *handle64);    /* another process's area */
FINCH_API void *finch_ep_peer_area(finch_ep_peer *peer);                                        /* device pointer of this rank's area */
FINCH_API int finch_ep_peer_attach(finch_ep_peer *peer, int src_rank, void *area);              /* an area of the same process */
FINCH_API int finch_ep_peer_set_wait_limit(finch_ep_peer *peer, long long polls);               /* ~100 ns each; default 4,000,000 */
FINCH_API int finch_ep_peer_reset(finch_ep_peer *peer);                                         /* waits for the device, clears the area, epoch = 1 */
FINCH_API int finch_ep_peer_destroy(finch_ep_peer *peer);
FINCH_API int finch_encode_ep_peer_dispatch(finch_ctx *ctx, finch_stream stream, finch_ep_peer *peer, const void *h_post,
                                            const int32_t *expert_ids, const float *weights, const uint8_t *valid);
/* Rows [world * tokens_per_rank] in source-rank order, this rank's own tokens among them (dispatch stores them into
 * its own area too).  mask_own != 0: the block of the rank's own tokens gets an all-zero mask (the caller has served
 * them in place); 0: it is an ordinary block, as finch_encode_moe_decode_multi wants it. */
FINCH_API int finch_encode_ep_peer_receive(finch_ctx *ctx, finch_stream stream, finch_ep_peer *peer, void *h_post,
                                           int32_t *expert_ids, float *weights, uint8_t *valid, int mask_own);
/* rows: fp32 [world * tokens_per_rank][hidden], block s = the partial sums of rank s's tokens. */
FINCH_API int finch_encode_ep_peer_return(finch_ctx *ctx, finch_stream stream, finch_ep_peer *peer, const float *rows);
/* The layer on this rank in ONE launch sequence over the rows of finch_encode_ep_peer_receive (mask_own = 0): batch c =
 * the tokens of rank c, served by the experts held here; the rank's own batch also gets h_mid and the shared expert and
 * lands in hidden_out; the last kernel of the sequence stores the other batches' rows straight into their ranks' areas
 * (the return step fused into the compute: no finch_encode_ep_peer_return, no local array of rows).  tokens_per_rank
 * <= 8 and tokens_per_rank * top_k <= 64, as finch_encode_moe_decode_multi wants.  Then finch_encode_ep_peer_combine. */
FINCH_API int finch_encode_ep_peer_decode(finch_ctx *ctx, finch_stream stream, finch_ep_peer *peer, finch_pool *pool, int layer, const void *rows_h_post,
                                          const int32_t *rows_expert_ids, const float *rows_weights, const uint8_t *rows_valid,
                                          const finch_shared *shared, const float *h_mid, float *hidden_out);
/* hidden_out[t] += the other ranks' partial rows of token t, in ascending rank order. */
FINCH_API int finch_encode_ep_peer_combine(finch_ctx *ctx, finch_stream stream, finch_ep_peer *peer, float *hidden_out);

/* Synthetic contents for one shard: experts [e0, e1) of layers [layer0, layer1) get the bytes
 * finch_pool_fill_synthetic gives them in a full pool; the pool needs n_layers * (e1 - e0) slots. */
FINCH_API int finch_pool_fill_synthetic_range(finch_pool *pool, int layer0, int layer1, int e0, int e1, uint64_t seed);

/* Failure injection for tests of the bounded device-side waits (no counterpart in the reference;
 * its waits are Metal's waitUntilCompleted, finchmoe/infer.m:7437-7454).  kind 1: in the following
 * finch_encode_moe_decode calls the warp of the gate/up kernel that owns the first piece of the
 * first tile withholds its first weight fetch
 * and every wait of that kernel gives up after microseconds instead of a fraction of a second.
 * The warps that wait in vain record FINCH_E_TIMEOUT in the device status word
 * (finch_device_status) and return; nothing faults, spins for long or is left in flight, and the
 * call's output is undefined.  kind 0 switches it off. */
FINCH_API int finch_debug_fault(finch_ctx *ctx, int kind);

/* Count of kernels launched by this context since creation (benchmark bookkeeping). */
FINCH_API uint64_t finch_launch_count(const finch_ctx *ctx);

#ifdef __cplusplus
}
#endif
#endif /* FINCH_CUDA_H */
