/*
 * tsugumi_cuda.h -- C ABI of libtsugumi_cuda.so, the B200 (sm_100a)
 * implementation of Tsugumi's MoE feed-forward block.
 *
 * The reference exposes this path as Swift encoder classes that encode into a
 * caller-owned MTLCommandBuffer (Sources/Tsugumi/Kernels/MoE/MoE.swift,
 * Sources/Tsugumi/Kernels/Prefill/MoE/*.swift).  Here every entry point
 * enqueues CUDA work on the context's stream and returns a tsg_status; nothing
 * aborts and no C++ exception crosses the boundary.  All tensor arguments are
 * device pointers owned by the caller; sizes are element counts unless named
 * *_bytes.  A context is not internally synchronised: use one per host
 * thread / stream (the reference's kernel objects are likewise not Sendable,
 * MoE.swift:505-512).
 *
 * Weight format (per expert blob, offsets in tsg_expert_offsets):
 *   gate codes [F][D/2] u8, gate scales [F][D/32] fp16, up codes, up scales,
 *   down codes [D][F/2] u8, down scales [D][F/32] fp16;
 *   int4 symmetric: w = s * (q - 8), low nibble = even element, group 32.
 * Activations are bf16; router weights fp32 [E][D].
 */
#ifndef TSUGUMI_CUDA_H
#define TSUGUMI_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TSG_ABI_VERSION 1

#if defined(__GNUC__)
#define TSG_API __attribute__((visibility("default")))
#else
#define TSG_API
#endif

/* Replaces the reference's three error channels (MoE.swift:31-40 typed
 * throws, precondition traps, "declined" return values) and
 * MetalContext.checkCommandBufferError (MetalContext.swift:40-45). */
typedef enum tsg_status {
    TSG_OK = 0,
    TSG_ERR_INVALID_ARG = 1,       /* replaces precondition failures and argument throws */
    TSG_ERR_UNSUPPORTED_SHAPE = 2, /* replaces "path declined" returns */
    TSG_ERR_OOM = 3,
    TSG_ERR_CUDA = 4,              /* replaces commandBuffer.error */
    TSG_ERR_NCCL = 5,
    TSG_ERR_TIMEOUT = 6,           /* a bounded device-side wait ran out */
    TSG_ERR_METADATA = 7           /* routing metadata failed device-side validation */
} tsg_status;

typedef struct tsg_ctx_s *tsg_ctx;
typedef struct tsg_moe_layer_s *tsg_moe_layer;

/* MoEExpertOffsets (Sources/Tsugumi/Kernels/MoE/MoE.swift:4-29): byte offsets
 * of one expert's sub-tensors in its blob.  Bias offsets alias the scales for
 * the symmetric scheme (ModelExpertIO.swift:56-84) and are never read. */
typedef struct tsg_expert_offsets {
    uint32_t gate_w_off, gate_s_off, gate_b_off;
    uint32_t up_w_off, up_s_off, up_b_off;
    uint32_t down_w_off, down_s_off, down_b_off;
} tsg_expert_offsets;

/* PrefillTokenExpertPair (Sources/Tsugumi/Kernels/Prefill/MoE/PrefillRouter.swift:4-28):
 * 16 bytes, fields at offsets 0/4/8/12; the weight is fp16 bits in the low
 * half of the last word. */
typedef struct tsg_token_expert_pair {
    uint32_t token, expert, rank, weight_bits_and_reserved;
} tsg_token_expert_pair;

/* PrefillMoEGroup / PrefillMoETile (PrefillMoEGrouping.swift:4-30). */
typedef struct tsg_moe_group {
    uint32_t expert, pair_start, pair_count;
} tsg_moe_group;

typedef struct tsg_moe_tile {
    uint32_t group_start, group_count, pair_start, pair_count;
} tsg_moe_tile;

/* PrefillRoutedGEMMBlock (PrefillGroupedRoutedMoE.swift:20-25). */
typedef struct tsg_routed_gemm_block {
    uint32_t local_slot, pair_start, row_count, local_row;
} tsg_routed_gemm_block;

/* MoE.GateActivation (MoE.swift:100-121). */
typedef enum tsg_gate_activation {
    TSG_ACT_GELU_PYTORCH_TANH = 0, /* Gemma 4 (GeGLU) */
    TSG_ACT_SILU = 1               /* Qwen3.5-MoE (SwiGLU) */
} tsg_gate_activation;

typedef enum tsg_dtype { TSG_DTYPE_BF16 = 0, TSG_DTYPE_F32 = 1, TSG_DTYPE_F16 = 2 } tsg_dtype;

/* One MoE layer's resident weights.  Replaces the per-layer state the Swift
 * runners hold (RealForwardRunner.swift:542-566 effective scale,
 * ModelExpertIO.routedExpertOffsets, QwenForwardRunner MoEWeights).  All
 * pointers are device pointers and must stay valid for the layer's life. */
typedef struct tsg_moe_layer_desc {
    uint32_t d;               /* hidden size, multiple of 256 */
    uint32_t f;               /* expert FFN width, multiple of 64 */
    uint32_t num_experts;     /* <= 512 */
    uint32_t top_k;           /* 1..32, <= num_experts */
    uint32_t group_size;      /* must be 32 */
    tsg_gate_activation activation;
    const void *experts;      /* expert 0's blob; blobs expert_stride bytes apart */
    uint64_t expert_stride;   /* multiple of 16 */
    tsg_expert_offsets offsets;
    const float *router_weight;    /* [E][D] */
    const float *effective_scale;  /* [D] or NULL; folded into the router rows */
    const float *per_expert_scale; /* [E] or NULL */
    const float *logit_bias;       /* [E] or NULL (routing-skew experiments) */
    uint32_t router_norm;          /* 1: no-scale RMSNorm of the block input */
    float norm_eps;
    const void *shared_expert;     /* optional shared expert blob, NULL if none */
    uint32_t shared_f;             /* its intermediate width (multiple of 64): equal to f,
                                      a shared expert (a slot of the routed kernels);
                                      else a dense branch (Gemma's dense MLP,
                                      SharedExpertInt4.swift:30-94), run beside the
                                      routed experts and added: y = residual + dense(x)
                                      + sum_r w_r expert_r(x) */
    tsg_expert_offsets shared_offsets;
    const float *shared_gate;      /* [D] sigmoid gate vector, or NULL (shared_f == f only) */
} tsg_moe_layer_desc;

/* ---- context (MetalContext analogue, Infrastructure/Metal/MetalContext.swift) ---- */
TSG_API int tsg_abi_version(void);
/* stream: a cudaStream_t, or NULL for the legacy default stream. */
TSG_API tsg_status tsg_ctx_create(int device, void *stream, tsg_ctx *out);
TSG_API tsg_status tsg_ctx_destroy(tsg_ctx ctx);
TSG_API tsg_status tsg_ctx_set_stream(tsg_ctx ctx, void *stream);
/* Largest T handled by the decode regime; default 3 (the single streaming
 * kernel; at most 4).  Larger T goes to the batched GEMVs (up to
 * "gemv_max_tokens") or the grouped tcgen05 contraction. */
TSG_API tsg_status tsg_ctx_set_decode_max_tokens(tsg_ctx ctx, uint32_t t);
/* Tuning switches: "fused_decode" (1: T <= 4 runs the whole block as one
 * cooperative kernel, default; 0: router / gate-up / down kernels) and
 * "programmatic_launch" (1, the default: a decode kernel lets the next
 * one on the stream launch early and start its input-independent prologue
 * as each SM frees up; 0: plain stream order), "cooperative_launch" (1, the
 * default: decode kernels are launched cooperatively, so the driver checks
 * that all their CTAs are resident at once; 0 launches them plainly -- one
 * CTA per SM on an otherwise idle GPU, every cross-CTA wait bounded -- which
 * lets a programmatic launch start the next layer's CTAs as this one's exit,
 * ~3 µs per layer less between eagerly launched layers; no change inside a
 * CUDA graph), "gemv_max_tokens" (router-driven batches above
 * decode_max_tokens and up to this size, at most 64, run the expert products
 * as batched GEMVs; default 16, 0 for the tensor-core contraction only) and
 * "debug_phase_stamps" (a device address of num_sms x 96 uint64 the
 * streaming decode kernel fills with %globaltimer stamps at its phase
 * boundaries, or 0 for none; only a library built with
 * TSG_NVCC_DEFINES="-DTSG_PHASE_STAMPS=1" has the stamping code), "ep_transport" (expert
 * parallelism: 1, the default, moves rows through peer memory; 0 through
 * NCCL all-to-all; every rank of a group sets the same value) and
 * "ep_return" (peer transport: 1, the default, runs the down contraction in
 * one chunk per source rank and copies each finished chunk to its rank with
 * the copy engines while the next computes; 0 lets the contraction's
 * epilogue store the rows into the peers' buffers) and "ep_dispatch" (peer
 * transport, every rank alike: 0, the default, lets the dispatch kernel
 * store the token rows into the owners' buffers; 1 converts the rows for
 * each remote owner into one local run and sends it with the copy engines). */
TSG_API tsg_status tsg_ctx_set_option(tsg_ctx ctx, const char *name, int64_t value);
/* Pre-allocates the workspace for up to max_tokens tokens of this layer's
 * shape, so later calls allocate nothing (required before stream capture). */
TSG_API tsg_status tsg_ctx_reserve(tsg_ctx ctx, tsg_moe_layer layer, uint32_t max_tokens);
/* Waits for the stream, then reports device-side errors (bounded-wait
 * timeouts, metadata validation) and clears them. */
TSG_API tsg_status tsg_sync(tsg_ctx ctx);
TSG_API const char *tsg_last_error_string(tsg_ctx ctx);

/* ---- layers ----
 * A layer must be destroyed before its context is used with another device;
 * destroying the context first is allowed (the layer then only frees its own
 * router copy). */
TSG_API tsg_status tsg_moe_layer_create(tsg_ctx ctx, const tsg_moe_layer_desc *desc, tsg_moe_layer *out);
TSG_API tsg_status tsg_moe_layer_destroy(tsg_moe_layer layer);

/* ---- the block, and its stages ---- */

/* Whole MoE block: router, permutation, routed experts, shared expert,
 * combine; picks the decode regime for T <= decode_max_tokens, else prefill.
 * y[t] = residual[t] + shared(t) + sum_r w[t,r] * expert_{id[t,r]}(x[t]).
 * Replaces the per-layer sequences in RealForwardRunner.swift:3079-3330
 * (decode), :1840-2640 (prefill) and QwenForwardRunner.swift:1460-1612. */
TSG_API tsg_status tsg_moe_block_forward(tsg_ctx ctx, tsg_moe_layer layer, const void *hidden_bf16,
                                 uint32_t hidden_stride, uint32_t T, const float *residual_f32,
                                 void *y, uint32_t y_stride, tsg_dtype y_dtype);

/* A speculative-verify block of T rows, each row's y bit for bit what
 * tsg_moe_block_forward gives that row alone in the decode regime (T = 1):
 * "a verify block is decode generalized to k rows".  Replaces
 * PrefillGroupedRoutedMoE.encodeStreamedRows / usesExpertRowsPath
 * (PrefillGroupedRoutedMoE.swift:768-800), whose contract is pinned by
 * PrefillRoutedMoERowsVsDecodeTests.swift:23-166.  Runs the streaming decode
 * kernel on the rows two at a time; TSG_ERR_UNSUPPORTED_SHAPE when that
 * kernel does not take the layer (or option fused_decode is not 1).
 * Arguments as tsg_moe_block_forward. */
TSG_API tsg_status tsg_moe_verify_rows_forward(tsg_ctx ctx, tsg_moe_layer layer, const void *hidden_bf16,
                                       uint32_t hidden_stride, uint32_t T, const float *residual_f32,
                                       void *y, uint32_t y_stride, tsg_dtype y_dtype);

/* Router + top-K.  Replaces MoE.encodeRouterGemma4BF16 (MoE.swift:259-302),
 * encodeRouterGemma4BF16Rows (:413-466), PrefillRouter.encodeGemma4BF16Block
 * and encodeGemma4BF16GEMM (PrefillRouter.swift:127-236).  Outputs [T][K]:
 * expert ids, fp32 weights, and optionally fp16 weights (the reference's
 * output type). */
TSG_API tsg_status tsg_router_topk(tsg_ctx ctx, tsg_moe_layer layer, const void *hidden_bf16,
                           uint32_t hidden_stride, uint32_t T, uint32_t *out_indices,
                           float *out_weights, uint16_t *out_weights_f16);

/* The router's GEMV alone, with no selection behind it.  Replaces
 * MoE.encodeRouterLogitsBF16 (MoE.swift:316-345).  out_logits [T][E] fp32
 * (device) receives exactly the scores tsg_router_topk ranks: the dot of the
 * layer's router row (effective scale folded in) with the hidden row, times
 * the row's no-scale RMSNorm factor when the layer normalises its input,
 * plus the layer's logit bias when it has one. */
TSG_API tsg_status tsg_router_logits(tsg_ctx ctx, tsg_moe_layer layer, const void *hidden_bf16,
                             uint32_t hidden_stride, uint32_t T, float *out_logits);

/* PrefillRouter.makeTokenExpertPairs (PrefillRouter.swift:238-258), on device. */
TSG_API tsg_status tsg_make_token_expert_pairs(tsg_ctx ctx, const uint32_t *indices,
                                       const uint16_t *weights_f16, uint32_t T, uint32_t K,
                                       tsg_token_expert_pair *out_pairs);

/* PrefillMoEGrouping.groupTokenExpertPairs (PrefillMoEGrouping.swift:91-201),
 * on device.  pairs may be in any order; sort_keys (device, [num_experts]) may
 * be NULL; tile_break_after_group < 0 means none.  Argument errors return
 * TSG_ERR_INVALID_ARG at once; per-pair errors (token/rank/expert out of
 * range, duplicate token+rank) are reported by tsg_sync as TSG_ERR_METADATA.
 * Outputs are device arrays: sorted_pairs [n_pairs], offsets/counts
 * [num_experts] (offset 0xFFFFFFFF when empty), groups [num_experts],
 * n_groups [1], tiles [num_experts], n_tiles [1]. */
TSG_API tsg_status tsg_moe_group_pairs(tsg_ctx ctx, const tsg_token_expert_pair *pairs, uint32_t n_pairs,
                               int32_t query_count, int32_t top_k, int32_t num_experts,
                               int32_t tile_expert_count, const uint64_t *sort_keys,
                               int32_t n_sort_keys, int32_t tile_break_after_group,
                               tsg_token_expert_pair *sorted_pairs, uint32_t *per_expert_offsets,
                               uint32_t *per_expert_counts, tsg_moe_group *groups,
                               uint32_t *n_groups, tsg_moe_tile *tiles, uint32_t *n_tiles);

/* No counterpart in the reference.  Same arguments, checks and outputs as
 * tsg_moe_group_pairs, but the call allocates no device memory: the
 * permutation's scratch (token-major ids and fp16 weights, the per-slot
 * occupancy flags that share the sorted positions' space, the row-tile
 * schedule and the per-chunk expert histograms)
 * lives in one fixed static device array of
 * TSG_GROUP_NOALLOC_SCRATCH_BYTES inside this library, instead of the
 * context's workspace, which tsg_moe_group_pairs may grow with cudaMalloc.
 * It is for hosts that must not allocate from inside their enqueue path:
 * a runtime that has reserved its device memory up front, or one for which
 * the device-wide synchronisation of cudaFree would stall other streams.
 * Limits: n_pairs <= TSG_GROUP_NOALLOC_MAX_PAIRS and num_experts <= 512;
 * larger calls return TSG_ERR_UNSUPPORTED_SHAPE with a message naming the
 * limit, before any work is enqueued.
 * - The first call on each device resolves the array's address for that
 *   device (cudaGetSymbolAddress, with the context's device current); make
 *   that first call before recording the context's stream into anything.
 *   After a cudaDeviceReset the next call resolves it again, so that call,
 *   too, must come before any stream capture.
 * - Nothing in the array has to start at zero: each call clears the
 *   occupancy flags itself (an async memset on the stream) and writes every
 *   other word it reads before reading it.
 * - The array is shared by every caller on a device: two calls whose work
 *   can overlap on the GPU (different streams, or different contexts of the
 *   same device, without an ordering between them) race on it and corrupt
 *   each other's results.  Order such calls, or use tsg_moe_group_pairs. */
#define TSG_GROUP_NOALLOC_MAX_PAIRS 65536u
#define TSG_GROUP_NOALLOC_SCRATCH_BYTES (1u << 20)
TSG_API tsg_status tsg_moe_group_pairs_noalloc(
    tsg_ctx ctx, const tsg_token_expert_pair *pairs, uint32_t n_pairs, int32_t query_count,
    int32_t top_k, int32_t num_experts, int32_t tile_expert_count, const uint64_t *sort_keys,
    int32_t n_sort_keys, int32_t tile_break_after_group, tsg_token_expert_pair *sorted_pairs,
    uint32_t *per_expert_offsets, uint32_t *per_expert_counts, tsg_moe_group *groups,
    uint32_t *n_groups, tsg_moe_tile *tiles, uint32_t *n_tiles);

/* PrefillRoutedGEMMPlanner.plan (PrefillGroupedRoutedMoE.swift:42-83), host
 * function on host arrays.  Writes up to max_blocks blocks and up to
 * max_batches batches (rows, first block, block count); returns
 * TSG_ERR_INVALID_ARG when the capacity is too small. */
TSG_API tsg_status tsg_plan_routed_gemm(const tsg_moe_group *groups, uint32_t n_groups,
                                uint32_t max_rows_per_batch, uint32_t tile_rows,
                                tsg_routed_gemm_block *blocks, uint32_t max_blocks,
                                uint32_t *n_blocks, uint32_t *batch_rows,
                                uint32_t *batch_first_block, uint32_t *batch_block_count,
                                uint32_t max_batches, uint32_t *n_batches);

/* Routed experts for caller-supplied routing, decode regime (batched GEMV).
 * Replaces MoE.encodeRoutedPersistentPhase1U16Load + Phase2Reduce
 * (MoE.swift:529-644): y = residual + (shared) + sum_r w * expert(x). */
TSG_API tsg_status tsg_moe_experts_decode(tsg_ctx ctx, tsg_moe_layer layer, const void *x_bf16,
                                  uint32_t x_stride, uint32_t T, const uint32_t *indices,
                                  const float *weights, const float *residual_f32, void *y,
                                  uint32_t y_stride, tsg_dtype y_dtype);

/* Routed experts for caller-supplied routing, prefill regime (grouped tcgen05
 * contraction).  Replaces PrefillGroupedRoutedMoE.encodeStreamedTiled
 * (PrefillGroupedRoutedMoE.swift:931-1051) + PrefillMoE.encodeReduceTokenMajor. */
TSG_API tsg_status tsg_moe_experts_prefill(tsg_ctx ctx, tsg_moe_layer layer, const void *x_bf16,
                                   uint32_t x_stride, uint32_t T, const uint32_t *indices,
                                   const float *weights, const float *residual_f32, void *y,
                                   uint32_t y_stride, tsg_dtype y_dtype);

/* prefill_moe_reduce_token_major (prefill.metal:796-817) via
 * PrefillMoE.encodeReduceTokenMajor (PrefillMoE.swift:11-39):
 * h2[t][d] = sum_r fma(w[t][r], partials[(t*K + r)*D + d]); partials fp16. */
TSG_API tsg_status tsg_moe_reduce_token_major(tsg_ctx ctx, const uint16_t *partials_f16,
                                      const float *weights, uint32_t T, uint32_t K, uint32_t D,
                                      void *h2, tsg_dtype h2_dtype);

/* Shared-expert branch alone, with its sigmoid gate when the layer has one.
 * Replaces SharedExpertRuntime.encode (SharedExpertInt4.swift:115-136),
 * PrefillSharedExpert.encodeBlock (PrefillSharedExpert.swift:44-272) and
 * QwenKernels.encodeMoESharedGate(Logit) (QwenKernels.swift:311-355). */
TSG_API tsg_status tsg_shared_expert(tsg_ctx ctx, tsg_moe_layer layer, const void *x_bf16,
                             uint32_t x_stride, uint32_t T, void *y, uint32_t y_stride,
                             tsg_dtype y_dtype);

/* The norm weights around Gemma's MoE block (BF16 [D] each; RMSNorm is
 * x * rsqrt(mean(x^2) + eps) * w), as fused_post_attn_setup and
 * fused_layer_tail (fused.metal:190-374) and the dense branch's post-norm
 * (RealForwardRunner.swift:3236-3242) take them. */
typedef struct {
    const uint16_t *post_attn;    /* norm of the attention output */
    const uint16_t *pre_ffn;      /* the dense branch's input norm */
    const uint16_t *pre_ffn2;     /* the routed experts' input norm */
    const uint16_t *post_dense;   /* the dense branch's output norm */
    const uint16_t *post_routed;  /* the routed output's norm */
    const uint16_t *post_ffn;     /* the summed branches' norm */
    float eps;
    float layer_scalar;
} tsg_gemma_norms;

/* Gemma's layer FFN with the adjacent norms and residuals fused, per token
 * (bf16 activations, rounded where the reference rounds to fp16):
 *   h       = hidden + norm(attn, post_attn)          (hidden updated)
 *   x^      = h * rsqrt(mean(h^2) + eps)
 *   d       = norm(dense(x^ * pre_ffn), post_dense)     (the dense branch)
 *   r       = norm(moe(route: x^, experts: x^ * pre_ffn2), post_routed)
 *   hidden  = (h + norm(d + r, post_ffn)) * layer_scalar
 * Replaces fused_post_attn_setup / fused_layer_tail (fused.metal:190-374)
 * and the sequence around them in RealForwardRunner.swift:3079-3330.  The
 * layer is created with router_norm = 0 and a dense branch
 * (shared_f != f; without one d = 0). */
TSG_API tsg_status tsg_gemma_ffn_forward(tsg_ctx ctx, tsg_moe_layer layer, const tsg_gemma_norms *norms,
                                 void *hidden_bf16, uint32_t hidden_stride,
                                 const void *attn_bf16, uint32_t attn_stride, uint32_t T);

/* Import of one int4 projection of a .moepack expert blob
 * (MoEPackPackedExpertsLayoutV1.swift:3-212; sub-tensors "gate", "gate_scales",
 * "gate_biases", ... as ModelExpertIO.swift:55-84 reads them) into this
 * library's expert layout, on the device.  In: codes_u32 [rows][cols/8] U32
 * words (MLX affine packing), scales_bf16 [rows][cols/group_size] BF16 bits,
 * biases_bf16 (same shape) or NULL for a `sym` blob.  Out: out_codes
 * [rows][cols/2] bytes and out_scales_f16 [rows][cols/32] (the layout of
 * tsg_expert_offsets).  Exact or fails: each BF16 scale must be an fp16 value,
 * a group of group_size > 32 gives its scale to each of its 32-groups, and
 * biases when given must be -8 x scale as BF16 bits (MoEPackAffineV1.swift:
 * 14-26); a failure is reported by tsg_sync as TSG_ERR_METADATA.  Device
 * pointers; codes 16-byte aligned. */
TSG_API tsg_status tsg_import_int4_affine(tsg_ctx ctx, const void *codes_u32,
                                  const uint16_t *scales_bf16, const uint16_t *biases_bf16,
                                  uint32_t rows, uint32_t cols, uint32_t group_size,
                                  void *out_codes, uint16_t *out_scales_f16);

/* Stage timing, the analogue of PrefillGPUProfile
 * (Runtime/Prefill/PrefillGPUProfile.swift:1-40): between begin and end,
 * every tsg_moe_block_forward records CUDA events on the context's stream at
 * its stage boundaries (also inside a captured CUDA graph, where the events
 * become graph nodes and are re-recorded by every replay).  end waits for
 * the stream and returns, summed over the recorded calls (at most
 * max_calls), the milliseconds of: [0] router + grouping, [1] gate/up,
 * [2] down (+ combine in the decode regime), [3] combine (prefill regime). */
TSG_API tsg_status tsg_ctx_profile_begin(tsg_ctx ctx, uint32_t max_calls);
TSG_API tsg_status tsg_ctx_profile_end(tsg_ctx ctx, float *stage_ms, uint32_t *n_calls);

/* Device-side scratch of the last forward, for tests and tooling: the routing
 * of the most recent call on this context (ids [T][K], fp32 weights [T][K],
 * sorted pairs [T*K]); valid until the next call. */
TSG_API tsg_status tsg_last_routing(tsg_ctx ctx, const uint32_t **ids, const float **weights,
                            const tsg_token_expert_pair **sorted_pairs, uint32_t *T,
                            uint32_t *K);

/* ---- Expert parallelism across the GPUs of one node ----------------------
 * No counterpart in the reference, which runs on one device: its per-layer
 * sequence (RealForwardRunner.swift:1840-2640 prefill) is kept on each rank,
 * with the experts split contiguously over R ranks.  Per layer, each rank
 * routes its own tokens, exchanges per-expert pair counts, sends each
 * normalised fp16 token row to the rank that owns its expert, runs the
 * grouped contraction on the rows it received (plus the shared expert on its
 * own tokens), returns the expert outputs and combines its tokens in rank
 * order -- the same arithmetic as one GPU, so the outputs are bit-equal.
 * With the peer transport (default, at most 16 ranks) a kernel stores each
 * token row once per owner rank straight into the owners' buffers over
 * NVLink (the owner expands them into pair rows), and the expert outputs
 * go back into the token's rank's buffer by copy engine, a chunk per source
 * rank as the down contraction finishes it (buffers mapped between the
 * processes with CUDA IPC); NCCL carries the counts and the barriers.  With "ep_transport" 0 NCCL all-to-all carries the rows.
 * NCCL (libnccl.so.2) is loaded when tsg_ep_init is first called. */
#define TSG_EP_UNIQUE_ID_BYTES 128

/* Writes a new NCCL unique id (TSG_EP_UNIQUE_ID_BYTES) on one rank; the
 * caller hands it to every rank (e.g. over its own process group). */
TSG_API tsg_status tsg_ep_unique_id(void *out_id);

/* Joins the expert-parallel group: rank in [0, world), on ctx's device. */
TSG_API tsg_status tsg_ep_init(tsg_ctx ctx, const void *unique_id, int rank, int world);

/* The MoE block of T local tokens under expert parallelism.  `layer` holds
 * this rank's experts: desc.num_experts is the global E (its router has all
 * E rows), desc.experts points at the blob of expert `expert_first` =
 * rank * E / world, and the blobs of the E / world local experts follow at
 * expert_stride.  E must be a multiple of world.  Every rank calls this
 * collectively, each with its own tokens (T may differ between ranks).
 * Synchronises the context's stream once (after the count exchange), and
 * again when an exchange buffer grows. */
TSG_API tsg_status tsg_ep_moe_block_forward(tsg_ctx ctx, tsg_moe_layer layer, uint32_t expert_first,
                                            const void *hidden_bf16, uint32_t hidden_stride,
                                            uint32_t T, const float *residual_f32, void *y,
                                            uint32_t y_stride, tsg_dtype y_dtype);

/* Device time, in ms, of the phases of this context's last peer-transport
 * tsg_ep_moe_block_forward (waits for it): [0] routing and sorting, [1] the
 * count exchange and the plan (host time included), [2] the row dispatch and
 * its barrier, [3] the expansion of received token rows into pair rows,
 * [4] the gate/up contraction, [5] the down contraction with the output
 * stores, [6] the return barrier, [7] the combine.  Writes min(n, 8)
 * values. */
TSG_API tsg_status tsg_ep_phase_ms(tsg_ctx ctx, float *ms, int n);

#ifdef __cplusplus
}
#endif

#endif /* TSUGUMI_CUDA_H */
