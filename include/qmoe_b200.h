/*
 * qmoe_b200.h -- C ABI of the B200 (sm_100a) 2-bit MoE layer.
 *
 * Drop-in boundary for qmoe-rs's MoE hot path.  Each entry point names the
 * qmoe-rs interface it replaces (paths relative to the qmoe-rs project root).
 * A Rust FFI crate binds these declarations one to one; qmoe-rs's public types
 * keep their signatures and call through them.
 *
 * Conventions
 *   - Every function returns QMOE_OK (0) or a QMOE_ERR_* code; no C++
 *     exception crosses the boundary.  qmoe_last_error() gives the calling
 *     thread's last message.
 *   - Plain pointers and sizes only.  `ptr_kind` says whether the data
 *     pointers of one call are host (QMOE_PTR_HOST) or device
 *     (QMOE_PTR_DEVICE) memory.  Host inputs are copied in and host outputs
 *     copied back on the context's stream (qmoe_layer_forward reads and
 *     writes page-locked host buffers in place instead, and replays the
 *     kernel sequence it captured on the previous call when x, out, T,
 *     dtype and path repeat and no routing is copied out; not on the
 *     legacy default stream), and the call returns after the results are
 *     in host memory.  Device calls are
 *     asynchronous on that stream.
 *   - Packed weights use qmoe-rs's layout verbatim (quantize.py:7-33,
 *     src/tensor.rs:16-23): uint8 [out, in/4], four 2-bit codes per byte,
 *     weight j of each group of four in bits 2j..2j+1, value = code - 1
 *     (0,1,2,3 -> -1,0,+1,+2), one f32 scale per output row.
 *   - A context, and the packed tensors and layers made from it, belong to
 *     one device and one stream; use one per host thread.  Distinct contexts
 *     are independent and may be used concurrently.
 */
#ifndef QMOE_B200_H
#define QMOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMOE_ABI_VERSION 1

#if defined(__GNUC__)
#define QMOE_API __attribute__((visibility("default")))
#else
#define QMOE_API
#endif

/* status codes */
#define QMOE_OK 0
#define QMOE_ERR_INVALID 1     /* bad argument, shape or configuration */
#define QMOE_ERR_CUDA 2        /* a CUDA runtime call failed */
#define QMOE_ERR_UNSUPPORTED 3 /* valid for qmoe-rs but not handled here */
#define QMOE_ERR_NOMEM 4       /* device allocation failed */

/* pointer kinds */
#define QMOE_PTR_DEVICE 0
#define QMOE_PTR_HOST 1

/* activation dtypes */
#define QMOE_DTYPE_F32 0
#define QMOE_DTYPE_BF16 1

/* scoring functions */
#define QMOE_SCORING_SOFTMAX 0 /* qmoe-rs semantics (src/moe.rs:64-81) */
#define QMOE_SCORING_SIGMOID 1 /* DeepSeek-V3 style; not in qmoe-rs */

typedef struct qmoe_ctx qmoe_ctx;
typedef struct qmoe_packed qmoe_packed;
typedef struct qmoe_layer qmoe_layer;

/*
 * MoE layer configuration.  The first four fields are qmoe-rs's MoEConfig
 * (src/moe.rs:6-11).  The rest extend it; their defaults
 * (shared_intermediate_dim 0, scoring SOFTMAX, n_group 1, topk_group 1,
 * norm_topk_prob 0, routed_scaling_factor 1, has_bias 0) reproduce qmoe-rs:
 * softmax over all experts, first top_k of a stable descending sort by
 * logit, no renormalisation.
 */
typedef struct qmoe_moe_config {
    int32_t num_experts;
    int32_t top_k;
    int32_t hidden_dim;
    int32_t intermediate_dim;
    int32_t shared_intermediate_dim; /* merged shared-expert width; 0 = none */
    int32_t scoring;                 /* QMOE_SCORING_* */
    int32_t n_group;                 /* expert groups for group-limited top-k */
    int32_t topk_group;              /* groups kept per token */
    int32_t norm_topk_prob;          /* renormalise the top_k weights */
    float routed_scaling_factor;     /* multiplies the routed weights */
    int32_t has_bias;                /* per-expert selection bias (sigmoid) */
    int32_t reserved;                /* must be 0 */
} qmoe_moe_config;

/* One expert's three packed projections (qmoe-rs PackedExpert,
 * src/moe.rs:15-19).  gate/up are [I, H/4] bytes + [I] scales; down is
 * [H, I/4] bytes + [H] scales.  The same struct carries the shared expert
 * (src/model.rs:318-322) with I = shared_intermediate_dim. */
typedef struct qmoe_expert_weights {
    const uint8_t *gate_packed;
    const float *gate_scales;
    const uint8_t *up_packed;
    const float *up_scales;
    const uint8_t *down_packed;
    const float *down_scales;
} qmoe_expert_weights;

/* ---- library --------------------------------------------------------- */

/* Last error message of the calling thread ("" if none). */
QMOE_API const char *qmoe_last_error(void);

/* QMOE_ABI_VERSION of the loaded library. */
QMOE_API int qmoe_abi_version(void);

/* ---- context ---------------------------------------------------------- */

/* Bind to CUDA device `device` and stream `stream` (a cudaStream_t; NULL =
 * the legacy default stream).  Fails with QMOE_ERR_UNSUPPORTED unless the
 * device is compute capability 10.0 (B200). */
QMOE_API int qmoe_ctx_create(int device, void *stream, qmoe_ctx **out);
QMOE_API int qmoe_ctx_destroy(qmoe_ctx *ctx);
/* Replace the stream later calls run on. */
QMOE_API int qmoe_ctx_set_stream(qmoe_ctx *ctx, void *stream);
/* Block until the context's stream is idle; reports asynchronous errors. */
QMOE_API int qmoe_ctx_synchronize(qmoe_ctx *ctx);

/* ---- packed tensor: PackedQMoETensor (src/tensor.rs:16-121) ------------ */

/* PackedQMoETensor::from_bytes (src/tensor.rs:47-53) and the data half of
 * ::mmap_from_file (:27-43): copy `packed` ([out_features, in_features/4]
 * bytes, in_features/4 rounded down as src/tensor.rs:74 does) and `scales`
 * ([out_features] f32) to device memory owned by the returned handle.  Any
 * positive in_features is accepted; rows whose width is not a multiple of 64
 * are kept padded with zero weights on the device (their activations are
 * staged into padded rows on each forward), and the in_features % 4
 * trailing activations of a row are never read (src/simd.rs:15). */
QMOE_API int qmoe_packed_create(qmoe_ctx *ctx, const uint8_t *packed, const float *scales,
                       int64_t out_features, int64_t in_features, int ptr_kind,
                       qmoe_packed **out);
QMOE_API int qmoe_packed_destroy(qmoe_packed *t);
/* Shape of the handle: PackedQMoETensor.shape (src/tensor.rs:20). */
QMOE_API int qmoe_packed_shape(const qmoe_packed *t, int64_t *out_features,
                      int64_t *in_features);

/* PackedQMoETensor::forward_simd / forward_simd_raw (src/tensor.rs:64-95,
 * :99-121): y[b, o] = scale[o] * sum_k (code[o,k] - 1) * x[b, k] for
 * x [batch, in_features] f32, y [batch, out_features] f32, k over the first
 * 4 * (in_features / 4) elements of a row.  Device x must be 16-byte aligned
 * when in_features is a multiple of 64. */
QMOE_API int qmoe_packed_forward(qmoe_packed *t, const float *x, int64_t batch, float *y,
                        int ptr_kind);

/* ---- packer: quantize.py (format producer) ----------------------------- */

/*
 * The offline quantizer of qmoe-rs on the device, bit for bit:
 * quantize_and_pack (quantize.py:7-33) with the row scale of the packing
 * loop (quantize.py:97-100).  w [out_features, in_features] f32, row-major
 * -> packed [out_features, in_features/4] bytes, code = clamp(round half to
 * even(w / scale), -1, 1) + 1, weight j of each group of four in bits
 * 2j..2j+1.  With scales_given == 0 the scales [out_features] f32 are
 * computed and written: max(unbiased std of the row, 1e-5)
 * (`tensor.std(dim=1)`, `torch.clamp(scale, min=1e-5)`); otherwise they are
 * read (`quantize_and_pack(weight, scale)`).  in_features must be a
 * positive multiple of 4 (the reference's assertion, quantize.py:26); device
 * w must be 16-byte aligned.  Host buffers (QMOE_PTR_HOST) are staged
 * through the device in row chunks; the call returns when they are written.
 */
QMOE_API int qmoe_quantize_pack(qmoe_ctx *ctx, const float *w, int64_t out_features,
                       int64_t in_features, float *scales, int scales_given,
                       uint8_t *packed, int ptr_kind);

/* ---- MoE layer: QMoELayer (src/moe.rs:23-130) + SharedExpert ----------- */

/*
 * QMoELayer::new (src/moe.rs:31-37) plus the layer's optional SharedExpert
 * (src/model.rs:318-348).
 *   gate_weight  [num_experts, hidden_dim] f32 (QMoELayer.gate_weight);
 *                may be NULL when expert_count is 0
 *   bias         [num_experts] f32 selection bias, or NULL (has_bias = 0)
 *   experts      expert_count entries: experts expert_begin ..
 *                expert_begin + expert_count - 1 (QMoELayer.experts).
 *                A single-process layer passes expert_begin = 0 and
 *                expert_count = num_experts; an expert-parallel rank passes
 *                the contiguous range it owns.  expert_count 0 is qmoe-rs's
 *                empty `experts` (src/moe.rs:46-48; a flattened layer,
 *                src/loader.rs:452-456): the forward is the shared expert
 *                alone, or zeros without one, and the routing outputs read
 *                -1 / 0; the routing entry points reject such a layer.
 *   shared       the shared expert, or NULL
 * All weight pointers are of `ptr_kind`; they are copied, not retained.
 */
QMOE_API int qmoe_layer_create(qmoe_ctx *ctx, const qmoe_moe_config *cfg,
                      const float *gate_weight, const float *bias,
                      const qmoe_expert_weights *experts, int32_t expert_begin,
                      int32_t expert_count, const qmoe_expert_weights *shared,
                      int ptr_kind, qmoe_layer **out);
QMOE_API int qmoe_layer_destroy(qmoe_layer *layer);

/* Pre-allocate the layer's device scratch for up to max_tokens tokens per
 * call, so later forwards allocate nothing (required before capturing a
 * forward into a CUDA graph).  Forwards grow the scratch on demand. */
QMOE_API int qmoe_layer_reserve(qmoe_layer *layer, int64_t max_tokens);

/*
 * The MoE block of a decoder layer without the residual: QMoELayer::forward
 * (src/moe.rs:40-130) followed by `moe_out + SharedExpert::forward`
 * (src/model.rs:386-389, :407-410).
 *   x        [T, hidden_dim], dtype QMOE_DTYPE_F32 or QMOE_DTYPE_BF16
 *   out      [T, hidden_dim], same dtype as x
 *   topk_idx optional [T, top_k] int32: selected experts, selection order
 *   topk_w   optional [T, top_k] f32: their combine weights
 * Requires expert_begin = 0 and expert_count = num_experts.
 */
QMOE_API int qmoe_layer_forward(qmoe_layer *layer, const void *x, int dtype, int64_t T,
                       void *out, int32_t *topk_idx, float *topk_w, int ptr_kind);

/* The router alone (src/moe.rs:51-82): gate logits, scoring, top-k and
 * combine weights for every token.  topk_idx [T, top_k] int32 and
 * topk_w [T, top_k] f32 are required. */
QMOE_API int qmoe_layer_route(qmoe_layer *layer, const void *x, int dtype, int64_t T,
                     int32_t *topk_idx, float *topk_w, int ptr_kind);

/*
 * Routed experts for rows whose routing is already known (the expert half of
 * src/moe.rs:84-129, run by an expert-parallel rank on the rows it
 * received).  topk_idx [R, top_k] holds LOCAL expert ids in
 * 0..expert_count-1, or -1 for a slot this rank does not own; topk_w the
 * matching weights.  out [R, hidden_dim] = sum over valid slots, in
 * ascending expert order, of w * expert(x).  No shared expert.
 */
QMOE_API int qmoe_layer_forward_routed(qmoe_layer *layer, const void *x, int dtype,
                              int64_t R, const int32_t *topk_idx,
                              const float *topk_w, void *out, int ptr_kind);

/* SharedExpert::forward (src/model.rs:325-347) for x [T, hidden_dim];
 * out [T, hidden_dim] in x's dtype.  With accumulate != 0, adds into out
 * (the `moe_out + shared_out` of src/model.rs:388). */
QMOE_API int qmoe_layer_shared_forward(qmoe_layer *layer, const void *x, int dtype,
                              int64_t T, void *out, int accumulate, int ptr_kind);

/* ---- decoder-layer MoE block (src/model.rs:359-412) ----------------------- */

/* The decoder layer's post_attention_layernorm (candle_nn::layer_norm,
 * src/model.rs:366-367): weight and bias [hidden_dim] f32, eps (1e-6 there).
 * Copied; a later call replaces them.  Needed by qmoe_layer_forward_block. */
QMOE_API int qmoe_layer_set_norm(qmoe_layer *layer, const float *weight, const float *bias,
                                 float eps, int ptr_kind);

/*
 * The MoE half of DecoderLayer::forward_with_cache / forward_prefill
 * (src/model.rs:400-412, :380-389): with x the residual stream after the
 * attention add,
 *     y   = post_attention_layernorm(x)
 *     out = x + (QMoELayer::forward(y) + SharedExpert::forward(y))
 * The normalisation runs as one kernel in a pinned order (64-wide chunk
 * sums added in order; the CPU oracle computes the same operations); the
 * residual add is the last operation of the combine.  x, out [T, hidden_dim]
 * in dtype; topk_idx / topk_w optional as in qmoe_layer_forward.  A layer
 * without routed experts gives x + shared(y) (or x).
 */
QMOE_API int qmoe_layer_forward_block(qmoe_layer *layer, const void *x, int dtype, int64_t T,
                                      void *out, int32_t *topk_idx, float *topk_w, int ptr_kind);

/*
 * Consecutive blocks: the layer loop of DeepSeekCoderV2::forward_next /
 * forward_prefill (src/model.rs:447-453, :481-489) over the MoE halves of
 * the decoder layers, the attention halves left out:
 *     out = block_{n-1}( ... block_1(block_0(x)) ... )
 * with block_l = qmoe_layer_forward_block of layers[l] (each with its
 * LayerNorm set; all on one context and of one hidden_dim).  The first call
 * for a given x, out, T and dtype captures the whole launch sequence into one
 * CUDA graph; repeats replay it (one graph launch for all layers; not on the
 * legacy default stream, which cannot be captured).  Intermediate rows live
 * in two buffers the chain owns.
 */
typedef struct qmoe_chain qmoe_chain;
QMOE_API int qmoe_chain_create(qmoe_layer *const *layers, int n_layers, qmoe_chain **out);
QMOE_API int qmoe_chain_destroy(qmoe_chain *chain);
QMOE_API int qmoe_chain_forward(qmoe_chain *chain, const void *x, int dtype, int64_t T, void *out,
                                int ptr_kind);

/* ---- allocation-free packed GEMV ---------------------------------------- */

/* Limits of qmoe_packed_forward_noalloc. */
#define QMOE_NOALLOC_MAX_BATCH 16384
#define QMOE_NOALLOC_MAX_IN_FEATURES 8192

/*
 * y = forward_simd(x) for callers that may not allocate device memory.  It has
 * no counterpart in qmoe-rs; it is the same product as qmoe_packed_forward
 * for a host program that owns all device memory (for instance a server that
 * hands its whole HBM budget to its own pool at start-up and gives a plugin
 * only each call's buffers), or a latency-critical path where cudaMalloc's
 * implicit device synchronisation is not allowed.
 *
 * All of packed ([out_features, in_features/4] bytes), scales, x
 * ([batch, in_features] f32) and y ([batch, out_features] f32) are device
 * pointers on `device`; packed and x must be 16-byte aligned.  The call is
 * asynchronous on `stream` and calls no cudaMalloc, cudaFree or allocating
 * library routine: its work list lives in one fixed array of device memory
 * (about 52 KB) that the library holds on every GPU it is loaded on until the
 * process exits.  Limits: batch <= QMOE_NOALLOC_MAX_BATCH, in_features a
 * multiple of 64 and <= QMOE_NOALLOC_MAX_IN_FEATURES; larger sizes return
 * QMOE_ERR_INVALID with a message in qmoe_last_error().
 *
 * The first call on a device does a one-time set-up with that device current
 * (it looks up the array's device address and sizes the launch grid); make
 * that first call before any stream capture.  Every call
 * on a device uses the same array, so calls that overlap on the GPU (two
 * streams, or two host threads) race; serialise them.  Each call rewrites
 * everything its kernels read from the array, so nothing needs clearing.
 */
QMOE_API int qmoe_packed_forward_noalloc(int device, void *stream, const uint8_t *packed,
                                         const float *scales, int64_t out_features,
                                         int64_t in_features, const float *x,
                                         int64_t batch, float *y);

/* ---- expert-product path -------------------------------------------------- */

/* Which kernels form the expert products of a forward.  AUTO takes the
 * prefill GEMM for bf16 activations once the routed positions per expert
 * (or the batch, for a shared-only pass) reach 16, and the decode GEMV
 * otherwise.  DECODE: integer-limb GEMV, products exact, f32 or bf16
 * activations.  PREFILL: tcgen05 bf16 GEMM with f32 accumulation and bf16
 * SwiGLU rows, bf16 activations only (an f32 forward then fails with
 * QMOE_ERR_UNSUPPORTED); needs hidden % 128 == 0 and intermediate dims
 * % 64 == 0.  DECODE_SPLIT: the DECODE arithmetic with the activation limbs
 * and the final combine as kernels of their own; DECODE (and AUTO) make them
 * inside the two GEMV kernels, launched cooperatively, where the device
 * supports cooperative launches.  Same results bit for bit.  Replaces
 * nothing in qmoe-rs, whose path is one. */
#define QMOE_PATH_AUTO 0
#define QMOE_PATH_DECODE 1
#define QMOE_PATH_PREFILL 2
#define QMOE_PATH_DECODE_SPLIT 3
QMOE_API int qmoe_layer_set_path(qmoe_layer *layer, int path);

/* ---- expert parallelism ------------------------------------------------- */

/* Device-side steps of an expert-parallel layer over `world` ranks, each
 * holding experts_per_rank consecutive experts.  qmoe-rs has no such mode
 * (src/moe.rs:40-130 runs every expert in one process); the host issues the
 * exchanges (NCCL all-to-all) between these calls.  All pointers are device
 * pointers; the calls are asynchronous on the context's stream.
 *
 * qmoe_ep_plan: from this rank's routing (topk_idx [T, K] global ids, -1 =
 * none; topk_w [T, K]) the send list, destination-major with tokens in
 * order: send_counts [world], send_tok (token of each send row), send_meta
 * [rows, 2K] int32 (K local expert ids on the destination, -1 for slots
 * owned elsewhere, then the bits of the K f32 weights), and slot_pos [T,
 * world] (send row of (token, rank), -1 if none).  capacity 0: compact
 * rows (rows = sum of
 * send_counts <= T * world, the buffers sized T * world); capacity C >= T:
 * rank d's rows start at d * C, the unused ones with ids -1, token 0 and
 * weight 0 (buffers of world * C rows), so every exchange has fixed sizes.
 * world <= 32. */
QMOE_API int qmoe_ep_plan(qmoe_ctx *ctx, const int32_t *topk_idx, const float *topk_w,
                          int64_t T, int K, int experts_per_rank, int world,
                          int64_t capacity, int32_t *send_counts, int32_t *send_tok,
                          int32_t *send_meta, int32_t *slot_pos);
/* out[i] = x[idx[i]] for n rows of H elements (f32 or bf16); H % 8 == 0. */
QMOE_API int qmoe_gather_rows(qmoe_ctx *ctx, const void *x, int dtype, int64_t H,
                              const int32_t *idx, int64_t n, void *out);
/* out[t] = rows[slot_pos[t][0]] + rows[slot_pos[t][1]] + ... (ascending s,
 * -1 skipped) + extra[t] (if extra is not NULL), f32 accumulation, for T
 * rows of H elements in dtype: the origin-side sum of the partials each
 * rank returned, then the shared expert's row. */
QMOE_API int qmoe_combine_rows(qmoe_ctx *ctx, const void *rows, int dtype, int64_t H,
                               const int32_t *slot_pos, int S, int64_t T, const void *extra,
                               void *out);
/* One rank's experts over R received rows plus the shared expert: rows carry
 * their routing as meta [R, 2K] int32 (local expert ids, -1 = skip, then the
 * f32 weight bits, the layout of qmoe_ep_plan's send_meta); rows shared_row0
 * .. R-1 also get the shared expert (the rank's own tokens, appended with
 * ids -1).  out [R, H]: per row the weighted sum of its local experts in
 * ascending order, plus the shared output for the shared rows.  Device
 * pointers, asynchronous. */
QMOE_API int qmoe_layer_forward_ep(qmoe_layer *layer, const void *x, int dtype, int64_t R,
                                   const int32_t *meta, int64_t shared_row0, void *out);
/* qmoe_layer_route followed by qmoe_ep_plan (capacity >= T, padded rows)
 * on this rank's tokens, device pointers, asynchronous: for small batches
 * one launch (the decode front cluster with the send list built in place of
 * the permute), else the router kernels and the plan kernel. */
QMOE_API int qmoe_layer_route_plan(qmoe_layer *layer, const void *x, int dtype, int64_t T,
                                   int32_t *topk_idx, float *topk_w, int experts_per_rank, int world,
                                   int64_t capacity, int32_t *send_counts, int32_t *send_tok,
                                   int32_t *send_meta, int32_t *slot_pos);

/* ---- expert-parallel exchange over peer memory ------------------------
 *
 * The dispatch and return of the expert-parallel layer as kernels that
 * write straight into the other ranks' memory (NVLink peer stores through
 * CUDA IPC mappings; no collective library): each rank owns one device
 * allocation holding its receive rows, their metadata, the returned
 * partial rows and the arrival flags; the ranks exchange the allocations'
 * IPC handles (QMOE_EP_HANDLE_BYTES each, e.g. with an all-gather of the
 * process group) and open each other's.  Per forward, in stream order on
 * every rank:
 *
 *   qmoe_ep_dispatch     rows x[send_tok[d*C + i]] (i < send_counts[d]) and
 *                        all C metadata rows of block d go to rank d's
 *                        receive block `rank`; this rank's own tokens x[0..T)
 *                        go to its own receive rows world*C ..; every row
 *                        sent counts one arrival on its destination;
 *   qmoe_ep_wait         waits (bounded) until every other rank's C rows of
 *                        a phase have arrived (phase 0: dispatch, 1: return);
 *   qmoe_ep_return       rows y[d*C + i] (the partial sums of the rows
 *                        received from rank d) go to rank d's return block
 *                        `rank`, each counted on arrival;
 *   qmoe_ep_wait(1)      ends the forward (arrivals are counted against a
 *                        per-forward sequence number kept on the device, so
 *                        the whole forward can be captured in a CUDA graph).
 *
 * These replace the three all-to-alls (ExpertParallelMoE over
 * torch.distributed) with two peer-store phases; with the buffers used as
 * qmoe_layer_forward_ep's input and qmoe_combine_rows's input.  A wait that
 * gives up raises the device error word (reported by the next synchronising
 * call) instead of hanging.  world <= 32; every rank must use the same
 * world, capacity, H, K and dtype. */
#define QMOE_EP_HANDLE_BYTES 64
typedef struct qmoe_ep_peer qmoe_ep_peer;
QMOE_API int qmoe_ep_peer_create(qmoe_ctx *ctx, int world, int rank, int64_t capacity,
                                 int64_t H, int K, int dtype, qmoe_ep_peer **out);
QMOE_API int qmoe_ep_peer_destroy(qmoe_ep_peer *p);
/* This rank's IPC handle (QMOE_EP_HANDLE_BYTES bytes). */
QMOE_API int qmoe_ep_peer_handle(qmoe_ep_peer *p, void *handle);
/* All ranks' handles, world * QMOE_EP_HANDLE_BYTES bytes in rank order. */
QMOE_API int qmoe_ep_peer_connect(qmoe_ep_peer *p, const void *handles);
/* Device pointers of this rank's receive rows [world*C + C, H] (dtype),
 * receive metadata [world*C + C, 2K] int32 and returned rows [world*C, H]
 * (dtype). */
QMOE_API int qmoe_ep_peer_buffers(qmoe_ep_peer *p, void **recv_rows, int32_t **recv_meta,
                                  void **back_rows);
QMOE_API int qmoe_ep_dispatch(qmoe_ep_peer *p, const void *x, int64_t T, const int32_t *send_counts,
                              const int32_t *send_tok, const int32_t *send_meta);
QMOE_API int qmoe_ep_wait(qmoe_ep_peer *p, int phase);
QMOE_API int qmoe_ep_return(qmoe_ep_peer *p, const void *y);
/* qmoe_ep_wait(0), qmoe_layer_forward_ep on this rank's receive rows (R =
 * world*C + own tokens, shared_row0 = world*C) and qmoe_ep_return: the wait is
 * done by the expert pass's first kernel and the return folded
 * into the expert pass where it can be: the decode path's last phase stores
 * each received row's partial sum straight into its origin rank's return
 * block, one arrival per (row, 1024 columns); rows past world*C (this rank's
 * shared-expert rows) go to y.  Other paths run the return kernel. */
QMOE_API int qmoe_layer_forward_ep_return(qmoe_layer *layer, qmoe_ep_peer *p, const void *x, int dtype,
                                          int64_t R, const int32_t *meta, int64_t shared_row0, void *y);
/* qmoe_ep_wait(1) and qmoe_combine_rows over the return block in one launch:
 * out[t] = sum over ranks s ascending of the returned row slot_pos[t][s]
 * (-1: none) + extra[t] (nullable), T <= capacity, device pointers. */
QMOE_API int qmoe_ep_finish(qmoe_ep_peer *p, const int32_t *slot_pos, int64_t T, const void *extra, void *out);

/* ---- tracing ----------------------------------------------------------- */

/* Stage timing, the device-side counterpart of the Instant-based breakdown
 * of qmoe-rs's bench harness (benches/moe_layer.rs:105-195).  While enabled,
 * each forward records CUDA events on the context's stream around its
 * stages: 0 router, 1 permute, 2 activation limbs for gate/up (prefill:
 * the bf16 row gather), 3 gate/up + SwiGLU, 4 limbs for down (prefill:
 * none), 5 down, 6 combine. */
QMOE_API int qmoe_layer_set_profiling(qmoe_layer *layer, int enable);
/* Waits for the last profiled forward and writes min(capacity, 7) stage
 * durations in milliseconds to ms; *count receives the number written. */
QMOE_API int qmoe_layer_stage_times(qmoe_layer *layer, float *ms, int capacity,
                                    int *count);

#ifdef __cplusplus
}
#endif

#endif /* QMOE_B200_H */
