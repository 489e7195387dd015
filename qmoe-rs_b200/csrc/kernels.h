// kernels.h -- launch interface of the qmoe_b200 kernels (library-internal).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qmoe {

// Rows per work item of the decode kernels (qgemv.cu); a permute chunk fed to
// them must not exceed it.
constexpr int kQgemvTokens = 5;

// Sets the message qmoe_last_error() returns on this thread (api.cu).
void set_last_error_message(const char *msg);

// ---- router -------------------------------------------------------------
struct RouterParams {
    const void *x;          // [T, H] f32 or bf16
    int dtype;              // 0 f32, 1 bf16
    int64_t T;
    int H, E, K;
    const float *gate_w;    // [E, H]
    const float *gate_t;    // [H, gate_t_ld] f32: gate_w transposed (large-batch logits), or nullptr
    int gate_t_ld;          // row stride of gate_t in floats (E rounded up to 4)
    const float *bias;      // [E] or nullptr
    int scoring;            // 0 softmax, 1 sigmoid
    int n_group, topk_group;
    int norm_topk;
    float routed_scale;
    int32_t *topk_idx;      // [T, K]
    float *topk_w;          // [T, K]
    float *scratch;         // router_scratch_floats(T, H, E) floats
};
size_t router_smem_bytes(int H, int E);
// Host: gate_t[k][e] = gate_w[e][k] for the large-batch logit kernel (ld =
// E rounded up to 4; the padding columns are zero).
cudaError_t launch_transpose_gate(const float *gate_w, int E, int H, float *gate_t, int ld, cudaStream_t s);
int gate_t_ld(int E);
bool router_uses_partials(int64_t T, int H, int E);
size_t router_scratch_floats(int64_t T, int H, int E);
// With a tail (tail->counter != nullptr), the last CTA of the selection
// kernel also builds the expert segments and the work list (the permute),
// for batches with router_tail_ok.
struct FrontParams {
    int32_t *counter;          // zero before the launch; the last CTA resets it
    int chunk;                 // tokens per group descriptor
    int64_t shared_count;      // shared-expert positions after the routed ones (0 or T)
    int32_t *seg_off;          // [E + 1]
    int32_t *assign_pos;       // [T, K]
    int32_t *pos_tok;          // [T * K]
    int4 *groups;
    int32_t *n_groups;         // [2]
    void *x_copy;              // front cluster kernel: device copy of x to write (nullable)
    // front cluster kernel, plan_world > 0: instead of the permute, the
    // expert-parallel send list of qmoe_ep_plan (padded layout, capacity >= T)
    int plan_world, plan_epr;
    int64_t plan_capacity;
    int32_t *send_counts, *send_tok, *send_meta, *slot_pos;
};
bool router_tail_ok(int64_t T, int E, int K);
cudaError_t launch_router(const RouterParams &p, const FrontParams *tail, cudaStream_t s);
// The whole decode front (logits, selection, permute) as one thread-block
// cluster (front.cu), for small batches: front_cluster_ok says whether this
// batch and layer shape, and the device, allow it.
bool front_cluster_ok(int64_t T, int H, int E, int K);
cudaError_t launch_front_cluster(const RouterParams &p, const FrontParams &f, cudaStream_t s);

// ---- expert-parallel exchange over peer memory (ep_p2p.cu) ---------------
// Every rank's allocation has the same layout: receive rows [G*C + C][H]
// (dtype), receive metadata [G*C + C][2K] int32, returned rows [G*C][H],
// arrival counters [2][G] int32; offsets below.  base[r] = rank r's allocation as this
// GPU addresses it (its own included).
constexpr int kEpMaxWorld = 32;
struct EpPeerDev {
    uint8_t *base[kEpMaxWorld];
    int world, rank, K;
    int64_t C, H, esize;
    int64_t off_rows, off_meta, off_back, off_flags;
    int *seq;                    // this rank's per-forward sequence number
    int *done;                   // exit count of the return-side kernel (zero between launches)
    int *cnt;                    // [2][kEpMaxWorld]; [phase][0]: CTAs of one launch done
                                 // (zero between launches; ep_signal.cuh)
    int *err;                    // device error word
};

// ---- permute ------------------------------------------------------------
// Builds per-expert segments of routed (token, slot) assignments, stable in
// token order, and the token-group work list of the grouped kernels.
struct PermuteParams {
    const int32_t *topk_idx;   // [T, K] (row stride topk_ld); ids outside [e_begin,
                               // e_begin+e_count) skipped
    int64_t T;
    int K, topk_ld;
    int e_begin, e_count;
    int chunk;                 // tokens per group descriptor
    int64_t shared_count;      // append groups over this many shared positions (segment e_count)
    int32_t *seg_off;          // [e_count + 1] routed segment offsets
    int32_t *assign_pos;       // [T, K] position of each assignment, -1 if skipped
    int32_t *pos_tok;          // [T*K] token of each routed position
    int4 *groups;              // (segment, pos_begin, count, 0)
    int32_t *n_groups;         // [2]: routed groups, shared groups
    int ep_wait;               // expert parallel: first wait (bounded) until every peer's
    EpPeerDev ep;              //    rows of this forward have arrived (the topk rows are theirs)
};
size_t permute_smem_bytes(int e_count);
cudaError_t launch_permute(const PermuteParams &p, cudaStream_t s);

// ---- decode grouped GEMV (int8-limb mma.sync, in-register 2-bit unpack) --
struct QgemvParams {
    // work list
    const int4 *groups;
    const int32_t *n_groups;     // [0] routed groups, [1] shared groups
    // routed weights, experts stacked: matrix m at w[m] + seg*w_stride
    const uint8_t *w[2];
    const float *s[2];
    int64_t w_stride;            // bytes per expert matrix
    int64_t s_stride;            // scales per expert matrix
    int rows, K;                 // rows per matrix, reduction length
    // shared segment weights (segment id == n_routed_segs)
    const uint8_t *ws[2];
    const float *ss[2];
    int rows_s, K_s;
    // activations: rows of f32 or bf16
    const void *act;
    int act_dtype;
    int64_t act_ld;
    const int32_t *pos_tok;      // routed position -> activation row (nullable)
    int64_t shared_base;         // first shared position
    // output rows by position
    float *out;
    int64_t out_ld;
};
// mode 0: gate+up matrices fused with SwiGLU (128 rows of each per item)
// mode 1: one matrix (256 rows per item)
cudaError_t launch_qgemv(int mode, const QgemvParams &p, int grid, cudaStream_t s);
int qgemv_max_grid(int mode, int K_max);
size_t qgemv_smem_bytes(int K_max);

// ---- activation quantisation for the integer tensor-core GEMV -----------
struct QuantParams {
    const void *act;             // rows of f32 or bf16
    int dtype;
    int64_t act_ld;
    const int32_t *pos_tok;      // routed position -> row (nullable: row = pos)
    int64_t shared_base;         // positions >= this are shared: row shared_row0 + pos - base
    int64_t shared_row0;
    const int32_t *n_valid;      // routed positions >= *n_valid are skipped (nullable)
    int64_t npos;                // positions (grid size)
    int K, K_s;                  // row length of routed / shared rows
    int Kp;                      // row stride of xq (>= both padded to 256)
    int8_t *xq;                  // [npos][3][Kp] limbs
    longlong2 *meta;             // [npos] (exponent, sum of Q)
};
cudaError_t launch_quant(const QuantParams &p, cudaStream_t s);

// ---- weighted combine (combine.cu / combine.cuh) -------------------------
struct CombineParams {
    const float *y;              // [positions, H] expert outputs
    const int32_t *assign_pos;   // [T, K]
    const int32_t *topk_idx;     // [T, K] row stride topk_ld (expert order of the accumulation)
    const float *topk_w;         // [T, K] row stride topk_ld
    int64_t T;
    int K, topk_ld, H;
    const float *y_shared;       // [shared_count, H] for rows shared_row0.. or nullptr
    int64_t shared_row0, shared_count;
    int accumulate;              // add into out instead of overwriting
    const void *residual;        // [T, H] in out_dtype, added last (nullable): the decoder
                                 // layer's residual stream (src/model.rs:409-412)
    void *out;                   // [T, H]
    int out_dtype;
    // expert parallel (combine kernel): rows t < world * C are received rows;
    // each goes straight to its origin rank's return block (peer memory),
    // skipped when it has no live slot; every CTA signals once after its
    // stores (ep_signal.cuh)
    int ep_ret;
    EpPeerDev ret;
};
cudaError_t launch_combine(const CombineParams &p, cudaStream_t s);

// ---- post-attention LayerNorm (norm.cu) ----------------------------------
struct NormParams {
    const void *x;               // [T, H] f32 or bf16
    int dtype;
    int64_t T;
    int H;                       // multiple of 64
    const float *w, *b;          // [H]
    float eps;
    void *y;                     // [T, H] in x's dtype
};
cudaError_t launch_layernorm(const NormParams &p, cudaStream_t s);

// 2-bit packer (pack.cu): qmoe-rs quantize.py:7-33 with the row scale of
// :97-100.  w [out_f, in_f] f32 (16-byte aligned, in_f a multiple of 4) ->
// packed [out_f, in_f / 4]; scales [out_f] written, or read when
// scales_given.
struct PackParams {
    const float *w;
    int64_t out_f, in_f;
    float *scales;
    int scales_given;
    uint8_t *packed;
    int *err;                    // device error word (a bounded wait that gave up)
};
constexpr size_t kPackStageMax = 100 * 1024;   // widest row staged in shared memory (bytes)
cudaError_t launch_pack_rows(const PackParams &p, int sm_count, cudaStream_t s);

// ---- decode grouped GEMV (qgemv_imma.cu): work list and operands ---------
struct DecodeMaps {
    CUtensorMap a0, a1;          // routed matrices (mode 0: gate, up; mode 1: down, down)
    CUtensorMap s0, s1;          // shared-expert matrices (copies of a0/a1 if none)
    CUtensorMap b;               // limb rows xq [npos*3][kp_b], 128-byte swizzle
    // 3-D views for the IMMA kernel: a matrix as [64-byte chunk][row][byte]
    // (one box = two chunks of 128 rows), the limb rows as
    // [128-byte block][row][byte] (one box = 16 rows x every block)
    CUtensorMap a0_3, a1_3, s0_3, s1_3, b3;
};
struct DecodeParams {
    const int4 *groups;
    const int32_t *n_groups;
    int rows, K;                 // routed matrices
    int rows_s, K_s;             // shared segment (rows_s = 0: none)
    const float *s[2];           // routed scales, expert stride s_stride
    int64_t s_stride;
    const float *ss[2];          // shared scales
    const longlong2 *meta;       // per position (exponent, sum of Q)
    int kp_b;                    // row length of the limb rows (>= every item's padded K)
    int b_buffers;               // limb-tile buffers (2, or 1 for very long rows)
    float *out;
    int64_t out_ld;
    int *err;                    // device error word
    int *sched;                  // [3] item counter, exit count, grid-barrier count;
                                 // zero between launches
    // Cooperative launch only (both 0 otherwise):
    int quant_in;                // 1: first make the limb rows and metadata of q
    QuantParams q;               //    (quant.cuh) in the kernel, then a grid barrier
    int combine;                 // mode 1: after a grid barrier, the combine of c
    CombineParams c;             //    (combine.cuh) as the last phase
    int ep_ret;                  // with combine: rows r < ret.world * ret.C go straight to
    EpPeerDev ret;               //    rank r / C's return block (peer memory), one signal per CTA
};
cudaError_t launch_qgemv_imma(int mode, const DecodeMaps &maps, const DecodeParams &p,
                              int grid, cudaStream_t s);
size_t qgemv_imma_smem_bytes(int kp_b, int b_buffers);
int qgemv_imma_buffers(int kp_b);

cudaError_t launch_ep_dispatch(const EpPeerDev &d, const void *x, int64_t T, const int32_t *send_counts,
                               const int32_t *send_tok, const int32_t *send_meta, cudaStream_t s);
cudaError_t launch_ep_return(const EpPeerDev &d, const void *y, cudaStream_t s);
cudaError_t launch_ep_wait(const EpPeerDev &d, int phase, cudaStream_t s);
// Return side of a forward in one launch: wait (bounded) for every peer's
// returned rows, then out[t] = sum over ranks s ascending of back[slot_pos[t][s]]
// (skipping -1) + extra[t] (the combine_rows arithmetic); the last CTA out
// advances the sequence number.
cudaError_t launch_ep_finish(const EpPeerDev &d, const int32_t *slot_pos, int64_t T, const void *extra,
                             void *out, cudaStream_t s);

// Device-side error word (device_state.cu) raised by a bounded wait that gives
// up: its address on the current device.
int *device_error_flag();

// Host: the current device's SM count (cached per device; 148 if the query
// fails).
int device_sm_count();
// CTAs per SM of the grid-stride copy and return kernels of the expert-
// parallel exchange (each CTA fences its peer stores once).
constexpr int kEpCopyCtasPerSm = 4;

// Host: raise `func`'s dynamic shared-memory opt-in on the current device to
// at least `bytes` (never lowers it; remembered per kernel and device).
cudaError_t ensure_dyn_smem(const void *func, size_t bytes);

// Host: a 2-D uint8 tensor map over [rows][row_bytes] with the given box and
// swizzle (CU_TENSOR_MAP_SWIZZLE_*); returns false if encoding fails.
bool make_tmap_u8(CUtensorMap *tm, const void *base, uint64_t row_bytes, uint64_t rows,
                  uint32_t box_bytes, uint32_t box_rows, int swizzle);
// Host: a 3-D uint8 tensor map (extents d0..d2, byte strides of dims 1 and 2).
// 4-D u8 view (strides need not grow with the dimension).
bool make_tmap_u8_4d(CUtensorMap *tm, const void *base, const uint64_t (&dims)[4],
                     const uint64_t (&strides)[3], const uint32_t (&box)[4], int swizzle);
bool make_tmap_u8_3d(CUtensorMap *tm, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                     uint64_t stride1, uint64_t stride2, uint32_t b0, uint32_t b1, uint32_t b2,
                     int swizzle);

// ---- prefill grouped GEMM (tcgen05 kind::f16; 2-bit -> bf16 into TMEM) ---
// Activation and SwiGLU rows are stored with every 16-element block in the
// order kPrefillPerm16 (position -> element), the order in which one shift
// and one mask split a 32-bit word of packed codes into bf16 pairs.
struct GatherParams {
    const void *x;               // [T, H] bf16
    int64_t H;
    const int32_t *pos_tok;      // routed position -> token
    const int32_t *n_valid;      // routed positions in use (device)
    int64_t shared_base;         // first shared position: row shared_row0 + pos - base
    int64_t shared_row0;
    int64_t npos;                // positions (routed slots + shared rows)
    void *xg;                    // [npos, H] bf16, blocks permuted
};
cudaError_t launch_gather_bf16(const GatherParams &p, cudaStream_t s);

struct QgemmMaps {
    CUtensorMap w0, w1;          // routed 2-bit matrices (mode 0: gate, up; mode 1: down)
    CUtensorMap s0, s1;          // shared-expert matrices (copies of w0/w1 if none)
    CUtensorMap b;               // bf16 activation rows [npos][ld], 128-byte swizzle, 256-row box
    CUtensorMap b2;              // the same rows, 128-row box
    CUtensorMap b3;              // the same rows, 192-row box
};
struct QgemmParams {
    const int4 *groups;          // (segment, first position, count <= 256)
    const int32_t *n_groups;     // [0] routed groups, [1] shared groups
    int rows, K;                 // routed matrices: rows per expert, reduction length
    int rows_s, K_s;             // shared matrices (rows_s = 0: none)
    const float *s[2];           // routed row scales, expert stride s_stride
    int64_t s_stride;
    const float *ss[2];          // shared row scales
    void *out;                   // mode 0: bf16 SwiGLU rows (blocks permuted); mode 1: f32
    int64_t out_ld;              // elements per output row
    int *err;                    // device error word
};
cudaError_t launch_qgemm_prefill(int mode, const QgemmMaps &maps, const QgemmParams &p, int grid,
                                 cudaStream_t s);
size_t qgemm_prefill_smem_bytes();
constexpr int kPrefillTile = 256;  // tokens per work item (group chunk)

// Host: a 2-D bf16 tensor map over rows of `cols` elements, `row_stride`
// bytes apart.
bool make_tmap_bf16(CUtensorMap *tm, const void *base, uint64_t cols, uint64_t rows,
                    uint64_t row_stride, uint32_t box_cols, uint32_t box_rows, int swizzle);

// ---- expert parallelism (ep.cu) -----------------------------------------
struct EpPlanParams {
    const int32_t *topk_idx;     // [T, K] global expert ids (-1 = none)
    const float *topk_w;         // [T, K]
    int64_t T;
    int K;
    int experts_per_rank, world; // world <= 32
    int64_t capacity;            // 0: compact rows; > 0: rows of rank d at d * capacity (>= T)
    int32_t *send_counts;        // [world]
    int32_t *send_tok;           // [T * world] token of each send row
    int32_t *send_meta;          // [rows, 2K]: local expert ids on the destination (-1
                                 // elsewhere), then the f32 weight bits
    int32_t *slot_pos;           // [T, world] send row of (token, rank), -1 if none
};
cudaError_t launch_ep_plan(const EpPlanParams &p, cudaStream_t s);
cudaError_t launch_gather_rows(const void *x, int dtype, int64_t H, const int32_t *idx, int64_t n,
                               void *out, cudaStream_t s);
cudaError_t launch_combine_rows(const void *rows, int dtype, int64_t H, const int32_t *slot_pos, int S,
                                int64_t T, const void *extra, void *out, cudaStream_t s);

// ---- combine -----------------------------------------------------------


}  // namespace qmoe
