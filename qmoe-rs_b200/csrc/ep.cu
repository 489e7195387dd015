// ep.cu -- device side of the expert-parallel layer (experts split over
// ranks, contiguous blocks of experts_per_rank).
//
// qmoe-rs runs the whole layer in one process (src/moe.rs:40-130); across G
// GPUs each rank routes its own tokens, sends every token once to each rank
// that owns one of its experts, runs its experts on what it received, and
// returns one partial sum per (token, rank).  The origin then adds the
// partials in ascending rank order, i.e. ascending expert blocks, and the
// shared expert last (src/model.rs:386-389).  These kernels build the send
// lists and the return map, gather rows, and add the returned partials; the
// exchanges themselves are NCCL all-to-alls issued by the host.
#include "common.cuh"
#include "kernels.h"

namespace qmoe {
namespace {

// Send list, destination-major and in token order within a destination
// (compact: destination d's rows follow those of d-1; padded, capacity C > 0:
// destination d's rows start at d*C and the unused rows carry ids -1, so
// every exchange has fixed sizes and needs no count on the host):
//   send_counts[d]          tokens sent to rank d
//   send_tok[s]             token of send row s
//   send_meta[s][k]         local expert id of slot k on the destination, -1
//                           if slot k goes elsewhere (k < K)
//   send_meta[s][K + k]     the bits of that slot's f32 combine weight (0 if -1)
//   slot_pos[t][d]          send row of (t, d), -1 if t sends nothing to d
// One CTA per tile of 256 tokens, none waiting on another: every CTA counts
// the destinations of all tokens (those before its tile give its base in
// each destination, all of them the totals), a block scan of the "sends to
// d" bits gives each token of the tile its row, and the CTAs share out the
// unused padded rows.
constexpr int kPlanThreads = 256;

QMOE_DEV uint32_t dest_mask(const EpPlanParams &p, int64_t t) {
    uint32_t m = 0;
    for (int k = 0; k < p.K; ++k) {
        const int e = p.topk_idx[t * p.K + k];
        if (e >= 0) m |= 1u << (e / p.experts_per_rank);
    }
    return m;
}

__global__ void __launch_bounds__(kPlanThreads)
ep_plan_kernel(const EpPlanParams p) {
    __shared__ int s_before[kEpMaxWorld], s_total[kEpMaxWorld], s_base[kEpMaxWorld];
    __shared__ int wsum[kPlanThreads / 32][kEpMaxWorld];
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = p.world, K = p.K;
    const int64_t t0 = (int64_t)blockIdx.x * kPlanThreads;
    if (tid < kEpMaxWorld) {
        s_before[tid] = 0;
        s_total[tid] = 0;
    }
    __syncthreads();
    // destinations of every token: counts before this tile and in total
    for (int64_t t = tid; t < p.T; t += kPlanThreads) {
        uint32_t m = dest_mask(p, t);
        const bool before = t < t0;
        while (m) {
            const int d = __ffs(m) - 1;
            m &= m - 1;
            atomicAdd(&s_total[d], 1);
            if (before) atomicAdd(&s_before[d], 1);
        }
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int d = 0; d < G; ++d) {
            s_base[d] = p.capacity > 0 ? (int)(d * p.capacity) : run;
            run += s_total[d];
        }
        if (blockIdx.x == 0)
            for (int d = 0; d < G; ++d) p.send_counts[d] = s_total[d];
    }
    // this tile: one token per thread, per destination a block scan
    const int64_t t = t0 + tid;
    const uint32_t m = t < p.T ? dest_mask(p, t) : 0u;
    for (int d = 0; d < G; ++d) {
        const unsigned b = __ballot_sync(0xffffffffu, (m >> d) & 1u);
        if (lane == 0) wsum[warp][d] = __popc(b);
    }
    __syncthreads();
    for (int d = 0; d < G; ++d) {
        const bool bit = t < p.T && ((m >> d) & 1u);
        const unsigned b = __ballot_sync(0xffffffffu, bit);
        if (t < p.T) {
            int pos = -1;
            if (bit) {
                int before_warps = 0;
                for (int w = 0; w < warp; ++w) before_warps += wsum[w][d];
                pos = s_base[d] + s_before[d] + before_warps + __popc(b & ((1u << lane) - 1u));
                p.send_tok[pos] = (int32_t)t;
                int32_t *mt = p.send_meta + (int64_t)pos * 2 * K;
                for (int k = 0; k < K; ++k) {
                    const int e = p.topk_idx[t * K + k];
                    const bool mine = e >= 0 && e / p.experts_per_rank == d;
                    mt[k] = mine ? e - d * p.experts_per_rank : -1;
                    mt[K + k] = mine ? __float_as_int(p.topk_w[t * K + k]) : 0;
                }
            }
            p.slot_pos[t * G + d] = pos;
        }
    }
    // padded layout: the unused rows of every destination, shared out
    if (p.capacity > 0) {
        const int64_t C = p.capacity;
        const int64_t stride = (int64_t)gridDim.x * kPlanThreads;
        for (int d = 0; d < G; ++d)
            for (int64_t i = s_total[d] + (int64_t)blockIdx.x * kPlanThreads + tid; i < C; i += stride) {
                const int64_t r = d * C + i;
                p.send_tok[r] = 0;
                int32_t *mt = p.send_meta + r * 2 * K;
                for (int k = 0; k < K; ++k) {
                    mt[k] = -1;
                    mt[K + k] = 0;
                }
            }
    }
}

// out[r] = x[idx[r]] for rows of H elements (f32 or bf16): CTA (r, slice),
// 16 bytes per thread.
__global__ void __launch_bounds__(256)
gather_rows_kernel(const void *x, int dtype, int64_t H, const int32_t *idx, int64_t n, void *out) {
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int64_t per_row = H * (dtype ? 2 : 4) / 16;
    const int64_t r = blockIdx.x;
    const int64_t c = (int64_t)blockIdx.y * 256 + threadIdx.x;
    if (c >= per_row) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(x) + (int64_t)idx[r] * per_row + c;
    reinterpret_cast<uint4 *>(out)[r * per_row + c] = __ldg(src);
}

// out[t] = sum over s ascending of rows[slot_pos[t][s]] (skipping -1), then
// + extra[t] if given; f32 accumulation, rows, extra and out in `dtype`.
__global__ void __launch_bounds__(256)
combine_rows_kernel(const void *rows, int dtype, int64_t H, const int32_t *slot_pos, int S, int64_t T,
                    const void *extra, void *out) {
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    // CTA (token t, slice of 256 x 4 elements)
    const int64_t t = blockIdx.x;
    const int64_t h = ((int64_t)blockIdx.y * 256 + threadIdx.x) * 4;
    if (h >= H) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < S; ++s) {
        const int pos = slot_pos[t * S + s];
        if (pos < 0) continue;
        const float4 v = load_act4(rows, dtype, (int64_t)pos * H + h);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    if (extra) {
        const float4 v = load_act4(extra, dtype, t * H + h);
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
    }
    store_act4(out, dtype, t * H + h, acc);
}

}  // namespace

cudaError_t launch_ep_plan(const EpPlanParams &p, cudaStream_t s) {
    const int64_t tiles = p.T > 0 ? (p.T + kPlanThreads - 1) / kPlanThreads : 1;
    return launch_pdl(ep_plan_kernel, dim3((unsigned)tiles), dim3(kPlanThreads), 0, s, p);
}

cudaError_t launch_gather_rows(const void *x, int dtype, int64_t H, const int32_t *idx, int64_t n,
                               void *out, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const int64_t per_row = H * (dtype ? 2 : 4) / 16;
    const dim3 grid((unsigned)n, (unsigned)((per_row + 255) / 256));
    return launch_pdl(gather_rows_kernel, grid, dim3(256), 0, s, x, dtype, H, idx, n, out);
}

cudaError_t launch_combine_rows(const void *rows, int dtype, int64_t H, const int32_t *slot_pos, int S,
                                int64_t T, const void *extra, void *out, cudaStream_t s) {
    if (T == 0 || H == 0) return cudaSuccess;
    const dim3 grid((unsigned)T, (unsigned)((H / 4 + 255) / 256));
    return launch_pdl(combine_rows_kernel, grid, dim3(256), 0, s, rows, dtype, H, slot_pos, S, T, extra,
                      out);
}

}  // namespace qmoe
