// permute.cu -- per-expert segments of the routed assignments.
//
// Replaces the binning of QMoELayer::forward (qmoe-rs src/moe.rs:57, :80):
// bins[e] lists the (token, weight) pairs routed to expert e in token order.
// Here every routed assignment gets a position; positions are grouped by
// expert (ascending), and inside an expert they follow token order, so
// position order is exactly the reference's bin order.
//
// One CTA of 1024 threads:
//   1. per-expert counts (shared-memory atomics);
//   2. exclusive scan of the counts -> segment offsets, and of the token-group
//      counts -> the work list the grouped kernels walk;
//   3. token tiles of 1024 (one thread per token): each warp sets one bit per
//      (lane, expert) in a per-warp bitmap; a scan over the 32 warps' popcounts
//      per expert plus popc(bitmap & lanes-below) gives every assignment its
//      stable rank within the expert.
#include "common.cuh"
#include "kernels.h"

namespace qmoe {
namespace {

constexpr int kPermThreads = 1024;
constexpr int kWarps = kPermThreads / 32;

__global__ void __launch_bounds__(kPermThreads)
permute_kernel(const PermuteParams p) {
    extern __shared__ int sm[];
    const int E = p.e_count;
    int *cnt = sm;                       // [E]
    int *off = cnt + E;                  // [E + 1]
    int *run = off + E + 1;              // [E] running rank base per expert
    int *scan_tmp = run + E;             // [kWarps + 1] position scan
    int *gscan = scan_tmp + kWarps + 1;  // [kWarps + 1] group scan
    uint32_t *bm = reinterpret_cast<uint32_t *>(gscan + kWarps + 1);  // [kWarps][E]
    int *wpre = reinterpret_cast<int *>(bm + kWarps * E);               // [kWarps][E]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int64_t T = p.T;
    const int K = p.K;
    const int64_t TK = T * K;

    for (int e = tid; e < E; e += kPermThreads) { cnt[e] = 0; run[e] = 0; }
    __syncthreads();

    // 1. counts
    for (int64_t a = tid; a < TK; a += kPermThreads) {
        const int e = p.topk_idx[(a / K) * p.topk_ld + a % K] - p.e_begin;
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();

    // 2. block-wide exclusive scans (E <= 1024*?, looped in tiles of 1024)
    //    of counts and of token-group counts
    int carry_pos = 0, carry_grp = 0;
    for (int e0 = 0; e0 < E; e0 += kPermThreads) {
        const int e = e0 + tid;
        const int c = e < E ? cnt[e] : 0;
        const int ng = (c + p.chunk - 1) / p.chunk;
        // warp inclusive scans of (c, ng)
        int ic = c, ig = ng;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int vc = __shfl_up_sync(0xffffffffu, ic, o);
            const int vg = __shfl_up_sync(0xffffffffu, ig, o);
            if (lane >= o) { ic += vc; ig += vg; }
        }
        if (lane == 31) { scan_tmp[warp] = ic; gscan[warp] = ig; }
        __syncthreads();
        if (warp == 0) {
            int vc = scan_tmp[lane], vg = gscan[lane];
            int sc = vc, sg = vg;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int uc = __shfl_up_sync(0xffffffffu, sc, o);
                const int ug = __shfl_up_sync(0xffffffffu, sg, o);
                if (lane >= o) { sc += uc; sg += ug; }
            }
            scan_tmp[lane] = sc - vc;   // exclusive warp offsets
            gscan[lane] = sg - vg;
            if (lane == 31) { scan_tmp[kWarps] = sc; gscan[kWarps] = sg; }
        }
        __syncthreads();
        const int pos0 = carry_pos + scan_tmp[warp] + ic - c;
        const int grp0 = carry_grp + gscan[warp] + ig - ng;
        if (e < E) {
            off[e] = pos0;
            p.seg_off[e] = pos0;
            for (int g = 0; g < ng; ++g) {
                const int b = g * p.chunk;
                p.groups[grp0 + g] = make_int4(e, pos0 + b, min(p.chunk, c - b), 0);
            }
        }
        const int tot_pos = scan_tmp[kWarps], tot_grp = gscan[kWarps];
        __syncthreads();
        carry_pos += tot_pos;
        carry_grp += tot_grp;
    }
    if (tid == 0) {
        off[E] = carry_pos;
        p.seg_off[E] = carry_pos;
        p.n_groups[0] = carry_grp;
        int ns = 0;
        if (p.shared_count) ns = (int)((p.shared_count + p.chunk - 1) / p.chunk);
        p.n_groups[1] = ns;
    }
    if (p.shared_count) {
        const int64_t S = p.shared_count;
        const int ns = (int)((S + p.chunk - 1) / p.chunk);
        for (int g = tid; g < ns; g += kPermThreads) {
            const int64_t b = (int64_t)g * p.chunk;
            p.groups[carry_grp + g] =
                make_int4(E, (int)(TK + b), (int)(S - b < p.chunk ? S - b : p.chunk), 0);
        }
    }
    __syncthreads();

    // 3. stable ranks, one token per thread, tiles of 1024 tokens
    for (int64_t t0 = 0; t0 < T; t0 += kPermThreads) {
        for (int i = tid; i < kWarps * E; i += kPermThreads) bm[i] = 0u;
        __syncthreads();
        const int64_t t = t0 + tid;
        const bool live = t < T;
        if (live) {
            for (int j = 0; j < K; ++j) {
                const int e = p.topk_idx[t * p.topk_ld + j] - p.e_begin;
                if (e >= 0 && e < E) atomicOr(&bm[warp * E + e], 1u << lane);
            }
        }
        __syncthreads();
        for (int e = tid; e < E; e += kPermThreads) {
            int r = run[e];
            for (int w = 0; w < kWarps; ++w) {
                wpre[w * E + e] = r;
                r += __popc(bm[w * E + e]);
            }
            run[e] = r;
        }
        __syncthreads();
        if (live) {
            const uint32_t below = (1u << lane) - 1u;
            for (int j = 0; j < K; ++j) {
                const int e = p.topk_idx[t * p.topk_ld + j] - p.e_begin;
                int pos = -1;
                if (e >= 0 && e < E) {
                    pos = off[e] + wpre[warp * E + e] + __popc(bm[warp * E + e] & below);
                    p.pos_tok[pos] = (int32_t)t;
                }
                p.assign_pos[t * K + j] = pos;
            }
        }
        __syncthreads();
    }
}

}  // namespace

size_t permute_smem_bytes(int e_count) {
    return sizeof(int) * ((size_t)3 * e_count + 1 + 2 * (kWarps + 1) + (size_t)2 * kWarps * e_count);
}

cudaError_t launch_permute(const PermuteParams &p, cudaStream_t s) {
    size_t smem = permute_smem_bytes(p.e_count);
    static size_t smem_set = 0;  // raise the opt-in limit only when needed
    if (smem > smem_set) {
        cudaError_t e = cudaFuncSetAttribute(permute_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        smem_set = smem;
    }
    return launch_pdl(permute_kernel, dim3(1), dim3(kPermThreads), smem, s, p);
}

}  // namespace qmoe
