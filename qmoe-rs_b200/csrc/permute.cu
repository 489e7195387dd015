// permute.cu -- per-expert segments of the routed assignments.
//
// Replaces the binning of QMoELayer::forward (qmoe-rs src/moe.rs:57, :80):
// bins[e] lists the (token, weight) pairs routed to expert e in token order.
// Here every routed assignment gets a position; positions are grouped by
// expert (ascending), and inside an expert they follow token order, so
// position order is exactly the reference's bin order.
//
// One CTA per tile of kPermTok tokens, each on its own: every CTA counts the
// assignments of all tokens per expert (private per-warp counters) -- the
// totals give the segment offsets, the counts of earlier tokens this tile's
// base in each segment -- so no CTA waits on another.  Inside the tile, one
// thread per token sets one bit per (lane, expert) in a per-warp bitmap; a
// scan over the tile's warps plus popc(bitmap & lanes below) gives every
// assignment its stable rank within the expert.  CTA 0 also writes the
// segment offsets and the token-group work list the grouped kernels walk.
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace qmoe {
namespace {

constexpr int kPermThreads = 512;
constexpr int kWarps = kPermThreads / 32;
constexpr int kPermTok = 128;              // tokens per CTA
constexpr int kTokWarps = kPermTok / 32;

// Exclusive scans over e < E of c[e] and of its group count ceil(c / chunk);
// returns the totals.  All threads call it.
QMOE_DEV int2 block_scan2(const int *c, int *off, int *goff, int E, int chunk, int *tmp) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int carry_c = 0, carry_g = 0;
    for (int e0 = 0; e0 < E; e0 += kPermThreads) {
        const int e = e0 + tid;
        const int v = e < E ? c[e] : 0;
        const int g = (v + chunk - 1) / chunk;
        int ic = v, ig = g;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int uc = __shfl_up_sync(0xffffffffu, ic, o), ug = __shfl_up_sync(0xffffffffu, ig, o);
            if (lane >= o) { ic += uc; ig += ug; }
        }
        if (lane == 31) { tmp[warp] = ic; tmp[kWarps + warp] = ig; }
        __syncthreads();
        int bc = 0, bg = 0, tc = 0, tg = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            if (w < warp) { bc += tmp[w]; bg += tmp[kWarps + w]; }
            tc += tmp[w];
            tg += tmp[kWarps + w];
        }
        if (e < E) {
            off[e] = carry_c + bc + ic - v;
            goff[e] = carry_g + bg + ig - g;
        }
        carry_c += tc;
        carry_g += tg;
        __syncthreads();
    }
    return make_int2(carry_c, carry_g);
}

__global__ void __launch_bounds__(kPermThreads)
permute_kernel(const PermuteParams p) {
    extern __shared__ int sm[];
    const int E = p.e_count;
    int *hist_t = sm;                        // [kWarps][E] all tokens, per warp
    int *hist_p = hist_t + kWarps * E;       // [kWarps][E] tokens before this tile
    int *tot = hist_p + kWarps * E;          // [E]
    int *pre = tot + E;                      // [E]
    int *off = pre + E;                      // [E]
    int *goff = off + E;                     // [E]
    int *tmp = goff + E;                     // [2 kWarps]
    uint32_t *bm = reinterpret_cast<uint32_t *>(tmp + 2 * kWarps);   // [kTokWarps][E]
    int *wpre = reinterpret_cast<int *>(bm + kTokWarps * E);           // [kTokWarps][E]

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    if (p.ep_wait) {
        // the rows and their metadata come from the peers' dispatch: wait
        // (bounded) until each peer's C rows of this forward have arrived
        if (warp == 0) {
            const uint32_t want = (uint32_t)(*p.ep.seq + 1);   // forwards whose dispatch arrived
            bool ok = true;
            for (int r = lane; r < p.ep.world; r += 32) {
                if (r == p.ep.rank) continue;
                const int *f = reinterpret_cast<const int *>(p.ep.base[p.ep.rank] + p.ep.off_flags) + r;
                uint32_t n = 0;
                while (!arrived(ld_acquire_sys_i32(f), want)) {
                    if (++n >= sm100::kMaxWaitProbes) {
                        ok = false;
                        break;
                    }
                    __nanosleep(64);
                }
            }
            if (!__all_sync(0xffffffffu, ok) && lane == 0) atomicOr(p.ep.err, sm100::kErrWaitTimeout);
        }
        __syncthreads();
    }
    const int64_t T = p.T;
    const int K = p.K;
    const int64_t TK = T * K;
    const int64_t t_start = (int64_t)blockIdx.x * kPermTok;

    for (int i = tid; i < 2 * kWarps * E; i += kPermThreads) hist_t[i] = 0;
    for (int i = tid; i < kTokWarps * E; i += kPermThreads) bm[i] = 0u;
    __syncthreads();

    // 1. counts per expert: all tokens, and tokens before this tile, one
    // token per thread at a time (no division), private per-warp counters
    for (int64_t t = tid; t < T; t += kPermThreads) {
        const int32_t *ids = p.topk_idx + t * p.topk_ld;
        const bool before = t < t_start;
        for (int j = 0; j < K; ++j) {
            const int e = ids[j] - p.e_begin;
            if (e >= 0 && e < E) {
                atomicAdd(&hist_t[warp * E + e], 1);
                if (before) atomicAdd(&hist_p[warp * E + e], 1);
            }
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += kPermThreads) {
        int a = 0, b = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            a += hist_t[w * E + e];
            b += hist_p[w * E + e];
        }
        tot[e] = a;
        pre[e] = b;
    }
    __syncthreads();

    // 2. segment offsets (and in CTA 0 the work list)
    const int2 totals = block_scan2(tot, off, goff, E, p.chunk, tmp);
    if (blockIdx.x == 0) {
        for (int e = tid; e < E; e += kPermThreads) {
            p.seg_off[e] = off[e];
            const int c = tot[e];
            for (int g = 0; g * p.chunk < c; ++g) {
                const int2 sg = split_group(c, p.chunk, g);
                p.groups[goff[e] + g] = make_int4(e, off[e] + sg.x, sg.y, 0);
            }
        }
        const int ns = p.shared_count ? (int)((p.shared_count + p.chunk - 1) / p.chunk) : 0;
        if (tid == 0) {
            p.seg_off[E] = totals.x;
            p.n_groups[0] = totals.y;
            p.n_groups[1] = ns;
        }
        for (int g = tid; g < ns; g += kPermThreads) {
            const int2 sg = split_group(p.shared_count, p.chunk, g);
            p.groups[totals.y + g] = make_int4(E, (int)(TK + sg.x), sg.y, 0);
        }
    }

    // 3. stable ranks inside the tile, one token per thread
    const int64_t t = t_start + tid;
    const bool live = tid < kPermTok && t < T;
    if (live)
        for (int j = 0; j < K; ++j) {
            const int e = p.topk_idx[t * p.topk_ld + j] - p.e_begin;
            if (e >= 0 && e < E) atomicOr(&bm[warp * E + e], 1u << lane);
        }
    __syncthreads();
    for (int e = tid; e < E; e += kPermThreads) {
        int r = off[e] + pre[e];
#pragma unroll
        for (int w = 0; w < kTokWarps; ++w) {
            wpre[w * E + e] = r;
            r += __popc(bm[w * E + e]);
        }
    }
    __syncthreads();
    if (live) {
        const uint32_t below = (1u << lane) - 1u;
        for (int j = 0; j < K; ++j) {
            const int e = p.topk_idx[t * p.topk_ld + j] - p.e_begin;
            int pos = -1;
            if (e >= 0 && e < E) {
                pos = wpre[warp * E + e] + __popc(bm[warp * E + e] & below);
                p.pos_tok[pos] = (int32_t)t;
            }
            p.assign_pos[t * K + j] = pos;
        }
    }
}

}  // namespace

size_t permute_smem_bytes(int e_count) {
    return sizeof(int) * ((size_t)2 * kWarps * e_count + 4 * (size_t)e_count + 2 * kWarps +
                          (size_t)2 * kTokWarps * e_count);
}

cudaError_t launch_permute(const PermuteParams &p, cudaStream_t s) {
    size_t smem = permute_smem_bytes(p.e_count);
    cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(permute_kernel), smem);
    if (e != cudaSuccess) return e;
    // without routed assignments (K = 0) only the shared groups are written
    const unsigned grid = (unsigned)(p.T > 0 && p.K > 0 ? (p.T + kPermTok - 1) / kPermTok : 1);
    return launch_pdl(permute_kernel, dim3(grid), dim3(kPermThreads), smem, s, p);
}

}  // namespace qmoe
