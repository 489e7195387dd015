// front.cu -- the decode front in one launch: gate logits, scoring, top-k,
// combine weights and the permute (expert segments and the token-group work
// list), for small batches, as one thread-block cluster.
//
// Replaces the router half of QMoELayer::forward (qmoe-rs src/moe.rs:51-82)
// and the grouping of its assignments by expert (src/moe.rs:90-118), with the
// same arithmetic as router.cu + permute.cu (bit-identical results):
//   phase A  each CTA of the cluster owns a contiguous run of 64-wide hidden
//            chunks and forms the chunk partials of every (token, expert) --
//            an fmaf chain over the chunk's 64 products from 0 -- and stores
//            each token's partials into the shared memory of the CTA that
//            owns the token (token t belongs to CTA t % cluster size;
//            distributed shared memory stores, which do not stall); the gate
//            tiles are fetched before the wait on the preceding kernel;
//   phase B  after a cluster barrier, one warp per token adds that token's
//            partials in chunk order from its own shared memory;
//   phase C  the same warp scores, applies the group limit and sorts the
//            experts (bitonic network over shuffles) in the stable
//            descending order, ties to the lower expert; the softmax sum runs
//            in descending-logit order; the warp writes the top-k ids and
//            weights, and the ids to CTA 0's shared memory;
//   phase D  after a second cluster barrier, CTA 0 builds the segments and
//            the work list (per-expert token masks, one thread per expert).
// One launch replaces the logits kernel, the selection kernel and the
// permute, and no partial sum goes through global memory.
#include <map>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "select.cuh"

namespace qmoe {
namespace {

constexpr int kFrontThreads = 256;
constexpr int kFrontWarps = kFrontThreads / 32;
constexpr int kFrontMaxT = 64, kFrontMaxE = 256, kFrontMaxK = 16;
constexpr int kFrontMaxTE = 4096;          // tokens x experts
constexpr size_t kFrontMaxSmem = 200 * 1024;

QMOE_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
QMOE_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
QMOE_DEV uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
QMOE_DEV void dsmem_st_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
QMOE_DEV void dsmem_st_v4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}

// Shared-memory layout, in floats from the (16-byte aligned) dynamic base.
struct FrontLayout {
    int ep, tp;          // experts / tokens rounded up to the compute tiles
    int ws_ld, xs_ld;    // row strides of the transposed gate and x tiles
    int town;            // tokens owned by one CTA (at most)
    int ws, xs, recv, warp, sel, selw, tail;
    int warp_floats;
    int total;
};

// Compute tiles: 32 tokens x 64 experts per 128 threads, 4 x 4 per thread.
__host__ __device__ inline FrontLayout front_layout(int T, int E, int nc, int cs, int lc) {
    FrontLayout L;
    L.ep = (E + 63) / 64 * 64;
    L.tp = (T + 31) / 32 * 32;
    L.ws_ld = L.ep + 4;
    L.xs_ld = L.tp + 4;
    L.town = (T + cs - 1) / cs;
    L.ws = 0;
    L.xs = L.ws + lc * 64 * L.ws_ld;
    L.recv = (L.xs + lc * 64 * L.xs_ld + 3) / 4 * 4;         // [town][nc][E] partials
    // per warp: sorted exp [E], logits [E] (each from a 16-byte boundary),
    // group scores [64], kept groups [64]
    L.warp_floats = 2 * ((E + 3) / 4 * 4) + 128;
    L.warp = L.recv + (L.town * nc * E + 3) / 4 * 4;
    L.sel = L.warp + kFrontWarps * L.warp_floats;            // [T][K] ids (CTA 0)
    L.selw = L.sel + kFrontMaxT * kFrontMaxK;                // [T][K] weight bits (CTA 0)
    L.tail = (L.selw + kFrontMaxT * kFrontMaxK + 3) / 4 * 4; // TailState (CTA 0)
    L.total = L.tail;
    return L;
}

struct TailState {
    uint32_t mlo[kFrontMaxE], mhi[kFrontMaxE];  // tokens 0-31 / 32-63 that picked each expert
    uint32_t dlo[kEpMaxWorld], dhi[kEpMaxWorld];  // plan: tokens sending to each rank
    int off[kFrontMaxE];                         // segment start of each expert
    int wsum[2][kFrontWarps];                    // per-warp totals of the scans
};

// Partial chains of one (32 tokens) x (64 experts) tile of chunk c: thread
// (tx, ty) of 128 owns tokens tb + 4 ty .. + 3 and experts eb + 4 tx .. + 3;
// each token's four experts go to the owner CTA's partials [t / cs][c][e]
// (recv_s: the local address of that array, at the same offset in every
// CTA).
QMOE_DEV void partial_tile(const float *w, const float *x, int ws_ld, int xs_ld, int tb, int eb, int tx,
                           int ty, int T, int E, int nc, int c, int cs, uint32_t recv_s) {
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
#pragma unroll 8
    for (int k = 0; k < kGateChunk; ++k) {
        const float4 wb = *reinterpret_cast<const float4 *>(w + k * ws_ld + eb + 4 * tx);
        const float4 xv = *reinterpret_cast<const float4 *>(x + k * xs_ld + tb + 4 * ty);
        const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            acc[a][0] = __fmaf_rn(xa[a], wb.x, acc[a][0]);
            acc[a][1] = __fmaf_rn(xa[a], wb.y, acc[a][1]);
            acc[a][2] = __fmaf_rn(xa[a], wb.z, acc[a][2]);
            acc[a][3] = __fmaf_rn(xa[a], wb.w, acc[a][3]);
        }
    }
    const int e = eb + 4 * tx;
    if (e >= E) return;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int t = tb + 4 * ty + a;
        if (t >= T) continue;
        const uint32_t owner = (uint32_t)(t % cs);
        const uint32_t addr = dsmem_map(recv_s + 4u * (uint32_t)(((t / cs) * nc + c) * E + e), owner);
        if ((E & 3) == 0) {
            dsmem_st_v4(addr, acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
        } else {
#pragma unroll
            for (int b = 0; b < 4; ++b)
                if (e + b < E) dsmem_st_f32(addr + 4u * b, acc[a][b]);
        }
    }
}

// The permute of all T tokens from their selections sel[T][K] (one CTA, one
// thread per expert): expert segments in expert order, tokens in order
// inside a segment, groups of at most f.chunk positions (split_group), the
// shared groups last.
QMOE_DEV void permute_tail(const FrontParams &f, int T, int E, int K, const int *sel, TailState &S) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += kFrontThreads) {
        S.mlo[e] = 0u;
        S.mhi[e] = 0u;
    }
    __syncthreads();
    const int TK = T * K;
    for (int a = tid; a < TK; a += kFrontThreads) {
        const int t = a / K;
        atomicOr(t < 32 ? &S.mlo[sel[a]] : &S.mhi[sel[a]], 1u << (t & 31));
    }
    __syncthreads();
    const int e = tid;               // E <= kFrontThreads
    const uint64_t mask = e < E ? ((uint64_t)S.mhi[e] << 32) | S.mlo[e] : 0ull;
    const int cnt = __popcll(mask);
    const int ng = (cnt + f.chunk - 1) / f.chunk;
    int ci = cnt, gi = ng;           // inclusive warp scans
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int uc = __shfl_up_sync(0xffffffffu, ci, o), ug = __shfl_up_sync(0xffffffffu, gi, o);
        if (lane >= o) {
            ci += uc;
            gi += ug;
        }
    }
    if (lane == 31) {
        S.wsum[0][warp] = ci;
        S.wsum[1][warp] = gi;
    }
    __syncthreads();
    int cb = 0, gb = 0, ct = 0, gt = 0;
#pragma unroll
    for (int w = 0; w < kFrontWarps; ++w) {
        if (w < warp) {
            cb += S.wsum[0][w];
            gb += S.wsum[1][w];
        }
        ct += S.wsum[0][w];
        gt += S.wsum[1][w];
    }
    if (e < E) {
        const int off = cb + ci - cnt, goff = gb + gi - ng;
        S.off[e] = off;
        f.seg_off[e] = off;
        for (int g = 0; g < ng; ++g) {
            const int2 sg = split_group(cnt, f.chunk, g);
            f.groups[goff + g] = make_int4(e, off + sg.x, sg.y, 0);
        }
    }
    __syncthreads();
    // each assignment's position: its token's rank among the expert's tokens
    for (int a = tid; a < TK; a += kFrontThreads) {
        const int t = a / K, ea = sel[a];
        const uint64_t m = ((uint64_t)S.mhi[ea] << 32) | S.mlo[ea];
        const int pos = S.off[ea] + __popcll(m & ((1ull << t) - 1ull));
        f.pos_tok[pos] = t;
        f.assign_pos[a] = pos;
    }
    const int ns = (int)((f.shared_count + f.chunk - 1) / f.chunk);
    if (tid == 0) {
        f.seg_off[E] = ct;
        f.n_groups[0] = gt;
        f.n_groups[1] = ns;
    }
    for (int g = tid; g < ns; g += kFrontThreads) {
        const int2 sg = split_group(f.shared_count, f.chunk, g);
        f.groups[gt + g] = make_int4(E, TK + sg.x, sg.y, 0);
    }
}

// The expert-parallel send list of all T tokens (qmoe_ep_plan's padded
// layout) from their selections sel[T][K] and weight bits selw[T][K] (one
// CTA): rank d's rows start at d * C, tokens in order, each row's metadata
// the local ids on d (-1 for slots owned elsewhere) and the weights' bits;
// unused rows carry token 0, ids -1 and weight 0.
QMOE_DEV void plan_tail(const FrontParams &f, int T, int K, const int *sel, const int *selw, TailState &S) {
    const int tid = threadIdx.x, G = f.plan_world, epr = f.plan_epr;
    const int64_t C = f.plan_capacity;
    for (int d = tid; d < G; d += kFrontThreads) {
        S.dlo[d] = 0u;
        S.dhi[d] = 0u;
    }
    __syncthreads();
    for (int a = tid; a < T * K; a += kFrontThreads) {
        const int t = a / K, e = sel[a];
        if (e >= 0) atomicOr(t < 32 ? &S.dlo[e / epr] : &S.dhi[e / epr], 1u << (t & 31));
    }
    __syncthreads();
    for (int d = tid; d < G; d += kFrontThreads) f.send_counts[d] = __popc(S.dlo[d]) + __popc(S.dhi[d]);
    // rows past each destination's count: unused
    for (int64_t r = tid; r < (int64_t)G * C; r += kFrontThreads) {
        const int d = (int)(r / C);
        const int64_t i = r - (int64_t)d * C;
        if (i >= __popc(S.dlo[d]) + __popc(S.dhi[d])) {
            f.send_tok[r] = 0;
            int32_t *m = f.send_meta + r * 2 * K;
            for (int k = 0; k < K; ++k) {
                m[k] = -1;
                m[K + k] = 0;
            }
        }
    }
    // (token, destination) pairs: the row is d * C + the token's rank among
    // the tokens sending to d
    for (int a = tid; a < T * G; a += kFrontThreads) {
        const int t = a / G, d = a - t * G;
        const uint32_t lo = S.dlo[d], hi = S.dhi[d];
        const uint32_t below = (1u << (t & 31)) - 1u;
        const bool sends = ((t < 32 ? lo : hi) >> (t & 31)) & 1u;
        if (!sends) {
            f.slot_pos[a] = -1;
            continue;
        }
        const int64_t r = (int64_t)d * C + (t < 32 ? __popc(lo & below) : __popc(lo) + __popc(hi & below));
        f.send_tok[r] = t;
        int32_t *m = f.send_meta + r * 2 * K;
        for (int k = 0; k < K; ++k) {
            const int e = sel[t * K + k];
            const bool mine = e >= 0 && e / epr == d;
            m[k] = mine ? e - d * epr : -1;
            m[K + k] = mine ? selw[t * K + k] : 0;
        }
        f.slot_pos[a] = (int32_t)r;
    }
}

// One cluster of gridDim.x CTAs; CTA r owns hidden chunks [r*lc, r*lc + lc)
// and tokens r, r + cs, ... (one per warp).  N: experts per lane of the
// selection (E <= 32 N), one instantiation per size so that each holds one
// selection's code.
template <int N>
__global__ void __launch_bounds__(kFrontThreads, 1)
front_cluster_kernel(const RouterParams p, const FrontParams f, int lc) {
    extern __shared__ float4 front_smem4[];
    float *sm = reinterpret_cast<float *>(front_smem4);
    const int T = (int)p.T, E = p.E, K = p.K, H = p.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cs = (int)gridDim.x;
    const int rank = (int)cluster_ctarank();
    const int nc = H / kGateChunk;
    const FrontLayout L = front_layout(T, E, nc, cs, lc);
    const int c0 = rank * lc;
    const int nloc = max(0, min(lc, nc - c0));
    float *ws = sm + L.ws, *xs = sm + L.xs;

    // A.1 gate tiles of the local chunks, transposed to [k][expert] (lanes
    // along experts, so the transposing stores spread over the banks); loads
    // batched four per thread before their stores
    {
        const int n4 = nloc * E * 16;
        for (int i0 = 0; i0 < n4; i0 += 4 * kFrontThreads) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kFrontThreads + tid;
                if (i < n4) {
                    const int e = i % E, r = i / E, k4 = r & 15, cl = r >> 4;
                    v[u] = __ldg(reinterpret_cast<const float4 *>(p.gate_w + (int64_t)e * H +
                                                                  (c0 + cl) * kGateChunk + 4 * k4));
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kFrontThreads + tid;
                if (i < n4) {
                    const int e = i % E, r = i / E, k4 = r & 15, cl = r >> 4;
                    float *w = ws + cl * kGateChunk * L.ws_ld + e;
                    w[(4 * k4 + 0) * L.ws_ld] = v[u].x;
                    w[(4 * k4 + 1) * L.ws_ld] = v[u].y;
                    w[(4 * k4 + 2) * L.ws_ld] = v[u].z;
                    w[(4 * k4 + 3) * L.ws_ld] = v[u].w;
                }
            }
        }
    }
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    // A.2 activation tiles, transposed to [k][token]
    {
        const int n4 = nloc * T * 16;
        for (int i0 = 0; i0 < n4; i0 += 4 * kFrontThreads) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kFrontThreads + tid;
                if (i < n4) {
                    const int t = i % T, r = i / T, k4 = r & 15, cl = r >> 4;
                    const int64_t xi = (int64_t)t * H + (c0 + cl) * kGateChunk + 4 * k4;
                    v[u] = load_act4(p.x, p.dtype, xi);
                    // x may be host memory read over the bus: the CTAs'
                    // chunks together leave a device copy for later kernels
                    if (f.x_copy) store_act4(f.x_copy, p.dtype, xi, v[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kFrontThreads + tid;
                if (i < n4) {
                    const int t = i % T, r = i / T, k4 = r & 15, cl = r >> 4;
                    float *x = xs + cl * kGateChunk * L.xs_ld + t;
                    x[(4 * k4 + 0) * L.xs_ld] = v[u].x;
                    x[(4 * k4 + 1) * L.xs_ld] = v[u].y;
                    x[(4 * k4 + 2) * L.xs_ld] = v[u].z;
                    x[(4 * k4 + 3) * L.xs_ld] = v[u].w;
                }
            }
        }
    }
    __syncthreads();
    // A.3 chunk partials, pushed to the token owners
    const uint32_t recv_s = (uint32_t)__cvta_generic_to_shared(sm + L.recv);
    {
        // the two halves of the CTA take alternate (chunk, token tile,
        // expert tile) items
        const int h = tid >> 7, tx = tid & 15, ty = (tid >> 4) & 7;
        const int ntt = L.tp / 32, net = L.ep / 64, per = ntt * net;
        for (int it = h; it < nloc * per; it += 2) {
            const int cl = it / per, tile = it - cl * per;
            partial_tile(ws + cl * kGateChunk * L.ws_ld, xs + cl * kGateChunk * L.xs_ld, L.ws_ld, L.xs_ld,
                         (tile / net) * 32, (tile % net) * 64, tx, ty, T, E, nc, c0 + cl, cs, recv_s);
        }
    }
    cluster_sync_all();  // every token's partials are in its owner

    // B + C: warp w takes token t = rank + cs * w
    const int t = rank + cs * warp;
    if (t < T) {
        float *wsc = sm + L.warp + warp * L.warp_floats;
        const int e4 = (E + 3) / 4 * 4;
        float *ex = wsc, *lg = wsc + e4, *gs = wsc + 2 * e4;
        int *gk = reinterpret_cast<int *>(gs + 64);
        const float *rv = sm + L.recv + warp * nc * E;   // [nc][E] of this token
        for (int e = lane; e < E; e += 32) {
            float tot = 0.0f;
            int c = 0;
            for (; c + 8 <= nc; c += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = rv[(c + j) * E + e];
#pragma unroll
                for (int j = 0; j < 8; ++j) tot = __fadd_rn(tot, v[j]);
            }
            for (; c < nc; ++c) tot = __fadd_rn(tot, rv[c * E + e]);
            lg[e] = tot;
        }
        __syncwarp();
        const uint32_t sel0 = dsmem_map((uint32_t)__cvta_generic_to_shared(sm + L.sel), 0u);
        const uint32_t selw0 = dsmem_map((uint32_t)__cvta_generic_to_shared(sm + L.selw), 0u);
        select_token<N>(p, t, lane, lg, ex, gs, gk, sel0, selw0, true);
    }
    cluster_sync_all();  // every selection in CTA 0
    if (rank != 0) return;
    if (f.plan_world > 0)
        plan_tail(f, T, K, reinterpret_cast<const int *>(sm + L.sel), reinterpret_cast<const int *>(sm + L.selw),
                  *reinterpret_cast<TailState *>(sm + L.tail));
    else
        permute_tail(f, T, E, K, reinterpret_cast<const int *>(sm + L.sel),
                     *reinterpret_cast<TailState *>(sm + L.tail));
}

}  // namespace
}  // namespace qmoe

namespace qmoe {

// Cluster shape for a batch: cs CTAs of lc chunks each, or false when the
// batch or the layer is outside what one cluster handles.
static bool front_shape(int64_t T, int H, int E, int K, int max_cs, int *cs, int *lc, size_t *smem) {
    if (T < 1 || T > kFrontMaxT || E > kFrontMaxE || K > kFrontMaxK || T * E > kFrontMaxTE ||
        H % kGateChunk)
        return false;
    const int nc = H / kGateChunk;
    int c = nc < max_cs ? nc : max_cs;
    const int l = (nc + c - 1) / c;
    c = (nc + l - 1) / l;                 // no CTA without a chunk
    if (T > (int64_t)kFrontWarps * c) return false;
    const FrontLayout L = front_layout((int)T, E, nc, c, l);
    const size_t bytes = (size_t)L.total * 4 + sizeof(TailState);
    if (bytes > kFrontMaxSmem) return false;
    *cs = c;
    *lc = l;
    *smem = bytes;
    return true;
}

template <int N>
static cudaError_t launch_front_n(const RouterParams &p, const FrontParams &f, int cs, int lc, size_t smem,
                                  cudaStream_t s) {
    auto kern = front_cluster_kernel<N>;
    cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(kern), smem);
    if (e != cudaSuccess) return e;
    if (cs > 8) {
        // per-device attribute, idempotent
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)cs);
    cfg.blockDim = dim3(kFrontThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)cs;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, p, f, lc);
}

// Largest cluster (16, else 8) that the device can schedule for this
// kernel configuration; 0 if none.
static int front_max_cluster(size_t smem) {
    for (int cs : {16, 8}) {
        auto kern = front_cluster_kernel<8>;
        if (cs > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        if (ensure_dyn_smem(reinterpret_cast<const void *>(kern), smem) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3((unsigned)cs);
        cfg.blockDim = dim3(kFrontThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)cs;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) return cs;
        cudaGetLastError();
    }
    return 0;
}

// Per device (the kernel attributes and the occupancy query are per device).
static int front_cluster_size() {
    static std::mutex mu;
    static std::map<int, int> known;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    auto it = known.find(dev);
    if (it != known.end()) return it->second;
    const int mc = front_max_cluster(kFrontMaxSmem);
    known[dev] = mc;
    return mc;
}

bool front_cluster_ok(int64_t T, int H, int E, int K) {
    int cs, lc;
    size_t smem;
    if (!front_shape(T, H, E, K, 16, &cs, &lc, &smem)) return false;
    const int mc = front_cluster_size();
    return mc > 0 && front_shape(T, H, E, K, mc, &cs, &lc, &smem);
}

cudaError_t launch_front_cluster(const RouterParams &p, const FrontParams &f, cudaStream_t s) {
    const int mc = front_cluster_size();
    int cs, lc;
    size_t smem;
    if (mc <= 0 || !front_shape(p.T, p.H, p.E, p.K, mc, &cs, &lc, &smem))
        return cudaErrorInvalidConfiguration;
    if (p.E <= 32) return launch_front_n<1>(p, f, cs, lc, smem, s);
    if (p.E <= 64) return launch_front_n<2>(p, f, cs, lc, smem, s);
    if (p.E <= 128) return launch_front_n<4>(p, f, cs, lc, smem, s);
    return launch_front_n<8>(p, f, cs, lc, smem, s);
}

}  // namespace qmoe
