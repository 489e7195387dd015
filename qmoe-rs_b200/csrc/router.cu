// router.cu -- gate logits, scoring, top-k selection and combine weights.
//
// Replaces the router half of QMoELayer::forward (qmoe-rs src/moe.rs:51-82).
// One CTA routes one token.
//
// Logit order (pinned; qmoe-rs delegates the gate matmul to candle, whose
// order is not observable): the hidden dim is cut into 64-wide chunks; the
// partial of chunk c is an fmaf chain over its 64 products starting from 0;
// the logit is ((0 + p_0) + p_1) + ... in chunk order.  All chains run in
// parallel, one per thread; a second pass adds the partials of each expert
// in order.  The CPU oracle computes the same operations in the same order,
// so the logits, and the routing built from them, agree bit for bit.
//
// Selection: stable descending order with ties to the lower expert index
// (src/moe.rs:68-71), computed as a rank per expert.  Softmax weights use
// the max and the sum of exp(l - max) over all experts accumulated in that
// sorted order (src/moe.rs:74-79); sigmoid scoring uses the deterministic
// qexp, so scores and the selection on them are bit-exact as well.
#include "common.cuh"
#include "kernels.h"

namespace qmoe {
namespace {

constexpr int kRouterThreads = 256;
constexpr int kChunkBatch = 32;              // chunks per partials pass
constexpr int kXStride = kGateChunk + 1;     // padded chunk stride in smem

struct RouterSmem {
    // offsets in floats within the dynamic buffer
    int xs, part, logit, choice, ex, gscore, misc;
};

__host__ __device__ inline RouterSmem router_layout(int H, int E) {
    int nc = (H + kGateChunk - 1) / kGateChunk;
    RouterSmem L;
    L.xs = 0;
    L.part = L.xs + nc * kXStride;
    L.logit = L.part + E * kChunkBatch;
    L.choice = L.logit + E;
    L.ex = L.choice + E;
    L.gscore = L.ex + E;
    L.misc = L.gscore + 64;                  // n_group <= 64
    return L;
}

__global__ void __launch_bounds__(kRouterThreads)
router_kernel(const RouterParams p) {
    extern __shared__ float smem[];
    const RouterSmem L = router_layout(p.H, p.E);
    float *xs = smem + L.xs;
    float *part = smem + L.part;
    float *logit = smem + L.logit;
    float *choice = smem + L.choice;
    float *ex = smem + L.ex;
    float *gscore = smem + L.gscore;
    float *misc = smem + L.misc;             // [0] max, [1] sum
    int *sel = reinterpret_cast<int *>(misc + 4);        // [K]
    int *gkeep = reinterpret_cast<int *>(misc + 4 + 256); // [n_group]

    const int t = blockIdx.x;
    const int tid = threadIdx.x;
    const int H = p.H, E = p.E, K = p.K;
    const int nc = (H + kGateChunk - 1) / kGateChunk;

    // 1. token row -> smem (f32), chunk-padded
    for (int k = tid; k < nc * kGateChunk; k += kRouterThreads) {
        float v = k < H ? load_act(p.x, p.dtype, (int64_t)t * H + k) : 0.0f;
        xs[(k / kGateChunk) * kXStride + (k % kGateChunk)] = v;
    }
    for (int e = tid; e < E; e += kRouterThreads) logit[e] = 0.0f;
    __syncthreads();

    // 2. chunk partials, 32 chunks per pass, then ordered per-expert sums
    for (int c0 = 0; c0 < nc; c0 += kChunkBatch) {
        const int cb = min(kChunkBatch, nc - c0);
        for (int i = tid; i < E * cb; i += kRouterThreads) {
            const int e = i / cb, c = c0 + i % cb;
            const int k0 = c * kGateChunk;
            const int k1 = min(H, k0 + kGateChunk);
            const float *w = p.gate_w + (int64_t)e * H;
            const float *xc = xs + c * kXStride;
            float acc = 0.0f;
            if (k1 - k0 == kGateChunk && (H % 4) == 0) {
                const float4 *w4 = reinterpret_cast<const float4 *>(w + k0);
#pragma unroll 4
                for (int j = 0; j < kGateChunk / 4; ++j) {
                    float4 wv = __ldg(w4 + j);
                    acc = __fmaf_rn(xc[4 * j + 0], wv.x, acc);
                    acc = __fmaf_rn(xc[4 * j + 1], wv.y, acc);
                    acc = __fmaf_rn(xc[4 * j + 2], wv.z, acc);
                    acc = __fmaf_rn(xc[4 * j + 3], wv.w, acc);
                }
            } else {
                for (int k = k0; k < k1; ++k) acc = __fmaf_rn(xc[k - k0], __ldg(w + k), acc);
            }
            part[e * kChunkBatch + (c - c0)] = acc;
        }
        __syncthreads();
        for (int e = tid; e < E; e += kRouterThreads) {
            float tot = logit[e];
            for (int c = 0; c < cb; ++c) tot = __fadd_rn(tot, part[e * kChunkBatch + c]);
            logit[e] = tot;
        }
        __syncthreads();
    }

    // 3. scores for the selection
    const bool sigm = p.scoring == 1;
    for (int e = tid; e < E; e += kRouterThreads) {
        float c = logit[e];
        if (sigm) {
            c = qsigmoid(c);
            if (p.bias) c = __fadd_rn(c, p.bias[e]);
        }
        choice[e] = c;
    }
    __syncthreads();

    // 4. group limit: group score = best (softmax) or best + second
    //    (sigmoid); keep the topk_group best groups, ties to the lower index
    const int G = p.n_group > 1 ? p.n_group : 1;
    const float NEG = __int_as_float(0xff800000);
    if (G > 1) {
        const int per = E / G;
        for (int g = tid; g < G; g += kRouterThreads) {
            const float *c = choice + g * per;
            int bi = 0;
            float best = c[0];
            for (int j = 1; j < per; ++j)
                if (c[j] > best) { best = c[j]; bi = j; }
            float second = NEG;
            bool have2 = false;
            for (int j = 0; j < per; ++j)
                if (j != bi && (!have2 || c[j] > second)) { second = c[j]; have2 = true; }
            gscore[g] = (!sigm || per < 2) ? best : __fadd_rn(best, second);
        }
        __syncthreads();
        for (int g = tid; g < G; g += kRouterThreads) {
            int r = 0;
            for (int h = 0; h < G; ++h) r += ranks_before(gscore[h], h, gscore[g], g);
            gkeep[g] = r < p.topk_group;
        }
        __syncthreads();
        for (int e = tid; e < E; e += kRouterThreads)
            if (!gkeep[e / per]) choice[e] = NEG;
        __syncthreads();
    }

    // 5. rank of every expert; the first K ranks are the selection
    for (int e = tid; e < E; e += kRouterThreads) {
        const float v = choice[e];
        int r = 0;
        for (int j = 0; j < E; ++j) r += ranks_before(choice[j], j, v, e);
        if (r < K) sel[r] = e;
    }

    if (!sigm) {
        // softmax over all experts (src/moe.rs:74-79): max, then the sum of
        // exp(l - max) accumulated in descending-logit order
        float m = NEG;
        for (int e = tid; e < E; e += kRouterThreads) m = fmaxf(m, logit[e]);
        m = warp_max(m);
        if ((tid & 31) == 0) part[tid >> 5] = m;
        __syncthreads();
        if (tid == 0) {
            float mm = part[0];
            for (int w = 1; w < kRouterThreads / 32; ++w) mm = fmaxf(mm, part[w]);
            misc[0] = mm;
        }
        __syncthreads();
        const float mx = misc[0];
        for (int e = tid; e < E; e += kRouterThreads) {
            const float v = logit[e];
            int r = 0;
            for (int j = 0; j < E; ++j) r += ranks_before(logit[j], j, v, e);
            ex[r] = expf(__fsub_rn(v, mx));
        }
        __syncthreads();
        if (tid == 0) {
            float s = 0.0f;
            for (int i = 0; i < E; ++i) s = __fadd_rn(s, ex[i]);
            misc[1] = s;
        }
    }
    __syncthreads();

    // 6. combine weights
    if (tid == 0) {
        float w[64];
        const float mx = misc[0], s = misc[1];
        for (int j = 0; j < K; ++j) {
            const int e = sel[j];
            w[j] = sigm ? qsigmoid(logit[e]) : __fdiv_rn(expf(__fsub_rn(logit[e], mx)), s);
        }
        if (p.norm_topk) {
            float den = 0.0f;
            for (int j = 0; j < K; ++j) den = __fadd_rn(den, w[j]);
            den = __fadd_rn(den, 1e-20f);
            for (int j = 0; j < K; ++j) w[j] = __fdiv_rn(w[j], den);
        }
        if (p.routed_scale != 1.0f)
            for (int j = 0; j < K; ++j) w[j] = __fmul_rn(w[j], p.routed_scale);
        for (int j = 0; j < K; ++j) {
            p.topk_idx[(int64_t)t * K + j] = sel[j];
            p.topk_w[(int64_t)t * K + j] = w[j];
        }
    }
}

}  // namespace

size_t router_smem_bytes(int H, int E) {
    RouterSmem L = router_layout(H, E);
    return (size_t)(L.misc + 4 + 256 + 64) * sizeof(float);
}

cudaError_t launch_router(const RouterParams &p, cudaStream_t s) {
    if (p.T == 0) return cudaSuccess;
    size_t smem = router_smem_bytes(p.H, p.E);
    static size_t smem_set = 0;  // raise the opt-in limit only when needed
    if (smem > smem_set) {
        cudaError_t e = cudaFuncSetAttribute(router_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        smem_set = smem;
    }
    router_kernel<<<(unsigned)p.T, kRouterThreads, smem, s>>>(p);
    return cudaGetLastError();
}

}  // namespace qmoe
