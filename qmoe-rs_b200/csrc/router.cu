// router.cu -- gate logits, scoring, top-k selection and combine weights.
//
// Replaces the router half of QMoELayer::forward (qmoe-rs src/moe.rs:51-82).
//
// Logit order (pinned; qmoe-rs delegates the gate matmul to candle, whose
// order is not observable): the hidden dim is cut into 64-wide chunks; the
// partial of chunk c is an fmaf chain over its 64 products starting from 0;
// the logit is ((0 + p_0) + p_1) + ... in chunk order.  The CPU oracle
// computes the same operations in the same order, so the logits, and the
// routing built from them, agree bit for bit.  Two ways to get there:
//   few tokens   router_partials_kernel: one thread per (token, expert,
//                chunk) chain, all chains in parallel; the selection kernel
//                adds each expert's partials in chunk order;
//   many tokens  router_logits_kernel: 64x64 (token x expert) tiles staged
//                in shared memory chunk by chunk, each thread owning 4x4
//                logits and running the same chains and chunk sums.
// Then router_select_kernel, one CTA per token, scores and selects.
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

struct RouterSmem {
    // offsets in floats within the dynamic buffer
    int xs, part, logit, choice, ex, gscore, misc;
};

__host__ __device__ inline RouterSmem router_layout(int E) {
    RouterSmem L;
    L.xs = 0;
    L.part = 0;                              // 8 floats of warp maxima
    L.logit = L.part + 8;
    L.choice = L.logit + E;
    L.ex = L.choice + E;
    L.gscore = L.ex + E;
    L.misc = L.gscore + 64;                  // n_group <= 64
    return L;
}

// One thread per (token, expert, chunk): partial[t][e][c] = fmaf chain.
__global__ void __launch_bounds__(256)
router_partials_kernel(const RouterParams p) {
    const int nc = (p.H + kGateChunk - 1) / kGateChunk;
    const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
    if (i >= p.T * p.E * nc) return;
    const int c = (int)(i % nc);
    const int64_t te = i / nc;
    const int e = (int)(te % p.E);
    const int64_t t = te / p.E;
    const int k0 = c * kGateChunk, k1 = min(p.H, k0 + kGateChunk);
    const float *w = p.gate_w + (int64_t)e * p.H;
    float acc = 0.0f;
    if (k1 - k0 == kGateChunk) {
#pragma unroll 4
        for (int j = 0; j < kGateChunk; j += 4) {
            const float4 xv = load_act4(p.x, p.dtype, t * p.H + k0 + j);
            const float4 wv = __ldg(reinterpret_cast<const float4 *>(w + k0 + j));
            acc = __fmaf_rn(xv.x, wv.x, acc);
            acc = __fmaf_rn(xv.y, wv.y, acc);
            acc = __fmaf_rn(xv.z, wv.z, acc);
            acc = __fmaf_rn(xv.w, wv.w, acc);
        }
    } else {
        for (int k = k0; k < k1; ++k)
            acc = __fmaf_rn(load_act(p.x, p.dtype, t * p.H + k), __ldg(w + k), acc);
    }
    p.scratch[i] = acc;
}

// Tiled logits: CTA = 64 tokens x 64 experts, thread = 4 x 4 logits.
constexpr int kTileT = 64, kTileE = 64;
__global__ void __launch_bounds__(256)
router_logits_kernel(const RouterParams p) {
    __shared__ float xs[kGateChunk][kTileT + 1];
    __shared__ float ws[kGateChunk][kTileE + 1];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t t0 = (int64_t)blockIdx.x * kTileT;
    const int e0 = blockIdx.y * kTileE;
    float tot[4][4], acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) tot[a][b] = 0.0f;
    for (int k0 = 0; k0 < p.H; k0 += kGateChunk) {
        const int kn = min(kGateChunk, p.H - k0);
        for (int i = tid; i < kTileT * kGateChunk; i += 256) {
            const int rr = i / kGateChunk, k = i % kGateChunk;
            const int64_t t = t0 + rr;
            xs[k][rr] = (t < p.T && k < kn) ? load_act(p.x, p.dtype, t * p.H + k0 + k) : 0.0f;
            const int e = e0 + rr;
            ws[k][rr] = (e < p.E && k < kn) ? __ldg(p.gate_w + (int64_t)e * p.H + k0 + k) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
        for (int k = 0; k < kn; ++k) {
            float xa[4], wb[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) xa[a] = xs[k][ty * 4 + a];
#pragma unroll
            for (int b = 0; b < 4; ++b) wb[b] = ws[k][tx * 4 + b];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) acc[a][b] = __fmaf_rn(xa[a], wb[b], acc[a][b]);
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) tot[a][b] = __fadd_rn(tot[a][b], acc[a][b]);
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int64_t t = t0 + ty * 4 + a;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int e = e0 + tx * 4 + b;
            if (t < p.T && e < p.E) p.scratch[t * p.E + e] = tot[a][b];
        }
    }
}

// Scoring and selection, one CTA per token; logits from the partials
// (summed here in chunk order) or from router_logits_kernel.
__global__ void __launch_bounds__(kRouterThreads)
router_select_kernel(const RouterParams p, int from_partials) {
    extern __shared__ float smem[];
    const RouterSmem L = router_layout(p.E);
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
    const int E = p.E, K = p.K;
    const int nc = (p.H + kGateChunk - 1) / kGateChunk;
    for (int e = tid; e < E; e += kRouterThreads) {
        if (from_partials) {
            const float *pp = p.scratch + ((int64_t)t * E + e) * nc;
            float tot = 0.0f;
            for (int c = 0; c < nc; ++c) tot = __fadd_rn(tot, pp[c]);
            logit[e] = tot;
        } else {
            logit[e] = p.scratch[(int64_t)t * E + e];
        }
    }
    __syncthreads();

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
    (void)H;
    RouterSmem L = router_layout(E);
    return (size_t)(L.misc + 4 + 256 + 64) * sizeof(float);
}

constexpr int64_t kPartialsMaxLogits = 32768;  // T * E up to which the partials path runs

bool router_uses_partials(int64_t T, int E) { return T * E <= kPartialsMaxLogits; }

// Enough for every token count up to T on either path (monotonic in T, so a
// buffer reserved for a larger batch serves every smaller one).
size_t router_scratch_floats(int64_t T, int H, int E) {
    const int64_t nc = (H + kGateChunk - 1) / kGateChunk;
    const int64_t logits = T * E;
    const int64_t parts = (logits < kPartialsMaxLogits ? logits : kPartialsMaxLogits) * nc;
    return (size_t)(parts > logits ? parts : logits);
}

cudaError_t launch_router(const RouterParams &p, cudaStream_t s) {
    if (p.T == 0) return cudaSuccess;
    const bool parts = router_uses_partials(p.T, p.E);
    if (parts) {
        const int nc = (p.H + kGateChunk - 1) / kGateChunk;
        const int64_t n = p.T * p.E * nc;
        router_partials_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(p);
    } else {
        dim3 grid((unsigned)((p.T + kTileT - 1) / kTileT), (unsigned)((p.E + kTileE - 1) / kTileE));
        router_logits_kernel<<<grid, 256, 0, s>>>(p);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = router_smem_bytes(p.H, p.E);
    static size_t smem_set = 0;  // raise the opt-in limit only when needed
    if (smem > smem_set) {
        e = cudaFuncSetAttribute(router_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return e;
        smem_set = smem;
    }
    router_select_kernel<<<(unsigned)p.T, kRouterThreads, smem, s>>>(p, parts ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace qmoe
