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
//   partials     router_chunk_kernel: every (token, expert, chunk) chain in
//                parallel, tiles of tokens x 64 experts x one chunk staged
//                in shared memory; the selection kernel adds each expert's
//                partials in chunk order;
//   whole        router_logits_kernel, for batches whose partials would not
//                fit the scratch: 64x64 (token x expert) tiles over all
//                chunks, each thread owning 4x4 logits and running the same
//                chains and chunk sums.
// Then router_select_kernel, one CTA per token, scores and selects.
//
// Selection: stable descending order with ties to the lower expert index
// (src/moe.rs:68-71), computed as a rank per expert.  Softmax weights use
// the max and the sum of exp(l - max) over all experts accumulated in that
// sorted order (src/moe.rs:74-79); sigmoid scoring uses the deterministic
// qexp, so scores and the selection on them are bit-exact as well.
#include "common.cuh"
#include "kernels.h"
#include "select.cuh"

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

// Chunk partials, partial[c][t][e] = fmaf chain of chunk c.  CTA = 16*TT
// tokens x 64 experts x one chunk; thread = TT tokens x 4 experts.  Every
// chain is independent, so the grid covers tokens, experts and chunks.
template <int TT>
__global__ void __launch_bounds__(256)
router_chunk_kernel(const RouterParams p) {
    constexpr int kT = 16 * TT;
    __shared__ float xs[kGateChunk][kT + 1];
    __shared__ float ws[kGateChunk][64 + 1];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t t0 = (int64_t)blockIdx.x * kT;
    const int e0 = blockIdx.y * 64;
    const int c = blockIdx.z;
    const int k0 = c * kGateChunk;
    // the gate tile does not depend on the preceding kernel: stage it first
    for (int i = tid; i < 64 * (kGateChunk / 4); i += 256) {
        const int rr = i / (kGateChunk / 4), k4 = i % (kGateChunk / 4);
        const int e = e0 + rr;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e < p.E) v = __ldg(reinterpret_cast<const float4 *>(p.gate_w + (int64_t)e * p.H + k0 + 4 * k4));
        ws[4 * k4 + 0][rr] = v.x;
        ws[4 * k4 + 1][rr] = v.y;
        ws[4 * k4 + 2][rr] = v.z;
        ws[4 * k4 + 3][rr] = v.w;
    }
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    for (int i = tid; i < kT * (kGateChunk / 4); i += 256) {
        const int rr = i / (kGateChunk / 4), k4 = i % (kGateChunk / 4);
        const int64_t t = t0 + rr;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < p.T) v = load_act4(p.x, p.dtype, t * p.H + k0 + 4 * k4);
        xs[4 * k4 + 0][rr] = v.x;
        xs[4 * k4 + 1][rr] = v.y;
        xs[4 * k4 + 2][rr] = v.z;
        xs[4 * k4 + 3][rr] = v.w;
    }
    __syncthreads();
    float acc[TT][4];
#pragma unroll
    for (int a = 0; a < TT; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
#pragma unroll 8
    for (int k = 0; k < kGateChunk; ++k) {
        float xa[TT], wb[4];
#pragma unroll
        for (int a = 0; a < TT; ++a) xa[a] = xs[k][ty * TT + a];
#pragma unroll
        for (int b = 0; b < 4; ++b) wb[b] = ws[k][tx * 4 + b];
#pragma unroll
        for (int a = 0; a < TT; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) acc[a][b] = __fmaf_rn(xa[a], wb[b], acc[a][b]);
    }
    float *part = p.scratch + (int64_t)c * p.T * p.E;
#pragma unroll
    for (int a = 0; a < TT; ++a) {
        const int64_t t = t0 + ty * TT + a;
        if (t >= p.T) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int e = e0 + tx * 4 + b;
            if (e < p.E) part[t * p.E + e] = acc[a][b];
        }
    }
}

// Whole logits for batches whose partials would not fit the scratch: CTA =
// 64 tokens x 64 experts over all chunks, thread = 4 x 4 logits, each chunk
// an fmaf chain added to the running total in chunk order.  The next
// chunk's tiles are fetched into registers while this one is computed.
constexpr int kTileT = 64, kTileE = 64;
__global__ void __launch_bounds__(256, 2)
router_logits_kernel(const RouterParams p) {
    __shared__ float xs[kGateChunk][kTileT + 1];
    __shared__ float ws[kGateChunk][kTileE + 1];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int64_t t0 = (int64_t)blockIdx.x * kTileT;
    const int e0 = blockIdx.y * kTileE;
    const int nc = p.H / kGateChunk;
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    // this thread's loads: rows rr = (tid + 256 j) / 16, float4 k4 = tid % 16
    float4 xv[4], wv[4];
    auto fetch = [&](int c) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + 256 * j, rr = i >> 4, k4 = i & 15;
            const int64_t t = t0 + rr;
            const int e = e0 + rr;
            xv[j] = t < p.T ? load_act4(p.x, p.dtype, t * p.H + c * kGateChunk + 4 * k4)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
            wv[j] = e < p.E ? __ldg(reinterpret_cast<const float4 *>(p.gate_w + (int64_t)e * p.H +
                                                                    c * kGateChunk + 4 * k4))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    float tot[4][4], acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) tot[a][b] = 0.0f;
    fetch(0);
    for (int c = 0; c < nc; ++c) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = tid + 256 * j, rr = i >> 4, k4 = i & 15;
            xs[4 * k4 + 0][rr] = xv[j].x;
            xs[4 * k4 + 1][rr] = xv[j].y;
            xs[4 * k4 + 2][rr] = xv[j].z;
            xs[4 * k4 + 3][rr] = xv[j].w;
            ws[4 * k4 + 0][rr] = wv[j].x;
            ws[4 * k4 + 1][rr] = wv[j].y;
            ws[4 * k4 + 2][rr] = wv[j].z;
            ws[4 * k4 + 3][rr] = wv[j].w;
        }
        __syncthreads();
        if (c + 1 < nc) fetch(c + 1);
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
#pragma unroll 8
        for (int k = 0; k < kGateChunk; ++k) {
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

// Whole logits for large batches: fma.rn.f32x2 does two IEEE fused
// multiply-adds per lane, each rounded exactly as fmaf, so every (token,
// expert) chain is the pinned one: per 64-wide chunk an fmaf chain from 0
// over k in order, the chunk added to the running total in chunk order
// (add.rn.f32x2, two IEEE adds).
//
// The loop is bound by shared-memory wavefronts: a warp-wide 16-byte load
// takes four of them whatever the broadcast, one per eight lanes.  So each
// thread owns an 8 x 8 tile (8 tokens x 8 experts, 32 accumulator pairs)
// and reads per k two 16-byte loads of x and two of the gate -- 16
// wavefronts per warp for 64 FMAs per lane, which keeps pace with the FP32
// pipe at four warps per SM -- and duplicates each x value into the pair
// operand (x, x) with a register move.  CTA = 128 threads (2 x 2 warps)
// over 64 tokens x 128 experts; per chunk the shared memory holds x as
// [k][token] and the transposed gate (gate_t, made once per layer) as
// [k][expert].  Lanes are 4 token groups x 8 expert groups, so the eight
// lanes of a load phase read consecutive 16-byte chunks.  Two stages: the
// next chunk's gate tile arrives by cp.async and its x tile through
// registers (converted from bf16 when needed) while this chunk is computed.
constexpr int kGemmThreads = 128;
constexpr int kGemmK = kGateChunk;       // 64: one chunk per stage
constexpr int kGemmTokens = 64, kGemmExperts = 128;
constexpr int kGemmXFloats = kGemmK * kGemmTokens;
constexpr int kGemmWFloats = kGemmK * kGemmExperts;
constexpr int kGemmStageFloats = kGemmXFloats + kGemmWFloats;

QMOE_DEV unsigned long long ffma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

QMOE_DEV unsigned long long fadd2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

QMOE_DEV unsigned long long dup2(float v) {
    unsigned long long d;
    asm("mov.b64 %0, {%1, %1};" : "=l"(d) : "f"(v));
    return d;
}

QMOE_DEV void cp_async16(void *smem, const void *gmem, bool valid) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    const int n = valid ? 16 : 0;                 // 0: fill the 16 bytes with zeros
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sa), "l"(gmem), "r"(n) : "memory");
}

size_t router_gemm_smem_bytes() { return 2 * sizeof(float) * kGemmStageFloats; }

__global__ void __launch_bounds__(kGemmThreads, 1)
router_gemm_kernel(const RouterParams p) {
    extern __shared__ __align__(16) float gsm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wt = warp & 1, we = warp >> 1;        // 2 x 2 warps
    const int tg = lane & 3, eg = lane >> 2;
    const int64_t t0 = (int64_t)blockIdx.x * kGemmTokens;
    const int e0 = blockIdx.y * kGemmExperts;
    const int nc = p.H / kGemmK;
    const int ld = p.gate_t_ld;

    // gate tile of chunk c into stage st: rows k, 16-byte segments of experts
    auto load_w = [&](int c, int st) {
        float *ws = gsm + st * kGemmStageFloats + kGemmXFloats;
        constexpr int kSegs = kGemmExperts / 4;                  // per row
#pragma unroll
        for (int q = 0; q < kGemmK * kSegs / kGemmThreads; ++q) {
            const int i = q * kGemmThreads + tid;
            const int k = i / kSegs, sgm = i % kSegs;
            const int e = e0 + 4 * sgm;
            const bool ok = e < ld;
            const float *src = p.gate_t + (int64_t)(c * kGemmK + k) * ld + (ok ? e : 0);
            cp_async16(ws + k * kGemmExperts + 4 * sgm, src, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // x tile of chunk c: thread -> token r = tid / 2, half h = tid % 2 (32
    // consecutive k of that token)
    uint4 xr[8];                                                 // 32 f32 or 32 bf16 (4 used)
    const int xr_r = tid >> 1, xr_h = tid & 1;
    auto fetch_x = [&](int c) {
        const int64_t t = t0 + xr_r;
        const int64_t base = t * p.H + c * kGemmK + xr_h * 32;
#pragma unroll
        for (int q = 0; q < 8; ++q) xr[q] = make_uint4(0, 0, 0, 0);
        if (t < p.T) {
            if (p.dtype == 0) {
                const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const float *>(p.x) + base);
#pragma unroll
                for (int q = 0; q < 8; ++q) xr[q] = __ldg(src + q);
            } else {
                const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const __nv_bfloat16 *>(p.x) + base);
#pragma unroll
                for (int q = 0; q < 4; ++q) xr[q] = __ldg(src + q);
            }
        }
    };
    auto store_x = [&](int st) {
        float *xs = gsm + st * kGemmStageFloats;
        float v[32];
        if (p.dtype == 0) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                v[4 * q + 0] = __uint_as_float(xr[q].x);
                v[4 * q + 1] = __uint_as_float(xr[q].y);
                v[4 * q + 2] = __uint_as_float(xr[q].z);
                v[4 * q + 3] = __uint_as_float(xr[q].w);
            }
        } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t u[4] = {xr[q].x, xr[q].y, xr[q].z, xr[q].w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v[8 * q + 2 * j] = __uint_as_float(u[j] << 16);
                    v[8 * q + 2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) xs[(xr_h * 32 + j) * kGemmTokens + xr_r] = v[j];
    };

    // the gate is the layer's, independent of the preceding kernel
    load_w(0, 0);
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    fetch_x(0);
    store_x(0);

    unsigned long long acc[8][4], tot[8][4];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) tot[a][b] = 0ull;

    // this thread's tokens: 4 tg + 16 j + u (j < 2, u < 4) in the warp's 32;
    // experts: 4 eg + 32 q + v (q < 2, v < 4) in the warp's 64
    const int xo = wt * 8 + tg;          // float4 index in an x row (+ 4 j)
    const int wo = we * 16 + eg;         // float4 index in a gate row (+ 8 q)

    for (int c = 0; c < nc; ++c) {
        const int st = c & 1;
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();                               // stage st complete, stage st^1 free
        if (c + 1 < nc) {
            load_w(c + 1, st ^ 1);
            fetch_x(c + 1);
        }
        const float4 *xs = reinterpret_cast<const float4 *>(gsm + st * kGemmStageFloats);
        const ulonglong2 *ws = reinterpret_cast<const ulonglong2 *>(gsm + st * kGemmStageFloats + kGemmXFloats);
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) acc[a][b] = 0ull;
#pragma unroll 4
        for (int k = 0; k < kGemmK; ++k) {
            const float4 x0 = xs[k * (kGemmTokens / 4) + xo];
            const float4 x1 = xs[k * (kGemmTokens / 4) + xo + 4];
            const ulonglong2 w0 = ws[k * (kGemmExperts / 4) + wo];
            const ulonglong2 w1 = ws[k * (kGemmExperts / 4) + wo + 8];
            const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
            for (int a = 0; a < 8; ++a) {
                const unsigned long long xx = dup2(xv[a]);
                acc[a][0] = ffma2(xx, w0.x, acc[a][0]);
                acc[a][1] = ffma2(xx, w0.y, acc[a][1]);
                acc[a][2] = ffma2(xx, w1.x, acc[a][2]);
                acc[a][3] = ffma2(xx, w1.y, acc[a][3]);
            }
        }
#pragma unroll
        for (int a = 0; a < 8; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) tot[a][b] = fadd2(tot[a][b], acc[a][b]);
        if (c + 1 < nc) store_x(st ^ 1);
    }
    // acc row a = token 4 (wt*8 + tg) + 16 (a / 4) + a % 4; column pair b =
    // experts 4 (we*16 + eg) + 32 (b / 2) + 2 (b % 2) + {0, 1}
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        const int64_t t = t0 + 4 * (wt * 8 + tg) + 16 * (a >> 2) + (a & 3);
        if (t >= p.T) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const unsigned long long v = tot[a][b];
            const int e = e0 + 4 * (we * 16 + eg) + 32 * (b >> 1) + 2 * (b & 1);
            if (e < p.E) p.scratch[t * p.E + e] = __uint_as_float((uint32_t)v);
            if (e + 1 < p.E) p.scratch[t * p.E + e + 1] = __uint_as_float((uint32_t)(v >> 32));
        }
    }
}

// Chunk partials for layers that keep the transposed gate (E > 64), small
// batches: CTA = 32 tokens x 128 experts x one chunk, 128 threads; warp w
// owns experts 32w..32w+31, lane (tg = lane % 4, eg = lane / 4) 8 tokens x 4
// experts, i.e. 16 accumulator pairs of fma.rn.f32x2 (each lane two IEEE
// fused multiply-adds, rounded as fmaf: the chain of every (token, expert)
// over the chunk's 64 k in order, from 0).  Per k a warp reads two 16-byte
// loads of x and one of the gate: 12 shared-memory wavefronts for 32 FMAs
// per lane, against 10 for 8 in router_chunk_kernel.
constexpr int kChunkTTok = 32, kChunkTExp = 128, kChunkTThreads = 128;

__global__ void __launch_bounds__(kChunkTThreads)
router_chunk_t_kernel(const RouterParams p) {
    __shared__ __align__(16) float xs[kGateChunk][kChunkTTok];
    __shared__ __align__(16) float ws[kGateChunk][kChunkTExp];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t t0 = (int64_t)blockIdx.x * kChunkTTok;
    const int e0 = blockIdx.y * kChunkTExp;
    const int c = blockIdx.z;
    const int ld = p.gate_t_ld;
    // gate rows k of the chunk, experts e0 .. e0+127 (zero past ld): the
    // layer's, independent of the preceding kernel
    constexpr int kSegs = kChunkTExp / 4;
#pragma unroll
    for (int q = 0; q < kGateChunk * kSegs / kChunkTThreads; ++q) {
        const int i = q * kChunkTThreads + tid;
        const int k = i / kSegs, sgm = i % kSegs;
        const int e = e0 + 4 * sgm;
        const bool ok = e < ld;
        cp_async16(&ws[k][4 * sgm], p.gate_t + (int64_t)(c * kGateChunk + k) * ld + (ok ? e : 0), ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    {
        // x: warp w stores k = 16w .. 16w+15 of token lane (no bank conflicts)
        const int r = lane, kq = warp * 16;
        const int64_t t = t0 + r;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.0f;
        if (t < p.T) {
            const int64_t base = t * p.H + (int64_t)c * kGateChunk + kq;
            if (p.dtype == 0) {
                const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(p.x) + base);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 a = __ldg(src + q);
                    v[4 * q] = a.x;
                    v[4 * q + 1] = a.y;
                    v[4 * q + 2] = a.z;
                    v[4 * q + 3] = a.w;
                }
            } else {
                const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const __nv_bfloat16 *>(p.x) + base);
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const uint4 a = __ldg(src + q);
                    const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        v[8 * q + 2 * j] = __uint_as_float(u[j] << 16);
                        v[8 * q + 2 * j + 1] = __uint_as_float(u[j] & 0xffff0000u);
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) xs[kq + j][r] = v[j];
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const int tg = lane & 3, eg = lane >> 2;
    const float4 *xs4 = reinterpret_cast<const float4 *>(&xs[0][0]);
    const ulonglong2 *ws2 = reinterpret_cast<const ulonglong2 *>(&ws[0][0]);
    const int xo = 2 * tg, wo = warp * 8 + eg;     // float4 index in an x row / a gate row
    unsigned long long acc[8][2];
#pragma unroll
    for (int a = 0; a < 8; ++a) acc[a][0] = acc[a][1] = 0ull;
#pragma unroll 8
    for (int k = 0; k < kGateChunk; ++k) {
        const float4 x0 = xs4[k * (kChunkTTok / 4) + xo];
        const float4 x1 = xs4[k * (kChunkTTok / 4) + xo + 1];
        const ulonglong2 w = ws2[k * (kChunkTExp / 4) + wo];
        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int a = 0; a < 8; ++a) {
            const unsigned long long xx = dup2(xv[a]);
            acc[a][0] = ffma2(xx, w.x, acc[a][0]);
            acc[a][1] = ffma2(xx, w.y, acc[a][1]);
        }
    }
    // acc[a] = token 8 tg + a, experts 4 (8 warp + eg) + {0, 1, 2, 3}
    float *part = p.scratch + (int64_t)c * p.T * p.E;
    const int e = e0 + 4 * wo;
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        const int64_t t = t0 + 8 * tg + a;
        if (t >= p.T) continue;
        const float v[4] = {__uint_as_float((uint32_t)acc[a][0]), __uint_as_float((uint32_t)(acc[a][0] >> 32)),
                            __uint_as_float((uint32_t)acc[a][1]), __uint_as_float((uint32_t)(acc[a][1] >> 32))};
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (e + j < p.E) part[t * p.E + e + j] = v[j];
    }
}

// Whole logits from the chunk partials, one thread per (token, expert): the
// ordered chunk sum, loads issued thirty-two at a time, written over the
// slot of chunk 0 that only this thread reads.  For batches too small to
// give the one-warp-per-token selection enough warps to sum its partials
// quickly.
constexpr int kSumThreads = 128;

__global__ void __launch_bounds__(kSumThreads)
router_sum_kernel(const RouterParams p) {
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int64_t i = (int64_t)blockIdx.x * kSumThreads + threadIdx.x;
    const int64_t n = p.T * p.E;
    if (i >= n) return;
    const int nc = p.H / kGateChunk;
    const float *pp = p.scratch + i;
    float tot = 0.0f;
    int c = 0;
    for (; c + 32 <= nc; c += 32) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __ldcg(pp + (c + j) * n);
#pragma unroll
        for (int j = 0; j < 32; ++j) tot = __fadd_rn(tot, v[j]);
    }
    for (; c < nc; ++c) tot = __fadd_rn(tot, __ldcg(pp + c * n));
    p.scratch[i] = tot;
}

__global__ void transpose_gate_kernel(const float *w, int E, int H, float *wt, int ld) {
    __shared__ float tile[32][33];
    const int e0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int e = e0 + i, k = k0 + threadIdx.x;
        tile[i][threadIdx.x] = (e < E && k < H) ? w[(int64_t)e * H + k] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int k = k0 + i, e = e0 + threadIdx.x;
        if (k < H && e < ld) wt[(int64_t)k * ld + e] = tile[threadIdx.x][i];
    }
}

// Permute run by the selection kernel's last CTA (small batches).
constexpr int kTailMaxT = 64, kTailMaxE = 256, kTailMaxK = 16;
struct TailSmem {
    unsigned long long mask[kTailMaxE];   // tokens that picked each expert
    int cnt[kTailMaxE], off[kTailMaxE + 1], goff[kTailMaxE + 1];
    int sel[kTailMaxT][kTailMaxK];
    int is_last;
};

// With f.counter set: the last CTA of the selection kernel to finish builds
// the expert segments and the work list from every token's selection (what
// permute_kernel does), saving a launch for small batches.  Called by every
// thread of every CTA after its own selections are stored.
QMOE_DEV void permute_tail(const RouterParams &p, const FrontParams &f) {
    if (!f.counter) return;
    __shared__ TailSmem S;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int E = p.E, K = p.K;
    __threadfence();
    __syncthreads();
    if (tid == 0) S.is_last = atomicAdd(f.counter, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!S.is_last) return;
    __threadfence();
    const int T = (int)p.T;
    const int lane = tid & 31, warp = tid >> 5;
    for (int a = tid; a < T * K; a += nthr) S.sel[a / K][a % K] = __ldcg(p.topk_idx + a);
    __syncthreads();
    // expert segments in expert order, tokens in order inside a segment (the
    // rank of token t in expert e's segment is the number of earlier tokens
    // in e's token mask), groups of at most f.chunk positions, shared groups
    // last
    for (int e = tid; e < E; e += nthr) S.mask[e] = 0ull;
    __syncthreads();
    const int TK = T * K;
    for (int a = tid; a < TK; a += nthr) {
        const int t = a / K;
        atomicOr(&S.mask[S.sel[t][a - t * K]], 1ull << t);
    }
    __syncthreads();
    if (warp == 0) {
        // exclusive scans over experts of counts and of group counts, 8
        // experts per lane
        int c8[8], g8[8], cs = 0, gsum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = lane * 8 + j;
            c8[j] = e < E ? __popcll(S.mask[e]) : 0;
            g8[j] = (c8[j] + f.chunk - 1) / f.chunk;
            cs += c8[j];
            gsum += g8[j];
        }
        int ci = cs, gi = gsum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int uc = __shfl_up_sync(0xffffffffu, ci, o), ug = __shfl_up_sync(0xffffffffu, gi, o);
            if (lane >= o) { ci += uc; gi += ug; }
        }
        int run = ci - cs, grun = gi - gsum;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = lane * 8 + j;
            if (e < E) {
                S.off[e] = run;
                S.goff[e] = grun;
                S.cnt[e] = c8[j];
            }
            run += c8[j];
            grun += g8[j];
        }
        if (lane == 31) {
            S.off[E] = run;
            S.goff[E] = grun;
            f.seg_off[E] = run;
            f.n_groups[0] = grun;
            f.n_groups[1] = (int)((f.shared_count + f.chunk - 1) / f.chunk);
        }
    }
    __syncthreads();
    for (int e = tid; e < E; e += nthr) {
        f.seg_off[e] = S.off[e];
        const int c = S.cnt[e];
        for (int g = 0; g * f.chunk < c; ++g) {
            const int2 sg = split_group(c, f.chunk, g);
            f.groups[S.goff[e] + g] = make_int4(e, S.off[e] + sg.x, sg.y, 0);
        }
    }
    {
        const int ns = (int)((f.shared_count + f.chunk - 1) / f.chunk);
        for (int g = tid; g < ns; g += nthr) {
            const int2 sg = split_group(f.shared_count, f.chunk, g);
            f.groups[S.goff[E] + g] = make_int4(E, (int)(TK + sg.x), sg.y, 0);
        }
    }
    for (int a = tid; a < TK; a += nthr) {
        const int t = a / K, e = S.sel[t][a - t * K];
        const int pos = S.off[e] + __popcll(S.mask[e] & ((1ull << t) - 1ull));
        f.pos_tok[pos] = t;
        f.assign_pos[a] = pos;
    }
    __syncthreads();
    if (tid == 0) *f.counter = 0;
}

// Warp: the value at the first index (lane) of the largest non-NaN value
// among the lanes other than `skip` -- the result of the scan
// `best = v[first]; for later j: if (v[j] > best) best = v[j]` when the
// first considered value is not NaN; its lane in *idx.
QMOE_DEV float first_max(float v, int ln, int skip, int *idx) {
    const float NEG = __int_as_float(0xff800000);
    const bool out = ln == skip || v != v;
    float bv = out ? NEG : v;
    int bi = out ? 64 + ln : ln;                   // excluded lanes lose every tie
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    *idx = bi;
    return bv;
}

// Scoring and selection, one CTA per token; logits from the partials
// (summed here in chunk order) or from router_logits_kernel.  With f.counter
// set, the last CTA to finish also builds the expert segments and the work
// list (what permute_kernel does), saving a launch for small batches.
__global__ void __launch_bounds__(kRouterThreads)
router_select_kernel(const RouterParams p, int from_partials, const FrontParams f) {
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
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    for (int e = tid; e < E; e += kRouterThreads) {
        if (from_partials) {
            const float *pp = p.scratch + (int64_t)t * E + e;
            const int64_t stride = (int64_t)p.T * E;
            float tot = 0.0f;
            for (int c = 0; c < nc; ++c) tot = __fadd_rn(tot, pp[c * stride]);
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
        if (per == 32 && G <= kRouterThreads / 32) {
            // warp g, lane j: expert g*32 + j; the scans below as shuffle
            // reductions with the same results
            const int wg = tid >> 5, ln = tid & 31;
            if (wg < G) {
                const float v = choice[wg * 32 + ln];
                const float c0 = __shfl_sync(0xffffffffu, v, 0);
                float best = c0;
                int bi = 0;
                if (c0 == c0) best = first_max(v, ln, -1, &bi);   // else NaN first: never replaced
                float second = NEG;
                if (sigm) {
                    const float cj0 = __shfl_sync(0xffffffffu, v, bi == 0 ? 1 : 0);
                    int si;
                    second = cj0 == cj0 ? first_max(v, ln, bi, &si) : cj0;
                }
                if (ln == 0) gscore[wg] = !sigm ? best : __fadd_rn(best, second);
            }
        } else {
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

    // 5. rank of every expert (a count: any order of the terms); the first
    //    K ranks are the selection.  When at least K experts of the kept
    //    groups score above -inf and no score is NaN, the K best are kept
    //    experts that every dropped expert (-inf) ranks after, so only kept
    //    experts are ranked, against kept experts alone.
    int n_real = 0, n_nan = 0;
    for (int e = tid; e < E; e += kRouterThreads) {
        const float v = choice[e];
        n_real += v > NEG;
        n_nan += v != v;
    }
    {
        __shared__ int s_cnt[2];
        if (tid < 2) s_cnt[tid] = 0;
        __syncthreads();
        if (n_real) atomicAdd(&s_cnt[0], n_real);
        if (n_nan) atomicAdd(&s_cnt[1], n_nan);
        __syncthreads();
        n_real = s_cnt[0];
        n_nan = s_cnt[1];
    }
    const bool kept_only = G > 1 && n_nan == 0 && n_real >= K;
    const int per = E / G;
    for (int e = tid; e < E; e += kRouterThreads) {
        const float v = choice[e];
        if (kept_only && !(v > NEG)) continue;     // ranks after the K best
        int r = 0;
        if (kept_only) {
            for (int g = 0; g < G; ++g) {
                if (!gkeep[g]) continue;
#pragma unroll 8
                for (int j = g * per; j < (g + 1) * per; ++j) r += ranks_before(choice[j], j, v, e);
            }
        } else {
#pragma unroll 16
            for (int j = 0; j < E; ++j) r += ranks_before(choice[j], j, v, e);
        }
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
#pragma unroll 16
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

    // 6. combine weights: slot j's by thread j, then the ordered sums by
    //    thread 0
    float *wsel = choice;                          // free after the ranking
    if (tid < K) {
        const float mx = misc[0], s = misc[1];
        const int e = sel[tid];
        wsel[tid] = sigm ? qsigmoid(logit[e]) : __fdiv_rn(expf(__fsub_rn(logit[e], mx)), s);
    }
    __syncthreads();
    if (tid == 0) {
        float w[64];
        for (int j = 0; j < K; ++j) w[j] = wsel[j];
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
    permute_tail(p, f);
}

// Scoring and selection with one warp per token, eight tokens per CTA (E <=
// 256, K <= 32): the logits from the partials (added in chunk order, loads
// issued eight at a time) or from the other logit kernels, then the warp's
// sort-based selection; with f.counter set the last CTA then runs the
// permute.
constexpr int kSelWarps = 8;

__host__ __device__ inline int sel_warp_floats(int E) { return 2 * ((E + 3) / 4 * 4) + 128; }

// One warp: token t's logits into lg, then its selection.
QMOE_DEV void select_warp_token(const RouterParams &p, int from_partials, int64_t t, int lane, float *lg,
                                float *ex, float *gs, int *gk) {
    const int E = p.E;
    const int nc = p.H / kGateChunk;
    for (int e = lane; e < E; e += 32) {
        if (from_partials) {
            const float *pp = p.scratch + t * E + e;
            const int64_t stride = p.T * E;
            float tot = 0.0f;
            int c = 0;
            for (; c + 8 <= nc; c += 8) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = pp[(c + j) * stride];
#pragma unroll
                for (int j = 0; j < 8; ++j) tot = __fadd_rn(tot, v[j]);
            }
            for (; c < nc; ++c) tot = __fadd_rn(tot, pp[c * stride]);
            lg[e] = tot;
        } else {
            lg[e] = p.scratch[t * E + e];
        }
    }
    __syncwarp();
    if (E <= 32)
        select_token<1>(p, (int)t, lane, lg, ex, gs, gk, 0u, 0u, false);
    else if (E <= 64)
        select_token<2>(p, (int)t, lane, lg, ex, gs, gk, 0u, 0u, false);
    else if (E <= 128)
        select_token<4>(p, (int)t, lane, lg, ex, gs, gk, 0u, 0u, false);
    else
        select_token<8>(p, (int)t, lane, lg, ex, gs, gk, 0u, 0u, false);
}

__global__ void __launch_bounds__(kSelWarps * 32)
router_select_warp_kernel(const RouterParams p, int from_partials, const FrontParams f) {
    extern __shared__ float wsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int E = p.E, e4 = (E + 3) / 4 * 4;
    float *ex = wsm + warp * sel_warp_floats(E), *lg = ex + e4, *gs = lg + e4;
    int *gk = reinterpret_cast<int *>(gs + 64);
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int64_t t = (int64_t)blockIdx.x * kSelWarps + warp;
    if (t < p.T) select_warp_token(p, from_partials, t, lane, lg, ex, gs, gk);
    permute_tail(p, f);
}

}  // namespace

size_t router_smem_bytes(int H, int E) {
    (void)H;
    RouterSmem L = router_layout(E);
    return (size_t)(L.misc + 4 + 256 + 64) * sizeof(float);
}

// Chunk partials (T * E * H/64 floats) up to this size; whole logits beyond.
constexpr int64_t kPartialsMaxFloats = int64_t(32) << 20;

bool router_uses_partials(int64_t T, int H, int E) {
    return T * E * (H / kGateChunk) <= kPartialsMaxFloats;
}

// The paired-FP32 tile kernel (layers of more than 64 experts, whose gate
// the layer keeps transposed) once the batch fills at least ~half the SMs
// with its 8192-logit tiles, and always where the partials do not fit.
static bool router_uses_gemm(const RouterParams &p) {
    return p.gate_t != nullptr && p.E > 64 &&
           (p.T * p.E >= (int64_t)1 << 19 || !router_uses_partials(p.T, p.H, p.E));
}

int gate_t_ld(int E) { return (E + 3) / 4 * 4; }

cudaError_t launch_transpose_gate(const float *gate_w, int E, int H, float *gate_t, int ld, cudaStream_t s) {
    dim3 grid((unsigned)((H + 31) / 32), (unsigned)((ld + 31) / 32));
    transpose_gate_kernel<<<grid, dim3(32, 8), 0, s>>>(gate_w, E, H, gate_t, ld);
    return cudaGetLastError();
}

// Enough for every token count up to T on either path (monotonic in T, so a
// buffer reserved for a larger batch serves every smaller one).
size_t router_scratch_floats(int64_t T, int H, int E) {
    const int64_t nc = H / kGateChunk;
    const int64_t logits = T * E;
    const int64_t parts = logits * nc <= kPartialsMaxFloats ? logits * nc : kPartialsMaxFloats;
    return (size_t)(parts > logits ? parts : logits);
}

bool router_tail_ok(int64_t T, int E, int K) {
    return T >= 1 && T <= kTailMaxT && E <= kTailMaxE && K <= kTailMaxK;
}

cudaError_t launch_router(const RouterParams &p, const FrontParams *tail, cudaStream_t s) {
    if (p.T == 0) return cudaSuccess;
    FrontParams f{};
    if (tail) f = *tail;
    const bool gemm = router_uses_gemm(p);
    const bool parts = !gemm && router_uses_partials(p.T, p.H, p.E);
    if (gemm) {
        const size_t smem = router_gemm_smem_bytes();
        cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(router_gemm_kernel), smem);
        if (e != cudaSuccess) return e;
        dim3 grid((unsigned)((p.T + kGemmTokens - 1) / kGemmTokens),
                  (unsigned)((p.E + kGemmExperts - 1) / kGemmExperts));
        e = launch_pdl(router_gemm_kernel, grid, dim3(kGemmThreads), smem, s, p);
        if (e != cudaSuccess) return e;
    } else if (parts && p.gate_t && p.E > 64 && p.T <= 64) {
        dim3 grid((unsigned)((p.T + kChunkTTok - 1) / kChunkTTok), (unsigned)((p.E + kChunkTExp - 1) / kChunkTExp),
                  (unsigned)(p.H / kGateChunk));
        cudaError_t e = launch_pdl(router_chunk_t_kernel, grid, dim3(kChunkTThreads), 0, s, p);
        if (e != cudaSuccess) return e;
    } else if (parts) {
        const int nc = p.H / kGateChunk;
        const int TT = p.T <= 16 ? 1 : p.T <= 32 ? 2 : 4;
        dim3 grid((unsigned)((p.T + 16 * TT - 1) / (16 * TT)), (unsigned)((p.E + 63) / 64), (unsigned)nc);
        cudaError_t e = TT == 1 ? launch_pdl(router_chunk_kernel<1>, grid, dim3(256), 0, s, p)
                      : TT == 2 ? launch_pdl(router_chunk_kernel<2>, grid, dim3(256), 0, s, p)
                                : launch_pdl(router_chunk_kernel<4>, grid, dim3(256), 0, s, p);
        if (e != cudaSuccess) return e;
    } else {
        dim3 grid((unsigned)((p.T + kTileT - 1) / kTileT), (unsigned)((p.E + kTileE - 1) / kTileE));
        cudaError_t e = launch_pdl(router_logits_kernel, grid, dim3(256), 0, s, p);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // few tokens and many chunks: the partials are summed by one thread per
    // logit first (a warp or CTA per token would read them nearly serially)
    bool from_parts = parts;
    if (parts && p.T < 256 && p.H / kGateChunk >= 16) {
        e = launch_pdl(router_sum_kernel, dim3((unsigned)((p.T * p.E + kSumThreads - 1) / kSumThreads)),
                       dim3(kSumThreads), 0, s, p);
        if (e != cudaSuccess) return e;
        from_parts = false;
    }
    // (with the permute hand-off the CTA-per-token selection is faster for
    // these few tokens: the warp selection of 8 of 256 experts measured
    // 55 us against 19 us at 32 tokens)
    if (!f.counter && p.E <= 256 && p.K <= 32) {
        const size_t wsmem = sizeof(float) * kSelWarps * sel_warp_floats(p.E);
        e = ensure_dyn_smem(reinterpret_cast<const void *>(router_select_warp_kernel), wsmem);
        if (e != cudaSuccess) return e;
        return launch_pdl(router_select_warp_kernel, dim3((unsigned)((p.T + kSelWarps - 1) / kSelWarps)),
                          dim3(kSelWarps * 32), wsmem, s, p, from_parts ? 1 : 0, f);
    }
    const size_t smem = router_smem_bytes(p.H, p.E);
    e = ensure_dyn_smem(reinterpret_cast<const void *>(router_select_kernel), smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(router_select_kernel, dim3((unsigned)p.T), dim3(kRouterThreads), smem, s, p,
                      from_parts ? 1 : 0, f);
}

}  // namespace qmoe

