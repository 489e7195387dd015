// select.cuh -- per-token expert selection by one warp (sort-based), shared
// by the decode front (front.cu) and the batched selection kernel (router.cu).
//
// Same arithmetic as the reference's router (qmoe-rs src/moe.rs:51-82):
// scores, group limit, stable descending order with ties to the lower expert,
// softmax with its sum taken in descending-logit order, renormalisation and
// scaling of the top-k weights.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace qmoe {

// Warp-wide bitonic sort of 32*N keys (value, id), element i = 32 r + lane
// in (v[r], id[r]), into the order of ranks_before: descending value, ties
// to the lower id.  Afterwards element i has rank i.
template <int N>
QMOE_DEV void warp_sort(float (&v)[N], int (&id)[N], int lane) {
#pragma unroll
    for (int k = 2; k <= 32 * N; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32) {
                // partners in the same lane: registers r and r ^ (j / 32)
#pragma unroll
                for (int r = 0; r < N; ++r) {
                    const int pr = r ^ (j >> 5);
                    if (pr > r) {
                        const bool up = ((r * 32 + lane) & k) == 0;
                        const bool hi_first = ranks_before(v[pr], id[pr], v[r], id[r]);
                        if (hi_first == up) {
                            const float tv = v[r];
                            v[r] = v[pr];
                            v[pr] = tv;
                            const int ti = id[r];
                            id[r] = id[pr];
                            id[pr] = ti;
                        }
                    }
                }
            } else {
#pragma unroll
                for (int r = 0; r < N; ++r) {
                    const float pv = __shfl_xor_sync(0xffffffffu, v[r], j);
                    const int pi = __shfl_xor_sync(0xffffffffu, id[r], j);
                    const bool up = ((r * 32 + lane) & k) == 0;
                    const bool lower = (lane & j) == 0;
                    const bool partner_first = ranks_before(pv, pi, v[r], id[r]);
                    if (lower == up ? partner_first : !partner_first) {
                        v[r] = pv;
                        id[r] = pi;
                    }
                }
            }
        }
    }
}

// Scoring, group limit, top-k and combine weights of token t by one warp,
// from its logits lg[E] (the arithmetic of router_select_kernel; the ranks
// come from a sort instead of counting).  Lanes j < K write slot j's id and
// weight, and, when `gather`, the id and the weight's bits to a cluster CTA's
// gather arrays at the shared::cluster addresses sel0 and selw0.  E <= 32 N, K <= 32; ex, gs, gk: warp
// scratch of E, 64 and 64 entries.
template <int N>
QMOE_DEV void select_token(const RouterParams &p, int t, int lane, const float *lg, float *ex, float *gs,
                           int *gk, uint32_t sel0, uint32_t selw0, bool gather) {
    const int E = p.E, K = p.K;
    const bool sigm = p.scoring == 1;
    const float NEG = __int_as_float(0xff800000);
    float v[N];
    int id[N];
#pragma unroll
    for (int r = 0; r < N; ++r) {
        const int e = r * 32 + lane;
        id[r] = e;
        float c = NEG;               // padding ranks after every expert (id >= E)
        if (e < E) {
            c = lg[e];
            if (sigm) {
                c = qsigmoid(c);
                if (p.bias) c = __fadd_rn(c, p.bias[e]);
            }
        }
        v[r] = c;
    }
    const int G = p.n_group > 1 ? p.n_group : 1;
    if (G > 1) {
        // group score = best (softmax) or best + second (sigmoid); keep the
        // topk_group best groups, ties to the lower index
        const int per = E / G;
        float *ch = ex;              // choice by expert, until ex is needed
#pragma unroll
        for (int r = 0; r < N; ++r)
            if (r * 32 + lane < E) ch[r * 32 + lane] = v[r];
        __syncwarp();
        for (int g = lane; g < G; g += 32) {
            const float *c = ch + g * per;
            int bi = 0;
            float best = c[0];
            for (int j = 1; j < per; ++j)
                if (c[j] > best) {
                    best = c[j];
                    bi = j;
                }
            float second = NEG;
            bool have2 = false;
            for (int j = 0; j < per; ++j)
                if (j != bi && (!have2 || c[j] > second)) {
                    second = c[j];
                    have2 = true;
                }
            gs[g] = (!sigm || per < 2) ? best : __fadd_rn(best, second);
        }
        __syncwarp();
        for (int g = lane; g < G; g += 32) {
            int r = 0;
            for (int h = 0; h < G; ++h) r += ranks_before(gs[h], h, gs[g], g);
            gk[g] = r < p.topk_group;
        }
        __syncwarp();
#pragma unroll
        for (int r = 0; r < N; ++r)
            if (r * 32 + lane < E && !gk[(r * 32 + lane) / per]) v[r] = NEG;
        __syncwarp();
    }
    warp_sort<N>(v, id, lane);
    const int my_sel = id[0];        // rank `lane`: slot lane of the selection when lane < K

    float mx = 0.0f, s = 0.0f;
    if (!sigm) {
        // softmax over all experts (src/moe.rs:74-79): max, then the sum of
        // exp(l - max) in descending-logit order
        float lv[N];
        int lid[N];
#pragma unroll
        for (int r = 0; r < N; ++r) {
            lv[r] = v[r];
            lid[r] = id[r];
        }
        if (G > 1) {                 // the choice order dropped groups: sort the logits
#pragma unroll
            for (int r = 0; r < N; ++r) {
                const int e = r * 32 + lane;
                lid[r] = e;
                lv[r] = e < E ? lg[e] : NEG;
            }
            warp_sort<N>(lv, lid, lane);
        }
        mx = __shfl_sync(0xffffffffu, lv[0], 0);
#pragma unroll
        for (int r = 0; r < N; ++r)
            if (r * 32 + lane < E) ex[r * 32 + lane] = expf(__fsub_rn(lv[r], mx));
        __syncwarp();
        if (lane == 0) {
            int i = 0;
            for (; i + 4 <= E; i += 4) {
                const float4 q = *reinterpret_cast<const float4 *>(ex + i);
                s = __fadd_rn(s, q.x);
                s = __fadd_rn(s, q.y);
                s = __fadd_rn(s, q.z);
                s = __fadd_rn(s, q.w);
            }
            for (; i < E; ++i) s = __fadd_rn(s, ex[i]);
        }
        s = __shfl_sync(0xffffffffu, s, 0);
    }
    float w = 0.0f;
    if (lane < K) {
        // without a group limit slot j is rank j of the logits: its exp is ex[j]
        const float l = lg[my_sel];
        w = sigm ? qsigmoid(l) : __fdiv_rn(G > 1 ? expf(__fsub_rn(l, mx)) : ex[lane], s);
    }
    if (p.norm_topk) {
        float den = 0.0f;
        for (int j = 0; j < K; ++j) den = __fadd_rn(den, __shfl_sync(0xffffffffu, w, j));
        den = __fadd_rn(den, 1e-20f);
        w = __fdiv_rn(w, den);
    }
    if (p.routed_scale != 1.0f) w = __fmul_rn(w, p.routed_scale);
    if (lane < K) {
        p.topk_idx[(int64_t)t * K + lane] = my_sel;
        p.topk_w[(int64_t)t * K + lane] = w;
        if (gather) {
            asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(sel0 + 4u * (uint32_t)(t * K + lane)),
                         "r"(my_sel)
                         : "memory");
            asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(selw0 + 4u * (uint32_t)(t * K + lane)),
                         "r"(__float_as_int(w))
                         : "memory");
        }
    }
}

}  // namespace qmoe
