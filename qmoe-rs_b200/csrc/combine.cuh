// combine.cuh -- weighted combine of the expert outputs plus the shared expert.
//
// Replaces the accumulation of QMoELayer::forward (qmoe-rs src/moe.rs:121-125:
// output_buf[t] += down_out * weight, experts visited in ascending index
// order) and the shared-expert add of the decoder layer (src/model.rs:386-389:
// moe_out + shared_out).  Per output element the operations and their order
// are the reference's: acc = 0; for each of the token's experts in ascending
// index, acc = acc + (y * w) (two roundings, no FMA); then acc + shared.
//
// Used by the combine kernel (combine.cu) and by the last phase of the
// cooperative down GEMV (qgemv_imma.cu); y may have been written by other
// CTAs of the same grid, so its rows are read through L2.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace qmoe {

constexpr int kCombineMaxK = 64;

// Warp: token t's live slots (assignment position >= 0) in ascending expert
// order, equal ids in slot order (the reference's stable order), into
// s_pos / s_w; returns their count (the same in every lane).
QMOE_DEV int combine_rank(const CombineParams &p, int64_t t, int lane, int *s_pos, float *s_w) {
    const int K = p.K, ld = p.topk_ld;
    int n_live = 0;
    for (int j0 = 0; j0 < K; j0 += 32) {
        const int j = j0 + lane;
        int pos = -1, e = 0x7fffffff;
        float w = 0.0f;
        if (j < K) {
            pos = p.assign_pos[t * K + j];
            e = p.topk_idx[t * ld + j];
            w = p.topk_w[t * ld + j];
        }
        const bool live = pos >= 0;
        int r = 0;
        for (int i0 = 0; i0 < K; i0 += 32)
#pragma unroll
            for (int l = 0; l < 32; ++l) {
                const int i = i0 + l;
                // slot i of the other 32-block is reloaded from memory
                int ei, pi;
                if (i0 == j0) {
                    ei = __shfl_sync(0xffffffffu, e, l);
                    pi = __shfl_sync(0xffffffffu, pos, l);
                } else {
                    ei = i < K ? p.topk_idx[t * ld + i] : 0x7fffffff;
                    pi = i < K ? p.assign_pos[t * K + i] : -1;
                }
                if (i < K && pi >= 0 && (ei < e || (ei == e && i < j))) ++r;
            }
        if (j < K && live) {
            s_pos[r] = pos;
            s_w[r] = w;
        }
        n_live += __popc(__ballot_sync(0xffffffffu, j < K && live));
    }
    return n_live;
}

// Output columns h .. h + 3 of token t from its n ranked rows, into the row
// at orow (p.out_dtype; nullptr: row t of p.out).
QMOE_DEV void combine_float4(const CombineParams &p, int64_t t, int h, int n, const int *s_pos,
                             const float *s_w, void *orow = nullptr) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    const bool shared = p.y_shared && t >= p.shared_row0 && t < p.shared_row0 + p.shared_count;
    // the shared row's load is issued with the first batch
    float4 sv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (shared) sv = __ldcg(reinterpret_cast<const float4 *>(p.y_shared + (t - p.shared_row0) * p.H + h));
    for (int q = 0; q < n; q += 8) {
        float4 y[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (q + u < n) y[u] = __ldcg(reinterpret_cast<const float4 *>(p.y + (int64_t)s_pos[q + u] * p.H + h));
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (q + u >= n) break;
            const float w = s_w[q + u];
            a0 = __fadd_rn(a0, __fmul_rn(y[u].x, w));
            a1 = __fadd_rn(a1, __fmul_rn(y[u].y, w));
            a2 = __fadd_rn(a2, __fmul_rn(y[u].z, w));
            a3 = __fadd_rn(a3, __fmul_rn(y[u].w, w));
        }
    }
    if (shared) {
        a0 = __fadd_rn(a0, sv.x);
        a1 = __fadd_rn(a1, sv.y);
        a2 = __fadd_rn(a2, sv.z);
        a3 = __fadd_rn(a3, sv.w);
    }
    if (p.residual) {
        // residual + (moe_out + shared_out) (src/model.rs:409-412)
        const float4 r = load_act4_cg(p.residual, p.out_dtype, t * p.H + h);
        a0 = __fadd_rn(r.x, a0);
        a1 = __fadd_rn(r.y, a1);
        a2 = __fadd_rn(r.z, a2);
        a3 = __fadd_rn(r.w, a3);
    }
    const int64_t o = orow ? h : t * p.H + h;
    void *ob = orow ? orow : p.out;
    if (p.out_dtype == 0) {
        float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(ob) + o);
        if (p.accumulate) {
            const float4 c = *dst;
            a0 = __fadd_rn(c.x, a0);
            a1 = __fadd_rn(c.y, a1);
            a2 = __fadd_rn(c.z, a2);
            a3 = __fadd_rn(c.w, a3);
        }
        *dst = make_float4(a0, a1, a2, a3);
    } else {
        __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(ob) + o;
        if (p.accumulate) {
            a0 = __fadd_rn(__bfloat162float(dst[0]), a0);
            a1 = __fadd_rn(__bfloat162float(dst[1]), a1);
            a2 = __fadd_rn(__bfloat162float(dst[2]), a2);
            a3 = __fadd_rn(__bfloat162float(dst[3]), a3);
        }
        __nv_bfloat162 lo = __floats2bfloat162_rn(a0, a1);
        __nv_bfloat162 hi = __floats2bfloat162_rn(a2, a3);
        *reinterpret_cast<__nv_bfloat162 *>(dst) = lo;
        *reinterpret_cast<__nv_bfloat162 *>(dst + 2) = hi;
    }
}

}  // namespace qmoe
