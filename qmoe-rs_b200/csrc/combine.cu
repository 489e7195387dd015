// combine.cu -- weighted combine of the expert outputs plus the shared expert.
//
// Replaces the accumulation of QMoELayer::forward (qmoe-rs src/moe.rs:121-125:
// output_buf[t] += down_out * weight, experts visited in ascending index
// order) and the shared-expert add of the decoder layer (src/model.rs:386-389:
// moe_out + shared_out).  Per output element the operations and their order
// are the reference's: acc = 0; for each of the token's experts in ascending
// index, acc = acc + (y * w) (two roundings, no FMA); then acc + shared.
#include "common.cuh"
#include "kernels.h"

namespace qmoe {
namespace {

constexpr int kCombThreads = 256;
constexpr int kMaxK = 64;

__global__ void __launch_bounds__(kCombThreads)
combine_kernel(const CombineParams p) {
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int H4 = p.H >> 2;
    const int64_t i = (int64_t)blockIdx.x * kCombThreads + threadIdx.x;
    if (i >= p.T * H4) return;
    const int64_t t = i / H4;
    const int h = (int)(i % H4) * 4;
    const int K = p.K, ld = p.topk_ld;

    // slots of this token in ascending expert order (insertion sort, K small)
    int ord[kMaxK];
    int n = 0;
    for (int j = 0; j < K; ++j) {
        if (p.assign_pos[t * K + j] < 0) continue;
        const int e = p.topk_idx[t * ld + j];
        int b = n - 1;
        while (b >= 0 && p.topk_idx[t * ld + ord[b]] > e) {
            ord[b + 1] = ord[b];
            --b;
        }
        ord[b + 1] = j;
        ++n;
    }
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    for (int q = 0; q < n; ++q) {
        const int j = ord[q];
        const float w = p.topk_w[t * ld + j];
        const float4 y = *reinterpret_cast<const float4 *>(
            p.y + (int64_t)p.assign_pos[t * K + j] * p.H + h);
        a0 = __fadd_rn(a0, __fmul_rn(y.x, w));
        a1 = __fadd_rn(a1, __fmul_rn(y.y, w));
        a2 = __fadd_rn(a2, __fmul_rn(y.z, w));
        a3 = __fadd_rn(a3, __fmul_rn(y.w, w));
    }
    if (p.y_shared && t >= p.shared_row0 && t < p.shared_row0 + p.shared_count) {
        const float4 s = *reinterpret_cast<const float4 *>(p.y_shared + (t - p.shared_row0) * p.H + h);
        a0 = __fadd_rn(a0, s.x);
        a1 = __fadd_rn(a1, s.y);
        a2 = __fadd_rn(a2, s.z);
        a3 = __fadd_rn(a3, s.w);
    }
    const int64_t o = t * p.H + h;
    if (p.out_dtype == 0) {
        float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.out) + o);
        if (p.accumulate) {
            const float4 c = *dst;
            a0 = __fadd_rn(c.x, a0); a1 = __fadd_rn(c.y, a1);
            a2 = __fadd_rn(c.z, a2); a3 = __fadd_rn(c.w, a3);
        }
        *dst = make_float4(a0, a1, a2, a3);
    } else {
        __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(p.out) + o;
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

}  // namespace

cudaError_t launch_combine(const CombineParams &p, cudaStream_t s) {
    const int64_t n = p.T * (p.H / 4);
    if (n == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((n + kCombThreads - 1) / kCombThreads);
    return launch_pdl(combine_kernel, dim3(grid), dim3(kCombThreads), 0, s, p);
}

}  // namespace qmoe
