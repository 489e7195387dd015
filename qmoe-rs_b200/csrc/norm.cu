// norm.cu -- the decoder layer's post-attention LayerNorm in front of the MoE
// block (qmoe-rs src/model.rs:366-367 builds it with candle_nn::layer_norm,
// eps 1e-6; :401-403 and :380-382 apply it before the router and experts).
//
// candle's summation order is not observable, so the order is pinned, in the
// same 64-wide chunks as the gate logits, and the CPU oracle computes the
// same operations:
//   s1 = ((0 + p_0) + p_1) + ...   p_c = sequential f32 sum of chunk c
//   mean = s1 / H
//   s2 = ((0 + q_0) + q_1) + ...   q_c = fmaf chain of d * d, d = x - mean
//   rstd = 1 / sqrt(s2 / H + eps)
//   y = ((x - mean) * rstd) * w + b, each operation rounded once
// One warp per row: lane l forms the chunk sums l, l + 32, ...; lane 0 adds
// them in chunk order; the row is read three times (the later passes from
// L1/L2) and y written once in the activation dtype.
#include "common.cuh"
#include "kernels.h"

namespace qmoe {
namespace {

constexpr int kNormWarps = 8;

// Sixteen consecutive elements of row `row` starting at k (f32 or bf16).
QMOE_DEV void load16(const void *x, int dtype, int64_t idx, float (&v)[16]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 f = load_act4(x, dtype, idx + 4 * q);
        v[4 * q + 0] = f.x;
        v[4 * q + 1] = f.y;
        v[4 * q + 2] = f.z;
        v[4 * q + 3] = f.w;
    }
}

__global__ void __launch_bounds__(kNormWarps * 32)
layernorm_kernel(const NormParams p) {
    extern __shared__ float part_all[];      // [kNormWarps][H / 64]
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t t = (int64_t)blockIdx.x * kNormWarps + warp;
    if (t >= p.T) return;                    // whole warps; no CTA barrier follows
    const int H = p.H, nc = H / kGateChunk;
    float *part = part_all + warp * nc;
    const int64_t base = t * H;

    // pass 1: mean
    for (int c = lane; c < nc; c += 32) {
        float s = 0.0f;
        for (int k = 0; k < kGateChunk; k += 16) {
            float v[16];
            load16(p.x, p.dtype, base + c * kGateChunk + k, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) s = __fadd_rn(s, v[j]);
        }
        part[c] = s;
    }
    __syncwarp();
    float mean = 0.0f;
    if (lane == 0) {
        float s1 = 0.0f;
        for (int c = 0; c < nc; ++c) s1 = __fadd_rn(s1, part[c]);
        mean = __fdiv_rn(s1, (float)H);
    }
    mean = __shfl_sync(0xffffffffu, mean, 0);
    __syncwarp();
    // pass 2: variance
    for (int c = lane; c < nc; c += 32) {
        float q = 0.0f;
        for (int k = 0; k < kGateChunk; k += 16) {
            float v[16];
            load16(p.x, p.dtype, base + c * kGateChunk + k, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float d = __fsub_rn(v[j], mean);
                q = __fmaf_rn(d, d, q);
            }
        }
        part[c] = q;
    }
    __syncwarp();
    float rstd = 0.0f;
    if (lane == 0) {
        float s2 = 0.0f;
        for (int c = 0; c < nc; ++c) s2 = __fadd_rn(s2, part[c]);
        rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s2, (float)H), p.eps)));
    }
    rstd = __shfl_sync(0xffffffffu, rstd, 0);
    // pass 3: normalise, scale, shift
    for (int k = 4 * lane; k < H; k += 128) {
        const float4 v = load_act4(p.x, p.dtype, base + k);
        const float4 w = __ldg(reinterpret_cast<const float4 *>(p.w + k));
        const float4 b = __ldg(reinterpret_cast<const float4 *>(p.b + k));
        float4 o;
        o.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, mean), rstd), w.x), b.x);
        o.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, mean), rstd), w.y), b.y);
        o.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, mean), rstd), w.z), b.z);
        o.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, mean), rstd), w.w), b.w);
        store_act4(p.y, p.dtype, base + k, o);
    }
}

}  // namespace

cudaError_t launch_layernorm(const NormParams &p, cudaStream_t s) {
    if (p.T == 0) return cudaSuccess;
    const size_t smem = sizeof(float) * kNormWarps * (p.H / kGateChunk);
    cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(layernorm_kernel), smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(layernorm_kernel, dim3((unsigned)((p.T + kNormWarps - 1) / kNormWarps)),
                      dim3(kNormWarps * 32), smem, s, p);
}

}  // namespace qmoe
