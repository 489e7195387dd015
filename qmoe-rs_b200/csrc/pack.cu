// pack.cu -- the 2-bit packer on the device: qmoe-rs's offline quantizer
// (quantize.py:97-100 for the row scale, quantize_and_pack quantize.py:7-33
// for the codes and the byte layout), bit for bit.
//
// Per row r of w [out, in] f32:
//   scale[r] = max(std_unbiased(w[r]), 1e-5)       (quantize.py:98-100)
//   code     = clamp(round_half_even(w / scale), -1, 1) + 1
//                                                   (quantize.py:18-22)
//   byte q of the row = code[4q] | code[4q+1] << 2 | code[4q+2] << 4 |
//                       code[4q+3] << 6             (quantize.py:28-31)
//
// The scale: torch's CPU std of an f32 row accumulates in double (Welford)
// and rounds the double sqrt once to f32; here the mean and the sum of
// squared deviations are block reductions in double and the same single
// rounding follows, so the f32 scale is the same value (both doubles carry
// ~1e-16 relative error, far below half an f32 ulp).
//
// The codes need no division.  With q = fl(w / s) (IEEE f32 quotient,
// round to nearest even) the code is 2 iff rint(q) >= 1 iff q > 0.5, and
// q > 0.5 iff the exact w / s > 0.5 + 2^-25 (0.5 + 2^-25 is the tie between
// 0.5 and the next float, and ties go to 0.5, the even one).  For s > 0 that
// is w > t with t = s * (0.5 + 2^-25), a product exact in double (24 + 25
// significant bits), and for a float w, w > t iff w > RD_f32(t).  So one
// threshold per row, rounded down to f32, and two compares per weight give
// exactly the reference's codes: code 0 iff w < -thr, code 2 iff w > thr.
// A negative scale (given scales only; -0 included) flips the sign of w; NaN
// in w or s fails both compares, code 1, as the reference's int32 cast of NaN
// on its x86 host (INT_MIN, +1, & 3 = 1); s = 0 gives 2 / 0 / 1 for w > 0,
// w < 0, w = 0 as w / 0 = +inf / -inf / NaN does.
//
// HBM-bound byte work (4 bytes read per weight, 1/4 byte written), rows
// streamed into shared memory by 1-D bulk copies (cp.async.bulk, no
// multicast) completing on mbarriers, so later rows arrive while the three
// passes (sum, squared deviations, codes) run over the current one:
//   * rows of up to kPackWarpRowMax floats (the V2-Lite widths): one warp per
//     row, each warp with a ring of 3 (or 2) row buffers, warp-shuffle
//     reductions only, one CTA of 8 warps per SM;
//   * wider rows up to kPackStageMax bytes: one CTA per row, two rows
//     double-buffered, CTA reductions;
//   * wider still: one CTA per row with plain loads, the second and third
//     passes served by L2.
// In every form a grid of one wave of resident CTAs loops over the rows.
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace qmoe {
namespace {

using namespace sm100;

constexpr int kPackThreads = 256;
constexpr int kPackWarps = kPackThreads / 32;
constexpr int kPackCtasPerSm = 6;          // resident CTAs per SM (40 registers a thread)
constexpr double kTieAboveHalf = 0.500000029802322387695312500;   // 0.5 + 2^-25
constexpr int kPackRingMax = 3;            // row buffers per warp in the warp-per-row packer
constexpr int kPackWarpRowMax = 3520;      // widest row (floats) of the warp-per-row packer

// Sum over the CTA (every thread gets the same value).
QMOE_DEV double block_sum(double v, double *s_red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();                       // the previous call's reads are done
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < kPackWarps; ++i) t += s_red[i];
    return t;
}

struct Thr {
    float t;                               // RD_f32(|s| * (0.5 + 2^-25))
    bool neg;                              // s has its sign bit set
};

QMOE_DEV Thr threshold(float s) {
    Thr h;
    h.neg = (__float_as_uint(s) >> 31) != 0;
    h.t = __double2float_rd((double)fabsf(s) * kTieAboveHalf);
    return h;
}

// t >= 0 (or NaN): code 2 iff x > t iff |x| > t with x positive, code 0
// iff x < -t iff |x| > t with x negative; NaN fails |x| > t.
QMOE_DEV uint32_t code_of(float w, const Thr &h) {
    const uint32_t u = __float_as_uint(w) ^ (h.neg ? 0x80000000u : 0u);
    return fabsf(__uint_as_float(u)) > h.t ? 2u - ((u >> 31) << 1) : 1u;
}

QMOE_DEV uint32_t byte_of(float4 v, const Thr &h) {
    return code_of(v.x, h) | code_of(v.y, h) << 2 | code_of(v.z, h) << 4 | code_of(v.w, h) << 6;
}

QMOE_DEV void bulk_load(void *smem_dst, const void *gsrc, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// The three passes over one row held in `row` (shared memory, or global
// memory read through L2), n4 float4 entries; thread t takes t, t + 256, ...
template <bool SMEM>
QMOE_DEV void pack_row(const PackParams &p, int64_t r, const float4 *row, int64_t n4, double *s_red) {
    uint8_t *dst = p.packed + r * n4;
    float s;
    if (p.scales_given) {
        s = p.scales[r];
    } else {
        double a = 0.0;
        for (int64_t i = threadIdx.x; i < n4; i += kPackThreads) {
            const float4 v = SMEM ? row[i] : __ldcs(row + i);
            a += (double)v.x;
            a += (double)v.y;
            a += (double)v.z;
            a += (double)v.w;
        }
        const double mean = block_sum(a, s_red) / (double)p.in_f;
        double q = 0.0;
        for (int64_t i = threadIdx.x; i < n4; i += kPackThreads) {
            const float4 v = SMEM ? row[i] : __ldcg(row + i);
            const double d0 = (double)v.x - mean, d1 = (double)v.y - mean;
            const double d2 = (double)v.z - mean, d3 = (double)v.w - mean;
            q = __fma_rn(d0, d0, q);
            q = __fma_rn(d1, d1, q);
            q = __fma_rn(d2, d2, q);
            q = __fma_rn(d3, d3, q);
        }
        const double var = block_sum(q, s_red) / (double)(p.in_f - 1);
        s = (float)sqrt(var);
        s = s < 1e-5f ? 1e-5f : s;         // clamp(min=1e-5); NaN stays NaN, as in torch
        if (threadIdx.x == 0) p.scales[r] = s;
    }
    const Thr h = threshold(s);
    for (int64_t i = threadIdx.x; i < n4; i += kPackThreads) {
        const float4 v = SMEM ? row[i] : (p.scales_given ? __ldcs(row + i) : __ldcg(row + i));
        dst[i] = (uint8_t)byte_of(v, h);
    }
}

// One warp per row (rows of at most kPackWarpRowMax floats): the three
// passes with warp-shuffle reductions only, four independent double
// accumulators per lane.  row: the staged row in shared memory.
QMOE_DEV void pack_row_warp(const PackParams &p, int64_t r, const float4 *row, int n4, int lane) {
    uint8_t *dst = p.packed + r * n4;
    float s;
    if (p.scales_given) {
        s = p.scales[r];
    } else {
        double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
        for (int i = lane; i < n4; i += 32) {
            const float4 v = row[i];
            a0 += (double)v.x;
            a1 += (double)v.y;
            a2 += (double)v.z;
            a3 += (double)v.w;
        }
        double a = (a0 + a1) + (a2 + a3);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        const double mean = a / (double)p.in_f;
        double q0 = 0.0, q1 = 0.0, q2 = 0.0, q3 = 0.0;
        for (int i = lane; i < n4; i += 32) {
            const float4 v = row[i];
            const double d0 = (double)v.x - mean, d1 = (double)v.y - mean;
            const double d2 = (double)v.z - mean, d3 = (double)v.w - mean;
            q0 = __fma_rn(d0, d0, q0);
            q1 = __fma_rn(d1, d1, q1);
            q2 = __fma_rn(d2, d2, q2);
            q3 = __fma_rn(d3, d3, q3);
        }
        double q = (q0 + q1) + (q2 + q3);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        const double var = q / (double)(p.in_f - 1);
        s = (float)sqrt(var);
        s = s < 1e-5f ? 1e-5f : s;         // clamp(min=1e-5); NaN stays NaN, as in torch
        if (lane == 0) p.scales[r] = s;
    }
    const Thr h = threshold(s);
    for (int i = lane; i < n4; i += 32) dst[i] = (uint8_t)byte_of(row[i], h);
}

// Warp-per-row packer: each warp owns a ring of `depth` row buffers in
// shared memory fed by bulk copies (lane 0 issues, one mbarrier per buffer),
// keeping depth - 1 rows in flight while it packs the current one; rows are
// dealt to the grid's warps round-robin.
__global__ void __launch_bounds__(kPackThreads, 2)
pack_rows_warp(const PackParams p, int depth) {
    extern __shared__ __align__(128) float4 s_ring[];    // [warps][depth][n4]
    __shared__ uint64_t bar[kPackWarps][kPackRingMax];
    __shared__ int abort_flag[kPackWarps];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n4 = (int)(p.in_f >> 2);
    const uint32_t row_bytes = (uint32_t)n4 * 16u;
    float4 *ring = s_ring + (size_t)warp * depth * n4;
    if (lane == 0) {
        for (int b = 0; b < depth; ++b) mbar_init(&bar[warp][b], 1);
        abort_flag[warp] = 0;
        fence_mbar_init();
    }
    __syncwarp();
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    volatile int *abort = &abort_flag[warp];
    const int64_t nw = (int64_t)gridDim.x * kPackWarps;
    const int64_t r0 = (int64_t)blockIdx.x * kPackWarps + warp;
    int64_t issued = 0;                    // lane 0: rows of this warp issued so far
    auto issue = [&](int64_t j) {          // this warp's j-th row into buffer j % depth
        const int b = (int)(j % depth);
        mbar_arrive_expect_tx(&bar[warp][b], row_bytes);
        bulk_load(ring + (size_t)b * n4, p.w + (r0 + j * nw) * p.in_f, row_bytes, &bar[warp][b]);
        issued = j + 1;
    };
    if (lane == 0)
        for (int64_t j = 0; j < depth - 1 && r0 + j * nw < p.out_f; ++j) issue(j);
    int64_t k = 0;
    for (int64_t r = r0; r < p.out_f; r += nw, ++k) {
        // buffer (k + depth - 1) % depth was read last for row k - 1
        if (lane == 0 && r + (depth - 1) * nw < p.out_f) issue(k + depth - 1);
        const int b = (int)(k % depth);
        if (!mbar_wait_warp(&bar[warp][b], (uint32_t)((k / depth) & 1), abort, p.err)) break;
        pack_row_warp(p, r, ring + (size_t)b * n4, n4, lane);
        __syncwarp();                      // every lane's reads of buffer b are done
    }
    // after a time-out: wait (bounded) for this warp's copies still in flight
    if (lane == 0 && *abort) {
        for (int64_t j = k; j < issued; ++j)
            for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                if (mbar_try_wait(&bar[warp][j % depth], (uint32_t)((j / depth) & 1))) break;
    }
}

// Rows staged in shared memory: two buffers of row_bytes, the bulk copy of
// this CTA's next row issued before the passes over the current one.
__global__ void __launch_bounds__(kPackThreads, kPackCtasPerSm)
pack_rows_staged(const PackParams p) {
    extern __shared__ __align__(128) float4 s_rows[];     // [2][n4]
    __shared__ uint64_t bar[2];
    __shared__ double s_red[kPackWarps];
    __shared__ int abort_flag;
    const int64_t n4 = p.in_f >> 2;
    const uint32_t row_bytes = (uint32_t)(p.in_f * 4);
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    volatile int *abort = &abort_flag;
    uint32_t issued[2] = {0u, 0u};         // thread 0: copies issued into each buffer
    auto issue = [&](int64_t r, int b) {
        mbar_arrive_expect_tx(&bar[b], row_bytes);
        bulk_load(s_rows + b * n4, p.w + r * p.in_f, row_bytes, &bar[b]);
        ++issued[b];
    };
    if (threadIdx.x == 0 && (int64_t)blockIdx.x < p.out_f) issue(blockIdx.x, 0);
    int k = 0;
    for (int64_t r = blockIdx.x; r < p.out_f; r += gridDim.x, ++k) {
        const int b = k & 1;
        const int64_t rn = r + gridDim.x;
        // buffer b ^ 1 was released by the barrier that ended the last row
        if (threadIdx.x == 0 && rn < p.out_f) issue(rn, b ^ 1);
        mbar_wait(&bar[b], (k >> 1) & 1, abort, p.err);
        __syncthreads();
        if (*abort) break;                 // the same decision in every thread
        pack_row<true>(p, r, s_rows + b * n4, n4, s_red);
        __syncthreads();                   // every read of buffer b is done
    }
    // after a time-out: wait (bounded) for the last copy issued into each
    // buffer, so none is in flight when the CTA exits
    if (threadIdx.x == 0 && *abort) {
        for (int b = 0; b < 2; ++b) {
            if (!issued[b]) continue;
            for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                if (mbar_try_wait(&bar[b], (issued[b] - 1) & 1)) break;
        }
    }
}

// Rows wider than the staging limit: each pass reads the row (the second
// and third from L2).
__global__ void __launch_bounds__(kPackThreads, kPackCtasPerSm)
pack_rows_direct(const PackParams p) {
    __shared__ double s_red[kPackWarps];
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int64_t n4 = p.in_f >> 2;
    for (int64_t r = blockIdx.x; r < p.out_f; r += gridDim.x) {
        pack_row<false>(p, r, reinterpret_cast<const float4 *>(p.w + r * p.in_f), n4, s_red);
        __syncthreads();                   // s_red reuse by the next row
    }
}

}  // namespace

cudaError_t launch_pack_rows(const PackParams &p, int sm_count, cudaStream_t s) {
    if (p.out_f == 0) return cudaSuccess;
    if (p.in_f < 4 || (p.in_f & 3)) return cudaErrorInvalidValue;
    const size_t row_bytes = (size_t)p.in_f * sizeof(float);
    // one wave of resident CTAs, each looping over rows: kPackCtasPerSm per
    // SM unless the two staged rows fill the SM's 228 KB of shared memory
    // first (1 KB reserved per CTA)
    const int64_t rows = p.out_f;
    if (p.in_f <= kPackWarpRowMax) {
        // 8 warps a CTA, each with a ring of 3 rows (2 where 3 do not fit
        // 220 KB); CTAs per SM as the shared memory allows, at most 2
        const int depth = 24 * row_bytes <= 220 * 1024 ? 3 : 2;
        const size_t smem = (size_t)kPackWarps * depth * row_bytes;
        cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(pack_rows_warp), smem);
        if (e != cudaSuccess) return e;
        int64_t per_sm = (int64_t)(228 * 1024) / (int64_t)(smem + 1024 + 256);
        per_sm = per_sm > 2 ? 2 : (per_sm < 1 ? 1 : per_sm);
        const int64_t warps = (rows + kPackWarps - 1) / kPackWarps;
        const int64_t wave = (int64_t)sm_count * per_sm;
        const int64_t grid = warps < wave ? warps : wave;
        return launch_pdl(pack_rows_warp, dim3((unsigned)grid), dim3(kPackThreads), smem, s, p, depth);
    }
    if (row_bytes <= kPackStageMax) {
        cudaError_t e = ensure_dyn_smem(reinterpret_cast<const void *>(pack_rows_staged), 2 * row_bytes);
        if (e != cudaSuccess) return e;
        int64_t per_sm = (int64_t)(228 * 1024) / (int64_t)(2 * row_bytes + 1024 + 256);
        per_sm = per_sm > kPackCtasPerSm ? kPackCtasPerSm : (per_sm < 1 ? 1 : per_sm);
        const int64_t wave = (int64_t)sm_count * per_sm;
        const int64_t grid = rows < wave ? rows : wave;
        return launch_pdl(pack_rows_staged, dim3((unsigned)grid), dim3(kPackThreads), 2 * row_bytes, s, p);
    }
    const int64_t wave = (int64_t)sm_count * kPackCtasPerSm;
    const int64_t grid = rows < wave ? rows : wave;
    return launch_pdl(pack_rows_direct, dim3((unsigned)grid), dim3(kPackThreads), 0, s, p);
}

}  // namespace qmoe
