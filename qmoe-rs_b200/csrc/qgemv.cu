// qgemv.cu -- decode-sized grouped GEMV over 2-bit packed expert weights.
//
// Replaces the per-assignment GEMVs of QMoELayer::forward (qmoe-rs
// src/moe.rs:96-118, via PackedQMoETensor::forward_simd src/tensor.rs:64-95
// and simd::fused_dequantize_and_dot src/simd.rs:6-45) and the batched
// shared-expert GEMVs (src/model.rs:325-347).
//
// Work item: (token group of <= 5 tokens of one segment, row block).  One
// 256-thread CTA per item in a persistent grid.
//
// Arithmetic.  A weight is code - 1 with code in 0..3, so for a row r
//     dot(w_r, x) = sum_k code_rk * x_k - sum_k x_k.
// Each token's activations are put on a per-token fixed-point grid,
// x_k ~= 2^e * Q_k with |Q_k| <= 2^22 (e chosen from max |x|; the scaling by
// a power of two is exact, only the rounding to the grid loses anything,
// at most 2^-23 of max |x|), and Q_k is split into three balanced int8 limbs
// Q = q2 * 2^16 + q1 * 2^8 + q0.  The tensor pipe computes
// sum_k code_rk * q_lk exactly in int32 (mma.sync m16n8k32, A = s8 limbs,
// B = u8 codes), the epilogue recombines the limbs in int64, subtracts
// sum_k Q_k and scales by 2^e and by the row scale.  Apart from the grid
// rounding the dot product is exact, i.e. at least as accurate as the f32
// sum qmoe-rs computes.
//
// Data movement.  Weights: each thread streams 64 codes of one row per
// 128-bit load, four threads cover 256 contiguous codes of a row (one 64 B
// coalesced segment), and the next k-step's loads are issued before the
// current step's math.  Unpacking: for a 32-bit word of 16 codes,
// (w >> 2j) & 0x03030303 is the u8 B-fragment register holding codes
// j, j+4, j+8, j+12 -- one shift and one mask per 4 weights.  Activations:
// the limbs of the group's tokens sit in shared memory in the matching
// order (each 16-element block stored as x0,x4,x8,x12,x1,x5,...), XOR-
// swizzled so the 128-bit fragment loads are free of bank conflicts.
#include "common.cuh"
#include "kernels.h"

namespace qmoe {
namespace {

constexpr int kThreads = 256;
constexpr int kTok = 5;        // tokens per item: 3 limbs each -> 15 of 16 MMA rows
constexpr int kKStep = 256;    // codes per row per k-step (4 threads x 64)
constexpr int kEpiCols = 256;  // output rows per item (both modes)

QMOE_DEV void mma_s8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                       uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// physical 16-byte chunk of logical 16-element block b within a limb row
QMOE_DEV int swz(int b) { return b ^ (((b >> 3) & 1) << 1); }

QMOE_DEV uint4 ldg_nc_v4(const uint8_t *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

struct ItemInfo {
    int seg, pos0, count, rb;
    bool shared;
};

QMOE_DEV ItemInfo decode_item(const QgemvParams &p, int item, int nr, int rb_r,
                              int rb_s) {
    ItemInfo it;
    int g;
    if (item < nr * rb_r) {
        g = item / rb_r;
        it.rb = item % rb_r;
        it.shared = false;
    } else {
        const int j = item - nr * rb_r;
        g = nr + j / rb_s;
        it.rb = j % rb_s;
        it.shared = true;
    }
    const int4 d = p.groups[g];
    it.seg = d.x;
    it.pos0 = d.y;
    it.count = d.z;
    return it;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads)
qgemv_kernel(const QgemvParams p) {
    extern __shared__ __align__(16) uint8_t sm[];
    __shared__ int s_exp[kTok];
    __shared__ long long s_sumq[kTok];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g8 = lane >> 2, t4 = lane & 3;

    // rows per matrix per item: mode 0 -> 128 (gate) + 128 (up); mode 1 -> 256
    constexpr int kRowsItem = MODE == 0 ? 128 : 256;
    const int rb_r = (p.rows + kRowsItem - 1) / kRowsItem;
    const int rb_s = p.ws[0] ? (p.rows_s + kRowsItem - 1) / kRowsItem : 1;
    const int nr = p.n_groups[0], ns = p.n_groups[1];
    const int total = nr * rb_r + ns * rb_s;

    const int mat = MODE == 0 ? (warp >> 2) : 0;
    const int wrow0 = MODE == 0 ? (warp & 3) * 32 : warp * 32;

    for (int item = blockIdx.x; item < total; item += gridDim.x) {
        const ItemInfo it = decode_item(p, item, nr, rb_r, rb_s);
        const int K = it.shared ? p.K_s : p.K;
        const int rows = it.shared ? p.rows_s : p.rows;
        const int Kp = (K + kKStep - 1) / kKStep * kKStep;
        const int stride = Kp + 16;            // limb-row stride in bytes
        const int bpr = K >> 2;                // bytes per packed row
        const uint8_t *wbase = it.shared ? p.ws[mat] : p.w[mat] + (int64_t)it.seg * p.w_stride;
        const float *sbase = it.shared ? p.ss[mat] : p.s[mat] + (int64_t)it.seg * p.s_stride;
        const int row0 = it.rb * kRowsItem + wrow0;

        // --- issue the first k-step's weight loads before the prologue
        const uint8_t *wr[4];
        bool rv[4];
#pragma unroll
        for (int rg = 0; rg < 4; ++rg) {
            const int r = row0 + rg * 8 + g8;
            rv[rg] = r < rows;
            wr[rg] = wbase + (int64_t)(rv[rg] ? r : 0) * bpr;
        }
        uint4 wcur[4], wnxt[4];
#pragma unroll
        for (int rg = 0; rg < 4; ++rg) {
            const int off = 16 * t4;
            wcur[rg] = (rv[rg] && off < bpr) ? ldg_nc_v4(wr[rg] + off) : make_uint4(0, 0, 0, 0);
        }

        // --- prologue: activation rows of the group -> int8 limbs in smem.
        //     One warp per token: max |x| and sum(Q) by shuffle reductions.
        const int nblk = Kp >> 4;  // 16-element blocks per row (incl. padding)
        if (warp < it.count) {
            const int c = warp;
            const int64_t pos = it.pos0 + c;
            int64_t row = pos;
            if (p.pos_tok)
                row = pos < p.shared_base ? (int64_t)p.pos_tok[pos] : pos - p.shared_base;
            const int64_t base = row * p.act_ld;
            float m = 0.0f;
            for (int q = lane; q < (K >> 2); q += 32) {
                const float4 v = load_act4(p.act, p.act_dtype, base + 4 * q);
                m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            }
            m = warp_max(m);
            int e = 0;
            if (m > 0.0f) {
                int ex;
                frexpf(m, &ex);          // m = f * 2^ex, f in [0.5, 1)
                e = max(ex - 22, -120);  // m * 2^-e in [2^21, 2^22)
            }
            const float sc = pow2i(-e);
            long long sq = 0;
            for (int b = lane; b < nblk; b += 32) {
                int Q[16];
                const bool in = b * 16 < K;  // K % 16 == 0: blocks are all in or out
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (in) v = load_act4(p.act, p.act_dtype, base + b * 16 + 4 * j4);
                    Q[4 * j4 + 0] = __float2int_rn(v.x * sc);
                    Q[4 * j4 + 1] = __float2int_rn(v.y * sc);
                    Q[4 * j4 + 2] = __float2int_rn(v.z * sc);
                    Q[4 * j4 + 3] = __float2int_rn(v.w * sc);
                }
                uint32_t l0[4], l1[4], l2[4];
#pragma unroll
                for (int w = 0; w < 4; ++w) { l0[w] = l1[w] = l2[w] = 0u; }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int q = Q[j];
                    sq += q;
                    const int d0 = ((q + 128) & 255) - 128;
                    const int q1 = (q - d0) >> 8;
                    const int d1 = ((q1 + 128) & 255) - 128;
                    const int d2 = (q1 - d1) >> 8;
                    // element j -> byte (j % 4) * 4 + j / 4 of the block
                    const int word = j & 3, sh = (j >> 2) * 8;
                    l0[word] |= (uint32_t)(d0 & 255) << sh;
                    l1[word] |= (uint32_t)(d1 & 255) << sh;
                    l2[word] |= (uint32_t)(d2 & 255) << sh;
                }
                const int pc = swz(b) * 16;
                *reinterpret_cast<uint4 *>(sm + (0 * kTok + c) * stride + pc) = make_uint4(l0[0], l0[1], l0[2], l0[3]);
                *reinterpret_cast<uint4 *>(sm + (1 * kTok + c) * stride + pc) = make_uint4(l1[0], l1[1], l1[2], l1[3]);
                *reinterpret_cast<uint4 *>(sm + (2 * kTok + c) * stride + pc) = make_uint4(l2[0], l2[1], l2[2], l2[3]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
            if (lane == 0) {
                s_exp[c] = e;
                s_sumq[c] = sq;
            }
        }
        __syncthreads();

        // --- main loop
        int acc[4][4];
#pragma unroll
        for (int rg = 0; rg < 4; ++rg)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[rg][j] = 0;

        const uint8_t *arow_lo = sm + g8 * stride;
        const uint8_t *arow_hi = sm + (g8 + 8) * stride;
        const int nks = Kp / kKStep;
        for (int ks = 0; ks < nks; ++ks) {
            if (ks + 1 < nks) {
                const int off = (ks + 1) * 64 + 16 * t4;
#pragma unroll
                for (int rg = 0; rg < 4; ++rg)
                    wnxt[rg] = (rv[rg] && off < bpr) ? ldg_nc_v4(wr[rg] + off) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int pc = swz(ks * 16 + 4 * t4 + q) * 16;
                const uint4 alo = *reinterpret_cast<const uint4 *>(arow_lo + pc);
                const uint4 ahi = *reinterpret_cast<const uint4 *>(arow_hi + pc);
#pragma unroll
                for (int rg = 0; rg < 4; ++rg) {
                    const uint32_t w = q == 0 ? wcur[rg].x : q == 1 ? wcur[rg].y
                                     : q == 2 ? wcur[rg].z : wcur[rg].w;
                    mma_s8u8(acc[rg], alo.x, ahi.x, alo.y, ahi.y,
                             w & 0x03030303u, (w >> 2) & 0x03030303u);
                    mma_s8u8(acc[rg], alo.z, ahi.z, alo.w, ahi.w,
                             (w >> 4) & 0x03030303u, (w >> 6) & 0x03030303u);
                }
            }
#pragma unroll
            for (int rg = 0; rg < 4; ++rg) wcur[rg] = wnxt[rg];
        }
        __syncthreads();  // all warps done with the limb tile

        // --- epilogue: int32 tile [16 token-limb rows][256 cols] in smem
        int *ct = reinterpret_cast<int *>(sm);
        {
            const int colw = (MODE == 0 ? mat * 128 : 0) + wrow0;
#pragma unroll
            for (int rg = 0; rg < 4; ++rg) {
                const int col = colw + rg * 8 + 2 * t4;
                *reinterpret_cast<int2 *>(ct + g8 * kEpiCols + col) = make_int2(acc[rg][0], acc[rg][1]);
                *reinterpret_cast<int2 *>(ct + (g8 + 8) * kEpiCols + col) = make_int2(acc[rg][2], acc[rg][3]);
            }
        }
        __syncthreads();
        if (MODE == 0) {
            const int r = tid & 127;
            const int grow = it.rb * 128 + r;
            if (grow < rows) {
                // scales by matrix, not by this warp's matrix: threads 128..255
                // belong to the up-projection warps but combine both
                const float sg = __ldg((it.shared ? p.ss[0] : p.s[0] + (int64_t)it.seg * p.s_stride) + grow);
                const float su = __ldg((it.shared ? p.ss[1] : p.s[1] + (int64_t)it.seg * p.s_stride) + grow);
                for (int c = tid >> 7; c < it.count; c += 2) {
                    const double s2 = (double)pow2i(s_exp[c]);
                    const long long gi = (long long)ct[(2 * kTok + c) * kEpiCols + r] * 65536LL +
                                         (long long)ct[(kTok + c) * kEpiCols + r] * 256LL +
                                         (long long)ct[c * kEpiCols + r] - s_sumq[c];
                    const long long ui = (long long)ct[(2 * kTok + c) * kEpiCols + 128 + r] * 65536LL +
                                         (long long)ct[(kTok + c) * kEpiCols + 128 + r] * 256LL +
                                         (long long)ct[c * kEpiCols + 128 + r] - s_sumq[c];
                    const float g = __fmul_rn((float)((double)gi * s2), sg);
                    const float u = __fmul_rn((float)((double)ui * s2), su);
                    p.out[(int64_t)(it.pos0 + c) * p.out_ld + grow] = swiglu(g, u);
                }
            }
        } else {
            const int r = tid;
            const int grow = it.rb * 256 + r;
            if (grow < rows) {
                const float sc = __ldg(sbase + grow);
                for (int c = 0; c < it.count; ++c) {
                    const double s2 = (double)pow2i(s_exp[c]);
                    const long long di = (long long)ct[(2 * kTok + c) * kEpiCols + r] * 65536LL +
                                         (long long)ct[(kTok + c) * kEpiCols + r] * 256LL +
                                         (long long)ct[c * kEpiCols + r] - s_sumq[c];
                    p.out[(int64_t)(it.pos0 + c) * p.out_ld + grow] = __fmul_rn((float)((double)di * s2), sc);
                }
            }
        }
        __syncthreads();  // tile reused by the next item's prologue
    }
}

}  // namespace

size_t qgemv_smem_bytes(int K_max) {
    const int Kp = (K_max + kKStep - 1) / kKStep * kKStep;
    const size_t limbs = (size_t)16 * (Kp + 16);
    const size_t epi = (size_t)16 * kEpiCols * sizeof(int);
    return limbs > epi ? limbs : epi;
}

int qgemv_max_grid(int mode, int K_max) {
    int dev = 0, sms = 0, per = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = qgemv_smem_bytes(K_max);
    // only ever raises the kernel's opt-in (a smaller K_max here must not
    // lower the limit an earlier, wider tensor's launches rely on)
    if (mode == 0) {
        ensure_dyn_smem(reinterpret_cast<const void *>(qgemv_kernel<0>), smem);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, qgemv_kernel<0>, kThreads, smem);
    } else {
        ensure_dyn_smem(reinterpret_cast<const void *>(qgemv_kernel<1>), smem);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, qgemv_kernel<1>, kThreads, smem);
    }
    cudaGetLastError();
    if (per < 1) per = 1;
    return sms * per;
}

cudaError_t launch_qgemv(int mode, const QgemvParams &p, int grid, cudaStream_t s) {
    const size_t smem = qgemv_smem_bytes(p.ws[0] && p.K_s > p.K ? p.K_s : p.K);
    cudaError_t e = mode == 0 ? ensure_dyn_smem(reinterpret_cast<const void *>(qgemv_kernel<0>), smem)
                              : ensure_dyn_smem(reinterpret_cast<const void *>(qgemv_kernel<1>), smem);
    if (e != cudaSuccess) return e;
    if (mode == 0)
        qgemv_kernel<0><<<grid, kThreads, smem, s>>>(p);
    else
        qgemv_kernel<1><<<grid, kThreads, smem, s>>>(p);
    return cudaGetLastError();
}

}  // namespace qmoe
