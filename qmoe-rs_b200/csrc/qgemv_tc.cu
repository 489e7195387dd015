// qgemv_tc.cu -- decode-sized grouped GEMV on the sm_100a tensor cores.
//
// Replaces the per-assignment GEMVs of QMoELayer::forward (qmoe-rs
// src/moe.rs:96-118 via PackedQMoETensor::forward_simd, src/tensor.rs:64-95,
// and simd::fused_dequantize_and_dot, src/simd.rs:6-45) and the shared
// expert's batched GEMVs (src/model.rs:325-347).
//
// Arithmetic: a weight is code - 1 (code in 0..3) and each activation row is
// x ~= 2^e * Q with Q split into three int8 limbs (quant.cu), so
//     dot(w_r, x) = 2^e * (sum_l 256^l sum_k code_rk q_lk  -  sum_k Q_k).
// The tensor core forms every sum_k code_rk q_lk exactly (tcgen05.mma
// kind::i8, A = u8 codes, B = s8 limbs, s32 accumulators in TMEM); the
// epilogue recombines the limbs in int64 and scales once.
//
// One work item = (<= 5 positions of one segment) x 256 output rows, as two
// 128-row A tiles (gate and up rows in mode 0, two halves of 256 down rows
// in mode 1), i.e. two M=128, N=16 (5 positions x 3 limbs + 1 spare)
// accumulators.  Persistent grid, one CTA per SM, fourteen warps:
//   warp 0    TMA: 2-bit weight tiles [128 rows x 64 B] (64-byte swizzle)
//             into a 4-stage ring, and each item's limb tile [16 x Kp]
//             (128-byte swizzle) into a 2-deep buffer;
//   warp 1    TMEM allocation; one lane issues the MMAs;
//   warps 2-9 two sets of four, one TMEM lane quarter per warp, taking
//             alternate stages: unpack 2-bit codes to u8 in registers
//             ((w >> 2j) & 0x03030303: one shift + one mask per 4 weights)
//             and tcgen05.st them into a 3-stage TMEM ring that is the
//             MMA's A operand -- the unpacked weights never touch shared
//             memory;
//   warps 10-13 the epilogue, one lane quarter each: tcgen05.ld of the
//             double-buffered accumulators, limb recombination, scales,
//             SwiGLU, stores; their scale / row metadata loads are issued
//             before they wait for the MMAs.
// The CTA's work-item descriptors are decoded into shared memory once.
// Every wait is bounded: on a time-out the kernel flags the device error
// word, lets its TMA copies and MMAs drain (again bounded), frees TMEM and
// returns.
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace qmoe {

__device__ int g_device_error;

namespace {

using namespace sm100;

constexpr int kWarps = 14;  // TMA, MMA, two sets of four unpack warps, four epilogue warps
constexpr int kThreads = kWarps * 32;
constexpr int kNS = 6;              // weight stages in shared memory
constexpr int kNT = 3;              // A stages in TMEM
constexpr int kStageCodes = 256;    // codes per row per stage
constexpr int kStageRowBytes = 64;  // packed bytes per row per stage
constexpr int kTileBytes = 128 * kStageRowBytes;  // one 128-row tile
constexpr int kBRows = 16;          // positions x limbs in a B tile (15 used)
constexpr int kTokMax = 5;          // positions per work item
constexpr int kItemCache = 256;     // work items per CTA decoded into shared memory
constexpr int kBBlock = kBRows * 128;  // one 128-byte K block of the B tile
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAColStage = 128;   // TMEM columns per A stage (2 tiles x 64)
constexpr uint32_t kDCol = kNT * kAColStage;  // accumulators after the A ring
constexpr uint32_t kIdesc = idesc_i8(128, kBRows, /*a_signed=*/false, /*b_signed=*/true);

struct Smem {
    uint64_t smem_full[kNS], smem_empty[kNS];
    uint64_t tmem_full[kNT], tmem_empty[kNT];
    uint64_t bq_full[2], bq_empty[2];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    int4 items[kItemCache];
};

struct Item {
    int seg, pos0, count, rb;
    bool shared;
};

QMOE_DEV Item get_item(const QgemvTcParams &p, int item, int nr, int rb_r, int rb_s) {
    Item it;
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
__global__ void __launch_bounds__(kThreads, 1)
qgemv_tc_kernel(const __grid_constant__ CUtensorMap tm_a0, const __grid_constant__ CUtensorMap tm_a1,
                const __grid_constant__ CUtensorMap tm_s0, const __grid_constant__ CUtensorMap tm_s1,
                const __grid_constant__ CUtensorMap tm_b, const QgemvTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned tiles (swizzled TMA destinations / UMMA atoms)
    uint8_t *base = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *wring = base;                                   // kNS x 2 tiles
    uint8_t *btile = wring + kNS * 2 * kTileBytes;           // nbuf x (16 x kp_b)
    const int nbuf = p.b_buffers;
    const int bbytes = kBRows * p.kp_b;
    Smem *S = reinterpret_cast<Smem *>(btile + nbuf * bbytes);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rows_item = MODE == 0 ? 128 : 256;
    const int rb_r = (p.rows + rows_item - 1) / rows_item;
    const int rb_s = p.rows_s > 0 ? (p.rows_s + rows_item - 1) / rows_item : 1;
    const int nr = p.n_groups[0], ns = p.n_groups[1];
    const int total = nr * rb_r + ns * rb_s;
    const int my_items = total > (int)blockIdx.x ? (total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (tid == 0) {
        for (int i = 0; i < kNS; ++i) {
            mbar_init(&S->smem_full[i], 1);
            mbar_init(&S->smem_empty[i], 4);
        }
        for (int i = 0; i < kNT; ++i) {
            mbar_init(&S->tmem_full[i], 4);
            mbar_init(&S->tmem_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S->bq_full[i], 1);
            mbar_init(&S->bq_empty[i], 1);
            mbar_init(&S->acc_full[i], 1);
            mbar_init(&S->acc_empty[i], 4);
        }
        mbar_init(&S->drain, 1);
        S->abort = 0;
        fence_mbar_init();
    }
    // this CTA's work items, decoded once into shared memory
    for (int i = tid; i < my_items && i < kItemCache; i += kThreads) {
        const Item it = get_item(p, (int)blockIdx.x + i * (int)gridDim.x, nr, rb_r, rb_s);
        S->items[i] = make_int4(it.seg, it.pos0, it.count, it.rb | (it.shared ? (1 << 30) : 0));
    }
    if (warp == 1) {
        tmem_alloc(&S->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S->tmem_base;
    volatile int *abort = &S->abort;

    auto item_at = [&](int i) -> Item {
        if (i < kItemCache) {
            const int4 v = S->items[i];
            Item it;
            it.seg = v.x;
            it.pos0 = v.y;
            it.count = v.z;
            it.rb = v.w & ((1 << 30) - 1);
            it.shared = (v.w >> 30) & 1;
            return it;
        }
        return get_item(p, (int)blockIdx.x + i * (int)gridDim.x, nr, rb_r, rb_s);
    };

    if (warp == 0) {
        // ------------------------------------------------------------- TMA
        if (lane == 0) {
            tma_prefetch_desc(&tm_a0);
            tma_prefetch_desc(&tm_a1);
            tma_prefetch_desc(&tm_b);
            if (p.rows_s > 0) {
                tma_prefetch_desc(&tm_s0);
                tma_prefetch_desc(&tm_s1);
            }
            uint32_t us = 0;
            int i = 0;
            bool ok = true;
            for (; ok && i < my_items; ++i) {
                const Item it = item_at(i);
                const int K = it.shared ? p.K_s : p.K;
                const int nks = (K + kStageCodes - 1) / kStageCodes;
                const int nkb = nks * 2;  // 128-byte K blocks of the limb tile
                const uint32_t b = nbuf == 2 ? (i & 1) : 0, ub = nbuf == 2 ? (i >> 1) : i;
                if (!(ok = mbar_wait(&S->bq_empty[b], (ub & 1) ^ 1, abort, p.err))) break;
                mbar_arrive_expect_tx(&S->bq_full[b], (uint32_t)(nkb * kBBlock));
                for (int kb = 0; kb < nkb; ++kb)
                    tma_load_2d(btile + b * bbytes + kb * kBBlock, &tm_b, &S->bq_full[b],
                                kb * 128, it.pos0 * 3);
                const CUtensorMap *t0 = it.shared ? &tm_s0 : &tm_a0;
                const CUtensorMap *t1 = MODE == 0 ? (it.shared ? &tm_s1 : &tm_a1) : t0;
                const int rows = it.shared ? p.rows_s : p.rows;
                const int ybase = it.shared ? 0 : it.seg * rows;
                const int y0 = ybase + it.rb * rows_item;
                const int y1 = MODE == 0 ? y0 : y0 + 128;
                for (int ks = 0; ks < nks; ++ks, ++us) {
                    const uint32_t s = us % kNS;
                    if (!(ok = mbar_wait(&S->smem_empty[s], ((us / kNS) & 1) ^ 1, abort, p.err)))
                        break;
                    mbar_arrive_expect_tx(&S->smem_full[s], 2 * kTileBytes);
                    uint8_t *dst = wring + s * 2 * kTileBytes;
                    tma_load_2d(dst, t0, &S->smem_full[s], ks * kStageRowBytes, y0);
                    tma_load_2d(dst + kTileBytes, t1, &S->smem_full[s], ks * kStageRowBytes, y1);
                }
            }
            if (!ok) {
                // drain: wait (bounded) for the copies this thread issued
                for (uint32_t u = us > kNS ? us - kNS : 0; u < us; ++u)
                    for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                        if (mbar_try_wait(&S->smem_full[u % kNS], (u / kNS) & 1)) break;
                for (int j = i - nbuf < 0 ? 0 : i - nbuf; j <= i && j < my_items; ++j) {
                    const uint32_t b = nbuf == 2 ? (j & 1) : 0, ub = nbuf == 2 ? (j >> 1) : j;
                    for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                        if (mbar_try_wait(&S->bq_full[b], ub & 1)) break;
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA
        if (lane == 0) {
            uint32_t ut = 0;
            bool ok = true, issued = false;
            const uint32_t b_base = smem_u32(btile);
            for (int i = 0; ok && i < my_items; ++i) {
                const Item it = item_at(i);
                const int K = it.shared ? p.K_s : p.K;
                const int nks = (K + kStageCodes - 1) / kStageCodes;
                const uint32_t b = nbuf == 2 ? (i & 1) : 0, ub = nbuf == 2 ? (i >> 1) : i;
                const uint32_t a = i & 1, ua = i >> 1;
                if (!(ok = mbar_wait(&S->bq_full[b], ub & 1, abort, p.err))) break;
                if (!(ok = mbar_wait(&S->acc_empty[a], (ua & 1) ^ 1, abort, p.err))) break;
                tc_fence_after();
                // B descriptor of this item's limb tile; per MMA only the
                // start-address field (low 14 bits, in 16-byte units) moves
                const uint64_t bd0 = smem_desc(b_base + b * bbytes, 16, 1024, 2);
                const uint32_t bd_lo = (uint32_t)bd0, bd_hi = (uint32_t)(bd0 >> 32);
                const uint32_t d0 = tmem + kDCol + a * 32, d1 = d0 + 16;
                for (int ks = 0; ks < nks; ++ks, ++ut) {
                    const uint32_t t = ut % kNT;
                    if (!(ok = mbar_wait(&S->tmem_full[t], (ut / kNT) & 1, abort, p.err))) break;
                    tc_fence_after();
                    const uint32_t a0 = tmem + t * kAColStage;
                    // 32-byte K chunk kc = 8 ks + j lives at block kc / 4, offset 32 (kc % 4)
                    const uint32_t lo = bd_lo + (uint32_t)(ks * 2 * kBBlock >> 4);
                    const uint32_t first = ks != 0;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t off = (uint32_t)(((j >> 2) * kBBlock + (j & 3) * 32) >> 4);
                        mma_i8_ts_lohi(d0, a0 + 8 * j, lo + off, bd_hi, kIdesc, j ? 1u : first);
                        mma_i8_ts_lohi(d1, a0 + 64 + 8 * j, lo + off, bd_hi, kIdesc, j ? 1u : first);
                    }
                    issued = true;
                    mma_commit(&S->tmem_empty[t]);
                }
                if (!ok) break;
                mma_commit(&S->acc_full[a]);
                mma_commit(&S->bq_empty[b]);
            }
            // let every MMA issued so far finish before TMEM is freed
            if (issued) {
                mma_commit(&S->drain);
                for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                    if (mbar_try_wait(&S->drain, 0)) break;
            }
        }
    } else if (warp < 10) {
        // ---------------------------------------------------------- unpack
        // Two sets of four warps (one warp per TMEM lane quarter each) take
        // alternate weight stages, so two stages are unpacked at a time, and a
        // stage's TMEM stores are waited for only after the set has read its
        // next stage from shared memory.
        const int set = (warp - 2) >> 2;
        const int q = warp & 3;            // TMEM lane quarter of this warp
        const int r = q * 32 + lane;       // row within a 128-row tile
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        const int sw = (r >> 1) & 3;       // 64-byte swizzle of row r
        uint32_t us = 0;                   // stage counter over both sets
        int pend = -1;                     // TMEM stage stored but not yet published
        bool ok = true;
        for (int i = 0; ok && i < my_items; ++i) {
            const Item it = item_at(i);
            const int K = it.shared ? p.K_s : p.K;
            const int nks = (K + kStageCodes - 1) / kStageCodes;
            for (int ks = 0; ks < nks; ++ks, ++us) {
                if ((int)(us & 1) != set) continue;
                const uint32_t s = us % kNS;
                if (!(ok = mbar_wait_warp(&S->smem_full[s], (us / kNS) & 1, abort, p.err))) break;
                uint4 v[2][4];
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    const uint8_t *row = wring + s * 2 * kTileBytes + m * kTileBytes + r * kStageRowBytes;
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        v[m][c] = *reinterpret_cast<const uint4 *>(row + 16 * (c ^ sw));
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S->smem_empty[s]);
                if (pend >= 0) {
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S->tmem_full[pend]);
                    pend = -1;
                }
                const uint32_t t = us % kNT;
                if (!(ok = mbar_wait_warp(&S->tmem_empty[t], ((us / kNT) & 1) ^ 1, abort, p.err))) break;
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        const uint32_t w4[4] = {v[m][c].x, v[m][c].y, v[m][c].z, v[m][c].w};
                        uint32_t regs[16];
#pragma unroll
                        for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                regs[4 * wi + j] = (w4[wi] >> (2 * j)) & 0x03030303u;
                        tmem_st_x16(tmem + lane_addr + t * kAColStage + m * 64 + 16 * c, regs);
                    }
                }
                pend = (int)t;
            }
        }
        if (ok && pend >= 0) {
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S->tmem_full[pend]);
        }
    } else {
        // -------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        bool ok = true;
        for (int i = 0; ok && i < my_items; ++i) {
            const Item it = item_at(i);
            const int rows = it.shared ? p.rows_s : p.rows;
            const float *sc0 = it.shared ? p.ss[0] : p.s[0] + (int64_t)it.seg * p.s_stride;
            const float *sc1 = MODE == 0 ? (it.shared ? p.ss[1] : p.s[1] + (int64_t)it.seg * p.s_stride)
                                         : sc0;
            const int row0 = it.rb * rows_item + r;
            const int row1 = MODE == 0 ? row0 : row0 + 128;
            // operands of the epilogue, fetched while the MMAs run
            const float s0 = row0 < rows ? __ldg(sc0 + row0) : 0.0f;
            const float s1 = row1 < rows ? __ldg(sc1 + row1) : 0.0f;
            longlong2 mt[kTokMax];
#pragma unroll
            for (int c = 0; c < kTokMax; ++c)
                mt[c] = c < it.count ? p.meta[it.pos0 + c] : make_longlong2(0, 0);

            const uint32_t a = i & 1;
            if (!(ok = mbar_wait_warp(&S->acc_full[a], (i >> 1) & 1, abort, p.err))) break;
            tc_fence_after();
            uint32_t d0[16], d1[16];
            tmem_ld_x16(tmem + lane_addr + kDCol + a * 32, d0);
            tmem_ld_x16(tmem + lane_addr + kDCol + a * 32 + 16, d1);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S->acc_empty[a]);

#pragma unroll
            for (int c = 0; c < kTokMax; ++c) {
                if (c >= it.count) break;
                const int64_t pos = it.pos0 + c;
                const double s2 = (double)pow2i((int)mt[c].x);
                const long long v0 = (long long)(int)d0[3 * c + 2] * 65536LL +
                                     (long long)(int)d0[3 * c + 1] * 256LL +
                                     (long long)(int)d0[3 * c] - mt[c].y;
                const long long v1 = (long long)(int)d1[3 * c + 2] * 65536LL +
                                     (long long)(int)d1[3 * c + 1] * 256LL +
                                     (long long)(int)d1[3 * c] - mt[c].y;
                const float f0 = __fmul_rn((float)((double)v0 * s2), s0);
                const float f1 = __fmul_rn((float)((double)v1 * s2), s1);
                float *o = p.out + pos * p.out_ld;
                if (MODE == 0) {
                    if (row0 < rows) o[row0] = swiglu(f0, f1);
                } else {
                    if (row0 < rows) o[row0] = f0;
                    if (row1 < rows) o[row1] = f1;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

size_t qgemv_tc_smem_bytes(int kp_b, int b_buffers) {
    return 1024 + (size_t)kNS * 2 * kTileBytes + (size_t)b_buffers * kBRows * kp_b + sizeof(Smem);
}

int qgemv_tc_buffers(int kp_b) {
    return qgemv_tc_smem_bytes(kp_b, 2) <= 227 * 1024 ? 2 : 1;
}

cudaError_t launch_qgemv_tc(int mode, const QgemvTcMaps &maps, const QgemvTcParams &p, int grid,
                            cudaStream_t s) {
    const size_t smem = qgemv_tc_smem_bytes(p.kp_b, p.b_buffers);
    static size_t smem_set[2] = {0, 0};
    if (smem > smem_set[mode]) {
        cudaError_t e = mode == 0
            ? cudaFuncSetAttribute(qgemv_tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)
            : cudaFuncSetAttribute(qgemv_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        smem_set[mode] = smem;
    }
    if (mode == 0)
        qgemv_tc_kernel<0><<<grid, kThreads, smem, s>>>(maps.a0, maps.a1, maps.s0, maps.s1, maps.b, p);
    else
        qgemv_tc_kernel<1><<<grid, kThreads, smem, s>>>(maps.a0, maps.a1, maps.s0, maps.s1, maps.b, p);
    return cudaGetLastError();
}

int *device_error_flag() {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    return static_cast<int *>(p);
}

}  // namespace qmoe
