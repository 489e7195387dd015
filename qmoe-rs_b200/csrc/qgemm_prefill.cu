// qgemm_prefill.cu -- prefill-sized grouped expert products on tcgen05.
//
// Replaces, for large batches of bf16 activations, the per-assignment GEMVs
// of QMoELayer::forward (qmoe-rs src/moe.rs:89-125 via
// PackedQMoETensor::forward_simd, src/tensor.rs:64-95, and
// simd::fused_dequantize_and_dot, src/simd.rs:6-45) and the shared expert's
// batched GEMVs (src/model.rs:325-347).
//
// Arithmetic: weight = (code - 1) * scale(row) (src/simd.rs:28-31, :44).  The
// codes minus one are exact in bf16, the bf16 activations are exact, so the
// tensor core forms sum_k (code-1) x_k with f32 accumulation and the epilogue
// applies the row scale in f32.  The SwiGLU rows feeding the down product
// are rounded to bf16 (the only rounding beyond f32 accumulation order).
//
// Work item = one group (<= 256 positions of one expert segment) x one tile
// of 128 output rows: in mode 0 the 128 rows are 64 gate rows and the 64
// matching up rows, interleaved (TMEM lane 2i = gate row i, 2i+1 = up row i)
// so that the SwiGLU pairs sit in neighbouring lanes; in mode 1 they are 128
// down rows.  D[128 x N] += A[128 x 16] * B[N x 16]^T per instruction, with
//   A  the dequantised weights, written by the dequant warps straight into
//      tensor memory;
//   B  the activation rows of the group, bf16, 128-byte swizzle, one 3-D TMA
//      box per stage: two 64-element K blocks of 128, 192 or 256 rows (the
//      fewer boxes, the faster the activation ring refills: with one 2-D box
//      per K block the MMA thread waited for activations ~30 % of its time);
//   D  f32 in tensor memory columns 256..511.
// The pipeline moves in stages of two K blocks (128 K): a stage owns one
// 64-column TMEM slot for A and one 64 KB shared-memory slot for B, and has
// one "full" barrier (four dequant-warp arrivals + the TMA transaction
// bytes) and one "empty" barrier (the MMA commit), so the single MMA thread
// waits once per eight MMAs.  One producer thread can issue a TMA box only
// every few hundred cycles (the issue and the barrier round trips), so boxes
// are as large as the 128-byte swizzle allows and few per stage.
//
// Persistent grid, one CTA per SM, twenty-three warps:
//   warp 0      TMA producer of the packed weight stages (256 K each);
//   warp 22     TMA producer of the activation K blocks;
//   warp 1      TMEM owner and MMA issuer (one thread);
//   warps 2-5   dequant: one TMEM lane (weight row) per thread, 64 codes per
//               K block: ((w >> s) & 0x00030003) | 0x43004300 is the bf16
//               pair (128 + c_lo, 128 + c_hi), one bf16x2 FMA subtracts 129;
//               a stage's TMEM stores are waited for only after the next
//               stage is unpacked;
//   warps 6-21  epilogue: four warps per TMEM lane quarter, each draining
//               at most two 32-column chunks to registers, then releasing the
//               accumulator; scales, SwiGLU (mode 0) or f32 rows (mode 1).
// Every wait is bounded; on a time-out the kernel flags the device error
// word, drains its copies and MMAs (again bounded), frees TMEM and returns.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace qmoe {
namespace {

using namespace sm100;

constexpr int kWarps = 23;
constexpr int kThreads = kWarps * 32;
constexpr int kEpiWarp0 = 6;
constexpr int kEpiWarps = 16;                // four per TMEM lane quarter
constexpr int kBWarp = 22;                   // activation producer
constexpr int kNW = 3;                       // packed-weight stages
constexpr int kWStage = 8192;                // 128 rows x 64 B (256 codes per row)
constexpr int kNS = 3;                       // pipeline stages (2 K blocks each)
constexpr int kKbBytes = kPrefillTile * 128; // one K block of B: 256 rows x 128 B
constexpr int kSBytes = 2 * kKbBytes;        // B bytes of a stage
constexpr uint32_t kACols = 64;              // TMEM columns of A per stage
constexpr uint32_t kDCol = 256;              // accumulator columns 256..511
constexpr uint32_t kTmemCols = 512;
constexpr int kItemCache = 256;
static_assert(kNS * kACols <= kDCol, "A slots overlap the accumulator");

struct Smem {
    uint64_t wfull[kNW], wempty[kNW];
    uint64_t full[kNS], empty[kNS];
    uint64_t dfull, dempty, drain;
    uint32_t tmem_base;
    int abort;
    int4 items[kItemCache];
};

struct Item {
    int seg, pos0, count, mt;
    bool shared;
};

QMOE_DEV Item decode_item(const QgemmParams &p, int item, int nr, int mt_r, int mt_s) {
    Item it;
    int g;
    if (item < nr * mt_r) {
        g = item / mt_r;
        it.mt = item % mt_r;
        it.shared = false;
    } else {
        const int j = item - nr * mt_r;
        g = nr + j / mt_s;
        it.mt = j % mt_s;
        it.shared = true;
    }
    const int4 d = p.groups[g];
    it.seg = d.x;
    it.pos0 = d.y;
    it.count = d.z;
    return it;
}

// Rows of the activation box of a group of `count` positions.
QMOE_DEV int box_rows(int count) { return count <= 128 ? 128 : count <= 192 ? 192 : 256; }

// (128 + c_lo, 128 + c_hi) - (129, 129) = (c_lo - 1, c_hi - 1), exact in bf16
QMOE_DEV uint32_t codes_to_bf16x2(uint32_t biased) {
    uint32_t r;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(biased), "r"(0x3F803F80u), "r"(0xC301C301u));
    return r;
}

// SiLU(g) * u in the fast-math form (|relative error| ~1e-6, far inside the
// bf16 rounding of the result); g is clamped so 1 + exp(-g) stays finite.
QMOE_DEV float swiglu_fast(float g, float u) {
    return __fdividef(g, 1.0f + __expf(-fmaxf(g, -80.0f))) * u;
}

// One drained 32-column chunk: scale, then (mode 0) pair the gate/up lanes
// and store bf16 SwiGLU rows, or (mode 1) store f32 rows.
template <int MODE>
QMOE_DEV void epilogue_chunk(const QgemmParams &p, const Item &it, int c, const uint32_t (&v)[32],
                             int L, int row, int rows, float scale) {
    if (MODE == 0) {
        // lane pair (2i, 2i+1) = (gate, up) of row i: the even lane finishes
        // columns 0-15 of the chunk, the odd lane 16-31
        const bool odd = L & 1;
        const int hpos = (row & ~15) | (4 * (row & 3) + 2 * ((row >> 2) & 1) + ((row >> 3) & 1));
        __nv_bfloat16 *o = reinterpret_cast<__nv_bfloat16 *>(p.out) + hpos;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float mine_lo = __uint_as_float(v[j]) * scale;
            const float mine_hi = __uint_as_float(v[16 + j]) * scale;
            const float other = __shfl_xor_sync(0xffffffffu, odd ? mine_lo : mine_hi, 1);
            const float g = odd ? other : mine_lo;
            const float u = odd ? mine_hi : other;
            const int n = 32 * c + (odd ? 16 : 0) + j;
            if (n < it.count && row < rows)
                o[(int64_t)(it.pos0 + n) * p.out_ld] = __float2bfloat16_rn(swiglu_fast(g, u));
        }
    } else {
        float *o = reinterpret_cast<float *>(p.out) + row;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int n = 32 * c + j;
            if (n < it.count && row < rows)
                o[(int64_t)(it.pos0 + n) * p.out_ld] = __uint_as_float(v[j]) * scale;
        }
    }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
qgemm_prefill_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                     const __grid_constant__ CUtensorMap tm_s0, const __grid_constant__ CUtensorMap tm_s1,
                     const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_b2,
                     const __grid_constant__ CUtensorMap tm_b3, const QgemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *bring = base;                         // kNS x 64 KB activation stages
    uint8_t *wring = bring + kNS * kSBytes;        // kNW x 8 KB packed weights
    Smem *S = reinterpret_cast<Smem *>(wring + kNW * kWStage);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int rows_tile = MODE == 0 ? 64 : 128;    // matrix rows per item (per matrix)
    const int mt_r = (p.rows + rows_tile - 1) / rows_tile;
    const int mt_s = p.rows_s > 0 ? (p.rows_s + rows_tile - 1) / rows_tile : 1;
    const int nr = p.n_groups[0], ns = p.n_groups[1];
    const int total = nr * mt_r + ns * mt_s;
    const int my_items =
        total > (int)blockIdx.x ? (total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    if (my_items == 0) return;  // uniform across the CTA, before any barrier or TMEM use

    if (tid == 0) {
        for (int i = 0; i < kNW; ++i) {
            mbar_init(&S->wfull[i], 1);
            mbar_init(&S->wempty[i], 4);
        }
        for (int i = 0; i < kNS; ++i) {
            mbar_init(&S->full[i], 4 + 1);     // dequant warps + TMA bytes
            mbar_init(&S->empty[i], 1);
        }
        mbar_init(&S->dfull, 1);
        mbar_init(&S->dempty, kEpiWarps);
        mbar_init(&S->drain, 1);
        S->abort = 0;
        fence_mbar_init();
    }
    for (int i = tid; i < my_items && i < kItemCache; i += kThreads) {
        const Item it = decode_item(p, (int)blockIdx.x + i * (int)gridDim.x, nr, mt_r, mt_s);
        S->items[i] = make_int4(it.seg, it.pos0, it.count, it.mt | (it.shared ? (1 << 30) : 0));
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
            it.mt = v.w & ((1 << 30) - 1);
            it.shared = (v.w >> 30) & 1;
            return it;
        }
        return decode_item(p, (int)blockIdx.x + i * (int)gridDim.x, nr, mt_r, mt_s);
    };

    if (warp == 0) {
        // ------------------------------------------------- TMA: packed weights
        if (lane == 0) {
            tma_prefetch_desc(&tm_w0);
            if (MODE == 0) tma_prefetch_desc(&tm_w1);
            if (p.rows_s > 0) {
                tma_prefetch_desc(&tm_s0);
                if (MODE == 0) tma_prefetch_desc(&tm_s1);
            }
            uint32_t uw = 0;
            bool ok = true;
            for (int i = 0; ok && i < my_items; ++i) {
                const Item it = item_at(i);
                const int K = it.shared ? p.K_s : p.K;
                const int nws = (K / 64 + 3) / 4;             // stages of 256 codes
                const CUtensorMap *m0 = it.shared ? &tm_s0 : &tm_w0;
                const CUtensorMap *m1 = it.shared ? &tm_s1 : &tm_w1;
                const int rows = it.shared ? p.rows_s : p.rows;
                const int y = (it.shared ? 0 : it.seg * rows) + it.mt * rows_tile;
                for (int ws = 0; ws < nws; ++ws, ++uw) {
                    const uint32_t s = uw % kNW;
                    if (!(ok = mbar_wait(&S->wempty[s], ((uw / kNW) & 1) ^ 1, abort, p.err))) break;
                    mbar_arrive_expect_tx(&S->wfull[s], kWStage);
                    uint8_t *dst = wring + s * kWStage;
                    tma_load_2d(dst, m0, &S->wfull[s], ws * 64, y);
                    if (MODE == 0) tma_load_2d(dst + kWStage / 2, m1, &S->wfull[s], ws * 64, y);
                }
            }
            if (!ok)  // let the copies already issued land before the CTA exits
                for (uint32_t u = uw > kNW ? uw - kNW : 0; u < uw; ++u)
                    for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                        if (mbar_try_wait(&S->wfull[u % kNW], (u / kNW) & 1)) break;
        }
    } else if (warp == kBWarp) {
        // ---------------------------------------------- TMA: activation rows
        if (lane == 0) {
            tma_prefetch_desc(&tm_b);
            tma_prefetch_desc(&tm_b2);
            tma_prefetch_desc(&tm_b3);
            uint32_t us = 0;
            bool ok = true;
            for (int i = 0; ok && i < my_items; ++i) {
                const Item it = item_at(i);
                const int K = it.shared ? p.K_s : p.K;
                const int nkb = K / 64;
                // one box per stage (two K blocks), the smallest of 128 / 192 /
                // 256 rows that holds the group (the MMAs read N = count
                // rounded to 16 rows); a stage with one K block left gets the
                // second zero-filled (past the last K block) and unused
                const CUtensorMap *mb = it.count <= 128 ? &tm_b2 : it.count <= 192 ? &tm_b3 : &tm_b;
                const uint32_t box = (uint32_t)box_rows(it.count) * 128;
                if (it.count > kPrefillTile) {
                    // a group larger than the stage slots: nothing is loaded,
                    // every role gives up at its next wait
                    atomicOr(p.err, kErrBadGroup);
                    *abort = 1;
                    ok = false;
                    break;
                }
                for (int kb = 0; kb < nkb; kb += 2, ++us) {
                    const uint32_t s = us % kNS;
                    if (!(ok = mbar_wait(&S->empty[s], ((us / kNS) & 1) ^ 1, abort, p.err))) break;
                    mbar_arrive_expect_tx(&S->full[s], 2 * box);
                    tma_load_3d(bring + s * kSBytes, mb, &S->full[s], 0, it.pos0, kb);
                }
            }
            if (!ok)
                for (uint32_t u = us > kNS ? us - kNS : 0; u < us; ++u)
                    for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                        if (mbar_try_wait(&S->full[u % kNS], (u / kNS) & 1)) break;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA
        if (lane == 0) {
            uint32_t us = 0;
            bool ok = true, issued = false;
            const uint64_t bd0 = smem_desc(smem_u32(bring), 16, 1024, 2);
            const uint32_t bd_lo = (uint32_t)bd0, bd_hi = (uint32_t)(bd0 >> 32);
            for (int i = 0; ok && i < my_items; ++i) {
                const Item it = item_at(i);
                const int K = it.shared ? p.K_s : p.K;
                const int nkb = K / 64;
                const int N = (it.count + 15) & ~15;
                const uint32_t idesc = idesc_bf16(128, N);
                const int box = box_rows(it.count) * 128;   // bytes of one K block of B
                if (!(ok = mbar_wait(&S->dempty, (i & 1) ^ 1, abort, p.err))) break;
                tc_fence_after();
                for (int kb = 0; kb < nkb; kb += 2, ++us) {
                    const int nk = nkb - kb < 2 ? nkb - kb : 2;
                    const uint32_t s = us % kNS;
                    if (!(ok = mbar_wait(&S->full[s], (us / kNS) & 1, abort, p.err))) break;
                    tc_fence_after();
                    for (int j = 0; j < nk; ++j) {
                        const uint32_t lo = bd_lo + (uint32_t)((s * kSBytes + j * box) >> 4);
                        const uint32_t a = tmem + s * kACols + 32 * j;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)
                            mma_bf16_ts_lohi(tmem + kDCol, a + 8 * kk, lo + 2 * kk, bd_hi, idesc,
                                             (kb | j | kk) != 0);
                    }
                    issued = true;
                    mma_commit(&S->empty[s]);
                }
                if (!ok) break;
                mma_commit(&S->dfull);
            }
            // every MMA issued so far completes before TMEM is freed
            if (issued) {
                mma_commit(&S->drain);
                for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                    if (mbar_try_wait(&S->drain, 0)) break;
            }
        }
    } else if (warp < kEpiWarp0) {
        // ---------------------------------------------------------- dequant
        const int q = warp & 3;                       // TMEM lane quarter
        const int L = q * 32 + lane;                  // A row = TMEM lane
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        // packed row in the weight stage: mode 0 gate row L/2 (even L) or up
        // row L/2 (odd L), each a 64-row box; mode 1 down row L
        const int r = MODE == 0 ? (L >> 1) : L;
        const int box_off = MODE == 0 ? (L & 1) * (kWStage / 2) : 0;
        const int sw = (r >> 1) & 3;                  // 64-byte swizzle of row r
        uint32_t uw = 0, us = 0;
        int pend = -1;                                // stage stored, not yet published
        bool ok = true;
        for (int i = 0; ok && i < my_items; ++i) {
            const Item it = item_at(i);
            const int K = it.shared ? p.K_s : p.K;
            const int nkb = K / 64;
            for (int kb = 0; kb < nkb; kb += 2, ++us) {
                const int nk = nkb - kb < 2 ? nkb - kb : 2;
                const uint32_t ws = uw % kNW;         // kb and kb+1 share a weight stage
                if ((kb & 3) == 0) {
                    if (!(ok = mbar_wait_warp(&S->wfull[ws], (uw / kNW) & 1, abort, p.err))) break;
                }
                const uint8_t *wrow = wring + ws * kWStage + box_off + r * 64;
                const uint4 v0 = *reinterpret_cast<const uint4 *>(wrow + 16 * ((kb & 3) ^ sw));
                const uint4 v1 = *reinterpret_cast<const uint4 *>(wrow + 16 * (((kb + 1) & 3) ^ sw));
                if ((kb & 3) == 2 || kb + nk >= nkb) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S->wempty[ws]);
                    ++uw;
                }
                const uint32_t s = us % kNS;
                if (!(ok = mbar_wait_warp(&S->empty[s], ((us / kNS) & 1) ^ 1, abort, p.err))) break;
                tc_fence_after();
                // publish the previous stage (its stores had this stage's
                // unpacking to complete in), then store this one
                if (pend >= 0) {
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S->full[pend]);
                }
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if (j < nk) {
                        const uint4 v = j ? v1 : v0;
                        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
                        uint32_t regs[32];
#pragma unroll
                        for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                            for (int jj = 0; jj < 4; ++jj)
#pragma unroll
                                for (int pp = 0; pp < 2; ++pp)
                                    regs[8 * wi + 2 * jj + pp] = codes_to_bf16x2(
                                        ((w4[wi] >> (2 * jj + 8 * pp)) & 0x00030003u) | 0x43004300u);
                        tmem_st_x32(tmem + lane_addr + s * kACols + 32 * j, regs);
                    }
                }
                pend = (int)s;
            }
        }
        tmem_wait_st();
        if (ok && pend >= 0) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S->full[pend]);
        }
    } else if (warp < kEpiWarp0 + kEpiWarps) {
        // -------------------------------------------------------- epilogue
        // Each warp drains its (at most two) 32-column chunks of the
        // accumulator into registers and releases it at once, so the next
        // item's MMAs overlap the scaling, SwiGLU and stores.
        const int q = warp & 3;
        const int slot = (warp - kEpiWarp0) >> 2;     // chunks slot, slot + 4
        const int L = q * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        bool ok = true;
        for (int i = 0; ok && i < my_items; ++i) {
            const Item it = item_at(i);
            const int rows = it.shared ? p.rows_s : p.rows;
            const int nch = (it.count + 31) / 32;
            int row;
            float scale;
            if (MODE == 0) {
                row = it.mt * 64 + (L >> 1);
                const bool up = L & 1;
                const float *sc = it.shared ? (up ? p.ss[1] : p.ss[0])
                                            : (up ? p.s[1] : p.s[0]) + (int64_t)it.seg * p.s_stride;
                scale = row < rows ? __ldg(sc + row) : 0.0f;
            } else {
                row = it.mt * 128 + L;
                const float *sc = it.shared ? p.ss[0] : p.s[0] + (int64_t)it.seg * p.s_stride;
                scale = row < rows ? __ldg(sc + row) : 0.0f;
            }
            if (!(ok = mbar_wait_warp(&S->dfull, i & 1, abort, p.err))) break;
            tc_fence_after();
            uint32_t v0[32], v1[32];
            const int c0 = slot, c1 = slot + 4;
            if (c0 < nch) tmem_ld_x32(tmem + lane_addr + kDCol + 32 * c0, v0);
            if (c1 < nch) tmem_ld_x32(tmem + lane_addr + kDCol + 32 * c1, v1);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S->dempty);
            if (c0 < nch) epilogue_chunk<MODE>(p, it, c0, v0, L, row, rows, scale);
            if (c1 < nch) epilogue_chunk<MODE>(p, it, c1, v1, L, row, rows, scale);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Row of x (bf16) -> position row of xg with each 16-element block permuted
// (position 2q / 2q+1 of word q = 2j + pp holds element 4pp + j / 8 + 4pp +
// j).  One warp per position row, grid-stride over the rows; a lane moves
// the 32-byte blocks lane, lane + 32, ... with two blocks' loads in flight
// before their stores.
constexpr int kGatherWarps = 8;

QMOE_DEV void permute_block(const uint4 &a, const uint4 &c, uint4 &o0, uint4 &o1) {
    o0.x = __byte_perm(a.x, c.x, 0x5410);  // e0  | e8
    o0.y = __byte_perm(a.z, c.z, 0x5410);  // e4  | e12
    o0.z = __byte_perm(a.x, c.x, 0x7632);  // e1  | e9
    o0.w = __byte_perm(a.z, c.z, 0x7632);  // e5  | e13
    o1.x = __byte_perm(a.y, c.y, 0x5410);  // e2  | e10
    o1.y = __byte_perm(a.w, c.w, 0x5410);  // e6  | e14
    o1.z = __byte_perm(a.y, c.y, 0x7632);  // e3  | e11
    o1.w = __byte_perm(a.w, c.w, 0x7632);  // e7  | e15
}

__global__ void __launch_bounds__(kGatherWarps * 32)
gather_bf16_kernel(const GatherParams p) {
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int lane = threadIdx.x & 31;
    const int64_t nblk = p.H / 16;
    const int64_t nvalid = *p.n_valid;
    const int64_t warps = (int64_t)gridDim.x * kGatherWarps;
    for (int64_t pos = (int64_t)blockIdx.x * kGatherWarps + (threadIdx.x >> 5); pos < p.npos; pos += warps) {
        const bool routed = pos < p.shared_base;
        if (routed && pos >= nvalid) continue;
        const int64_t row = routed ? (int64_t)p.pos_tok[pos] : p.shared_row0 + pos - p.shared_base;
        const uint4 *src = reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(p.x) + row * p.H);
        uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.xg) + pos * p.H);
        int64_t b = lane;
        for (; b + 32 < nblk; b += 64) {
            const uint4 a0 = __ldg(src + 2 * b), c0 = __ldg(src + 2 * b + 1);
            const uint4 a1 = __ldg(src + 2 * (b + 32)), c1 = __ldg(src + 2 * (b + 32) + 1);
            uint4 o0, o1;
            permute_block(a0, c0, o0, o1);
            dst[2 * b] = o0;
            dst[2 * b + 1] = o1;
            permute_block(a1, c1, o0, o1);
            dst[2 * (b + 32)] = o0;
            dst[2 * (b + 32) + 1] = o1;
        }
        if (b < nblk) {
            const uint4 a0 = __ldg(src + 2 * b), c0 = __ldg(src + 2 * b + 1);
            uint4 o0, o1;
            permute_block(a0, c0, o0, o1);
            dst[2 * b] = o0;
            dst[2 * b + 1] = o1;
        }
    }
}

}  // namespace

size_t qgemm_prefill_smem_bytes() {
    return 1024 + (size_t)kNS * kSBytes + (size_t)kNW * kWStage + sizeof(Smem);
}

cudaError_t launch_qgemm_prefill(int mode, const QgemmMaps &maps, const QgemmParams &p, int grid,
                                 cudaStream_t s) {
    const size_t smem = qgemm_prefill_smem_bytes();
    cudaError_t e = mode == 0 ? ensure_dyn_smem(reinterpret_cast<const void *>(qgemm_prefill_kernel<0>), smem)
                              : ensure_dyn_smem(reinterpret_cast<const void *>(qgemm_prefill_kernel<1>), smem);
    if (e != cudaSuccess) return e;
    return mode == 0 ? launch_pdl(qgemm_prefill_kernel<0>, dim3(grid), dim3(kThreads), smem, s, maps.w0,
                                  maps.w1, maps.s0, maps.s1, maps.b, maps.b2, maps.b3, p)
                     : launch_pdl(qgemm_prefill_kernel<1>, dim3(grid), dim3(kThreads), smem, s, maps.w0,
                                  maps.w1, maps.s0, maps.s1, maps.b, maps.b2, maps.b3, p);
}

cudaError_t launch_gather_bf16(const GatherParams &p, cudaStream_t s) {
    if (p.npos == 0) return cudaSuccess;
    // enough warps for every SM (8 CTAs of 8 warps each), at most one per row
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t need = (p.npos + kGatherWarps - 1) / kGatherWarps;
    const int64_t cap = (int64_t)sms * 8;
    return launch_pdl(gather_bf16_kernel, dim3((unsigned)(need < cap ? need : cap)), dim3(kGatherWarps * 32), 0,
                      s, p);
}

}  // namespace qmoe
