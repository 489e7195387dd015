// qgemv_imma.cu -- decode-sized grouped GEMV over 2-bit packed expert weights.
//
// Replaces the per-assignment GEMVs of QMoELayer::forward (qmoe-rs
// src/moe.rs:96-118 via PackedQMoETensor::forward_simd, src/tensor.rs:64-95,
// and simd::fused_dequantize_and_dot, src/simd.rs:6-45) and the shared
// expert's batched GEMVs (src/model.rs:325-347).
//
// Arithmetic: a weight is code - 1 (code in 0..3) and each activation row is
// x ~= 2^e * Q with Q split into three int8 limbs (quant.cu), so
//     dot(w_r, x) = 2^e * (sum_l 256^l sum_k code_rk q_lk  -  sum_k Q_k).
// The tensor pipe forms every sum_k code_rk q_lk exactly (mma.sync
// m16n8k32, A = u8 codes of 16 weight rows, B = s8 limbs: one n8 tile holds
// 2 positions x 3 limbs, two tiles 5 positions), the epilogue recombines the
// limbs in int64 and scales once.
//
// Why mma.sync here: with only a few positions per expert the product is a
// stream of weights each used by <= 15 limb rows.  tcgen05.mma reads its A
// tile (the weights, 128 rows x 32 bytes) at a fixed ~4 KB per instruction
// whatever N is, i.e. ~37 weights per clock per SM -- below the HBM rate of
// ~93 packed weights per clock per SM.  The warp-level m16n8k32 consumes 512
// weights per instruction from registers against one n8 limb tile, one per
// ~8 cycles per scheduler, so the kernel can follow HBM.
//
// Work item = (<= 5 positions of one segment) x 256 output rows (gate+up
// rows 128+128 in mode 0, 256 down rows in mode 1).  Persistent grid, one CTA
// per SM, thirteen warps:
//   warp 0      TMA: per stage of 512 codes, the 2-bit weight tiles
//               [2 chunks x 128 rows x 64 B] (64-byte swizzle, one 3-D box per
//               tile) and the item's limb rows for those codes [4 blocks x 16
//               rows x 128 B] (128-byte swizzle, one 3-D box), 40 KB, into a
//               4-stage ring continuous across items: HBM latency under load
//               is several thousand cycles, so the bytes in flight set the
//               rate, and a thread issues a box only every few hundred
//               cycles, so boxes are few and large;
//   warps 1-8   compute: two groups of four warps take the two 256-code
//               chunks of a stage; a warp owns 32 rows of each weight tile
//               (four 16-row blocks): 128-bit shared loads of the packed
//               rows, unpack in registers ((w << (6 - 2j)) & 0xC0C0C0C0: one
//               shift + one mask per 4 weights, codes scaled by 64), m16n8k32
//               IMMAs against one limb tile for items of <= 2 positions, two
//               otherwise; at item end each group's int32 accumulators go to
//               its tile of a double-buffered pair in shared memory;
//   warps 9-12  epilogue: sum of the two groups' tiles, limb recombination,
//               scales, SwiGLU, stores, while the compute warps run the next
//               item.
// Every wait is bounded; on a time-out the kernel flags the device error
// word, lets its TMA copies drain (again bounded) and returns.
#include "combine.cuh"
#include "ep_signal.cuh"
#include "common.cuh"
#include "kernels.h"
#include "quant.cuh"
#include "sm100.cuh"

namespace qmoe {
namespace {

using namespace sm100;

constexpr int kWarps = 13;
constexpr int kThreads = kWarps * 32;
constexpr int kCompute = 8;            // compute warps (1..8)
constexpr int kEpiWarp0 = 9;           // first epilogue warp
constexpr int kNS = 4;                 // stages in shared memory
constexpr int kStageCodes = 512;       // codes per row per stage (two 64-byte chunks)
constexpr int kSubBytes = 128 * 64;    // one 128-row x 64-byte chunk (64-byte swizzle)
constexpr int kTileBytes = 2 * kSubBytes;  // one 128-row weight tile of a stage
constexpr int kBRows = 16;             // positions x limbs (15 used)
constexpr int kBBlock = kBRows * 128;  // one 128-byte K block of the limb rows
constexpr int kLimbBytes = 4 * kBBlock;            // limb blocks of a stage (512 codes)
constexpr int kStageBytes = 2 * kTileBytes + kLimbBytes;  // 40 KB
constexpr int kTokMax = 5;
constexpr int kOutCols = 256;          // output rows per item
constexpr int kLimbRows = 15;          // limb rows in use (5 positions x 3 limbs)
constexpr int kTileStride = 260;       // int32 row stride of an accumulator tile (2 x 260 = 8 mod 32 banks)
constexpr int kAccBytes = kLimbRows * kTileStride * 4;  // one group's int32 tile
constexpr int kQueue = 16;              // published items (> kNS + 2 items in flight)

struct Smem {
    uint64_t smem_full[kNS], smem_empty[kNS];
    uint64_t tile_full[2], tile_empty[2];
    int abort;
    int grid_ok;                       // the last grid barrier was passed
    int4 queue[kQueue];                // this CTA's items in run order; x < 0: no more
    float q_red[3][4];                 // limb phase: per row group, per warp
    long long q_sum[3][4];
    int c_pos[kCombineMaxK];           // combine phase: the token's rows, ranked
    float c_w[kCombineMaxK];
    int c_n;
};

QMOE_DEV void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

QMOE_DEV int ld_acquire_gpu(const int *p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Generic-proxy global writes of this thread become visible to (and later
// async-proxy reads, i.e. TMA, of this thread are ordered after) the fence.
QMOE_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Bounded wait until a grid-wide barrier count reaches `target` (every CTA of
// the cooperative launch has counted in).  On time-out: abort, error word.
QMOE_DEV bool grid_wait(const int *ctr, int target, volatile int *abort, int *err) {
    for (uint32_t n = 0; n < kMaxWaitProbes; ++n) {
        if (ld_acquire_gpu(ctr) >= target) return true;
        if (*abort) return false;
        __nanosleep(64);
    }
    *abort = 1;
    atomicOr(err, kErrWaitTimeout);
    return false;
}

// Limb phase of a cooperative launch: warps 1..12 as three groups of four,
// one position per group at a time (quant.cuh), then every CTA counts in on
// the grid barrier and the twelve warps wait for all of them.
QMOE_DEV void limb_phase(const DecodeParams &p, Smem *S, int tid, volatile int *abort) {
    const int g = (tid - 32) >> 7, ht = (tid - 32) & 127;
    const int kmax = p.q.K > p.q.K_s ? p.q.K : p.q.K_s;
    const int nblk = ((kmax + 255) / 256) * 16;
    const int bpt = (nblk + kQuantGroup - 1) / kQuantGroup;
    auto sync = [g] { named_bar(1 + g, kQuantGroup); };
    for (int64_t pos = (int64_t)blockIdx.x * 3 + g; pos < p.q.npos; pos += (int64_t)gridDim.x * 3) {
        // rows of up to 1024 float4 (the V3 hidden size) stay in registers:
        // every load in flight at once instead of two passes of dependent
        // loads
        if (bpt <= 1)
            quant_position<1>(p.q, pos, ht, S->q_red[g], S->q_sum[g], sync);
        else if (bpt <= 2)
            quant_position<2>(p.q, pos, ht, S->q_red[g], S->q_sum[g], sync);
        else if (bpt <= 4)
            quant_position<4>(p.q, pos, ht, S->q_red[g], S->q_sum[g], sync);
        else
            quant_position<0>(p.q, pos, ht, S->q_red[g], S->q_sum[g], sync);
    }
    fence_proxy_async_global();
    __threadfence();
    named_bar(4, 384);
    if (tid == 32) {
        atomicAdd(p.sched + 2, 1);
        S->grid_ok = grid_wait(p.sched + 2, (int)gridDim.x, abort, p.err);
    }
    named_bar(4, 384);
}

struct Item {
    int seg, pos0, count, rb;
    bool shared;
};

QMOE_DEV int4 pack_item(const Item &it) {
    return make_int4(it.seg, it.pos0, it.count, it.rb | (it.shared ? (1 << 30) : 0));
}

QMOE_DEV Item unpack_item(int4 v) {
    Item it;
    it.seg = v.x;
    it.pos0 = v.y;
    it.count = v.z;
    it.rb = v.w & ((1 << 30) - 1);
    it.shared = (v.w >> 30) & 1;
    return it;
}

QMOE_DEV Item decode_item(const DecodeParams &p, int item, int nr, int rb_r, int rb_s) {
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

QMOE_DEV void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                   uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A warp's share of one stage: rows 32 wq .. 32 wq + 31 of both weight tiles
// (16-row blocks b = 0..3: tile b / 2, rows 32 wq + 16 (b & 1) + {g8, g8 + 8})
// x the 256-code chunk grp, against NT n8 tiles of limb rows (8 per tile).
// m16n8k32 with A = weight codes (u8, unpacked in registers), B = limbs (s8):
// lane (g8, t4) holds 16 codes of rows g8 and g8 + 8 per 32-bit word, and
// (w << (6 - 2j)) & 0xC0C0C0C0 puts code j of each byte at bits 6-7, i.e.
// every A byte is 64 x code; the epilogue divides the exact int32 sums by 64.
// A 32-bit word q of a 64-code chunk covers 16 consecutive codes; codes
// {0,4,8,12} + j of it meet limb bytes 4j..4j+3 of the matching 16-byte limb
// fragment, whose positions are permuted to that order by the limb writer.
// The loads are done, and the stage released, before the IMMAs.
template <int NT>
QMOE_DEV void stage_mma(const uint8_t *stage, int grp, int wq, int g8, int t4, int (&acc)[8][4],
                        uint64_t *empty, int lane) {
    uint4 w[8], lo[4], hi[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const uint8_t *wt = stage + (b >> 1) * kTileBytes + grp * kSubBytes;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int rr = wq * 32 + (b & 1) * 16 + h * 8 + g8;
            w[2 * b + h] = *reinterpret_cast<const uint4 *>(wt + rr * 64 + 16 * (t4 ^ ((rr >> 1) & 3)));
        }
    }
    // limb fragments of the chunk: 16-code groups 4 t4 + q, i.e. 16-byte
    // chunk c of 128-byte block t4 / 2 of group grp; limb rows g8 (tile 0)
    // and g8 + 8 (tile 1).  The stage's limbs are 128-byte lines
    // [group][row][block] with the 128-byte swizzle (chunk ^ line % 8), so a
    // quarter-warp (rows 2i, 2i + 1 x four t4) meets four line phases
    // 2 row + block and two chunks each: eight distinct bank groups
    const int line = grp * 32 + g8 * 2 + (t4 >> 1);
    const uint8_t *lrow = stage + 2 * kTileBytes + line * 128;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int c = ((t4 & 1) << 2) | q;
        const int off = 16 * (c ^ (line & 7));
        lo[q] = *reinterpret_cast<const uint4 *>(lrow + off);
        if (NT == 2) hi[q] = *reinterpret_cast<const uint4 *>(lrow + 16 * 128 + off);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint32_t wl = q == 0 ? w[2 * b].x : q == 1 ? w[2 * b].y : q == 2 ? w[2 * b].z : w[2 * b].w;
            const uint32_t wh = q == 0 ? w[2 * b + 1].x : q == 1 ? w[2 * b + 1].y
                              : q == 2 ? w[2 * b + 1].z : w[2 * b + 1].w;
            const uint32_t m = 0xC0C0C0C0u;
            const uint32_t a0 = (wl << 6) & m, a1 = (wh << 6) & m, a2 = (wl << 4) & m, a3 = (wh << 4) & m;
            const uint32_t c0 = (wl << 2) & m, c1 = (wh << 2) & m, c2 = wl & m, c3 = wh & m;
            const uint4 l = lo[q];
            imma(acc[b], a0, a1, a2, a3, l.x, l.y);
            imma(acc[b], c0, c1, c2, c3, l.z, l.w);
            if (NT == 2) {
                const uint4 u = hi[q];
                imma(acc[4 + b], a0, a1, a2, a3, u.x, u.y);
                imma(acc[4 + b], c0, c1, c2, c3, u.z, u.w);
            }
        }
    }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
qgemv_imma_kernel(const __grid_constant__ DecodeMaps maps, const DecodeParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = base;                                   // kNS stages: 2 weight tiles + limbs
    int *acc_tile = reinterpret_cast<int *>(ring + kNS * kStageBytes);  // [2 bufs][2 groups][15][264]
    Smem *S = reinterpret_cast<Smem *>(reinterpret_cast<uint8_t *>(acc_tile) + 4 * kAccBytes);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // Separate-limb launches read the work list (groups, counts) and issue
    // the first weights before the wait on the preceding kernel: the list
    // comes from a kernel two launches back (the permute or the front, then
    // the limb kernel), which had completed before this grid was launched,
    // because every kernel of the library triggers its dependents only after
    // its own wait.  A cooperative launch (limbs or combine inside) follows
    // the kernel that builds the list, so it waits for that grid first.  The
    // limb rows, their metadata and every global write come after the wait.
    if (p.quant_in || p.combine) QMOE_PDL_WAIT();
    const int rows_item = MODE == 0 ? 128 : 256;
    const int rb_r = (p.rows + rows_item - 1) / rows_item;
    const int rb_s = p.rows_s > 0 ? (p.rows_s + rows_item - 1) / rows_item : 1;
    const int nr = p.n_groups[0], ns = p.n_groups[1];
    const int total = nr * rb_r + ns * rb_s;

    if (tid == 0) {
        for (int i = 0; i < kNS; ++i) {
            mbar_init(&S->smem_full[i], 1);
            mbar_init(&S->smem_empty[i], kCompute);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S->tile_full[i], kCompute);
            mbar_init(&S->tile_empty[i], 4);
        }
        S->abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    volatile int *abort = &S->abort;
    const bool producer = warp == 0 && lane == 0;
    if (!producer) {
        QMOE_PDL_WAIT();
        QMOE_PDL_TRIGGER();
    }
    if (p.quant_in && warp >= 1) limb_phase(p, S, tid, abort);

    // Work items are numbered in descending list order (the shared expert's,
    // the costliest, first).  A CTA runs number blockIdx.x first and then the
    // numbers the grid's counter hands out, so CTAs that finish early take
    // more; the TMA thread publishes each item in the queue before its first
    // stage, and after the last an end mark that rides on the next stage's
    // full barrier (compute warps) and then on a tile barrier (epilogue).
    if (warp == 0) {
        // ------------------------------------------------------------- TMA
        // Per stage: one 3-D box per weight tile (two 64-byte chunks of 128
        // rows; 2-D boxes per chunk where the stage reaches the ragged end of
        // a row) and one 3-D box of the item's limb rows for those 512 codes.
        if (lane == 0) {
            tma_prefetch_desc(&maps.a0_3);
            tma_prefetch_desc(&maps.b3);
            if (MODE == 0) tma_prefetch_desc(&maps.a1_3);
            if (p.rows_s > 0) {
                tma_prefetch_desc(&maps.s0_3);
                if (MODE == 0) tma_prefetch_desc(&maps.s1_3);
            }
            const uint64_t stream = l2_evict_first_policy();
            uint64_t keep;
            asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(keep));
            auto issue_weights = [&](const Item &it, int ks, uint32_t s) {
                const int K = it.shared ? p.K_s : p.K;
                const int nfull = K >> 8;                   // complete 64-byte chunks per row
                const CUtensorMap *t0 = it.shared ? &maps.s0 : &maps.a0;
                const CUtensorMap *t1 = MODE == 0 ? (it.shared ? &maps.s1 : &maps.a1) : t0;
                const CUtensorMap *t0_3 = it.shared ? &maps.s0_3 : &maps.a0_3;
                const CUtensorMap *t1_3 = MODE == 0 ? (it.shared ? &maps.s1_3 : &maps.a1_3) : t0_3;
                const int rows = it.shared ? p.rows_s : p.rows;
                const int ybase = it.shared ? 0 : it.seg * rows;
                const int y0 = ybase + it.rb * rows_item;
                const int y1 = MODE == 0 ? y0 : y0 + 128;
                uint8_t *dst = ring + s * kStageBytes;
                // routed weights: read by one group of positions (rarely
                // two), evict first; the shared expert's: every group
                const uint64_t pol = it.shared ? keep : stream;
                if (2 * ks + 1 < nfull) {
                    tma_load_3d_hint(dst, t0_3, &S->smem_full[s], 0, y0, 2 * ks, pol);
                    tma_load_3d_hint(dst + kTileBytes, t1_3, &S->smem_full[s], 0, y1, 2 * ks, pol);
                } else {
                    for (int sub = 0; sub < 2; ++sub) {
                        tma_load_2d_hint(dst + sub * kSubBytes, t0, &S->smem_full[s], (2 * ks + sub) * 64, y0,
                                         pol);
                        tma_load_2d_hint(dst + kTileBytes + sub * kSubBytes, t1, &S->smem_full[s],
                                         (2 * ks + sub) * 64, y1, pol);
                    }
                }
            };
            auto issue_limbs = [&](const Item &it, int ks, uint32_t s) {
                tma_load_4d(ring + s * kStageBytes + 2 * kTileBytes, &maps.b3, &S->smem_full[s], 0, 0,
                            it.pos0 * 3, 2 * ks);
            };
            // the first kNS stages' weights go out before the wait on the
            // preceding kernel, their limb rows after it
            Item pend_it[kNS];
            int pend_ks[kNS];
            uint32_t us = 0;
            bool ok = true, waited = false;
            auto wait_then_limbs = [&]() {
                QMOE_PDL_WAIT();
                QMOE_PDL_TRIGGER();
                waited = true;
                if (p.quant_in) {
                    // the limb rows come from every CTA's limb phase
                    if (!grid_wait(p.sched + 2, (int)gridDim.x, abort, p.err)) {
                        ok = false;
                        return;
                    }
                    fence_proxy_async_global();
                }
                for (uint32_t u = 0; u < us && u < kNS; ++u) issue_limbs(pend_it[u], pend_ks[u], u);
            };
            // the next item's number is taken once its first stage has a free
            // slot, so a CTA holds at most the ring's stages of work ahead
            for (int i = 0; ok; ++i) {
                const uint32_t s0 = us % kNS;
                if (us >= kNS) {
                    if (!waited) wait_then_limbs();
                    if (!ok || !(ok = mbar_wait(&S->smem_empty[s0], ((us / kNS) & 1) ^ 1, abort, p.err))) break;
                }
                const int num = i == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(p.sched, 1);
                if (num >= total) {
                    S->queue[i % kQueue] = make_int4(-1, 0, 0, 0);
                    mbar_arrive(&S->smem_full[s0]);
                    break;
                }
                const Item it = decode_item(p, total - 1 - num, nr, rb_r, rb_s);
                S->queue[i % kQueue] = pack_item(it);
                const int nks = ((it.shared ? p.K_s : p.K) + kStageCodes - 1) / kStageCodes;
                for (int ks = 0; ks < nks; ++ks, ++us) {
                    const uint32_t s = us % kNS;
                    if (ks > 0 && us >= kNS) {
                        if (!waited) wait_then_limbs();
                        if (!ok || !(ok = mbar_wait(&S->smem_empty[s], ((us / kNS) & 1) ^ 1, abort, p.err)))
                            break;
                    }
                    mbar_arrive_expect_tx(&S->smem_full[s], kStageBytes);
                    issue_weights(it, ks, s);
                    if (waited) {
                        issue_limbs(it, ks, s);
                    } else {
                        pend_it[s] = it;
                        pend_ks[s] = ks;
                    }
                }
            }
            if (!waited) wait_then_limbs();
            if (!ok)
                for (uint32_t u = us > kNS ? us - kNS : 0; u < us; ++u)
                    for (uint32_t n = 0; n < kMaxWaitProbes; ++n)
                        if (mbar_try_wait(&S->smem_full[u % kNS], (u / kNS) & 1)) break;
        }
    } else if (warp <= kCompute) {
        // --------------------------------------------------------- compute
        // Two groups of four warps take the two 256-code chunks of a stage;
        // a warp owns rows 32 wq .. 32 wq + 31 of both weight tiles (four
        // 16-row blocks), so every limb fragment it loads feeds 8 or 16 IMMAs.
        const int cw = warp - 1;                    // 0..7
        const int grp = cw >> 2;                    // chunk of each stage
        const int wq = cw & 3;
        const int g8 = lane >> 2, t4 = lane & 3;
        uint32_t us = 0;
        bool ok = true;
        for (int i = 0; ok; ++i) {
            // the item's first stage, or the end mark, completes the next
            // full barrier
            if (!(ok = mbar_wait_warp(&S->smem_full[us % kNS], (us / kNS) & 1, abort, p.err))) break;
            const int4 qv = S->queue[i % kQueue];
            const uint32_t tb = i & 1;
            if (qv.x < 0) {
                if (!(ok = mbar_wait_warp(&S->tile_empty[tb], ((i >> 1) & 1) ^ 1, abort, p.err))) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&S->tile_full[tb]);
                break;
            }
            const Item it = unpack_item(qv);
            const int K = it.shared ? p.K_s : p.K;
            const int nks = (K + kStageCodes - 1) / kStageCodes;
            // limb columns in use: 3 per position; <= 2 positions fit one n8 tile
            const bool two = it.count > 2;
            int acc[8][4];
#pragma unroll
            for (int rg = 0; rg < 8; ++rg)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[rg][j] = 0;

            const int nsub_all = (K + 255) / 256;        // 256-code chunks holding codes < K
            for (int ks = 0; ks < nks; ++ks, ++us) {
                const uint32_t s = us % kNS;
                if (ks > 0 && !(ok = mbar_wait_warp(&S->smem_full[s], (us / kNS) & 1, abort, p.err))) break;
                const bool live = 2 * ks + grp < nsub_all;
                const uint8_t *stage = ring + s * kStageBytes;
                if (live) {
                    if (two)
                        stage_mma<2>(stage, grp, wq, g8, t4, acc, &S->smem_empty[s], lane);
                    else
                        stage_mma<1>(stage, grp, wq, g8, t4, acc, &S->smem_empty[s], lane);
                } else {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S->smem_empty[s]);
                }
            }
            if (!ok) break;

            // accumulators -> this group's tile [15 limb rows][256 cols]:
            // acc[b] (+ acc[4 + b], limb rows 8..15) holds rows g8 / g8 + 8 of
            // 16-row block b, limb columns 2 t4, 2 t4 + 1
            if (!(ok = mbar_wait_warp(&S->tile_empty[tb], ((i >> 1) & 1) ^ 1, abort, p.err))) break;
            int *ct = acc_tile + (tb * 2 + grp) * (kAccBytes / 4);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int col = (b >> 1) * 128 + wq * 32 + (b & 1) * 16 + g8;
                int *c0 = ct + (2 * t4) * kTileStride + col;
                c0[0] = acc[b][0];
                c0[kTileStride] = acc[b][1];
                c0[8] = acc[b][2];
                c0[kTileStride + 8] = acc[b][3];
                if (two) {
                    int *c1 = c0 + 8 * kTileStride;
                    c1[0] = acc[4 + b][0];
                    c1[8] = acc[4 + b][2];
                    if (2 * t4 + 9 < kLimbRows) {
                        c1[kTileStride] = acc[4 + b][1];
                        c1[kTileStride + 8] = acc[4 + b][3];
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S->tile_full[tb]);
        }
    } else {
        // -------------------------------------------------------- epilogue
        const int r = (warp - kEpiWarp0) * 32 + lane;   // 0..127
        bool ok = true;
        for (int i = 0; ok; ++i) {
            const uint32_t tb = i & 1;
            if (!(ok = mbar_wait_warp(&S->tile_full[tb], (i >> 1) & 1, abort, p.err))) break;
            const int4 qv = S->queue[i % kQueue];
            if (qv.x < 0) break;
            const Item it = unpack_item(qv);
            const int rows = it.shared ? p.rows_s : p.rows;
            const float *sc0 = it.shared ? p.ss[0] : p.s[0] + (int64_t)it.seg * p.s_stride;
            const float *sc1 = MODE == 0 ? (it.shared ? p.ss[1] : p.s[1] + (int64_t)it.seg * p.s_stride)
                                         : sc0;
            const int row0 = it.rb * rows_item + r;
            const int row1 = MODE == 0 ? row0 : row0 + 128;
            const float s0 = row0 < rows ? __ldg(sc0 + row0) : 0.0f;
            const float s1 = row1 < rows ? __ldg(sc1 + row1) : 0.0f;
            longlong2 mt[kTokMax];
#pragma unroll
            for (int c = 0; c < kTokMax; ++c)
                mt[c] = c < it.count ? __ldcg(p.meta + it.pos0 + c) : make_longlong2(0, 0);

            const int *ct0 = acc_tile + (tb * 2) * (kAccBytes / 4);   // group 0 + group 1
            const int *ct1 = ct0 + kAccBytes / 4;
            int v0[kLimbRows], v1[kLimbRows];
#pragma unroll
            for (int n = 0; n < kLimbRows; ++n) {
                // the IMMAs saw 64 x code: exact multiples of 64
                v0[n] = (ct0[n * kTileStride + r] + ct1[n * kTileStride + r]) >> 6;
                v1[n] = (ct0[n * kTileStride + 128 + r] + ct1[n * kTileStride + 128 + r]) >> 6;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S->tile_empty[tb]);
#pragma unroll
            for (int c = 0; c < kTokMax; ++c) {
                if (c >= it.count) break;
                const int64_t pos = it.pos0 + c;
                const double s2 = (double)pow2i((int)mt[c].x);
                // limb rows of position c are 3c + l
                const long long a0 = (long long)v0[3 * c + 2] * 65536LL +
                                     (long long)v0[3 * c + 1] * 256LL + (long long)v0[3 * c] - mt[c].y;
                const long long a1 = (long long)v1[3 * c + 2] * 65536LL +
                                     (long long)v1[3 * c + 1] * 256LL + (long long)v1[3 * c] - mt[c].y;
                const float f0 = __fmul_rn((float)((double)a0 * s2), s0);
                const float f1 = __fmul_rn((float)((double)a1 * s2), s1);
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
    __syncthreads();
    if (MODE == 1 && p.combine) {
        // combine phase: every CTA's y rows are stored before it counts in
        // (the barrier above orders them before thread 0's fence, which
        // makes them visible device-wide before its count: one fence per
        // CTA, not one per warp); tasks are (token, 1024 columns), the
        // ranking of a task's rows done before the wait
        if (tid == 0) {
            __threadfence();
            atomicAdd(p.sched + 2, 1);
        }
        const int H4 = p.c.H >> 2;
        const int nch = (H4 + 255) / 256;
        const int64_t ntask = p.c.T * nch;
        bool first = true;
        for (int64_t task = blockIdx.x; task < ntask; task += gridDim.x) {
            const int64_t t = task / nch;
            const int ch = (int)(task - t * nch);
            if (warp == 0) {
                const int n = combine_rank(p.c, t, lane, S->c_pos, S->c_w);
                if (lane == 0) S->c_n = n;
                if (first && lane == 0)
                    S->grid_ok = grid_wait(p.sched + 2, (p.quant_in ? 2 : 1) * (int)gridDim.x, abort, p.err);
            }
            first = false;
            __syncthreads();
            if (!S->grid_ok) break;
            // expert parallel: a received row's partial sum goes straight to
            // its origin rank's return block
            void *orow = nullptr;
            int dst = -1;
            if (p.ep_ret && t < (int64_t)p.ret.world * p.ret.C) {
                dst = (int)(t / p.ret.C);
                const int64_t i = t - (int64_t)dst * p.ret.C;
                orow = p.ret.base[dst] + p.ret.off_back + ((int64_t)p.ret.rank * p.ret.C + i) * p.ret.H * p.ret.esize;
            }
            const int c4 = ch * 256 + tid;
            // a received row without live slots is never read by its origin:
            // not sent
            if (tid < 256 && c4 < H4 && (dst < 0 || S->c_n > 0))
                combine_float4(p.c, t, 4 * c4, S->c_n, S->c_pos, S->c_w, orow);
            __syncthreads();
        }
        // every CTA counts in once, after all of its stores into peer memory
        if (p.ep_ret && tid == 0) ep_signal_all(p.ret, 1, (int)gridDim.x);
    }
    // the last CTA out resets the grid's counters for the next launch
    // (every CTA's last counter use precedes its exit count)
    if (tid == 0 && atomicAdd(p.sched + 1, 1) == (int)gridDim.x - 1) {
        p.sched[0] = 0;
        p.sched[1] = 0;
        p.sched[2] = 0;
    }
}

}  // namespace

size_t qgemv_imma_smem_bytes(int kp_b, int b_buffers) {
    (void)kp_b;
    (void)b_buffers;
    return 1024 + (size_t)kNS * kStageBytes + 4 * (size_t)kAccBytes + sizeof(Smem);
}

int qgemv_imma_buffers(int kp_b) {
    (void)kp_b;
    return 0;
}

cudaError_t launch_qgemv_imma(int mode, const DecodeMaps &maps, const DecodeParams &p, int grid,
                              cudaStream_t s) {
    const size_t smem = qgemv_imma_smem_bytes(p.kp_b, p.b_buffers);
    cudaError_t e = mode == 0 ? ensure_dyn_smem(reinterpret_cast<const void *>(qgemv_imma_kernel<0>), smem)
                              : ensure_dyn_smem(reinterpret_cast<const void *>(qgemv_imma_kernel<1>), smem);
    if (e != cudaSuccess) return e;
    const bool coop = p.quant_in || p.combine;
    return mode == 0 ? launch_pdl_coop(qgemv_imma_kernel<0>, dim3(grid), dim3(kThreads), smem, s, coop, maps, p)
                     : launch_pdl_coop(qgemv_imma_kernel<1>, dim3(grid), dim3(kThreads), smem, s, coop, maps, p);
}

}  // namespace qmoe
