// ep_p2p.cu -- the expert-parallel exchanges as kernels over peer memory.
//
// qmoe-rs runs every expert in one process (src/moe.rs:40-130); split over
// G GPUs, each forward moves every token's row to the ranks that own its
// experts and each rank's partial sums back (the dispatch and combine of
// expert parallelism).  Here each rank owns one device allocation (receive
// rows, their metadata, returned partial rows, arrival flags) that the other
// ranks map through CUDA IPC, and the copies are plain stores into the
// peers' memory over NVLink from the kernels that read the data -- no
// collective library, no staging buffer, no TMA on peer memory.
//
// Ordering: the CTAs of a copy kernel stride over the rows (any destination);
// each fences its stores system-wide once, and the last CTA raises every
// peer's flag for (phase, this rank) (ep_signal.cuh).  A waiting rank polls
// its own flags with acquire loads until each peer's reaches the forward's
// sequence number (bounded; on time-out it raises the device error word);
// rows a rank sends to itself are ordered by its stream.  The sequence number lives on the device (read by every kernel of
// a forward, advanced by the last wait), so a whole forward can be replayed
// from a CUDA graph.  Rank d's receive buffer is
// rewritten only in the next forward, after d has returned its partial sums
// of this one (which it computes after reading the rows), so one flag per
// phase suffices.
#include "common.cuh"
#include "ep_signal.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace qmoe {
namespace {

using sm100::kErrWaitTimeout;
using sm100::kMaxWaitProbes;

constexpr int kCopyThreads = 256;

QMOE_DEV int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

QMOE_DEV int *flag_at(const EpPeerDev &d, int owner, int phase, int from) { return ep_flag(d, owner, phase, from); }

// Copies one row of `bytes` (a multiple of 16) with the CTA, four 16-byte
// loads in flight per thread before their stores.
QMOE_DEV void copy_row(uint8_t *dst, const uint8_t *src, int64_t bytes) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src);
    uint4 *o = reinterpret_cast<uint4 *>(dst);
    const int64_t n = bytes / 16;
    for (int64_t i0 = threadIdx.x; i0 < n; i0 += 4 * kCopyThreads) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i0 + u * kCopyThreads < n) v[u] = __ldg(s + i0 + u * kCopyThreads);
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i0 + u * kCopyThreads < n) o[i0 + u * kCopyThreads] = v[u];
    }
}

// After all of this CTA's stores: count it towards the phase's signal.
QMOE_DEV void arrive(const EpPeerDev &d, int phase) {
    __syncthreads();
    if (threadIdx.x == 0) ep_signal_all(d, phase, (int)gridDim.x);
}

// Row j < world*C: send row j (destination j / C, row j % C) if it is in use,
// and its metadata row; row world*C + t: this rank's own token t for the
// shared expert (metadata: no routed expert).  CTAs stride over the rows.
__global__ void __launch_bounds__(kCopyThreads)
ep_dispatch_kernel(const EpPeerDev d, const void *x, int64_t T, const int32_t *send_counts,
                   const int32_t *send_tok, const int32_t *send_meta) {
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int64_t GC = (int64_t)d.world * d.C;
    const int64_t rb = d.H * d.esize, mb = 2 * (int64_t)d.K * 4;
    const uint8_t *xs = static_cast<const uint8_t *>(x);
    for (int64_t j = blockIdx.x; j < GC + T; j += gridDim.x) {
        if (j < GC) {
            const int dst = (int)(j / d.C);
            const int64_t i = j - (int64_t)dst * d.C;
            const int64_t r = (int64_t)d.rank * d.C + i;           // row in the destination's block
            if (i < send_counts[dst]) copy_row(d.base[dst] + d.off_rows + r * rb, xs + send_tok[j] * rb, rb);
            int32_t *m = reinterpret_cast<int32_t *>(d.base[dst] + d.off_meta + r * mb);
            for (int k = threadIdx.x; k < 2 * d.K; k += kCopyThreads) m[k] = send_meta[j * 2 * d.K + k];
        } else {
            const int64_t t = j - GC, r = GC + t;
            copy_row(d.base[d.rank] + d.off_rows + r * rb, xs + t * rb, rb);
            int32_t *m = reinterpret_cast<int32_t *>(d.base[d.rank] + d.off_meta + r * mb);
            for (int k = threadIdx.x; k < 2 * d.K; k += kCopyThreads) m[k] = k < d.K ? -1 : 0;
        }
    }
    arrive(d, 0);
}

// Row j < world*C: the partial row j (rows received from rank j / C) goes to
// that rank's return block, unless no slot of the row was routed here (its
// metadata ids all -1: the origin never reads it).  CTAs stride over the
// rows.
__global__ void __launch_bounds__(kCopyThreads)
ep_return_kernel(const EpPeerDev d, const void *y) {
    __shared__ int s_live;
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int64_t rb = d.H * d.esize;
    for (int64_t j = blockIdx.x; j < (int64_t)d.world * d.C; j += gridDim.x) {
        const int dst = (int)(j / d.C);
        const int64_t i = j - (int64_t)dst * d.C;
        if (threadIdx.x < 32) {
            const int32_t *m = reinterpret_cast<const int32_t *>(d.base[d.rank] + d.off_meta) + j * 2 * d.K;
            const bool live = threadIdx.x < d.K && __ldcg(m + threadIdx.x) >= 0;
            const bool any = __any_sync(0xffffffffu, live) || d.K > 32;
            if (threadIdx.x == 0) s_live = any;
        }
        __syncthreads();
        if (s_live)
            copy_row(d.base[dst] + d.off_back + ((int64_t)d.rank * d.C + i) * rb,
                     static_cast<const uint8_t *>(y) + j * rb, rb);
        __syncthreads();                           // s_live is rewritten next row
    }
    arrive(d, 1);
}

// Lane p waits until rank p's C rows of `phase` of this forward have
// arrived; the return phase ends the forward and advances the sequence
// number.
__global__ void __launch_bounds__(32)
ep_wait_kernel(const EpPeerDev d, int phase) {
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int s = *d.seq + 1;
    const uint32_t want = (uint32_t)s;           // forwards whose phase arrived
    bool ok = true;
    for (int p = threadIdx.x; p < d.world; p += 32) {
        if (p == d.rank) continue;
        const int *f = flag_at(d, d.rank, phase, p);
        uint32_t n = 0;
        while (!arrived(ld_acquire_sys(f), want)) {
            if (++n >= kMaxWaitProbes) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!ok) atomicOr(d.err, kErrWaitTimeout);
    __syncwarp();
    if (phase == 1 && threadIdx.x == 0) *d.seq = s;
}

// CTA (token t, slice of 256 x 4 columns): lanes of warp 0 wait for every
// peer's returned rows of this forward (bounded), then the combine_rows sum
// (ep.cu) of t's returned partials and its shared row, read through L2.
__global__ void __launch_bounds__(256)
ep_finish_kernel(const EpPeerDev d, const int32_t *slot_pos, int64_t T, const void *extra, void *out) {
    __shared__ int s_ok;
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int seq = *d.seq + 1;
    if (threadIdx.x < 32) {
        const uint32_t want = (uint32_t)seq;
        bool ok = true;
        for (int p = threadIdx.x; p < d.world; p += 32) {
            if (p == d.rank) continue;
            const int *f = flag_at(d, d.rank, 1, p);
            uint32_t n = 0;
            while (!arrived(ld_acquire_sys(f), want)) {
                if (++n >= kMaxWaitProbes) {
                    ok = false;
                    break;
                }
                __nanosleep(64);
            }
        }
        ok = __all_sync(0xffffffffu, ok);
        if (threadIdx.x == 0) {
            if (!ok) atomicOr(d.err, kErrWaitTimeout);
            s_ok = ok;
        }
    }
    __syncthreads();
    const int dtype = d.esize == 2 ? 1 : 0;
    const int64_t t = blockIdx.x, h = ((int64_t)blockIdx.y * 256 + threadIdx.x) * 4;
    if (s_ok && h < d.H) {
        const uint8_t *rows = d.base[d.rank] + d.off_back;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < d.world; ++r) {
            const int pos = slot_pos[t * d.world + r];
            if (pos < 0) continue;
            const float4 v = load_act4_cg(rows, dtype, (int64_t)pos * d.H + h);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        if (extra) {
            const float4 v = load_act4_cg(extra, dtype, t * d.H + h);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        store_act4(out, dtype, t * d.H + h, acc);
    }
    // the last CTA out ends the forward (every CTA read seq above)
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(d.done, 1) == (int)(gridDim.x * gridDim.y) - 1) {
        *d.done = 0;
        *d.seq = seq;
    }
}

}  // namespace

cudaError_t launch_ep_finish(const EpPeerDev &d, const int32_t *slot_pos, int64_t T, const void *extra,
                             void *out, cudaStream_t s) {
    const dim3 grid((unsigned)T, (unsigned)((d.H / 4 + 255) / 256));
    return launch_pdl(ep_finish_kernel, grid, dim3(256), 0, s, d, slot_pos, T, extra, out);
}

cudaError_t launch_ep_dispatch(const EpPeerDev &d, const void *x, int64_t T, const int32_t *send_counts,
                               const int32_t *send_tok, const int32_t *send_meta, cudaStream_t s) {
    const int64_t rows = (int64_t)d.world * d.C + T;
    const int grid = (int)std::min<int64_t>(rows, (int64_t)device_sm_count() * kEpCopyCtasPerSm);
    return launch_pdl(ep_dispatch_kernel, dim3((unsigned)std::max(grid, 1)), dim3(kCopyThreads), 0, s, d, x, T,
                      send_counts, send_tok, send_meta);
}

cudaError_t launch_ep_return(const EpPeerDev &d, const void *y, cudaStream_t s) {
    const int64_t rows = (int64_t)d.world * d.C;
    const int grid = (int)std::min<int64_t>(rows, (int64_t)device_sm_count() * kEpCopyCtasPerSm);
    return launch_pdl(ep_return_kernel, dim3((unsigned)std::max(grid, 1)), dim3(kCopyThreads), 0, s, d, y);
}

cudaError_t launch_ep_wait(const EpPeerDev &d, int phase, cudaStream_t s) {
    return launch_pdl(ep_wait_kernel, dim3(1), dim3(32), 0, s, d, phase);
}

}  // namespace qmoe
