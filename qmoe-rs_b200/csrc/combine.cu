// combine.cu -- the combine kernel (arithmetic and order in combine.cuh): one
// CTA per (token, slice of kCombThreads * kCombVec float4 columns).  Warp 0
// puts the token's live slots in ascending expert order in shared memory;
// then every thread issues the loads of up to eight rows before their
// in-order sum.  The cooperative down GEMV does the same work as its last
// phase; this kernel serves the other callers.
#include "combine.cuh"
#include "ep_signal.cuh"

namespace qmoe {
namespace {

constexpr int kCombThreads = 256;
constexpr int kCombVec = 4;        // float4 columns per thread

__global__ void __launch_bounds__(kCombThreads)
combine_kernel(const CombineParams p, int vec) {
    __shared__ int s_pos[kCombineMaxK];
    __shared__ float s_w[kCombineMaxK];
    __shared__ int s_n;
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int64_t t = blockIdx.x;
    if (threadIdx.x < 32) {
        const int n = combine_rank(p, t, threadIdx.x, s_pos, s_w);
        if (threadIdx.x == 0) s_n = n;
    }
    __syncthreads();
    const int n = s_n;
    const int H4 = p.H >> 2;
    // expert parallel: a received row's partial sum goes to its origin
    // rank's return block; a row without live slots is not sent at all (its
    // origin never reads it), but still counted
    void *orow = nullptr;
    int dst = -1;
    if (p.ep_ret && t < (int64_t)p.ret.world * p.ret.C) {
        dst = (int)(t / p.ret.C);
        const int64_t i = t - (int64_t)dst * p.ret.C;
        orow = p.ret.base[dst] + p.ret.off_back + ((int64_t)p.ret.rank * p.ret.C + i) * p.ret.H * p.ret.esize;
    }
    if (dst < 0 || n > 0)
        for (int v = 0; v < vec; ++v) {
            const int c4 = (blockIdx.y * vec + v) * kCombThreads + threadIdx.x;
            if (c4 >= H4) break;
            combine_float4(p, t, 4 * c4, n, s_pos, s_w, orow);
        }
    if (dst >= 0 && dst != p.ret.rank) {
        __syncthreads();
        if (threadIdx.x == 0) ep_signal(p.ret, dst, 1, (int)(p.ret.C * gridDim.y));
    }
}

}  // namespace

cudaError_t launch_combine(const CombineParams &p, cudaStream_t s) {
    if (p.T == 0 || p.H == 0) return cudaSuccess;
    if (p.K > kCombineMaxK) return cudaErrorInvalidValue;
    // expert parallel: slices of 1024 columns (more CTAs in flight for the
    // NVLink stores)
    const int vec = p.ep_ret ? 1 : kCombVec;
    const int per_cta = kCombThreads * vec;
    const dim3 grid((unsigned)p.T, (unsigned)((p.H / 4 + per_cta - 1) / per_cta));
    return launch_pdl(combine_kernel, grid, dim3(kCombThreads), 0, s, p, vec);
}

}  // namespace qmoe
