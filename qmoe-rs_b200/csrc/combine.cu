// combine.cu -- the combine kernels (arithmetic and order in combine.cuh).
// Local: one CTA per (token, slice of kCombThreads * kCombVec float4
// columns).  Expert parallel (received rows summed and sent back to their
// origin ranks): CTAs stride over whole rows and fence their peer stores
// once at the end.  Warp 0 puts a row's live slots in ascending expert order
// in shared memory; then every thread issues the loads of up to eight rows
// before their in-order sum.  The cooperative down GEMV does the same work as
// its last phase; these kernels serve the other callers.
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
    for (int v = 0; v < vec; ++v) {
        const int c4 = (blockIdx.y * vec + v) * kCombThreads + threadIdx.x;
        if (c4 >= H4) break;
        combine_float4(p, t, 4 * c4, n, s_pos, s_w);
    }
}

// Expert parallel: row t < world*C (received from rank t / C) goes to that
// rank's return block, unless none of its slots was routed here (its origin
// never reads it); later rows (this rank's own tokens) stay local.
__global__ void __launch_bounds__(kCombThreads)
combine_return_kernel(const CombineParams p) {
    __shared__ int s_pos[kCombineMaxK];
    __shared__ float s_w[kCombineMaxK];
    __shared__ int s_n;
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    const int H4 = p.H >> 2;
    const int64_t GC = (int64_t)p.ret.world * p.ret.C;
    for (int64_t t = blockIdx.x; t < p.T; t += gridDim.x) {
        if (threadIdx.x < 32) {
            const int n = combine_rank(p, t, threadIdx.x, s_pos, s_w);
            if (threadIdx.x == 0) s_n = n;
        }
        __syncthreads();
        const int n = s_n;
        void *orow = nullptr;
        bool send = true;
        if (t < GC) {
            const int dst = (int)(t / p.ret.C);
            const int64_t i = t - (int64_t)dst * p.ret.C;
            orow = p.ret.base[dst] + p.ret.off_back + ((int64_t)p.ret.rank * p.ret.C + i) * p.ret.H * p.ret.esize;
            send = n > 0;
        }
        if (send)
            for (int c4 = threadIdx.x; c4 < H4; c4 += kCombThreads) combine_float4(p, t, 4 * c4, n, s_pos, s_w, orow);
        __syncthreads();                           // s_pos / s_w / s_n are rewritten next row
    }
    if (threadIdx.x == 0) ep_signal_all(p.ret, 1, (int)gridDim.x);
}

}  // namespace

cudaError_t launch_combine(const CombineParams &p, cudaStream_t s) {
    if (p.T == 0 || p.H == 0) return cudaSuccess;
    if (p.K > kCombineMaxK) return cudaErrorInvalidValue;
    if (p.ep_ret) {
        const int grid = (int)std::min<int64_t>(p.T, (int64_t)device_sm_count() * kEpCopyCtasPerSm);
        return launch_pdl(combine_return_kernel, dim3((unsigned)grid), dim3(kCombThreads), 0, s, p);
    }
    const int per_cta = kCombThreads * kCombVec;
    const dim3 grid((unsigned)p.T, (unsigned)((p.H / 4 + per_cta - 1) / per_cta));
    return launch_pdl(combine_kernel, grid, dim3(kCombThreads), 0, s, p, kCombVec);
}

}  // namespace qmoe
