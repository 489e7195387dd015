// quant.cu -- the limb kernel: every position's fixed-point limbs (format and
// arithmetic in quant.cuh), two positions per CTA.  The decode GEMVs do the
// same work in their first phase when they are launched cooperatively; this
// kernel serves the other callers.
#include "quant.cuh"

namespace qmoe {
namespace {

constexpr int kQuantThreads = 2 * kQuantGroup;     // two positions per CTA: one wave
                                                   // beside a resident GEMV CTA

template <int BPT>
__global__ void __launch_bounds__(kQuantThreads)
quant_kernel(const QuantParams p) {
    QMOE_PDL_WAIT();
    QMOE_PDL_TRIGGER();
    __shared__ float s_red[8];
    __shared__ long long s_sum[8];
    const int half = threadIdx.x / kQuantGroup, ht = threadIdx.x % kQuantGroup;
    const int64_t pos = (int64_t)blockIdx.x * 2 + half;
    quant_position<BPT>(p, pos, ht, s_red + 4 * half, s_sum + 4 * half, [] { __syncthreads(); });
}

}  // namespace

cudaError_t launch_quant(const QuantParams &p, cudaStream_t s) {
    if (p.npos == 0) return cudaSuccess;
    const int bpt = quant_bpt(p.K > p.K_s ? p.K : p.K_s);
    const dim3 grid((unsigned)((p.npos + 1) / 2)), block(kQuantThreads);
    if (bpt == 1) return launch_pdl(quant_kernel<1>, grid, block, 0, s, p);
    if (bpt == 2) return launch_pdl(quant_kernel<2>, grid, block, 0, s, p);
    if (bpt == 4) return launch_pdl(quant_kernel<4>, grid, block, 0, s, p);
    return launch_pdl(quant_kernel<0>, grid, block, 0, s, p);
}

}  // namespace qmoe
