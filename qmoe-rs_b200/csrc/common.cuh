// common.cuh -- device helpers shared by the qmoe_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

#define QMOE_DEV __device__ __forceinline__

// Programmatic dependent launch.  QMOE_PDL_WAIT blocks until the preceding
// kernel in the stream has completed and its writes are visible (a no-op
// when the launch carries no programmatic dependency); every read of a
// predecessor's output and every global write comes after it.
// QMOE_PDL_TRIGGER lets the next kernel in the stream begin launching while
// this one runs.
#define QMOE_PDL_WAIT() asm volatile("griddepcontrol.wait;" ::: "memory")
#define QMOE_PDL_TRIGGER() asm volatile("griddepcontrol.launch_dependents;" ::: "memory")

namespace qmoe {

constexpr int kGateChunk = 64;  // hidden-dim chunk of the pinned logit order

QMOE_DEV float to_f32(float v) { return v; }
QMOE_DEV float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

// Load element k of row `row` of an activation matrix stored as f32 or bf16.
QMOE_DEV float load_act(const void *base, int dtype, int64_t idx) {
    if (dtype == 0) return __ldg(reinterpret_cast<const float *>(base) + idx);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(base)[idx]);
}

// Four consecutive activations (f32 or bf16) starting at a multiple of 4.
QMOE_DEV float4 load_act4(const void *base, int dtype, int64_t idx) {
    if (dtype == 0) return __ldg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(base) + idx));
    const uint2 u = __ldg(reinterpret_cast<const uint2 *>(reinterpret_cast<const __nv_bfloat16 *>(base) + idx));
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

// System-scope acquire load (a flag another GPU sets after its stores).
QMOE_DEV int ld_acquire_sys_i32(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Arrival counters grow by a fixed amount per forward and wrap modulo 2^32
// over a long run; `count` has reached `want` when the wrapped difference is
// not negative (valid while the two are less than 2^31 apart).
QMOE_DEV bool arrived(int count, uint32_t want) { return (int32_t)((uint32_t)count - want) >= 0; }

// Group g of a segment of c positions cut into ceil(c / chunk) groups of
// near-equal size (each at most chunk): (first position, count).  Even
// groups keep the GEMMs' tiles full (300 rows as 150 + 150, not 256 + 44).
QMOE_DEV int2 split_group(int64_t c, int chunk, int g) {
    const int64_t ng = (c + chunk - 1) / chunk;
    const int64_t sz = (c + ng - 1) / ng;
    const int64_t b = (int64_t)g * sz;
    return make_int2((int)b, (int)(c - b < sz ? c - b : sz));
}

// load_act4 through L2 only, for rows other CTAs or other GPUs wrote after
// this kernel started (the read-only path of __ldg is not coherent with them).
QMOE_DEV float4 load_act4_cg(const void *base, int dtype, int64_t idx) {
    if (dtype == 0) return __ldcg(reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(base) + idx));
    const uint2 u = __ldcg(reinterpret_cast<const uint2 *>(reinterpret_cast<const __nv_bfloat16 *>(base) + idx));
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

QMOE_DEV void store_act4(void *base, int dtype, int64_t idx, float4 v) {
    if (dtype == 0) {
        *reinterpret_cast<float4 *>(reinterpret_cast<float *>(base) + idx) = v;
        return;
    }
    const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t *>(&lo);
    u.y = *reinterpret_cast<const uint32_t *>(&hi);
    *reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(base) + idx) = u;
}

QMOE_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

QMOE_DEV int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Stable-descending-sort precedence: a ranks before b when its value is
// larger, ties going to the lower index (qmoe-rs src/moe.rs:68-71 sorts an
// index-ordered list with a stable sort).
QMOE_DEV bool ranks_before(float va, int ia, float vb, int ib) {
    return va > vb || (va == vb && ia < ib);
}

// Exact power of two 2^n for -149 <= n <= 127.
QMOE_DEV float pow2i(int n) {
    uint32_t u = n >= -126 ? (uint32_t)(n + 127) << 23 : 1u << (n + 149);
    return __uint_as_float(u);
}

// Deterministic exp for sigmoid scoring: Cody & Waite reduction with a
// two-float ln2, degree-7 Taylor polynomial in Horner form, scaling by 2^n.
// Every step is one correctly rounded IEEE operation, so the CPU oracle's
// C version of the same steps returns the same bits.
QMOE_DEV float qexp(float x) {
    if (!(x == x)) return x;
    if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
    if (x < -103.97208404541016f) return 0.0f;
    float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
    float r = __fmaf_rn(n, -0.693145751953125f, x);
    r = __fmaf_rn(n, -1.428606765330187045037746429443359375e-06f, r);
    float p = 1.98412698412698412698e-4f;
    p = __fmaf_rn(p, r, 1.38888888888888888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333333333333333e-3f);
    p = __fmaf_rn(p, r, 4.16666666666666666667e-2f);
    p = __fmaf_rn(p, r, 1.66666666666666666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) return __fmul_rn(__fmul_rn(p, pow2i(127)), pow2i(ni - 127));
    if (ni < -126) return __fmul_rn(__fmul_rn(p, pow2i(-126)), pow2i(ni + 126));
    return __fmul_rn(p, pow2i(ni));
}

QMOE_DEV float qsigmoid(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, qexp(-x)));
}

// SwiGLU exactly as qmoe-rs writes it (src/moe.rs:109-115):
// (g * (1 / (1 + exp(-g)))) * u, each operation rounded separately.
QMOE_DEV float swiglu(float g, float u) {
    float s = __fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
    return __fmul_rn(s, u);
}

}  // namespace qmoe

namespace qmoe {
// Host: launch with the programmatic-stream-serialization attribute, so the
// kernel may start while its predecessor finishes (it waits in QMOE_PDL_WAIT).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl, optionally as a cooperative launch (every CTA co-resident, so
// the kernel may hold grid-wide barriers).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_coop(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                   cudaStream_t s, bool cooperative, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cooperative ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
}  // namespace qmoe
