// sm100.cuh -- thin wrappers over the sm_100a PTX the tensor-core kernels use:
// mbarriers, TMA tensor loads, TMEM allocation, tcgen05 MMA / commit / ld / st.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace qmoe {
namespace sm100 {

// Device-side failure flag: set by a kernel whose bounded wait ran out; the
// host reads it back (qmoe_ctx_synchronize and every host-pointer call).
constexpr int kErrWaitTimeout = 1;
constexpr int kErrBadGroup = 2;      // a work item larger than the kernel was configured for

// One bounded wait = this many failed try_wait probes (each try_wait itself
// suspends for up to a hardware-chosen time), on the order of a second.
constexpr uint32_t kMaxWaitProbes = 1u << 22;

QMOE_DEV uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ----------------------------------------------------------
QMOE_DEV void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

QMOE_DEV void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

QMOE_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

QMOE_DEV void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
            smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

QMOE_DEV bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase of `parity`.  Returns false when it gives up or
// when another role already gave up (*abort set); on a time-out it raises
// *abort and the global error flag.
QMOE_DEV bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    for (uint32_t n = 0; n < kMaxWaitProbes; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
    }
    *abort = 1;
    atomicOr(err, kErrWaitTimeout);
    return false;
}

// Warp-uniform bounded wait: every lane probes (so every lane acquires the
// phase) and the warp decides together, so .sync.aligned instructions after
// it run converged and a time-out never splits the warp.
QMOE_DEV bool mbar_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort, int *err) {
    for (uint32_t n = 0; n < kMaxWaitProbes; ++n) {
        const bool done = mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, done)) return true;
        if (__any_sync(0xffffffffu, *abort != 0)) return false;
    }
    if ((threadIdx.x & 31) == 0) {
        *abort = 1;
        atomicOr(err, kErrWaitTimeout);
    }
    __syncwarp();
    return false;
}

// ---- TMA ----------------------------------------------------------------
QMOE_DEV void tma_prefetch_desc(const CUtensorMap *tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// 2-D tiled load of the box at (x, y) (x in elements of the innermost
// dimension) into shared memory; completion is signalled on `bar` as
// transaction bytes.
QMOE_DEV void tma_load_2d(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 3-D tiled load of the box at (x, y, z).
QMOE_DEV void tma_load_3d(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

QMOE_DEV void tma_load_4d(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int x, int y, int z,
                          int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}

// L2 policy for streams read once: their lines are the first to go, so the
// small tensors, the code and the reused weights of the other kernels stay.
QMOE_DEV uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// tma_load_2d / tma_load_3d with an L2 cache policy.
QMOE_DEV void tma_load_2d_hint(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int x, int y,
                               uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(pol)
        : "memory");
}

QMOE_DEV void tma_load_3d_hint(void *smem_dst, const CUtensorMap *tm, uint64_t *bar, int x, int y, int z,
                               uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(pol)
        : "memory");
}

// ---- TMEM ---------------------------------------------------------------
// Whole-warp operations.
QMOE_DEV void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
QMOE_DEV void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
QMOE_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

QMOE_DEV void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
QMOE_DEV void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (TMA,
// tensor core).
QMOE_DEV void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05.mma ----------------------------------------------------------
// Instruction descriptor of a dense kind::i8 / kind::f16 MMA with K-major A
// and B: D format in bits 4-5, A / B formats in 7-9 / 10-12, N/8 in 17-22,
// M/16 in 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, bool a_signed, bool b_signed) {
    return (2u << 4)                       // D = s32
           | ((a_signed ? 1u : 0u) << 7)   // A: u8 / s8
           | ((b_signed ? 1u : 0u) << 10)  // B: u8 / s8
           | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4)          // D = f32
           | (1u << 7)        // A = bf16
           | (1u << 10)       // B = bf16
           | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor (K-major): start address, leading / stride
// byte offsets (all >> 4), version 1, layout type in bits 61-63
// (0 = no swizzle, 2 = 128-byte swizzle).
QMOE_DEV uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)(layout & 7) << 61;
    return d;
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::i8, issued by one thread.
QMOE_DEV void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                        uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(
            d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u),
        "r"(0u)
        : "memory");
}

// Same, with the B descriptor given as its two 32-bit halves (callers step the
// start-address field in the low half without 64-bit arithmetic) and the
// accumulate flag as a predicate value computed once.
QMOE_DEV void mma_i8_ts_lohi(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n .reg .b64 bd;\n setp.ne.b32 p, %5, 0;\n mov.b64 bd, {%2, %3};\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], bd, %4, {%6, %7, %8, %9}, p;\n}" ::"r"(
            d_tmem),
        "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (bf16 operands, f32 accumulate).
QMOE_DEV void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(
            d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u),
        "r"(0u)
        : "memory");
}

// kind::f16 with the B descriptor as two 32-bit halves (see mma_i8_ts_lohi).
QMOE_DEV void mma_bf16_ts_lohi(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n .reg .b64 bd;\n setp.ne.b32 p, %5, 0;\n mov.b64 bd, {%2, %3};\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, {%6, %7, %8, %9}, p;\n}" ::"r"(
            d_tmem),
        "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u)
        : "memory");
}

// Arrive on `bar` once every tcgen05.mma this thread issued so far is done.
QMOE_DEV void mma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// ---- tcgen05.ld / st (32 lanes x 32-bit columns, this warp's lane quarter) --
QMOE_DEV void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

QMOE_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

QMOE_DEV void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

QMOE_DEV void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

QMOE_DEV void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

QMOE_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace sm100
}  // namespace qmoe
