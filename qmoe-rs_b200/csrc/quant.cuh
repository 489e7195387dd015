// quant.cuh -- activations -> per-row fixed point, as three balanced int8 limbs.
//
// Feeds the integer tensor-core GEMV (qgemv_imma.cu).  For every row (one
// routed assignment or shared-expert token, in position order):
//   e   = exponent with max|x| * 2^-e in [2^21, 2^22)  (0 for an all-zero row)
//   Q_k = rint(x_k * 2^-e)      (scaling by a power of two is exact)
//   Q_k = q2 * 2^16 + q1 * 2^8 + q0 with every q in [-128, 127]
// written as xq[row][limb][Kp] (int8) and meta[row] = (e, sum_k Q_k).
// Inside each 16-element block the bytes are stored in the order
// 0,4,8,12, 1,5,9,13, 2,6,10,14, 3,7,11,15: the order in which the GEMV
// unpacks a 32-bit word of 2-bit codes (bits 2j..2j+1 of its four bytes are
// codes j, j+4, j+8, j+12), so activation k meets the weight of column k.
// Blocks past K up to the row's length padded to 256 are zero.
//
// One row is done by a group of kQuantGroup threads (four warps) that meet
// at a barrier the caller supplies: the whole CTA in the limb kernel
// (quant.cu), a named barrier of the group inside the GEMV (qgemv_imma.cu).
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace qmoe {

constexpr int kQuantGroup = 128;  // threads per row

// Limbs of one 16-element block from its Q values, in the block byte order.
QMOE_DEV void quant_store_block(int8_t *dst, int64_t Kp, int b, const int (&Q)[16], long long &sq) {
    uint32_t l0[4] = {0, 0, 0, 0}, l1[4] = {0, 0, 0, 0}, l2[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int q = Q[j];
        sq += q;
        const int d0 = ((q + 128) & 255) - 128;
        const int q1 = (q - d0) >> 8;
        const int d1 = ((q1 + 128) & 255) - 128;
        const int d2 = (q1 - d1) >> 8;
        const int word = j & 3, sh = (j >> 2) * 8;  // element j -> byte 4*(j%4) + j/4
        l0[word] |= (uint32_t)(d0 & 255) << sh;
        l1[word] |= (uint32_t)(d1 & 255) << sh;
        l2[word] |= (uint32_t)(d2 & 255) << sh;
    }
    *reinterpret_cast<uint4 *>(dst + 0 * Kp + 16 * b) = make_uint4(l0[0], l0[1], l0[2], l0[3]);
    *reinterpret_cast<uint4 *>(dst + 1 * Kp + 16 * b) = make_uint4(l1[0], l1[1], l1[2], l1[3]);
    *reinterpret_cast<uint4 *>(dst + 2 * Kp + 16 * b) = make_uint4(l2[0], l2[1], l2[2], l2[3]);
}

QMOE_DEV int quant_exponent(float m) {
    int e = 0;
    if (m > 0.0f) {
        int ex;
        frexpf(m, &ex);
        e = max(ex - 22, -120);
    }
    return e;
}

// One position's limbs and metadata by the group thread `ht` (0..127);
// s_red / s_sum: this group's four slots; sync(): the group's barrier.  BPT
// > 0: the row is read once, each thread holding BPT 16-element blocks in
// registers (rows up to 2048 * BPT); BPT == 0: any length, the row is read
// twice (max, limbs).  Every thread of the group calls it with the same pos.
template <int BPT, class Sync>
QMOE_DEV void quant_position(const QuantParams &p, int64_t pos, int ht, float *s_red, long long *s_sum,
                             Sync sync) {
    const int gw = ht >> 5;  // warp of the group
    const bool routed = pos < p.shared_base;
    // unused routed slots and the padding position are skipped
    const bool active = pos < p.npos && !(routed && p.n_valid && pos >= *p.n_valid);
    int64_t row = pos;
    if (active && p.pos_tok) row = routed ? (int64_t)p.pos_tok[pos] : p.shared_row0 + pos - p.shared_base;
    const int64_t base = row * p.act_ld;
    const int K = routed ? p.K : p.K_s;
    const int nblk = ((K + 255) / 256) * 16;  // blocks the GEMV reads (K padded to 256)
    int8_t *dst = p.xq + pos * 3 * (int64_t)p.Kp;
    long long sq = 0;
    float m = 0.0f;
    float4 v[BPT > 0 ? BPT : 1][4];
    if (BPT > 0) {
#pragma unroll
        for (int i = 0; i < BPT; ++i) {
            const int b = ht + i * kQuantGroup;
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4) {
                v[i][j4] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (active && b * 16 < K) v[i][j4] = load_act4(p.act, p.dtype, base + b * 16 + 4 * j4);
                m = fmaxf(m, fmaxf(fmaxf(fabsf(v[i][j4].x), fabsf(v[i][j4].y)),
                                   fmaxf(fabsf(v[i][j4].z), fabsf(v[i][j4].w))));
            }
        }
    } else if (active) {
        for (int q = ht; q < (K >> 2); q += kQuantGroup) {
            const float4 x = load_act4(p.act, p.dtype, base + 4 * q);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
        }
    }
    // max over the group
    m = warp_max(m);
    if ((ht & 31) == 0) s_red[gw] = m;
    sync();
    m = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
    const int e = quant_exponent(m);
    const float sc = pow2i(-e);
    if (BPT > 0) {
#pragma unroll
        for (int i = 0; i < BPT; ++i) {
            const int b = ht + i * kQuantGroup;
            if (!active || b >= nblk) continue;
            int Q[16];
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4) {
                Q[4 * j4 + 0] = __float2int_rn(v[i][j4].x * sc);
                Q[4 * j4 + 1] = __float2int_rn(v[i][j4].y * sc);
                Q[4 * j4 + 2] = __float2int_rn(v[i][j4].z * sc);
                Q[4 * j4 + 3] = __float2int_rn(v[i][j4].w * sc);
            }
            quant_store_block(dst, p.Kp, b, Q, sq);
        }
    } else if (active) {
        for (int b = ht; b < nblk; b += kQuantGroup) {
            int Q[16];
            const bool in = b * 16 < K;
#pragma unroll
            for (int j4 = 0; j4 < 4; ++j4) {
                float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                if (in) x = load_act4(p.act, p.dtype, base + b * 16 + 4 * j4);
                Q[4 * j4 + 0] = __float2int_rn(x.x * sc);
                Q[4 * j4 + 1] = __float2int_rn(x.y * sc);
                Q[4 * j4 + 2] = __float2int_rn(x.z * sc);
                Q[4 * j4 + 3] = __float2int_rn(x.w * sc);
            }
            quant_store_block(dst, p.Kp, b, Q, sq);
        }
    }
    // sum of Q over the group
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if ((ht & 31) == 0) s_sum[gw] = sq;
    sync();
    if (ht == 0 && active) p.meta[pos] = make_longlong2(e, s_sum[0] + s_sum[1] + s_sum[2] + s_sum[3]);
}

// Blocks a thread of the group holds for rows of up to kmax elements (0: the
// two-pass form).
inline int quant_bpt(int kmax) {
    const int nblk = ((kmax + 255) / 256) * 16;
    const int bpt = (nblk + kQuantGroup - 1) / kQuantGroup;
    return bpt <= 1 ? 1 : bpt <= 2 ? 2 : bpt <= 4 ? 4 : 0;
}

}  // namespace qmoe
