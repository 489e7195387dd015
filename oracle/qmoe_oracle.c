/*
 * qmoe_oracle.c -- CPU restatement of qmoe-rs's 2-bit MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * --impl reference legs load it.  Nothing in the shipped library links it,
 * and the library never falls back to it.
 *
 * What it restates (paths are relative to the qmoe-rs project root):
 *   qo_dequant_dot      src/simd.rs:6-45     4-lane f32 accumulators, codes
 *                                           LSB-first, value = code - 1.0
 *                                           (code 3 -> +2.0), tail ignored,
 *                                           reduce_sum() then * scale.
 *   qo_packed_forward   src/tensor.rs:64-95  batch-outer, row-inner GEMV.
 *   qo_route            src/moe.rs:57-82     stable descending sort, softmax
 *                                           over ALL experts summed in sorted
 *                                           order, first top_k, no renorm.
 *   qo_moe_forward      src/moe.rs:40-130    expert-ascending loop, SwiGLU
 *                                           g*(1/(1+exp(-g)))*u, down GEMV,
 *                                           out += d*w.
 *   qo_shared_forward   src/model.rs:325-347 batched shared-expert FFN.
 *   qo_layer_forward    src/model.rs:386-389 moe_out + shared_out.
 *
 * Pinned where the reference is not:
 *   - Gate logits (src/moe.rs:51) come from candle's CPU matmul, whose
 *     summation order is not observable here.  qo_gate_logits pins one order:
 *     for each 64-wide chunk c of the hidden dim, p_c = fmaf-chain over the
 *     chunk starting from 0; logit = ((0 + p_0) + p_1) + ...  The CUDA router
 *     computes exactly this, so routing indices are comparable bit for bit.
 *   - Extensions the reference lacks (DeepSeek-V2/V3 routing): sigmoid
 *     scoring, per-expert selection bias, group-limited top-k, top-k
 *     renormalisation, routed scaling.  Their spec is written here.  Sigmoid
 *     uses qo_exp (Cody-Waite reduction + degree-7 Taylor polynomial, all
 *     fmaf), which the CUDA router restates op for op, so sigmoid scores and
 *     the selection built on them are reproducible bit for bit.
 *
 * Compile with -ffp-contract=off: Rust does not contract a*b+c into an FMA
 * (src/simd.rs:40), and expf is glibc's, the libm that Rust's f32::exp calls
 * on Linux.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QO_REDUCE_ORDERED 0
#define QO_REDUCE_PAIRWISE 1

#define QO_SCORING_SOFTMAX 0
#define QO_SCORING_SIGMOID 1

#define QO_GATE_CHUNK 64

/* Layer configuration; field order mirrors qmoe_moe_config in the C ABI. */
typedef struct {
    int32_t num_experts;
    int32_t top_k;
    int32_t hidden_dim;
    int32_t intermediate_dim;
    int32_t shared_intermediate_dim; /* 0 = no shared expert */
    int32_t scoring;                 /* QO_SCORING_* */
    int32_t n_group;                 /* 1 = no group limit */
    int32_t topk_group;
    int32_t norm_topk_prob;          /* 0 = reference semantics */
    float routed_scaling_factor;     /* 1.0 = reference semantics */
    int32_t has_bias;                /* per-expert selection bias present */
    int32_t reduce_mode;             /* QO_REDUCE_* for qo_dequant_dot */
} qo_config;

/* ---------------------------------------------------------------------- */
/* L1: src/simd.rs:6-45                                                     */
/* ---------------------------------------------------------------------- */
float qo_dequant_dot(const uint8_t *packed, int64_t n_packed, const float *act,
                     int64_t n_act, float scale, int reduce_mode)
{
    /* lane accumulators of the f32x4 `sum` (src/simd.rs:11) */
    float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f, l3 = 0.0f;
    /* num_bytes = min(len, act.len()/4): a ragged activation tail is
     * ignored (src/simd.rs:15) */
    int64_t nb = n_packed < n_act / 4 ? n_packed : n_act / 4;
    for (int64_t i = 0; i < nb; ++i) {
        uint8_t b = packed[i];
        /* bits 2j..2j+1 hold weight j; value = code - 1.0 (src/simd.rs:22-31) */
        float f0 = (float)(int32_t)(b & 3u) - 1.0f;
        float f1 = (float)(int32_t)((b >> 2) & 3u) - 1.0f;
        float f2 = (float)(int32_t)((b >> 4) & 3u) - 1.0f;
        float f3 = (float)(int32_t)((b >> 6) & 3u) - 1.0f;
        const float *a = act + 4 * i;
        /* sum += w_vec * a_vec : lane-wise mul then add (src/simd.rs:40) */
        l0 = l0 + f0 * a[0];
        l1 = l1 + f1 * a[1];
        l2 = l2 + f2 * a[2];
        l3 = l3 + f3 * a[3];
    }
    float s;
    if (reduce_mode == QO_REDUCE_PAIRWISE)
        s = (l0 + l1) + (l2 + l3);
    else
        s = ((l0 + l1) + l2) + l3; /* ordered reduction, lane 0 first */
    return s * scale;            /* src/simd.rs:44 */
}

/* ---------------------------------------------------------------------- */
/* L2: src/tensor.rs:64-95 (forward_simd) / :99-121 (forward_simd_raw)      */
/* ---------------------------------------------------------------------- */
void qo_packed_forward(const uint8_t *packed, const float *scales, int64_t out_f,
                       int64_t in_f, const float *x, int64_t batch, float *y,
                       int reduce_mode)
{
    int64_t bpr = in_f / 4; /* bytes_per_row (src/tensor.rs:74) */
    for (int64_t b = 0; b < batch; ++b) {
        const float *xv = x + b * in_f;
        for (int64_t o = 0; o < out_f; ++o)
            y[b * out_f + o] = qo_dequant_dot(packed + o * bpr, bpr, xv, in_f,
                                              scales[o], reduce_mode);
    }
}

/* Same, parallel over the batch rows; each row is computed identically. */
static void packed_forward_mt(const uint8_t *packed, const float *scales,
                              int64_t out_f, int64_t in_f, const float *x,
                              int64_t batch, float *y, int reduce_mode,
                              int nthreads)
{
#ifdef _OPENMP
    if (nthreads > 1) {
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
        for (int64_t b = 0; b < batch; ++b)
            qo_packed_forward(packed, scales, out_f, in_f, x + b * in_f, 1,
                              y + b * out_f, reduce_mode);
        return;
    }
#endif
    (void)nthreads;
    qo_packed_forward(packed, scales, out_f, in_f, x, batch, y, reduce_mode);
}

/* ---------------------------------------------------------------------- */
/* Pinned gate-logit order (stands in for candle's matmul, src/moe.rs:51)   */
/* ---------------------------------------------------------------------- */
void qo_gate_logits(const float *x, const float *gate_w, int64_t T, int64_t E,
                    int64_t H, float *logits)
{
    for (int64_t t = 0; t < T; ++t) {
        const float *xv = x + t * H;
        for (int64_t e = 0; e < E; ++e) {
            const float *wv = gate_w + e * H;
            float total = 0.0f;
            for (int64_t c0 = 0; c0 < H; c0 += QO_GATE_CHUNK) {
                int64_t c1 = c0 + QO_GATE_CHUNK < H ? c0 + QO_GATE_CHUNK : H;
                float acc = 0.0f;
                for (int64_t k = c0; k < c1; ++k)
                    acc = fmaf(xv[k], wv[k], acc);
                total = total + acc;
            }
            logits[t * E + e] = total;
        }
    }
}

/* ---------------------------------------------------------------------- */
/* Deterministic exp for the sigmoid extension.                             */
/* Method: Cody & Waite argument reduction x = n*ln2 + r with ln2 split in  */
/* two floats (hi has 16 trailing zero bits so n*hi is exact), then the     */
/* Taylor series of e^r to degree 7 in Horner form (|r| <= ln2/2, so the    */
/* truncation term r^8/8! < 6e-9), then scaling by 2^n built from the       */
/* exponent bits.  Every step is an IEEE op (fmaf, mul, rint), so a CUDA    */
/* restatement with __fmaf_rn / __fmul_rn yields the same bits.             */
/* ---------------------------------------------------------------------- */
static float qo_pow2i(int n)
{
    /* 2^n for -149 <= n <= 127 as an exact float */
    union { uint32_t u; float f; } v;
    if (n >= -126) {
        v.u = (uint32_t)(n + 127) << 23;
    } else {
        v.u = 1u << (n + 149);
    }
    return v.f;
}

float qo_exp(float x)
{
    if (!(x == x)) return x;          /* NaN */
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.97208404541016f) return 0.0f;
    float n = rintf(x * 1.44269502162933349609375f); /* round(x*log2 e) */
    float r = fmaf(n, -0.693145751953125f, x);       /* x - n*ln2_hi (exact) */
    r = fmaf(n, -1.428606765330187045037746429443359375e-06f, r); /* - n*ln2_lo */
    float p = 1.98412698412698412698e-4f;            /* 1/7! */
    p = fmaf(p, r, 1.38888888888888888889e-3f);      /* 1/6! */
    p = fmaf(p, r, 8.33333333333333333333e-3f);      /* 1/5! */
    p = fmaf(p, r, 4.16666666666666666667e-2f);      /* 1/4! */
    p = fmaf(p, r, 1.66666666666666666667e-1f);      /* 1/3! */
    p = fmaf(p, r, 0.5f);                            /* 1/2! */
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) return p * qo_pow2i(127) * qo_pow2i(ni - 127);
    if (ni < -126) return (p * qo_pow2i(-126)) * qo_pow2i(ni + 126);
    return p * qo_pow2i(ni);
}

float qo_sigmoid(float x)
{
    return 1.0f / (1.0f + qo_exp(-x));
}

/* ---------------------------------------------------------------------- */
/* Routing: src/moe.rs:57-82 plus the DeepSeek-V2/V3 extensions.            */
/* ---------------------------------------------------------------------- */
/* a ranks before b in a stable descending sort of (value, index) pairs whose
 * input order is ascending index: larger value first, ties -> lower index.
 * (sort_by with partial_cmp is stable, src/moe.rs:68-71.) */
static int before(float va, int ia, float vb, int ib)
{
    if (va > vb) return 1;
    if (va < vb) return 0;
    return ia < ib;
}

/* Stable descending argsort of v[0..n) (insertion sort keeps stability). */
static void argsort_desc(const float *v, int n, int *idx)
{
    for (int i = 0; i < n; ++i) idx[i] = i;
    for (int i = 1; i < n; ++i) {
        int cur = idx[i];
        int j = i - 1;
        while (j >= 0 && before(v[cur], cur, v[idx[j]], idx[j])) {
            idx[j + 1] = idx[j];
            --j;
        }
        idx[j + 1] = cur;
    }
}

/*
 * Route one token.  Writes its top_k experts in selection order (descending
 * score, ties to the lower index) and their combine weights.
 *
 * softmax (reference, src/moe.rs:64-81): order by logit; max over all E;
 *   S = sum of expf(l - max) over all E in sorted order; w = expf(l-max)/S.
 *   With n_group > 1 (DeepSeek-V2 group_limited_greedy) a group's score is
 *   its max logit, the topk_group best groups survive, and the top_k come
 *   from the survivors.  Selection uses logits, which orders the same way
 *   as the softmax probabilities.
 * sigmoid (DeepSeek-V3): s = qo_sigmoid(l); choice = s + bias (bias
 *   optional); group score = sum of the two best choices in the group;
 *   topk_group groups survive; top_k by choice among survivors; w = s.
 * then, if norm_topk_prob: w /= (sum of the top_k w in selection order +
 * 1e-20); then w *= routed_scaling_factor (skipped when it is exactly 1).
 */
static int route_token(const qo_config *cfg, const float *logits,
                       const float *bias, int32_t *out_idx, float *out_w,
                       float *scratch_f, int *scratch_i)
{
    const int E = cfg->num_experts, K = cfg->top_k;
    const int G = cfg->n_group > 0 ? cfg->n_group : 1;
    const int TG = cfg->topk_group > 0 ? cfg->topk_group : G;
    float *choice = scratch_f;         /* [E] */
    float *gscore = scratch_f + E;     /* [G] */
    float *masked = scratch_f + E + G; /* [E] */
    int *order = scratch_i;            /* [E] */
    int *gorder = scratch_i + E;       /* [G] */
    if (K > E || E % G != 0 || TG > G) return -1;
    const int per_group = E / G;

    if (cfg->scoring == QO_SCORING_SOFTMAX) {
        for (int e = 0; e < E; ++e) choice[e] = logits[e];
    } else {
        for (int e = 0; e < E; ++e) {
            float s = qo_sigmoid(logits[e]);
            choice[e] = cfg->has_bias ? s + bias[e] : s;
        }
    }

    /* group limit */
    const float NEG = -INFINITY;
    if (G > 1) {
        for (int g = 0; g < G; ++g) {
            const float *c = choice + g * per_group;
            float best = NEG, second = NEG;
            int bi = -1;
            for (int j = 0; j < per_group; ++j)
                if (bi < 0 || c[j] > best) { best = c[j]; bi = j; }
            for (int j = 0; j < per_group; ++j)
                if (j != bi && (second == NEG || c[j] > second)) second = c[j];
            if (cfg->scoring == QO_SCORING_SOFTMAX || per_group < 2)
                gscore[g] = best;
            else
                gscore[g] = best + second;
        }
        argsort_desc(gscore, G, gorder);
        for (int e = 0; e < E; ++e) masked[e] = NEG;
        for (int r = 0; r < TG; ++r) {
            int g = gorder[r];
            for (int j = 0; j < per_group; ++j)
                masked[g * per_group + j] = choice[g * per_group + j];
        }
        /* masked experts sort after every survivor; among equal -inf the
         * lower index comes first, but K <= TG*per_group keeps them out. */
        if (K > TG * per_group) return -1;
        argsort_desc(masked, E, order);
    } else {
        argsort_desc(choice, E, order);
    }

    if (cfg->scoring == QO_SCORING_SOFTMAX) {
        /* src/moe.rs:74-81: max and sum over ALL experts in sorted-by-logit
         * order (the reference sorts by logit, no groups involved). */
        int *lorder = scratch_i + E + G;
        argsort_desc(logits, E, lorder);
        float mx = NEG;
        for (int i = 0; i < E; ++i) mx = fmaxf(mx, logits[lorder[i]]);
        float s = 0.0f;
        for (int i = 0; i < E; ++i) s = s + expf(logits[lorder[i]] - mx);
        for (int j = 0; j < K; ++j) {
            int e = order[j];
            out_idx[j] = e;
            out_w[j] = expf(logits[e] - mx) / s;
        }
    } else {
        for (int j = 0; j < K; ++j) {
            int e = order[j];
            out_idx[j] = e;
            out_w[j] = qo_sigmoid(logits[e]);
        }
    }
    if (cfg->norm_topk_prob) {
        float den = 0.0f;
        for (int j = 0; j < K; ++j) den = den + out_w[j];
        den = den + 1e-20f;
        for (int j = 0; j < K; ++j) out_w[j] = out_w[j] / den;
    }
    if (cfg->routed_scaling_factor != 1.0f)
        for (int j = 0; j < K; ++j) out_w[j] = out_w[j] * cfg->routed_scaling_factor;
    return 0;
}

int qo_route(const qo_config *cfg, const float *logits, const float *bias,
             int64_t T, int32_t *topk_idx, float *topk_w)
{
    const int E = cfg->num_experts, G = cfg->n_group > 0 ? cfg->n_group : 1;
    float *sf = (float *)malloc(sizeof(float) * (size_t)(2 * E + G));
    int *si = (int *)malloc(sizeof(int) * (size_t)(2 * E + G));
    int rc = 0;
    for (int64_t t = 0; t < T && rc == 0; ++t)
        rc = route_token(cfg, logits + t * E, bias, topk_idx + t * cfg->top_k,
                         topk_w + t * cfg->top_k, sf, si);
    free(sf);
    free(si);
    return rc;
}

/* ---------------------------------------------------------------------- */
/* SwiGLU as written in src/moe.rs:109-115 and src/model.rs:332-338.        */
/* ---------------------------------------------------------------------- */
static inline float swiglu(float g, float u)
{
    float swish = g * (1.0f / (1.0f + expf(-g)));
    return swish * u;
}

/* One (token, expert) assignment: gate/up GEMV, SwiGLU, down GEMV.  The
 * reference builds each as a batch-1 forward_simd call (src/moe.rs:98-118). */
static void expert_ffn(const uint8_t *wg, const float *sg, const uint8_t *wu,
                       const float *su, const uint8_t *wd, const float *sd,
                       int64_t H, int64_t I, const float *x, float *act_buf,
                       float *g_buf, float *u_buf, float *d_out, int rm)
{
    qo_packed_forward(wg, sg, I, H, x, 1, g_buf, rm);
    qo_packed_forward(wu, su, I, H, x, 1, u_buf, rm);
    for (int64_t i = 0; i < I; ++i) act_buf[i] = swiglu(g_buf[i], u_buf[i]);
    qo_packed_forward(wd, sd, H, I, act_buf, 1, d_out, rm);
}

/*
 * Routed experts: src/moe.rs:40-130.
 * w_packed / w_scales hold 3 entries per expert: gate, up, down.
 * topk_idx / topk_w (optional) receive the routing of every token.
 * nthreads <= 1 runs the reference's expert-outer loop verbatim; more
 * threads run tokens in parallel, which computes every (token, expert)
 * product the same way and accumulates each token's output in the same
 * ascending-expert order, so the bits are identical.
 */
int qo_moe_forward(const qo_config *cfg, const float *gate_w, const float *bias,
                   const uint8_t *const *w_packed, const float *const *w_scales,
                   const float *x, int64_t T, float *out, int32_t *topk_idx,
                   float *topk_w, int nthreads)
{
    const int64_t E = cfg->num_experts, K = cfg->top_k;
    const int64_t H = cfg->hidden_dim, I = cfg->intermediate_dim;
    const int rm = cfg->reduce_mode;
    memset(out, 0, sizeof(float) * (size_t)(T * H));
    if (E == 0) return 0; /* empty experts -> zeros (src/moe.rs:46-48) */

    float *logits = (float *)malloc(sizeof(float) * (size_t)(T * E));
    int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * (size_t)(T * K));
    float *wts = (float *)malloc(sizeof(float) * (size_t)(T * K));
    qo_gate_logits(x, gate_w, T, E, H, logits);
    int rc = qo_route(cfg, logits, bias, T, idx, wts);
    if (rc != 0) goto done;

    if (nthreads <= 1) {
        /* bins[e] = [(t, w)] in token order (src/moe.rs:57, :80) */
        int64_t *cnt = (int64_t *)calloc((size_t)E, sizeof(int64_t));
        for (int64_t a = 0; a < T * K; ++a) cnt[idx[a]]++;
        int64_t *off = (int64_t *)malloc(sizeof(int64_t) * (size_t)(E + 1));
        off[0] = 0;
        for (int64_t e = 0; e < E; ++e) off[e + 1] = off[e] + cnt[e];
        int64_t *bt = (int64_t *)malloc(sizeof(int64_t) * (size_t)(T * K + 1));
        float *bw = (float *)malloc(sizeof(float) * (size_t)(T * K + 1));
        int64_t *fill = (int64_t *)calloc((size_t)E, sizeof(int64_t));
        for (int64_t t = 0; t < T; ++t)
            for (int64_t j = 0; j < K; ++j) {
                int64_t e = idx[t * K + j];
                int64_t p = off[e] + fill[e]++;
                bt[p] = t;
                bw[p] = wts[t * K + j];
            }
        float *g = (float *)malloc(sizeof(float) * (size_t)I);
        float *u = (float *)malloc(sizeof(float) * (size_t)I);
        float *act = (float *)malloc(sizeof(float) * (size_t)I);
        float *d = (float *)malloc(sizeof(float) * (size_t)H);
        for (int64_t e = 0; e < E; ++e) {
            for (int64_t p = off[e]; p < off[e + 1]; ++p) {
                int64_t t = bt[p];
                expert_ffn(w_packed[3 * e], w_scales[3 * e], w_packed[3 * e + 1],
                           w_scales[3 * e + 1], w_packed[3 * e + 2],
                           w_scales[3 * e + 2], H, I, x + t * H, act, g, u, d, rm);
                float *o = out + t * H;
                for (int64_t h = 0; h < H; ++h) o[h] = o[h] + d[h] * bw[p];
            }
        }
        free(g); free(u); free(act); free(d);
        free(cnt); free(off); free(bt); free(bw); free(fill);
    } else {
#ifdef _OPENMP
#pragma omp parallel num_threads(nthreads)
#endif
        {
            float *g = (float *)malloc(sizeof(float) * (size_t)I);
            float *u = (float *)malloc(sizeof(float) * (size_t)I);
            float *act = (float *)malloc(sizeof(float) * (size_t)I);
            float *d = (float *)malloc(sizeof(float) * (size_t)H);
            int64_t *ord = (int64_t *)malloc(sizeof(int64_t) * (size_t)K);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
            for (int64_t t = 0; t < T; ++t) {
                /* this token's experts in ascending index order */
                for (int64_t j = 0; j < K; ++j) ord[j] = j;
                for (int64_t a = 1; a < K; ++a) {
                    int64_t c = ord[a], b = a - 1;
                    while (b >= 0 && idx[t * K + ord[b]] > idx[t * K + c]) {
                        ord[b + 1] = ord[b];
                        --b;
                    }
                    ord[b + 1] = c;
                }
                float *o = out + t * H;
                for (int64_t j = 0; j < K; ++j) {
                    int64_t e = idx[t * K + ord[j]];
                    float w = wts[t * K + ord[j]];
                    expert_ffn(w_packed[3 * e], w_scales[3 * e], w_packed[3 * e + 1],
                               w_scales[3 * e + 1], w_packed[3 * e + 2],
                               w_scales[3 * e + 2], H, I, x + t * H, act, g, u, d, rm);
                    for (int64_t h = 0; h < H; ++h) o[h] = o[h] + d[h] * w;
                }
            }
            free(g); free(u); free(act); free(d); free(ord);
        }
    }
    if (topk_idx) memcpy(topk_idx, idx, sizeof(int32_t) * (size_t)(T * K));
    if (topk_w) memcpy(topk_w, wts, sizeof(float) * (size_t)(T * K));
done:
    free(logits);
    free(idx);
    free(wts);
    return rc;
}

/* The expert half of src/moe.rs:84-129 for rows whose routing is given:
 * idx [R, K] holds expert ids in 0..E-1 or -1 (slot skipped), w [R, K] the
 * weights.  out[r] = sum over valid slots in ascending expert order of
 * w * expert(x[r]); the per-(row, expert) FFN is the reference's. */
void qo_experts_forward(const qo_config *cfg, const uint8_t *const *w_packed,
                        const float *const *w_scales, const float *x, int64_t R,
                        const int32_t *idx, const float *wts, float *out,
                        int nthreads)
{
    const int64_t K = cfg->top_k, H = cfg->hidden_dim, I = cfg->intermediate_dim;
    const int rm = cfg->reduce_mode;
    memset(out, 0, sizeof(float) * (size_t)(R * H));
#ifdef _OPENMP
#pragma omp parallel num_threads(nthreads > 1 ? nthreads : 1)
#endif
    {
        float *g = (float *)malloc(sizeof(float) * (size_t)I);
        float *u = (float *)malloc(sizeof(float) * (size_t)I);
        float *act = (float *)malloc(sizeof(float) * (size_t)I);
        float *d = (float *)malloc(sizeof(float) * (size_t)H);
        int64_t *ord = (int64_t *)malloc(sizeof(int64_t) * (size_t)(K > 0 ? K : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t r = 0; r < R; ++r) {
            int64_t n = 0;
            for (int64_t j = 0; j < K; ++j) {
                if (idx[r * K + j] < 0) continue;
                int64_t b = n - 1;
                while (b >= 0 && idx[r * K + ord[b]] > idx[r * K + j]) {
                    ord[b + 1] = ord[b];
                    --b;
                }
                ord[b + 1] = j;
                ++n;
            }
            float *o = out + r * H;
            for (int64_t q = 0; q < n; ++q) {
                int64_t e = idx[r * K + ord[q]];
                float w = wts[r * K + ord[q]];
                expert_ffn(w_packed[3 * e], w_scales[3 * e], w_packed[3 * e + 1],
                           w_scales[3 * e + 1], w_packed[3 * e + 2], w_scales[3 * e + 2],
                           H, I, x + r * H, act, g, u, d, rm);
                for (int64_t h = 0; h < H; ++h) o[h] = o[h] + d[h] * w;
            }
        }
        free(g); free(u); free(act); free(d); free(ord);
    }
}

/* ---------------------------------------------------------------------- */
/* Shared expert: src/model.rs:325-347 (batched forward_simd over T rows).  */
/* ---------------------------------------------------------------------- */
void qo_shared_forward(const uint8_t *wg, const float *sg, const uint8_t *wu,
                       const float *su, const uint8_t *wd, const float *sd,
                       int64_t H, int64_t Is, const float *x, int64_t T,
                       float *out, int reduce_mode, int nthreads)
{
    float *g = (float *)malloc(sizeof(float) * (size_t)(T * Is));
    float *u = (float *)malloc(sizeof(float) * (size_t)(T * Is));
    packed_forward_mt(wg, sg, Is, H, x, T, g, reduce_mode, nthreads);
    packed_forward_mt(wu, su, Is, H, x, T, u, reduce_mode, nthreads);
    for (int64_t i = 0; i < T * Is; ++i) g[i] = swiglu(g[i], u[i]);
    packed_forward_mt(wd, sd, H, Is, g, T, out, reduce_mode, nthreads);
    free(g);
    free(u);
}

/* Decoder-layer MoE block without the residual: moe_out + shared_out
 * (src/model.rs:386-389 / :407-410).  shared_* may be NULL. */
int qo_layer_forward(const qo_config *cfg, const float *gate_w, const float *bias,
                     const uint8_t *const *w_packed, const float *const *w_scales,
                     const uint8_t *const *shared_packed,
                     const float *const *shared_scales, const float *x, int64_t T,
                     float *out, int32_t *topk_idx, float *topk_w, int nthreads)
{
    int rc = qo_moe_forward(cfg, gate_w, bias, w_packed, w_scales, x, T, out,
                            topk_idx, topk_w, nthreads);
    if (rc != 0) return rc;
    if (shared_packed && cfg->shared_intermediate_dim > 0) {
        const int64_t H = cfg->hidden_dim;
        float *s = (float *)malloc(sizeof(float) * (size_t)(T * H));
        qo_shared_forward(shared_packed[0], shared_scales[0], shared_packed[1],
                          shared_scales[1], shared_packed[2], shared_scales[2], H,
                          cfg->shared_intermediate_dim, x, T, s, cfg->reduce_mode,
                          nthreads);
        for (int64_t i = 0; i < T * H; ++i) out[i] = out[i] + s[i];
        free(s);
    }
    return 0;
}

/* Unpack to the dequantised f32 matrix (code - 1) * scale[row]: the value
 * every kernel must reproduce exactly. */
void qo_dequantize(const uint8_t *packed, const float *scales, int64_t out_f,
                   int64_t in_f, float *w)
{
    int64_t bpr = in_f / 4;
    for (int64_t o = 0; o < out_f; ++o)
        for (int64_t k = 0; k < bpr * 4; ++k) {
            uint8_t b = packed[o * bpr + k / 4];
            float c = (float)(int32_t)((b >> (2 * (k % 4))) & 3u) - 1.0f;
            w[o * in_f + k] = c * scales[o];
        }
}

/* ---------------------------------------------------------------------- */
/* Decoder-layer MoE block: post-attention LayerNorm (src/model.rs:366-367, */
/* :400-403) and the residual add (:409-412)                                */
/* ---------------------------------------------------------------------- */
/*
 * candle_nn::layer_norm(hidden, 1e-6) normalises each row with its mean and
 * biased variance and applies weight and bias.  candle's summation order is
 * not observable here (third-party, not vendored), so this pins one, in the
 * same 64-wide chunks as the gate logits:
 *   s1   = ((0 + p_0) + p_1) + ...,  p_c = sequential f32 sum of chunk c
 *   mean = s1 / H
 *   s2   = ((0 + q_0) + q_1) + ...,  q_c = fmaf chain of d*d over chunk c,
 *          d = x - mean
 *   rstd = 1 / sqrtf(s2 / H + eps)
 *   y    = ((x - mean) * rstd) * w + b   (each operation rounded once)
 * The CUDA kernel computes the same operations in the same order.  With
 * round_bf16 the result is rounded to bf16 (round to nearest even), what a
 * bf16 forward hands to its router and experts.
 */
static float qo_round_bf16(float v)
{
    uint32_t u;
    memcpy(&u, &v, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {       /* inf / nan: keep, quiet nan */
        if (u & 0x007fffffu) u |= 0x00400000u;
        u &= 0xffff0000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);
        u &= 0xffff0000u;
    }
    float r;
    memcpy(&r, &u, 4);
    return r;
}

void qo_layernorm(const float *x, const float *w, const float *b, float eps, int64_t T,
                  int64_t H, int round_bf16, float *y)
{
    for (int64_t t = 0; t < T; ++t) {
        const float *xv = x + t * H;
        float s1 = 0.0f;
        for (int64_t c0 = 0; c0 < H; c0 += QO_GATE_CHUNK) {
            int64_t c1 = c0 + QO_GATE_CHUNK < H ? c0 + QO_GATE_CHUNK : H;
            float p = 0.0f;
            for (int64_t k = c0; k < c1; ++k) p = p + xv[k];
            s1 = s1 + p;
        }
        const float mean = s1 / (float)H;
        float s2 = 0.0f;
        for (int64_t c0 = 0; c0 < H; c0 += QO_GATE_CHUNK) {
            int64_t c1 = c0 + QO_GATE_CHUNK < H ? c0 + QO_GATE_CHUNK : H;
            float q = 0.0f;
            for (int64_t k = c0; k < c1; ++k) {
                const float d = xv[k] - mean;
                q = fmaf(d, d, q);
            }
            s2 = s2 + q;
        }
        const float rstd = 1.0f / sqrtf(s2 / (float)H + eps);
        for (int64_t k = 0; k < H; ++k) {
            const float n = (xv[k] - mean) * rstd;
            const float v = n * w[k] + b[k];
            y[t * H + k] = round_bf16 ? qo_round_bf16(v) : v;
        }
    }
}
