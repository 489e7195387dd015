// api.cu -- the C ABI (include/qmoe_b200.h): contexts, device-resident packed
// tensors and MoE layers, and the launch sequence of a forward.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/qmoe_b200.h"
#include "combine.cuh"
#include "kernels.h"

using namespace qmoe;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define QTRY_CUDA(call)                                                            \
    do {                                                                           \
        cudaError_t e_ = (call);                                                   \
        if (e_ != cudaSuccess)                                                     \
            return fail(e_ == cudaErrorMemoryAllocation ? QMOE_ERR_NOMEM           \
                                                        : QMOE_ERR_CUDA,           \
                        "%s failed: %s", #call, cudaGetErrorString(e_));          \
    } while (0)

#define QTRY(call)                \
    do {                          \
        int r_ = (call);          \
        if (r_ != QMOE_OK) return r_; \
    } while (0)

// Scoped switch to a context's device.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

struct DevBuf {
    void *p = nullptr;
    size_t n = 0;
    template <class T> T *as() const { return static_cast<T *>(p); }
};

int grow(DevBuf &b, size_t bytes) {
    if (bytes <= b.n) return QMOE_OK;
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.n = 0;
    size_t n = bytes < 256 ? 256 : bytes;
    QTRY_CUDA(cudaMalloc(&b.p, n));
    b.n = n;
    return QMOE_OK;
}

void release(DevBuf &b) {
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.n = 0;
}

cudaMemcpyKind kind_in(int ptr_kind) {
    return ptr_kind == QMOE_PTR_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
}

int check_ptr_kind(int k) {
    if (k != QMOE_PTR_HOST && k != QMOE_PTR_DEVICE)
        return fail(QMOE_ERR_INVALID, "ptr_kind must be QMOE_PTR_HOST or QMOE_PTR_DEVICE");
    return QMOE_OK;
}

int check_dtype(int d) {
    if (d != QMOE_DTYPE_F32 && d != QMOE_DTYPE_BF16)
        return fail(QMOE_ERR_INVALID, "dtype must be QMOE_DTYPE_F32 or QMOE_DTYPE_BF16");
    return QMOE_OK;
}

size_t dtype_size(int d) { return d == QMOE_DTYPE_F32 ? 4 : 2; }

// Device activations and outputs are read and written with 16-byte vectors.
int check_align(const void *p, int ptr_kind, const char *name) {
    if (ptr_kind == QMOE_PTR_DEVICE && p && (reinterpret_cast<uintptr_t>(p) & 15u))
        return fail(QMOE_ERR_INVALID, "device pointer %s must be 16-byte aligned", name);
    return QMOE_OK;
}

constexpr int kDecodeTok = 5;   // tokens per work item of the decode kernels
// Host outputs up to this size are stored by the kernels straight into
// page-locked host memory; larger ones are staged and copied back.
constexpr size_t kMappedOutMaxBytes = size_t(2) << 20;
// Auto path: the prefill GEMM once the routed positions per expert segment
// (or the batch, for a shared-only pass) reach this many.
constexpr int64_t kPrefillMinRows = 16;

// A kernel whose bounded wait timed out leaves a flag in device memory; report
// (and clear) it at the next host synchronisation point.
int *error_flag() { return qmoe::device_error_flag(); }   // the current device's word

int check_device_error() {
    int *flag = error_flag();
    if (!flag) return QMOE_OK;
    int v = 0;
    QTRY_CUDA(cudaMemcpy(&v, flag, sizeof(int), cudaMemcpyDeviceToHost));
    if (v) {
        const int z = 0;
        cudaMemcpy(flag, &z, sizeof(int), cudaMemcpyHostToDevice);
        return fail(QMOE_ERR_CUDA, "a device-side wait timed out; the kernel abandoned its work");
    }
    return QMOE_OK;
}

}  // namespace

// Waits for the stream and reads the device error word with it: the word is
// copied into a page-locked host int in stream order, so one wait covers
// both (no extra synchronous copy per call).
int sync_and_check(cudaStream_t st) {
    static thread_local int *pinned = nullptr;
    static thread_local bool tried = false;
    if (!tried) {
        tried = true;
        if (cudaHostAlloc(reinterpret_cast<void **>(&pinned), sizeof(int), cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            pinned = nullptr;
        }
    }
    int *flag = error_flag();
    if (!flag || !pinned) {
        QTRY_CUDA(cudaStreamSynchronize(st));
        return check_device_error();
    }
    *pinned = 0;
    QTRY_CUDA(cudaMemcpyAsync(pinned, flag, sizeof(int), cudaMemcpyDeviceToHost, st));
    QTRY_CUDA(cudaStreamSynchronize(st));
    if (*pinned) return check_device_error();     // clears the word and reports
    return QMOE_OK;
}

struct qmoe_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
};

struct qmoe_packed {
    qmoe_ctx *ctx = nullptr;
    int64_t out_f = 0, in_f = 0;
    // Rows whose width is not a multiple of 64 codes are stored padded to
    // k_pad codes (padding code 1 = weight 0) and their activations staged
    // into rows of k_pad f32 whose padding stays zero; the GEMV then runs
    // on whole 64-code blocks.  k_pad == in_f for widths it takes directly.
    int64_t k_pad = 0;
    uint8_t *w = nullptr;
    float *s = nullptr;
    DevBuf groups, ngroups, x, y;
    int grid = 0;
};

struct qmoe_layer {
    qmoe_ctx *ctx = nullptr;
    qmoe_moe_config cfg{};
    int e_begin = 0, e_count = 0;
    bool has_shared = false;
    float *gate_w = nullptr, *bias = nullptr;
    float *gate_t = nullptr;   // [H][gate_t_ld(E)] transposed gate (E > 64), for large-batch logits
    // the decoder layer's post-attention LayerNorm (qmoe_layer_set_norm)
    float *ln_w = nullptr, *ln_b = nullptr;
    float ln_eps = 1e-6f;
    DevBuf xn;                 // normalised rows of a block forward
    uint8_t *w[3] = {nullptr, nullptr, nullptr};
    float *s[3] = {nullptr, nullptr, nullptr};
    uint8_t *ws[3] = {nullptr, nullptr, nullptr};
    float *ss[3] = {nullptr, nullptr, nullptr};
    int grid0 = 0, grid1 = 0;
    // tensor-core GEMV: TMA maps over the stacked 2-bit matrices, one CTA per SM
    int sm_count = 0;
    bool coop = false;     // cooperative launches available: the GEMVs make their own
                           // limb rows and the down GEMV combines
    CUtensorMap tm_w[3], tm_ws[3];
    CUtensorMap tm_w3[3], tm_ws3[3];  // 3-D views: two 64-byte chunks of 128 rows per box
    int kp1 = 0, kp2 = 0;  // limb row strides: hidden dim / intermediate dims, padded to 256
    // scratch
    int64_t cap = -1;
    DevBuf topk_idx, topk_w, assign_pos, pos_tok, seg_off, groups, ngroups, h, y;
    DevBuf x_in, io_out, user_idx, user_w;
    DevBuf xq1, meta1, xq2, meta2, router_scratch;
    DevBuf front_counter;  // hand-off counter of the decode front kernel (kept at zero)
    DevBuf gemv_sched;     // [2 modes][4] work counters of the decode GEMVs (kept at zero)
    CUtensorMap tm_xq1, tm_xq2;
    CUtensorMap tm_xq1_3, tm_xq2_3;   // 4-D views: 16 limb rows x 512 codes per decode stage
    // prefill path: gate/up maps with 64-row boxes, bf16 activation / SwiGLU
    // rows (16-element blocks permuted) and their 128-byte-swizzled maps
    bool prefill_ok = false;
    int path = QMOE_PATH_AUTO;
    CUtensorMap tm_pw[2], tm_pws[2];
    DevBuf xg, hb;
    CUtensorMap tm_xg, tm_hb, tm_xg2, tm_hb2;  // 256-row and 128-row boxes
    CUtensorMap tm_xg3, tm_hb3;                // 192-row boxes
    // tracing
    bool profiling = false;
    // Host-buffer forwards that repeat with the same page-locked x and out:
    // the kernel sequence is captured once (on the second such call) and
    // replayed as one graph launch.
    struct {
        const void *x = nullptr;
        const void *out = nullptr;
        const void *x_in = nullptr;   // the device copy of x the captured kernels read
        int64_t T = 0, cap = 0;
        int dtype = -1, path = -1, calls = 0;
        cudaGraphExec_t exec = nullptr;
    } fg;
    cudaEvent_t ev[8] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
};

namespace {
constexpr int kStages = 7;  // router, permute, quant1, gate_up, quant2, down, combine
inline void mark(qmoe_layer *L, int i) {
    if (L->profiling) cudaEventRecord(L->ev[i], L->ctx->stream);
}
}  // namespace

extern "C" {

const char *qmoe_last_error(void) { return g_err.c_str(); }

int qmoe_abi_version(void) { return QMOE_ABI_VERSION; }

int qmoe_ctx_create(int device, void *stream, qmoe_ctx **out) {
    if (!out) return fail(QMOE_ERR_INVALID, "out is NULL");
    *out = nullptr;
    int n = 0;
    QTRY_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n)
        return fail(QMOE_ERR_INVALID, "device %d out of range (%d devices)", device, n);
    cudaDeviceProp prop;
    QTRY_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10 || prop.minor != 0)
        return fail(QMOE_ERR_UNSUPPORTED,
                    "device %d is sm_%d%d; this library is built for sm_100a (B200)",
                    device, prop.major, prop.minor);
    qmoe_ctx *c = new (std::nothrow) qmoe_ctx;
    if (!c) return fail(QMOE_ERR_NOMEM, "host allocation failed");
    c->device = device;
    c->stream = static_cast<cudaStream_t>(stream);
    *out = c;
    return QMOE_OK;
}

int qmoe_ctx_destroy(qmoe_ctx *ctx) {
    delete ctx;
    return QMOE_OK;
}

int qmoe_ctx_set_stream(qmoe_ctx *ctx, void *stream) {
    if (!ctx) return fail(QMOE_ERR_INVALID, "ctx is NULL");
    ctx->stream = static_cast<cudaStream_t>(stream);
    return QMOE_OK;
}

int qmoe_ctx_synchronize(qmoe_ctx *ctx) {
    if (!ctx) return fail(QMOE_ERR_INVALID, "ctx is NULL");
    DeviceGuard g(ctx->device);
    return sync_and_check(ctx->stream);
}

// ---------------------------------------------------------------------------
// packed tensor
// ---------------------------------------------------------------------------

int qmoe_packed_create(qmoe_ctx *ctx, const uint8_t *packed, const float *scales,
                       int64_t out_features, int64_t in_features, int ptr_kind,
                       qmoe_packed **out) {
    if (!ctx || !scales || !out) return fail(QMOE_ERR_INVALID, "NULL argument");
    QTRY(check_ptr_kind(ptr_kind));
    *out = nullptr;
    // src/tensor.rs:74: a row is in_features / 4 bytes; the in_features % 4
    // trailing activations of a row are never read (src/simd.rs:15)
    const int64_t bpr = in_features / 4;
    if (out_features <= 0 || in_features <= 0)
        return fail(QMOE_ERR_INVALID, "shape (%lld, %lld): both dimensions must be > 0",
                    (long long)out_features, (long long)in_features);
    if (bpr > 0 && !packed) return fail(QMOE_ERR_INVALID, "NULL argument");
    if (in_features > (1 << 20) || out_features > (1LL << 31))
        return fail(QMOE_ERR_UNSUPPORTED, "shape too large");
    DeviceGuard g(ctx->device);
    qmoe_packed *t = new (std::nothrow) qmoe_packed;
    if (!t) return fail(QMOE_ERR_NOMEM, "host allocation failed");
    t->ctx = ctx;
    t->out_f = out_features;
    t->in_f = in_features;
    t->k_pad = in_features % 64 == 0 ? in_features : (4 * bpr + 63) / 64 * 64;
    if (t->k_pad == 0) t->k_pad = 64;
    const size_t wb = (size_t)out_features * (t->k_pad / 4);
    cudaError_t e = cudaMalloc(&t->w, wb);
    if (e == cudaSuccess) e = cudaMalloc(&t->s, sizeof(float) * out_features);
    if (e == cudaSuccess && t->k_pad == in_features) {
        e = cudaMemcpyAsync(t->w, packed, wb, kind_in(ptr_kind), ctx->stream);
    } else if (e == cudaSuccess) {
        // padded rows: fill with code 1 (weight 0), then the bpr bytes of each row
        e = cudaMemsetAsync(t->w, 0x55, wb, ctx->stream);
        if (e == cudaSuccess && bpr > 0)
            e = cudaMemcpy2DAsync(t->w, (size_t)(t->k_pad / 4), packed, (size_t)bpr, (size_t)bpr,
                                  (size_t)out_features, kind_in(ptr_kind), ctx->stream);
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(t->s, scales, sizeof(float) * out_features, kind_in(ptr_kind), ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        qmoe_packed_destroy(t);
        return fail(e == cudaErrorMemoryAllocation ? QMOE_ERR_NOMEM : QMOE_ERR_CUDA,
                    "packed upload failed: %s", cudaGetErrorString(e));
    }
    t->grid = qgemv_max_grid(1, (int)t->k_pad);
    *out = t;
    return QMOE_OK;
}

int qmoe_packed_destroy(qmoe_packed *t) {
    if (!t) return QMOE_OK;
    DeviceGuard g(t->ctx->device);
    if (t->w) cudaFree(t->w);
    if (t->s) cudaFree(t->s);
    release(t->groups);
    release(t->ngroups);
    release(t->x);
    release(t->y);
    delete t;
    return QMOE_OK;
}

int qmoe_packed_shape(const qmoe_packed *t, int64_t *out_features, int64_t *in_features) {
    if (!t) return fail(QMOE_ERR_INVALID, "tensor is NULL");
    if (out_features) *out_features = t->out_f;
    if (in_features) *in_features = t->in_f;
    return QMOE_OK;
}

int qmoe_packed_forward(qmoe_packed *t, const float *x, int64_t batch, float *y,
                        int ptr_kind) {
    if (!t || (!x && batch > 0) || (!y && batch > 0)) return fail(QMOE_ERR_INVALID, "NULL argument");
    QTRY(check_ptr_kind(ptr_kind));
    if (batch < 0) return fail(QMOE_ERR_INVALID, "batch < 0");
    if (batch == 0) return QMOE_OK;
    const bool padded = t->k_pad != t->in_f;
    if (!padded) QTRY(check_align(x, ptr_kind, "x"));
    qmoe_ctx *ctx = t->ctx;
    DeviceGuard g(ctx->device);
    cudaStream_t st = ctx->stream;
    const int64_t ngr = (batch + kDecodeTok - 1) / kDecodeTok;
    QTRY(grow(t->groups, sizeof(int4) * ngr));
    QTRY(grow(t->ngroups, sizeof(int32_t) * 4));
    const float *xd = x;
    float *yd = y;
    if (padded) {
        // rows of k_pad f32: the 4 * (in/4) activations a row uses, then
        // zeros (written once per allocation; the copies never touch them)
        const void *before = t->x.p;
        QTRY(grow(t->x, sizeof(float) * batch * t->k_pad));
        if (t->x.p != before) QTRY_CUDA(cudaMemsetAsync(t->x.p, 0, t->x.n, st));
        const int64_t used = 4 * (t->in_f / 4);
        if (used > 0)
            QTRY_CUDA(cudaMemcpy2DAsync(t->x.p, sizeof(float) * t->k_pad, x, sizeof(float) * t->in_f,
                                        sizeof(float) * used, (size_t)batch, kind_in(ptr_kind), st));
        xd = t->x.as<float>();
        if (ptr_kind == QMOE_PTR_HOST) {
            QTRY(grow(t->y, sizeof(float) * batch * t->out_f));
            yd = t->y.as<float>();
        }
    } else if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(grow(t->x, sizeof(float) * batch * t->in_f));
        QTRY(grow(t->y, sizeof(float) * batch * t->out_f));
        QTRY_CUDA(cudaMemcpyAsync(t->x.p, x, sizeof(float) * batch * t->in_f,
                                  cudaMemcpyHostToDevice, st));
        xd = t->x.as<float>();
        yd = t->y.as<float>();
    }
    // one shared-style segment covering all rows: groups of kDecodeTok rows
    PermuteParams pp{};
    pp.topk_idx = nullptr;
    pp.T = batch;
    pp.K = 0;
    pp.e_begin = 0;
    pp.e_count = 1;
    pp.chunk = kDecodeTok;
    pp.shared_count = batch;
    pp.seg_off = t->ngroups.as<int32_t>() + 2;   // [2..3]: the one segment's offsets
    pp.assign_pos = nullptr;
    pp.pos_tok = nullptr;
    pp.groups = t->groups.as<int4>();
    pp.n_groups = t->ngroups.as<int32_t>();
    QTRY_CUDA(launch_permute(pp, st));

    QgemvParams q{};
    q.groups = t->groups.as<int4>();
    q.n_groups = t->ngroups.as<int32_t>();
    q.rows = 0;
    q.K = (int)t->k_pad;
    q.ws[0] = t->w;
    q.ss[0] = t->s;
    q.rows_s = (int)t->out_f;
    q.K_s = (int)t->k_pad;
    q.act = xd;
    q.act_dtype = 0;
    q.act_ld = padded ? t->k_pad : t->in_f;
    q.pos_tok = nullptr;
    q.shared_base = 0;
    q.out = yd;
    q.out_ld = t->out_f;
    QTRY_CUDA(launch_qgemv(1, q, t->grid, st));
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY_CUDA(cudaMemcpyAsync(y, yd, sizeof(float) * batch * t->out_f,
                                  cudaMemcpyDeviceToHost, st));
        QTRY_CUDA(cudaStreamSynchronize(st));
    }
    return QMOE_OK;
}

// ---------------------------------------------------------------------------
// packer
// ---------------------------------------------------------------------------

// Host rows go through the device in chunks of at most this many bytes of w.
constexpr size_t kPackChunkBytes = size_t(256) << 20;

static int pack_chunks(qmoe_ctx *ctx, const float *w, int64_t out_f, int64_t in_f, float *scales,
                       int scales_given, uint8_t *packed, int sm_count, DevBuf &wd, DevBuf &sd,
                       DevBuf &pd) {
    cudaStream_t st = ctx->stream;
    const size_t row_bytes = sizeof(float) * (size_t)in_f;
    int64_t chunk = (int64_t)(kPackChunkBytes / row_bytes);
    if (chunk < 1) chunk = 1;
    if (chunk > out_f) chunk = out_f;
    QTRY(grow(wd, row_bytes * chunk));
    QTRY(grow(sd, sizeof(float) * chunk));
    QTRY(grow(pd, (size_t)(in_f / 4) * chunk));
    for (int64_t r0 = 0; r0 < out_f; r0 += chunk) {
        const int64_t n = out_f - r0 < chunk ? out_f - r0 : chunk;
        QTRY_CUDA(cudaMemcpyAsync(wd.p, w + r0 * in_f, row_bytes * n, cudaMemcpyHostToDevice, st));
        if (scales_given)
            QTRY_CUDA(cudaMemcpyAsync(sd.p, scales + r0, sizeof(float) * n, cudaMemcpyHostToDevice, st));
        PackParams pp{wd.as<float>(), n, in_f, sd.as<float>(), scales_given, pd.as<uint8_t>(), error_flag()};
        QTRY_CUDA(launch_pack_rows(pp, sm_count, st));
        QTRY_CUDA(cudaMemcpyAsync(packed + r0 * (in_f / 4), pd.p, (size_t)(in_f / 4) * n,
                                  cudaMemcpyDeviceToHost, st));
        if (!scales_given)
            QTRY_CUDA(cudaMemcpyAsync(scales + r0, sd.p, sizeof(float) * n, cudaMemcpyDeviceToHost, st));
        // the staging buffers are reused by the next chunk
        QTRY(sync_and_check(st));
    }
    return QMOE_OK;
}

int qmoe_quantize_pack(qmoe_ctx *ctx, const float *w, int64_t out_features, int64_t in_features,
                       float *scales, int scales_given, uint8_t *packed, int ptr_kind) {
    if (!ctx) return fail(QMOE_ERR_INVALID, "ctx is NULL");
    QTRY(check_ptr_kind(ptr_kind));
    if (out_features < 0) return fail(QMOE_ERR_INVALID, "out_features < 0");
    // quantize.py:26 asserts in_features % 4 == 0
    if (in_features <= 0 || in_features % 4)
        return fail(QMOE_ERR_INVALID, "in_features (%lld) must be a positive multiple of 4",
                    (long long)in_features);
    if (out_features == 0) return QMOE_OK;
    if (!w || !scales || !packed) return fail(QMOE_ERR_INVALID, "NULL argument");
    QTRY(check_align(w, ptr_kind, "w"));
    DeviceGuard g(ctx->device);
    int sm_count = 0;
    QTRY_CUDA(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, ctx->device));
    if (ptr_kind == QMOE_PTR_DEVICE) {
        PackParams pp{w, out_features, in_features, scales, scales_given, packed, error_flag()};
        QTRY_CUDA(launch_pack_rows(pp, sm_count, ctx->stream));
        return QMOE_OK;
    }
    DevBuf wd, sd, pd;
    const int rc = pack_chunks(ctx, w, out_features, in_features, scales, scales_given, packed, sm_count,
                               wd, sd, pd);
    if (rc != QMOE_OK) cudaStreamSynchronize(ctx->stream);   // no copy in flight from freed memory
    release(wd);
    release(sd);
    release(pd);
    return rc;
}

// ---------------------------------------------------------------------------
// layer
// ---------------------------------------------------------------------------

static int validate_cfg(const qmoe_moe_config *c) {
    if (!c) return fail(QMOE_ERR_INVALID, "cfg is NULL");
    if (c->num_experts < 1 || c->top_k < 1 || c->top_k > c->num_experts)
        return fail(QMOE_ERR_INVALID, "need 1 <= top_k (%d) <= num_experts (%d)",
                    c->top_k, c->num_experts);
    if (c->top_k > 64) return fail(QMOE_ERR_UNSUPPORTED, "top_k > 64");
    if (c->num_experts > 4096) return fail(QMOE_ERR_UNSUPPORTED, "num_experts > 4096");
    if (c->hidden_dim <= 0 || c->hidden_dim % 64 || c->intermediate_dim <= 0 ||
        c->intermediate_dim % 64)
        return fail(QMOE_ERR_INVALID,
                    "hidden_dim (%d) and intermediate_dim (%d) must be positive multiples of 64",
                    c->hidden_dim, c->intermediate_dim);
    if (c->shared_intermediate_dim < 0 || c->shared_intermediate_dim % 64)
        return fail(QMOE_ERR_INVALID, "shared_intermediate_dim must be 0 or a multiple of 64");
    // the decode GEMV sums 64 x code x int8 limb over K in int32: K <= 65536
    if (c->hidden_dim > 65536 || c->intermediate_dim > 65536 || c->shared_intermediate_dim > 65536)
        return fail(QMOE_ERR_UNSUPPORTED, "hidden and intermediate dims above 65536");
    if (c->scoring != QMOE_SCORING_SOFTMAX && c->scoring != QMOE_SCORING_SIGMOID)
        return fail(QMOE_ERR_INVALID, "unknown scoring %d", c->scoring);
    const int G = c->n_group;
    if (G < 1 || G > 64 || c->num_experts % G)
        return fail(QMOE_ERR_INVALID, "n_group (%d) must divide num_experts and be <= 64", G);
    if (c->topk_group < 1 || c->topk_group > G)
        return fail(QMOE_ERR_INVALID, "need 1 <= topk_group <= n_group");
    if (c->top_k > c->topk_group * (c->num_experts / G))
        return fail(QMOE_ERR_INVALID, "top_k exceeds the experts of the kept groups");
    if (c->has_bias && c->scoring != QMOE_SCORING_SIGMOID)
        return fail(QMOE_ERR_INVALID, "a selection bias requires sigmoid scoring");
    if (c->reserved != 0) return fail(QMOE_ERR_INVALID, "reserved must be 0");
    return QMOE_OK;
}

int qmoe_layer_destroy(qmoe_layer *L) {
    if (!L) return QMOE_OK;
    DeviceGuard g(L->ctx->device);
    for (int m = 0; m < 3; ++m) {
        if (L->w[m]) cudaFree(L->w[m]);
        if (L->s[m]) cudaFree(L->s[m]);
        if (L->ws[m]) cudaFree(L->ws[m]);
        if (L->ss[m]) cudaFree(L->ss[m]);
    }
    if (L->gate_w) cudaFree(L->gate_w);
    if (L->gate_t) cudaFree(L->gate_t);
    if (L->ln_w) cudaFree(L->ln_w);
    if (L->ln_b) cudaFree(L->ln_b);
    release(L->xn);
    if (L->bias) cudaFree(L->bias);
    for (cudaEvent_t &e : L->ev)
        if (e) cudaEventDestroy(e);
    DevBuf *bufs[] = {&L->topk_idx, &L->topk_w, &L->assign_pos, &L->pos_tok,
                      &L->seg_off, &L->groups, &L->ngroups, &L->h, &L->y,
                      &L->x_in, &L->io_out, &L->user_idx, &L->user_w,
                      &L->xq1, &L->meta1, &L->xq2, &L->meta2, &L->router_scratch,
                      &L->xg, &L->hb, &L->front_counter, &L->gemv_sched};
    for (DevBuf *b : bufs) release(*b);
    if (L->fg.exec) cudaGraphExecDestroy(L->fg.exec);
    delete L;
    return QMOE_OK;
}

static int layer_alloc_copy(void **dst, const void *src, size_t bytes, int kind,
                            cudaStream_t st) {
    QTRY_CUDA(cudaMalloc(dst, bytes));
    QTRY_CUDA(cudaMemcpyAsync(*dst, src, bytes, kind_in(kind), st));
    return QMOE_OK;
}

static int shared_pass(qmoe_layer *L, const void *x, int dtype, int64_t T, void *out, int accumulate,
                       int ptr_kind);

// A layer without routed experts: the expert-side tensor maps are made over
// the shared expert's matrices (valid descriptors that no routed item ever
// reads, since no routed segment exists), or left unset without a shared
// expert (the forward then writes zeros and launches nothing).
static int empty_layer_maps(qmoe_layer *L) {
    const qmoe_moe_config &c = L->cfg;
    int dev = 0;
    cudaGetDevice(&dev);
    QTRY_CUDA(cudaDeviceGetAttribute(&L->sm_count, cudaDevAttrMultiProcessorCount, dev));
    int coop = 0;
    QTRY_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
    L->coop = coop != 0;
    const int64_t H = c.hidden_dim, Is = c.shared_intermediate_dim;
    const int64_t Imx = Is > c.intermediate_dim ? Is : c.intermediate_dim;
    L->kp1 = (int)((H + 255) / 256 * 256);       // limb strides (the scratch is laid out even
    L->kp2 = (int)((Imx + 255) / 256 * 256);     // when no kernel will read it)
    if (!L->has_shared) return QMOE_OK;
    const int64_t srows[3] = {Is, Is, H}, skin[3] = {H, H, Is};
    for (int m = 0; m < 3; ++m) {
        if (!make_tmap_u8(&L->tm_ws[m], L->ws[m], (uint64_t)(skin[m] / 4), (uint64_t)srows[m], 64, 128,
                          CU_TENSOR_MAP_SWIZZLE_64B))
            return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for shared matrix %d", m);
        L->tm_ws3[m] = L->tm_ws[m];
        if (skin[m] / 256 >= 2 &&
            !make_tmap_u8_3d(&L->tm_ws3[m], L->ws[m], 64, (uint64_t)srows[m], (uint64_t)(skin[m] / 256),
                             (uint64_t)(skin[m] / 4), 64, 64, 128, 2, CU_TENSOR_MAP_SWIZZLE_64B))
            return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed for shared matrix %d", m);
        L->tm_w[m] = L->tm_ws[m];
        L->tm_w3[m] = L->tm_ws3[m];
    }
    L->prefill_ok = H % 128 == 0 && Is % 64 == 0;
    if (L->prefill_ok)
        for (int m = 0; m < 2; ++m) {
            if (!make_tmap_u8(&L->tm_pws[m], L->ws[m], (uint64_t)(H / 4), (uint64_t)Is, 64, 64,
                              CU_TENSOR_MAP_SWIZZLE_64B))
                return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for shared matrix %d", m);
            L->tm_pw[m] = L->tm_pws[m];
        }
    if (qgemv_imma_smem_bytes(L->kp1, 1) > 227 * 1024 || qgemv_imma_smem_bytes(L->kp2, 1) > 227 * 1024)
        return fail(QMOE_ERR_UNSUPPORTED, "hidden or shared intermediate dim too large for the GEMV tiles");
    L->grid0 = qgemv_max_grid(0, (int)H);
    L->grid1 = qgemv_max_grid(1, (int)Is);
    return QMOE_OK;
}

static int layer_create_impl(qmoe_layer *L, const float *gate_weight, const float *bias,
                             const qmoe_expert_weights *experts,
                             const qmoe_expert_weights *shared, int ptr_kind) {
    const qmoe_moe_config &c = L->cfg;
    cudaStream_t st = L->ctx->stream;
    const int64_t E = c.num_experts, H = c.hidden_dim, I = c.intermediate_dim;
    const int64_t El = L->e_count;
    if (El > 0) {
        QTRY(layer_alloc_copy((void **)&L->gate_w, gate_weight, sizeof(float) * E * H, ptr_kind, st));
        if (E > 64) {
            const int ld = gate_t_ld((int)E);
            QTRY_CUDA(cudaMalloc((void **)&L->gate_t, sizeof(float) * (size_t)ld * H));
            QTRY_CUDA(launch_transpose_gate(L->gate_w, (int)E, (int)H, L->gate_t, ld, st));
        }
        if (c.has_bias)
            QTRY(layer_alloc_copy((void **)&L->bias, bias, sizeof(float) * E, ptr_kind, st));
    }
    const int64_t rows[3] = {I, I, H}, kin[3] = {H, H, I};
    for (int m = 0; m < 3 && El > 0; ++m) {
        const size_t wb = (size_t)rows[m] * (kin[m] / 4);
        QTRY_CUDA(cudaMalloc((void **)&L->w[m], wb * El));
        QTRY_CUDA(cudaMalloc((void **)&L->s[m], sizeof(float) * rows[m] * El));
        for (int64_t e = 0; e < El; ++e) {
            const qmoe_expert_weights &x = experts[e];
            const uint8_t *pk = m == 0 ? x.gate_packed : m == 1 ? x.up_packed : x.down_packed;
            const float *sc = m == 0 ? x.gate_scales : m == 1 ? x.up_scales : x.down_scales;
            if (!pk || !sc) return fail(QMOE_ERR_INVALID, "expert %lld has a NULL weight", (long long)e);
            QTRY_CUDA(cudaMemcpyAsync(L->w[m] + e * wb, pk, wb, kind_in(ptr_kind), st));
            QTRY_CUDA(cudaMemcpyAsync(L->s[m] + e * rows[m], sc, sizeof(float) * rows[m],
                                      kind_in(ptr_kind), st));
        }
    }
    if (L->has_shared) {
        const int64_t Is = c.shared_intermediate_dim;
        const int64_t srows[3] = {Is, Is, H}, skin[3] = {H, H, Is};
        for (int m = 0; m < 3; ++m) {
            const uint8_t *pk = m == 0 ? shared->gate_packed : m == 1 ? shared->up_packed : shared->down_packed;
            const float *sc = m == 0 ? shared->gate_scales : m == 1 ? shared->up_scales : shared->down_scales;
            if (!pk || !sc) return fail(QMOE_ERR_INVALID, "shared expert has a NULL weight");
            QTRY(layer_alloc_copy((void **)&L->ws[m], pk, (size_t)srows[m] * (skin[m] / 4), ptr_kind, st));
            QTRY(layer_alloc_copy((void **)&L->ss[m], sc, sizeof(float) * srows[m], ptr_kind, st));
        }
    }
    QTRY_CUDA(cudaStreamSynchronize(st));
    if (El == 0) return empty_layer_maps(L);
    // TMA maps: rows of 64-byte boxes, 128 rows per box, 64-byte swizzle
    for (int m = 0; m < 3; ++m) {
        if (!make_tmap_u8(&L->tm_w[m], L->w[m], (uint64_t)(kin[m] / 4), (uint64_t)(rows[m] * El),
                          64, 128, CU_TENSOR_MAP_SWIZZLE_64B))
            return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for expert matrix %d", m);
        L->tm_ws[m] = L->tm_w[m];
    }
    if (L->has_shared) {
        const int64_t Is = c.shared_intermediate_dim;
        const int64_t srows[3] = {Is, Is, H}, skin[3] = {H, H, Is};
        for (int m = 0; m < 3; ++m)
            if (!make_tmap_u8(&L->tm_ws[m], L->ws[m], (uint64_t)(skin[m] / 4), (uint64_t)srows[m],
                              64, 128, CU_TENSOR_MAP_SWIZZLE_64B))
                return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for shared matrix %d", m);
    }
    // 3-D views of the matrices for the decode GEMV (rows of whole 64-byte
    // chunks; a stage that reaches a ragged row end uses the 2-D map)
    for (int m = 0; m < 3; ++m) {
        L->tm_w3[m] = L->tm_w[m];
        if (kin[m] / 256 >= 2 &&
            !make_tmap_u8_3d(&L->tm_w3[m], L->w[m], 64, (uint64_t)(rows[m] * El),
                             (uint64_t)(kin[m] / 256), (uint64_t)(kin[m] / 4), 64, 64, 128, 2,
                             CU_TENSOR_MAP_SWIZZLE_64B))
            return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed for expert matrix %d", m);
        L->tm_ws3[m] = L->tm_w3[m];
    }
    if (L->has_shared) {
        const int64_t Is = c.shared_intermediate_dim;
        const int64_t srows[3] = {Is, Is, H}, skin[3] = {H, H, Is};
        for (int m = 0; m < 3; ++m) {
            L->tm_ws3[m] = L->tm_ws[m];
            if (skin[m] / 256 >= 2 &&
                !make_tmap_u8_3d(&L->tm_ws3[m], L->ws[m], 64, (uint64_t)srows[m],
                                 (uint64_t)(skin[m] / 256), (uint64_t)(skin[m] / 4), 64, 64, 128, 2,
                                 CU_TENSOR_MAP_SWIZZLE_64B))
                return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed for shared matrix %d", m);
        }
    }
    // prefill kernels: K blocks of 64 everywhere, down tiles of 128 rows
    L->prefill_ok = H % 128 == 0 && I % 64 == 0 &&
                    (!L->has_shared || c.shared_intermediate_dim % 64 == 0);
    if (L->prefill_ok) {
        for (int m = 0; m < 2; ++m) {
            if (!make_tmap_u8(&L->tm_pw[m], L->w[m], (uint64_t)(H / 4), (uint64_t)(I * El), 64, 64,
                              CU_TENSOR_MAP_SWIZZLE_64B))
                return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for expert matrix %d", m);
            L->tm_pws[m] = L->tm_pw[m];
            if (L->has_shared &&
                !make_tmap_u8(&L->tm_pws[m], L->ws[m], (uint64_t)(H / 4),
                              (uint64_t)c.shared_intermediate_dim, 64, 64, CU_TENSOR_MAP_SWIZZLE_64B))
                return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for shared matrix %d", m);
        }
    }
    {
        int dev = 0;
        cudaGetDevice(&dev);
        QTRY_CUDA(cudaDeviceGetAttribute(&L->sm_count, cudaDevAttrMultiProcessorCount, dev));
        int coop = 0;
        QTRY_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
        L->coop = coop != 0;
        const int64_t Imx = c.shared_intermediate_dim > I ? c.shared_intermediate_dim : I;
        L->kp1 = (int)((H + 255) / 256 * 256);
        L->kp2 = (int)((Imx + 255) / 256 * 256);
        if (qgemv_imma_smem_bytes(L->kp1, 1) > 227 * 1024 || qgemv_imma_smem_bytes(L->kp2, 1) > 227 * 1024)
            return fail(QMOE_ERR_UNSUPPORTED, "hidden or intermediate dim too large for the GEMV tiles");
    }
    const int kmax0 = (int)H;
    const int kmax1 = (int)(c.shared_intermediate_dim > I ? c.shared_intermediate_dim : I);
    L->grid0 = qgemv_max_grid(0, kmax0);
    L->grid1 = qgemv_max_grid(1, kmax1);
    return QMOE_OK;
}

int qmoe_layer_create(qmoe_ctx *ctx, const qmoe_moe_config *cfg, const float *gate_weight,
                      const float *bias, const qmoe_expert_weights *experts,
                      int32_t expert_begin, int32_t expert_count,
                      const qmoe_expert_weights *shared, int ptr_kind, qmoe_layer **out) {
    if (!ctx || !out) return fail(QMOE_ERR_INVALID, "NULL argument");
    *out = nullptr;
    QTRY(check_ptr_kind(ptr_kind));
    QTRY(validate_cfg(cfg));
    // expert_count 0: a layer without routed experts (qmoe-rs's empty
    // `experts`, src/moe.rs:46-48, e.g. a flattened layer loaded as its
    // shared FFN alone, src/loader.rs:452-456); its gate is never read
    if (expert_count > 0 && !gate_weight) return fail(QMOE_ERR_INVALID, "gate_weight is NULL");
    if (expert_count > 0 && cfg->has_bias && !bias)
        return fail(QMOE_ERR_INVALID, "has_bias set but bias is NULL");
    if (expert_begin < 0 || expert_count < 0 || expert_begin + expert_count > cfg->num_experts)
        return fail(QMOE_ERR_INVALID, "expert range [%d, %d) outside [0, %d)", expert_begin,
                    expert_begin + expert_count, cfg->num_experts);
    if (expert_count > 768) return fail(QMOE_ERR_UNSUPPORTED, "more than 768 local experts");
    if (expert_count > 0 && !experts) return fail(QMOE_ERR_INVALID, "experts is NULL");
    if ((cfg->shared_intermediate_dim > 0) != (shared != nullptr))
        return fail(QMOE_ERR_INVALID,
                    "shared must be given exactly when shared_intermediate_dim > 0");
    DeviceGuard g(ctx->device);
    qmoe_layer *L = new (std::nothrow) qmoe_layer;
    if (!L) return fail(QMOE_ERR_NOMEM, "host allocation failed");
    L->ctx = ctx;
    L->cfg = *cfg;
    L->e_begin = expert_begin;
    L->e_count = expert_count;
    L->has_shared = shared != nullptr;
    int rc = layer_create_impl(L, gate_weight, bias, experts, shared, ptr_kind);
    if (rc != QMOE_OK) {
        std::string msg = g_err;
        qmoe_layer_destroy(L);
        g_err = msg;
        return rc;
    }
    *out = L;
    return QMOE_OK;
}

static int layer_reserve(qmoe_layer *L, int64_t T) {
    if (T <= L->cap) return QMOE_OK;
    const qmoe_moe_config &c = L->cfg;
    const int64_t K = c.top_k, H = c.hidden_dim;
    const int64_t Imax = c.shared_intermediate_dim > c.intermediate_dim ? c.shared_intermediate_dim
                                                                        : c.intermediate_dim;
    const int64_t TK = T * K;
    const int64_t npos = TK + T;                 // routed + shared positions
    const int64_t ngroups = TK + L->e_count + T + 2;
    QTRY(grow(L->topk_idx, sizeof(int32_t) * TK));
    QTRY(grow(L->topk_w, sizeof(float) * TK));
    QTRY(grow(L->assign_pos, sizeof(int32_t) * TK));
    QTRY(grow(L->pos_tok, sizeof(int32_t) * (TK + 1)));
    QTRY(grow(L->seg_off, sizeof(int32_t) * (L->e_count + 1)));
    QTRY(grow(L->groups, sizeof(int4) * ngroups));
    QTRY(grow(L->ngroups, sizeof(int32_t) * 2));
    QTRY(grow(L->h, sizeof(float) * npos * Imax));
    QTRY(grow(L->y, sizeof(float) * npos * H));
    QTRY(grow(L->xq1, (size_t)npos * 3 * L->kp1));
    QTRY(grow(L->xq2, (size_t)npos * 3 * L->kp2));
    QTRY(grow(L->meta1, sizeof(longlong2) * npos));
    QTRY(grow(L->meta2, sizeof(longlong2) * npos));
    QTRY(grow(L->router_scratch, sizeof(float) * router_scratch_floats(T, c.hidden_dim, c.num_experts)));
    if (!L->front_counter.p) {
        QTRY(grow(L->front_counter, sizeof(int32_t)));
        QTRY_CUDA(cudaMemsetAsync(L->front_counter.p, 0, sizeof(int32_t), L->ctx->stream));
    }
    if (!L->gemv_sched.p) {
        QTRY(grow(L->gemv_sched, 8 * sizeof(int32_t)));
        QTRY_CUDA(cudaMemsetAsync(L->gemv_sched.p, 0, 8 * sizeof(int32_t), L->ctx->stream));
    }
    if (L->prefill_ok) {
        QTRY(grow(L->xg, 2 * (size_t)npos * H));
        QTRY(grow(L->hb, 2 * (size_t)npos * Imax));
        // 3-D views [K block of 128 bytes][row][K block index]: one box =
        // two K blocks of 128, 192 or 256 rows, i.e. one copy per GEMM stage
        auto rows3d = [&](CUtensorMap *tm, void *base, uint64_t cols, uint32_t box_rows) {
            return make_tmap_u8_3d(tm, base, 128, (uint64_t)npos, cols / 64, 2 * cols, 128, 128, box_rows, 2,
                                   CU_TENSOR_MAP_SWIZZLE_128B);
        };
        if (!rows3d(&L->tm_xg, L->xg.p, (uint64_t)H, kPrefillTile) ||
            !rows3d(&L->tm_xg2, L->xg.p, (uint64_t)H, kPrefillTile / 2) ||
            !rows3d(&L->tm_xg3, L->xg.p, (uint64_t)H, kPrefillTile * 3 / 4) ||
            !rows3d(&L->tm_hb, L->hb.p, (uint64_t)Imax, kPrefillTile) ||
            !rows3d(&L->tm_hb2, L->hb.p, (uint64_t)Imax, kPrefillTile / 2) ||
            !rows3d(&L->tm_hb3, L->hb.p, (uint64_t)Imax, kPrefillTile * 3 / 4))
            return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the prefill rows");
    }
    if (!make_tmap_u8(&L->tm_xq1, L->xq1.p, (uint64_t)L->kp1, (uint64_t)(npos * 3), 128, 16,
                      CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_u8(&L->tm_xq2, L->xq2.p, (uint64_t)L->kp2, (uint64_t)(npos * 3), 128, 16,
                      CU_TENSOR_MAP_SWIZZLE_128B))
        return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the limb scratch");
    // decode GEMV stage view: (128-byte block x, block of a 256-code group,
    // limb row, group); the box lands as [group][row][block] lines, so the
    // 128-byte swizzle phase (2 row + block) differs for the four (row pair,
    // block) combinations a quarter-warp reads
    {
        const uint64_t d1[4] = {128, 2, (uint64_t)(npos * 3), (uint64_t)(L->kp1 / 256)};
        const uint64_t d2[4] = {128, 2, (uint64_t)(npos * 3), (uint64_t)(L->kp2 / 256)};
        const uint64_t s1[3] = {128, (uint64_t)L->kp1, 256}, s2[3] = {128, (uint64_t)L->kp2, 256};
        const uint32_t box[4] = {128, 2, 16, 2};
        if (!make_tmap_u8_4d(&L->tm_xq1_3, L->xq1.p, d1, s1, box, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !make_tmap_u8_4d(&L->tm_xq2_3, L->xq2.p, d2, s2, box, CU_TENSOR_MAP_SWIZZLE_128B))
            return fail(QMOE_ERR_CUDA, "cuTensorMapEncodeTiled (4-D) failed for the limb scratch");
    }
    L->cap = T;
    return QMOE_OK;
}

int qmoe_layer_reserve(qmoe_layer *L, int64_t max_tokens) {
    if (!L || max_tokens < 0) return fail(QMOE_ERR_INVALID, "bad argument");
    DeviceGuard g(L->ctx->device);
    return layer_reserve(L, max_tokens);
}

// Stage a host input in device memory (device inputs pass through).
// The device address of page-locked host memory that kernels may access in
// place, or nullptr for other memory.
static const void *mapped_host(const void *p) {
    cudaPointerAttributes at{};
    if (!p || cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

static int stage_in(DevBuf &buf, const void *src, size_t bytes, int ptr_kind,
                    cudaStream_t st, const void **dev) {
    if (ptr_kind == QMOE_PTR_DEVICE) {
        *dev = src;
        return QMOE_OK;
    }
    QTRY(grow(buf, bytes));
    QTRY_CUDA(cudaMemcpyAsync(buf.p, src, bytes, cudaMemcpyHostToDevice, st));
    *dev = buf.p;
    return QMOE_OK;
}

static RouterParams router_params(qmoe_layer *L, const void *xd, int dtype, int64_t T) {
    const qmoe_moe_config &c = L->cfg;
    RouterParams rp{};
    rp.x = xd;
    rp.dtype = dtype;
    rp.T = T;
    rp.H = c.hidden_dim;
    rp.E = c.num_experts;
    rp.K = c.top_k;
    rp.gate_w = L->gate_w;
    rp.gate_t = L->gate_t;
    rp.gate_t_ld = gate_t_ld(c.num_experts);
    rp.bias = L->bias;
    rp.scoring = c.scoring;
    rp.n_group = c.n_group;
    rp.topk_group = c.topk_group;
    rp.norm_topk = c.norm_topk_prob;
    rp.routed_scale = c.routed_scaling_factor;
    rp.topk_idx = L->topk_idx.as<int32_t>();
    rp.topk_w = L->topk_w.as<float>();
    rp.scratch = L->router_scratch.as<float>();
    return rp;
}

static int run_router(qmoe_layer *L, const void *xd, int dtype, int64_t T) {
    const RouterParams rp = router_params(L, xd, dtype, T);
    mark(L, 0);
    QTRY_CUDA(launch_router(rp, nullptr, L->ctx->stream));
    return QMOE_OK;
}

// Expert products on the tcgen05 bf16 GEMM (large bf16 batches) or on the
// exact integer-limb GEMV.  Fails for a forced prefill path it cannot take.
static int choose_prefill(qmoe_layer *L, int dtype, int64_t T, int K, bool *prefill) {
    *prefill = false;
    if (L->path == QMOE_PATH_PREFILL) {
        if (!L->prefill_ok || dtype != QMOE_DTYPE_BF16)
            return fail(QMOE_ERR_UNSUPPORTED,
                        "the prefill path needs bf16 activations, hidden %% 128 == 0 and "
                        "intermediate dims %% 64 == 0");
        *prefill = true;
    } else if (L->path == QMOE_PATH_AUTO && L->prefill_ok && dtype == QMOE_DTYPE_BF16) {
        const int64_t per_seg = K > 0 ? T * K / (L->e_count > 0 ? L->e_count : 1) : T;
        *prefill = per_seg >= kPrefillMinRows;
    }
    return QMOE_OK;
}

// Small batches of a full layer: the router with the permute in the last
// CTA of its selection kernel.
static int run_front(qmoe_layer *L, const void *xd, int dtype, int64_t T, bool prefill,
                     void *x_copy = nullptr) {
    const RouterParams rp = router_params(L, xd, dtype, T);
    FrontParams f{};
    f.x_copy = x_copy;
    f.counter = L->front_counter.as<int32_t>();
    f.chunk = prefill ? kPrefillTile : kDecodeTok;
    f.shared_count = L->has_shared ? T : 0;
    f.seg_off = L->seg_off.as<int32_t>();
    f.assign_pos = L->assign_pos.as<int32_t>();
    f.pos_tok = L->pos_tok.as<int32_t>();
    f.groups = L->groups.as<int4>();
    f.n_groups = L->ngroups.as<int32_t>();
    mark(L, 0);
    if (front_cluster_ok(T, rp.H, rp.E, rp.K))
        QTRY_CUDA(launch_front_cluster(rp, f, L->ctx->stream));
    else
        QTRY_CUDA(launch_router(rp, &f, L->ctx->stream));
    return QMOE_OK;
}

// What one expert pass computes over its T rows: routed assignments
// (topk ids relative to e_begin, row stride topk_ld, -1 = skip) and the
// shared expert over rows shared_row0 .. shared_row0 + shared_count - 1.
struct ExpertsArgs {
    const int32_t *topk_idx = nullptr;
    const float *topk_w = nullptr;
    int topk_ld = 0;
    int e_begin = 0;
    int64_t shared_row0 = 0, shared_count = 0;
    bool permuted = false;  // segments and work list already built (run_front)
    EpPeerDev *ep_ret = nullptr;  // expert parallel: the down GEMV returns the received
                                  // rows' partial sums straight to their origin ranks
    bool *returned = nullptr;     // set when it did (else the caller runs the return kernel)
    bool wait_dispatch = false;   // the permute first waits for the peers' rows (ep_ret's flags)
    const void *residual = nullptr;  // block forward: the residual stream, added by the combine
};

// Weighted sum of each token's expert rows in ascending expert order, plus
// the shared expert's row (src/moe.rs:117-125, src/model.rs:386-389).
static CombineParams combine_params(qmoe_layer *L, int64_t T, const ExpertsArgs &a, void *outd, int dtype,
                                    int accumulate) {
    const qmoe_moe_config &c = L->cfg;
    CombineParams cp{};
    cp.y = L->y.as<float>();
    cp.assign_pos = L->assign_pos.as<int32_t>();
    cp.topk_idx = a.topk_idx;
    cp.topk_w = a.topk_w;
    cp.T = T;
    cp.K = c.top_k;
    cp.topk_ld = a.topk_ld;
    cp.H = c.hidden_dim;
    cp.y_shared = a.shared_count ? L->y.as<float>() + T * c.top_k * c.hidden_dim : nullptr;
    cp.shared_row0 = a.shared_row0;
    cp.shared_count = a.shared_count;
    cp.accumulate = accumulate;
    cp.residual = a.residual;
    cp.out = outd;
    cp.out_dtype = dtype;
    return cp;
}

static int run_combine(qmoe_layer *L, int64_t T, const ExpertsArgs &a, void *outd, int dtype,
                       int accumulate) {
    CombineParams cp = combine_params(L, T, a, outd, dtype, accumulate);
    if (a.ep_ret) {
        // received rows go straight back to their origin ranks
        cp.ep_ret = 1;
        cp.ret = *a.ep_ret;
        *a.returned = true;
    }
    mark(L, 6);
    QTRY_CUDA(launch_combine(cp, L->ctx->stream));
    mark(L, 7);
    return QMOE_OK;
}

// Prefill expert products: gather the bf16 rows of every position, gate/up
// GEMM with SwiGLU into bf16 rows, down GEMM into f32 rows of y.
static int run_prefill(qmoe_layer *L, const void *xd, int64_t T, int64_t npos, const ExpertsArgs &a,
                       const int32_t *n_valid, int *err) {
    const bool with_shared = a.shared_count > 0;
    const qmoe_moe_config &c = L->cfg;
    cudaStream_t st = L->ctx->stream;
    const int64_t TK = T * c.top_k;
    const int64_t Imax = c.shared_intermediate_dim > c.intermediate_dim ? c.shared_intermediate_dim
                                                                        : c.intermediate_dim;
    GatherParams gp{};
    gp.x = xd;
    gp.H = c.hidden_dim;
    gp.pos_tok = L->pos_tok.as<int32_t>();
    gp.n_valid = n_valid;
    gp.shared_base = TK;
    gp.shared_row0 = a.shared_row0;
    gp.npos = npos;
    gp.xg = L->xg.p;
    mark(L, 2);
    QTRY_CUDA(launch_gather_bf16(gp, st));
    mark(L, 3);

    QgemmMaps m0;
    m0.w0 = L->tm_pw[0];
    m0.w1 = L->tm_pw[1];
    m0.s0 = L->tm_pws[0];
    m0.s1 = L->tm_pws[1];
    m0.b = L->tm_xg;
    m0.b2 = L->tm_xg2;
    m0.b3 = L->tm_xg3;
    QgemmParams g0{};
    g0.groups = L->groups.as<int4>();
    g0.n_groups = L->ngroups.as<int32_t>();
    g0.rows = c.intermediate_dim;
    g0.K = c.hidden_dim;
    g0.rows_s = with_shared ? c.shared_intermediate_dim : 0;
    g0.K_s = c.hidden_dim;
    g0.s[0] = L->s[0];
    g0.s[1] = L->s[1];
    g0.s_stride = c.intermediate_dim;
    g0.ss[0] = L->ss[0];
    g0.ss[1] = L->ss[1];
    g0.out = L->hb.p;
    g0.out_ld = Imax;
    g0.err = err;
    QTRY_CUDA(launch_qgemm_prefill(0, m0, g0, L->sm_count, st));
    mark(L, 4);
    mark(L, 5);

    QgemmMaps m1;
    m1.w0 = m1.w1 = L->tm_w[2];
    m1.s0 = m1.s1 = L->tm_ws[2];
    m1.b = L->tm_hb;
    m1.b2 = L->tm_hb2;
    m1.b3 = L->tm_hb3;
    QgemmParams g1{};
    g1.groups = g0.groups;
    g1.n_groups = g0.n_groups;
    g1.rows = c.hidden_dim;
    g1.K = c.intermediate_dim;
    g1.rows_s = with_shared ? c.hidden_dim : 0;
    g1.K_s = with_shared ? c.shared_intermediate_dim : c.intermediate_dim;
    g1.s[0] = g1.s[1] = L->s[2];
    g1.s_stride = c.hidden_dim;
    g1.ss[0] = g1.ss[1] = L->ss[2];
    g1.out = L->y.p;
    g1.out_ld = c.hidden_dim;
    g1.err = err;
    QTRY_CUDA(launch_qgemm_prefill(1, m1, g1, L->sm_count, st));
    return QMOE_OK;
}

static int run_experts(qmoe_layer *L, const void *xd, int dtype, int64_t T, const ExpertsArgs &a,
                       void *outd, int accumulate) {
    const qmoe_moe_config &c = L->cfg;
    const bool with_shared = a.shared_count > 0;
    cudaStream_t st = L->ctx->stream;
    const int K = c.top_k;
    const int64_t TK = T * K;
    const int64_t Imax = c.shared_intermediate_dim > c.intermediate_dim ? c.shared_intermediate_dim
                                                                        : c.intermediate_dim;
    // expert products: tcgen05 bf16 GEMM for large bf16 batches, the exact
    // integer-limb GEMV otherwise
    bool prefill = false;
    QTRY(choose_prefill(L, dtype, T, K, &prefill));
    PermuteParams pp{};
    pp.topk_idx = a.topk_idx;
    pp.T = T;
    pp.K = K;
    pp.topk_ld = a.topk_ld;
    pp.e_begin = a.e_begin;
    pp.e_count = L->e_count;
    pp.chunk = prefill ? kPrefillTile : kDecodeTok;
    pp.shared_count = a.shared_count;
    pp.seg_off = L->seg_off.as<int32_t>();
    pp.assign_pos = L->assign_pos.as<int32_t>();
    pp.pos_tok = L->pos_tok.as<int32_t>();
    pp.groups = L->groups.as<int4>();
    pp.n_groups = L->ngroups.as<int32_t>();
    if (a.wait_dispatch && a.ep_ret) {
        pp.ep_wait = 1;
        pp.ep = *a.ep_ret;
    }
    mark(L, 1);
    if (!a.permuted) QTRY_CUDA(launch_permute(pp, st));

    const int64_t npos = TK + a.shared_count;
    const int32_t *n_valid = L->seg_off.as<int32_t>() + L->e_count;
    int *err = device_error_flag();
    if (prefill) {
        QTRY(run_prefill(L, xd, T, npos, a, n_valid, err));
        return run_combine(L, T, a, outd, dtype, accumulate);
    }

    // gate/up: activations -> limbs, then the tensor-core GEMV with SwiGLU
    QuantParams q1{};
    q1.act = xd;
    q1.dtype = dtype;
    q1.act_ld = c.hidden_dim;
    q1.pos_tok = L->pos_tok.as<int32_t>();
    q1.shared_base = TK;
    q1.shared_row0 = a.shared_row0;
    q1.n_valid = n_valid;
    q1.npos = npos;
    q1.K = c.hidden_dim;
    q1.K_s = c.hidden_dim;
    q1.Kp = L->kp1;
    q1.xq = L->xq1.as<int8_t>();
    q1.meta = L->meta1.as<longlong2>();
    // cooperative GEMVs: each makes its own limb rows in a first phase (no
    // limb kernels) and the down GEMV ends with the combine (no combine kernel)
    const bool coop = L->coop && L->path != QMOE_PATH_DECODE_SPLIT;
    mark(L, 2);
    if (!coop) QTRY_CUDA(launch_quant(q1, st));
    mark(L, 3);

    DecodeMaps m0;
    m0.a0 = L->tm_w[0];
    m0.a1 = L->tm_w[1];
    m0.s0 = L->tm_ws[0];
    m0.s1 = L->tm_ws[1];
    m0.b = L->tm_xq1;
    m0.a0_3 = L->tm_w3[0];
    m0.a1_3 = L->tm_w3[1];
    m0.s0_3 = L->tm_ws3[0];
    m0.s1_3 = L->tm_ws3[1];
    m0.b3 = L->tm_xq1_3;
    DecodeParams g0{};
    g0.groups = L->groups.as<int4>();
    g0.n_groups = L->ngroups.as<int32_t>();
    g0.rows = c.intermediate_dim;
    g0.K = c.hidden_dim;
    g0.rows_s = with_shared ? c.shared_intermediate_dim : 0;
    g0.K_s = c.hidden_dim;
    g0.s[0] = L->s[0];
    g0.s[1] = L->s[1];
    g0.s_stride = c.intermediate_dim;
    g0.ss[0] = L->ss[0];
    g0.ss[1] = L->ss[1];
    g0.meta = q1.meta;
    g0.kp_b = L->kp1;
    g0.b_buffers = qgemv_imma_buffers(L->kp1);
    g0.out = L->h.as<float>();
    g0.out_ld = Imax;
    g0.err = err;
    g0.sched = L->gemv_sched.as<int32_t>();
    if (coop) {
        g0.quant_in = 1;
        g0.q = q1;
    }
    QTRY_CUDA(launch_qgemv_imma(0, m0, g0, L->sm_count, st));

    // down: SwiGLU outputs -> limbs, then the tensor-core GEMV
    QuantParams q2 = q1;
    q2.act = L->h.p;
    q2.dtype = 0;
    q2.act_ld = Imax;
    q2.pos_tok = nullptr;
    q2.K = c.intermediate_dim;
    q2.K_s = with_shared ? c.shared_intermediate_dim : c.intermediate_dim;
    q2.Kp = L->kp2;
    q2.xq = L->xq2.as<int8_t>();
    q2.meta = L->meta2.as<longlong2>();
    mark(L, 4);
    if (!coop) QTRY_CUDA(launch_quant(q2, st));
    mark(L, 5);

    DecodeMaps m1;
    m1.a0 = m1.a1 = L->tm_w[2];
    m1.s0 = m1.s1 = L->tm_ws[2];
    m1.b = L->tm_xq2;
    m1.a0_3 = m1.a1_3 = L->tm_w3[2];
    m1.s0_3 = m1.s1_3 = L->tm_ws3[2];
    m1.b3 = L->tm_xq2_3;
    DecodeParams g1{};
    g1.groups = g0.groups;
    g1.n_groups = g0.n_groups;
    g1.rows = c.hidden_dim;
    g1.K = c.intermediate_dim;
    g1.rows_s = with_shared ? c.hidden_dim : 0;
    g1.K_s = with_shared ? c.shared_intermediate_dim : c.intermediate_dim;
    g1.s[0] = g1.s[1] = L->s[2];
    g1.s_stride = c.hidden_dim;
    g1.ss[0] = g1.ss[1] = L->ss[2];
    g1.meta = q2.meta;
    g1.kp_b = L->kp2;
    g1.b_buffers = qgemv_imma_buffers(L->kp2);
    g1.out = L->y.as<float>();
    g1.out_ld = c.hidden_dim;
    g1.err = err;
    g1.sched = L->gemv_sched.as<int32_t>() + 4;
    if (coop && c.top_k <= kCombineMaxK) {
        g1.quant_in = 1;
        g1.q = q2;
        g1.combine = 1;
        g1.c = combine_params(L, T, a, outd, dtype, accumulate);
        if (a.ep_ret) {
            // the combine tasks signal each destination once it has all
            // its rows (ep_signal.cuh)
            g1.ep_ret = 1;
            g1.ret = *a.ep_ret;
            *a.returned = true;
        }
        QTRY_CUDA(launch_qgemv_imma(1, m1, g1, L->sm_count, st));
        mark(L, 6);          // down GEMV with its limb and combine phases
        mark(L, 7);
        return QMOE_OK;
    }
    if (coop) {
        g1.quant_in = 1;
        g1.q = q2;
    }
    QTRY_CUDA(launch_qgemv_imma(1, m1, g1, L->sm_count, st));

    return run_combine(L, T, a, outd, dtype, accumulate);
}

static int finish_out(qmoe_layer *L, void *user, const void *dev, size_t bytes, int ptr_kind) {
    if (ptr_kind == QMOE_PTR_HOST && bytes)
        QTRY_CUDA(cudaMemcpyAsync(user, dev, bytes, cudaMemcpyDeviceToHost, L->ctx->stream));
    return QMOE_OK;
}

// A layer without routed experts: QMoELayer::forward returns zeros
// (src/moe.rs:46-48) and the block adds the shared expert's output
// (src/model.rs:386-389), so the result is the shared expert alone, or zeros
// without one.  No expert is selected: routing outputs read -1 / 0.
static int forward_without_experts(qmoe_layer *L, const void *x, int dtype, int64_t T, void *out,
                                   int32_t *topk_idx, float *topk_w, int ptr_kind) {
    cudaStream_t st = L->ctx->stream;
    const size_t xbytes = dtype_size(dtype) * T * L->cfg.hidden_dim;
    const size_t kb = sizeof(int32_t) * T * L->cfg.top_k;
    if (ptr_kind == QMOE_PTR_HOST) {
        if (topk_idx) std::memset(topk_idx, 0xff, kb);
        if (topk_w) std::memset(topk_w, 0, kb);
    } else {
        if (topk_idx) QTRY_CUDA(cudaMemsetAsync(topk_idx, 0xff, kb, st));
        if (topk_w) QTRY_CUDA(cudaMemsetAsync(topk_w, 0, kb, st));
    }
    if (L->has_shared) return shared_pass(L, x, dtype, T, out, 0, ptr_kind);
    if (ptr_kind == QMOE_PTR_HOST) {
        std::memset(out, 0, xbytes);
        return QMOE_OK;
    }
    QTRY_CUDA(cudaMemsetAsync(out, 0, xbytes, st));
    return QMOE_OK;
}

int qmoe_layer_forward(qmoe_layer *L, const void *x, int dtype, int64_t T, void *out,
                       int32_t *topk_idx, float *topk_w, int ptr_kind) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    QTRY(check_ptr_kind(ptr_kind));
    QTRY(check_dtype(dtype));
    if (T < 0) return fail(QMOE_ERR_INVALID, "T < 0");
    if (T > 0 && (!x || !out)) return fail(QMOE_ERR_INVALID, "NULL x or out");
    if (L->e_count > 0 && (L->e_begin != 0 || L->e_count != L->cfg.num_experts))
        return fail(QMOE_ERR_INVALID,
                    "qmoe_layer_forward needs all experts local; use the routed entry points");
    if (T == 0) return QMOE_OK;
    QTRY(check_align(x, ptr_kind, "x"));
    QTRY(check_align(out, ptr_kind, "out"));
    DeviceGuard g(L->ctx->device);
    if (L->e_count == 0) return forward_without_experts(L, x, dtype, T, out, topk_idx, topk_w, ptr_kind);
    cudaStream_t st = L->ctx->stream;
    QTRY(layer_reserve(L, T));
    const qmoe_moe_config &c = L->cfg;
    const size_t xbytes = dtype_size(dtype) * T * c.hidden_dim;
    ExpertsArgs a;
    a.topk_idx = L->topk_idx.as<int32_t>();
    a.topk_w = L->topk_w.as<float>();
    a.topk_ld = c.top_k;
    a.shared_count = L->has_shared ? T : 0;
    const bool front = L->e_count == c.num_experts && router_tail_ok(T, c.num_experts, c.top_k);
    bool prefill = false;
    if (front) QTRY(choose_prefill(L, dtype, T, c.top_k, &prefill));
    // Page-locked host buffers are read and written in place by the kernels
    // (no staging copies): x by the cluster front, which leaves a device copy
    // for the later kernels, out by the combine.  Other host memory is
    // staged through device buffers.
    const void *x_mapped = ptr_kind == QMOE_PTR_HOST && front && !prefill &&
                                   front_cluster_ok(T, c.hidden_dim, c.num_experts, c.top_k)
                               ? mapped_host(x)
                               : nullptr;
    // Outputs of decode-sized batches are written into page-locked host
    // memory in place by the combine (no copy launch); larger ones go to a
    // device buffer and back with one DMA copy, which moves bulk data over
    // the bus faster than the kernel's scattered stores do.
    void *out_mapped = ptr_kind == QMOE_PTR_HOST && xbytes <= kMappedOutMaxBytes
                           ? const_cast<void *>(mapped_host(out))
                           : nullptr;
    const void *xd;
    if (x_mapped) {
        QTRY(grow(L->x_in, xbytes));
        xd = L->x_in.p;                         // written by the front
    } else {
        QTRY(stage_in(L->x_in, x, xbytes, ptr_kind, st, &xd));
    }
    void *outd = out;
    if (ptr_kind == QMOE_PTR_HOST) {
        if (out_mapped) {
            outd = out_mapped;
        } else {
            QTRY(grow(L->io_out, xbytes));
            outd = L->io_out.p;
        }
    }
    auto enqueue = [&]() -> int {
        if (front) {
            QTRY(run_front(L, x_mapped ? x_mapped : xd, dtype, T, prefill,
                           x_mapped ? const_cast<void *>(xd) : nullptr));
            a.permuted = true;
        } else {
            QTRY(run_router(L, xd, dtype, T));
        }
        return run_experts(L, xd, dtype, T, a, outd, 0);
    };
    // whole forward in place on page-locked buffers, no routing copied out:
    // a repeat of the last call replays its captured graph
    if (x_mapped && out_mapped && !topk_idx && !topk_w && !L->profiling) {
        auto &G = L->fg;
        // every buffer the captured kernels touch is part of the key: the
        // scratch through cap (only layer_reserve reallocates it) and the
        // device copy of x, which other host-pointer calls may reallocate
        const bool same = G.x == x && G.out == out && G.T == T && G.dtype == dtype && G.path == L->path &&
                          G.cap == L->cap && G.x_in == L->x_in.p;
        if (!same) {
            if (G.exec) cudaGraphExecDestroy(G.exec);
            G.exec = nullptr;
            G.x = x;
            G.out = out;
            G.T = T;
            G.cap = L->cap;
            G.x_in = L->x_in.p;
            G.dtype = dtype;
            G.path = L->path;
            G.calls = 0;
        }
        if (!G.exec && ++G.calls >= 2) {
            cudaGraph_t graph = nullptr;
            if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
                const int rc = enqueue();
                const cudaError_t ec = cudaStreamEndCapture(st, &graph);
                if (rc == QMOE_OK && ec == cudaSuccess && graph &&
                    cudaGraphInstantiate(&G.exec, graph, 0) != cudaSuccess)
                    G.exec = nullptr;
                if (graph) cudaGraphDestroy(graph);
                cudaGetLastError();
                if (rc != QMOE_OK) return rc;
            } else {
                cudaGetLastError();   // e.g. the legacy default stream, which cannot be captured
            }
        }
        if (G.exec) {
            QTRY_CUDA(cudaGraphLaunch(G.exec, st));
            return sync_and_check(st);
        }
    }
    QTRY(enqueue());
    const size_t kb = sizeof(int32_t) * T * c.top_k;
    if (topk_idx)
        QTRY_CUDA(cudaMemcpyAsync(topk_idx, L->topk_idx.p, kb,
                                  ptr_kind == QMOE_PTR_HOST ? cudaMemcpyDeviceToHost
                                                            : cudaMemcpyDeviceToDevice, st));
    if (topk_w)
        QTRY_CUDA(cudaMemcpyAsync(topk_w, L->topk_w.p, kb,
                                  ptr_kind == QMOE_PTR_HOST ? cudaMemcpyDeviceToHost
                                                            : cudaMemcpyDeviceToDevice, st));
    if (!out_mapped) QTRY(finish_out(L, out, outd, xbytes, ptr_kind));
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(sync_and_check(st));
    }
    return QMOE_OK;
}

int qmoe_layer_route(qmoe_layer *L, const void *x, int dtype, int64_t T, int32_t *topk_idx,
                     float *topk_w, int ptr_kind) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    if (L->e_count == 0) return fail(QMOE_ERR_INVALID, "the layer has no routed experts");
    QTRY(check_ptr_kind(ptr_kind));
    QTRY(check_dtype(dtype));
    if (T < 0) return fail(QMOE_ERR_INVALID, "T < 0");
    if (T > 0 && (!x || !topk_idx || !topk_w)) return fail(QMOE_ERR_INVALID, "NULL argument");
    if (T == 0) return QMOE_OK;
    DeviceGuard g(L->ctx->device);
    cudaStream_t st = L->ctx->stream;
    QTRY(layer_reserve(L, T));
    const qmoe_moe_config &c = L->cfg;
    const void *xd;
    QTRY(stage_in(L->x_in, x, dtype_size(dtype) * T * c.hidden_dim, ptr_kind, st, &xd));
    QTRY(run_router(L, xd, dtype, T));
    const size_t kb = sizeof(int32_t) * T * c.top_k;
    const cudaMemcpyKind k = ptr_kind == QMOE_PTR_HOST ? cudaMemcpyDeviceToHost
                                                       : cudaMemcpyDeviceToDevice;
    QTRY_CUDA(cudaMemcpyAsync(topk_idx, L->topk_idx.p, kb, k, st));
    QTRY_CUDA(cudaMemcpyAsync(topk_w, L->topk_w.p, kb, k, st));
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(sync_and_check(st));
    }
    return QMOE_OK;
}

int qmoe_layer_route_plan(qmoe_layer *L, const void *x, int dtype, int64_t T, int32_t *topk_idx,
                          float *topk_w, int experts_per_rank, int world, int64_t capacity,
                          int32_t *send_counts, int32_t *send_tok, int32_t *send_meta, int32_t *slot_pos) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    if (L->e_count == 0) return fail(QMOE_ERR_INVALID, "the layer has no routed experts");
    QTRY(check_dtype(dtype));
    const qmoe_moe_config &c = L->cfg;
    if (T < 0 || world < 1 || world > kEpMaxWorld || experts_per_rank < 1 ||
        experts_per_rank * world != c.num_experts)
        return fail(QMOE_ERR_INVALID, "bad plan (T %lld, world %d, experts_per_rank %d, %d experts)",
                    (long long)T, world, experts_per_rank, c.num_experts);
    if (capacity < T) return fail(QMOE_ERR_INVALID, "capacity %lld < T %lld", (long long)capacity,
                                  (long long)T);
    if (T > 0 && (!x || !topk_idx || !topk_w || !send_counts || !send_tok || !send_meta || !slot_pos))
        return fail(QMOE_ERR_INVALID, "NULL argument");
    if (T == 0) return QMOE_OK;
    QTRY(check_align(x, QMOE_PTR_DEVICE, "x"));
    DeviceGuard g(L->ctx->device);
    cudaStream_t st = L->ctx->stream;
    QTRY(layer_reserve(L, T));
    RouterParams rp = router_params(L, x, dtype, T);
    rp.topk_idx = topk_idx;
    rp.topk_w = topk_w;
    mark(L, 0);
    if (front_cluster_ok(T, c.hidden_dim, c.num_experts, c.top_k)) {
        FrontParams f{};
        f.plan_world = world;
        f.plan_epr = experts_per_rank;
        f.plan_capacity = capacity;
        f.send_counts = send_counts;
        f.send_tok = send_tok;
        f.send_meta = send_meta;
        f.slot_pos = slot_pos;
        QTRY_CUDA(launch_front_cluster(rp, f, st));
        return QMOE_OK;
    }
    QTRY_CUDA(launch_router(rp, nullptr, st));
    EpPlanParams p{};
    p.topk_idx = topk_idx;
    p.topk_w = topk_w;
    p.T = T;
    p.K = c.top_k;
    p.experts_per_rank = experts_per_rank;
    p.world = world;
    p.capacity = capacity;
    p.send_counts = send_counts;
    p.send_tok = send_tok;
    p.send_meta = send_meta;
    p.slot_pos = slot_pos;
    QTRY_CUDA(launch_ep_plan(p, st));
    return QMOE_OK;
}

int qmoe_layer_forward_routed(qmoe_layer *L, const void *x, int dtype, int64_t R,
                              const int32_t *topk_idx, const float *topk_w, void *out,
                              int ptr_kind) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    if (L->e_count == 0) return fail(QMOE_ERR_INVALID, "the layer has no routed experts");
    QTRY(check_ptr_kind(ptr_kind));
    QTRY(check_dtype(dtype));
    if (R < 0) return fail(QMOE_ERR_INVALID, "R < 0");
    if (R > 0 && (!x || !topk_idx || !topk_w || !out)) return fail(QMOE_ERR_INVALID, "NULL argument");
    if (R == 0) return QMOE_OK;
    QTRY(check_align(x, ptr_kind, "x"));
    QTRY(check_align(out, ptr_kind, "out"));
    DeviceGuard g(L->ctx->device);
    cudaStream_t st = L->ctx->stream;
    QTRY(layer_reserve(L, R));
    const qmoe_moe_config &c = L->cfg;
    const size_t xbytes = dtype_size(dtype) * R * c.hidden_dim;
    const size_t kb = sizeof(int32_t) * R * c.top_k;
    const void *xd, *id, *wd;
    QTRY(stage_in(L->x_in, x, xbytes, ptr_kind, st, &xd));
    QTRY(stage_in(L->user_idx, topk_idx, kb, ptr_kind, st, &id));
    QTRY(stage_in(L->user_w, topk_w, kb, ptr_kind, st, &wd));
    void *outd = out;
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(grow(L->io_out, xbytes));
        outd = L->io_out.p;
    }
    ExpertsArgs a;
    a.topk_idx = static_cast<const int32_t *>(id);
    a.topk_w = static_cast<const float *>(wd);
    a.topk_ld = c.top_k;
    QTRY(run_experts(L, xd, dtype, R, a, outd, 0));
    QTRY(finish_out(L, out, outd, xbytes, ptr_kind));
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(sync_and_check(st));
    }
    return QMOE_OK;
}

int qmoe_layer_forward_ep(qmoe_layer *L, const void *x, int dtype, int64_t R, const int32_t *meta,
                          int64_t shared_row0, void *out) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    if (L->e_count == 0) return fail(QMOE_ERR_INVALID, "the layer has no routed experts");
    QTRY(check_dtype(dtype));
    if (R < 0 || shared_row0 < 0 || shared_row0 > R)
        return fail(QMOE_ERR_INVALID, "bad rows (R %lld, shared_row0 %lld)", (long long)R,
                    (long long)shared_row0);
    if (R > 0 && (!x || !meta || !out)) return fail(QMOE_ERR_INVALID, "NULL argument");
    if (R == 0) return QMOE_OK;
    QTRY(check_align(x, QMOE_PTR_DEVICE, "x"));
    QTRY(check_align(out, QMOE_PTR_DEVICE, "out"));
    DeviceGuard g(L->ctx->device);
    QTRY(layer_reserve(L, R));
    const int K = L->cfg.top_k;
    ExpertsArgs a;
    a.topk_idx = meta;
    a.topk_w = reinterpret_cast<const float *>(meta + K);
    a.topk_ld = 2 * K;
    a.shared_row0 = shared_row0;
    a.shared_count = L->has_shared ? R - shared_row0 : 0;
    return run_experts(L, x, dtype, R, a, out, 0);
}

// The shared expert alone over T rows (SharedExpert::forward,
// src/model.rs:325-347), written to out or added into it.
static int shared_pass(qmoe_layer *L, const void *x, int dtype, int64_t T, void *out, int accumulate,
                       int ptr_kind) {
    cudaStream_t st = L->ctx->stream;
    QTRY(layer_reserve(L, T));
    const qmoe_moe_config &c = L->cfg;
    const size_t xbytes = dtype_size(dtype) * T * c.hidden_dim;
    const void *xd;
    QTRY(stage_in(L->x_in, x, xbytes, ptr_kind, st, &xd));
    void *outd = out;
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(grow(L->io_out, xbytes));
        outd = L->io_out.p;
        if (accumulate)
            QTRY_CUDA(cudaMemcpyAsync(outd, out, xbytes, cudaMemcpyHostToDevice, st));
    }
    // a shared-only pass: no routed assignments (top_k slots all skipped)
    qmoe_moe_config saved = L->cfg;
    L->cfg.top_k = 0;
    ExpertsArgs a;
    a.shared_count = T;
    int rc = run_experts(L, xd, dtype, T, a, outd, accumulate);
    L->cfg = saved;
    if (rc != QMOE_OK) return rc;
    QTRY(finish_out(L, out, outd, xbytes, ptr_kind));
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(sync_and_check(st));
    }
    return QMOE_OK;
}

int qmoe_layer_shared_forward(qmoe_layer *L, const void *x, int dtype, int64_t T, void *out,
                              int accumulate, int ptr_kind) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    QTRY(check_ptr_kind(ptr_kind));
    QTRY(check_dtype(dtype));
    if (!L->has_shared) return fail(QMOE_ERR_INVALID, "layer has no shared expert");
    if (T < 0) return fail(QMOE_ERR_INVALID, "T < 0");
    if (T > 0 && (!x || !out)) return fail(QMOE_ERR_INVALID, "NULL argument");
    if (T == 0) return QMOE_OK;
    QTRY(check_align(x, ptr_kind, "x"));
    QTRY(check_align(out, ptr_kind, "out"));
    DeviceGuard g(L->ctx->device);
    return shared_pass(L, x, dtype, T, out, accumulate, ptr_kind);
}

// ---------------------------------------------------------------------------
// expert parallelism helpers
// ---------------------------------------------------------------------------

int qmoe_ep_plan(qmoe_ctx *ctx, const int32_t *topk_idx, const float *topk_w, int64_t T, int K,
                 int experts_per_rank, int world, int64_t capacity, int32_t *send_counts,
                 int32_t *send_tok, int32_t *send_meta, int32_t *slot_pos) {
    if (!ctx) return fail(QMOE_ERR_INVALID, "ctx is NULL");
    if (T < 0 || K <= 0 || experts_per_rank <= 0 || world <= 0 || world > 32)
        return fail(QMOE_ERR_INVALID, "bad plan shape (T %lld, K %d, experts_per_rank %d, world %d)",
                    (long long)T, K, experts_per_rank, world);
    if (capacity < 0 || (capacity > 0 && capacity < T))
        return fail(QMOE_ERR_INVALID, "capacity %lld < T %lld", (long long)capacity, (long long)T);
    if (!send_counts || (T > 0 && (!topk_idx || !topk_w || !send_tok || !send_meta || !slot_pos)))
        return fail(QMOE_ERR_INVALID, "NULL argument");
    DeviceGuard g(ctx->device);
    EpPlanParams p{};
    p.topk_idx = topk_idx;
    p.topk_w = topk_w;
    p.T = T;
    p.K = K;
    p.experts_per_rank = experts_per_rank;
    p.world = world;
    p.capacity = capacity;
    p.send_counts = send_counts;
    p.send_tok = send_tok;
    p.send_meta = send_meta;
    p.slot_pos = slot_pos;
    QTRY_CUDA(launch_ep_plan(p, ctx->stream));
    return QMOE_OK;
}

int qmoe_gather_rows(qmoe_ctx *ctx, const void *x, int dtype, int64_t H, const int32_t *idx, int64_t n,
                     void *out) {
    if (!ctx) return fail(QMOE_ERR_INVALID, "ctx is NULL");
    QTRY(check_dtype(dtype));
    if (H <= 0 || H % 8 || n < 0) return fail(QMOE_ERR_INVALID, "bad shape (H %% 8 must be 0)");
    if (n > 0 && (!x || !idx || !out)) return fail(QMOE_ERR_INVALID, "NULL argument");
    QTRY(check_align(x, QMOE_PTR_DEVICE, "x"));
    QTRY(check_align(out, QMOE_PTR_DEVICE, "out"));
    DeviceGuard g(ctx->device);
    QTRY_CUDA(launch_gather_rows(x, dtype, H, idx, n, out, ctx->stream));
    return QMOE_OK;
}

int qmoe_combine_rows(qmoe_ctx *ctx, const void *rows, int dtype, int64_t H, const int32_t *slot_pos,
                      int S, int64_t T, const void *extra, void *out) {
    if (!ctx) return fail(QMOE_ERR_INVALID, "ctx is NULL");
    QTRY(check_dtype(dtype));
    if (H <= 0 || H % 4 || S <= 0 || T < 0) return fail(QMOE_ERR_INVALID, "bad shape");
    if (T > 0 && (!slot_pos || !out)) return fail(QMOE_ERR_INVALID, "NULL argument");
    QTRY(check_align(out, QMOE_PTR_DEVICE, "out"));
    DeviceGuard g(ctx->device);
    if (extra) QTRY(check_align(extra, QMOE_PTR_DEVICE, "extra"));
    QTRY_CUDA(launch_combine_rows(rows, dtype, H, slot_pos, S, T, extra, out, ctx->stream));
    return QMOE_OK;
}

// ---------------------------------------------------------------------------
// expert-parallel exchange over peer memory
// ---------------------------------------------------------------------------

struct qmoe_ep_peer {
    qmoe_ctx *ctx = nullptr;
    EpPeerDev d{};
    uint8_t *mem = nullptr;
    cudaIpcMemHandle_t handle{};
    bool opened[kEpMaxWorld] = {};
};

static_assert(sizeof(cudaIpcMemHandle_t) == QMOE_EP_HANDLE_BYTES, "IPC handle size");

static int64_t align256(int64_t n) { return (n + 255) / 256 * 256; }

int qmoe_ep_peer_create(qmoe_ctx *ctx, int world, int rank, int64_t capacity, int64_t H, int K, int dtype,
                        qmoe_ep_peer **out) {
    if (!ctx || !out) return fail(QMOE_ERR_INVALID, "NULL argument");
    *out = nullptr;
    QTRY(check_dtype(dtype));
    if (world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world)
        return fail(QMOE_ERR_INVALID, "rank %d / world %d (world <= %d)", rank, world, kEpMaxWorld);
    const int64_t es = (int64_t)dtype_size(dtype);
    if (capacity < 1 || H <= 0 || (H * es) % 16 || K < 1)
        return fail(QMOE_ERR_INVALID, "bad exchange shape (capacity %lld, H %lld, K %d)",
                    (long long)capacity, (long long)H, K);
    DeviceGuard g(ctx->device);
    qmoe_ep_peer *p = new (std::nothrow) qmoe_ep_peer;
    if (!p) return fail(QMOE_ERR_NOMEM, "host allocation failed");
    p->ctx = ctx;
    EpPeerDev &d = p->d;
    d.world = world;
    d.rank = rank;
    d.K = K;
    d.C = capacity;
    d.H = H;
    d.esize = es;
    const int64_t rows = (int64_t)world * capacity + capacity;
    d.off_rows = 0;
    d.off_meta = align256(rows * H * es);
    d.off_back = d.off_meta + align256(rows * 2 * K * 4);
    d.off_flags = d.off_back + align256((int64_t)world * capacity * H * es);
    const int64_t off_local = d.off_flags + align256(2 * world * 4);
    const int64_t bytes = off_local + 256 + 2 * kEpMaxWorld * 4;
    if (cudaMalloc(&p->mem, (size_t)bytes) != cudaSuccess) {
        cudaGetLastError();
        delete p;
        return fail(QMOE_ERR_NOMEM, "cudaMalloc of %lld bytes failed", (long long)bytes);
    }
    int rc = QMOE_OK;
    if (cudaMemset(p->mem, 0, (size_t)bytes) != cudaSuccess ||
        cudaIpcGetMemHandle(&p->handle, p->mem) != cudaSuccess) {
        rc = fail(QMOE_ERR_CUDA, "exchange buffer setup: %s", cudaGetErrorString(cudaGetLastError()));
        cudaFree(p->mem);
        delete p;
        return rc;
    }
    d.base[rank] = p->mem;
    d.seq = reinterpret_cast<int *>(p->mem + off_local);
    d.done = d.seq + 1;
    d.cnt = reinterpret_cast<int *>(p->mem + off_local + 256);
    d.err = error_flag();
    *out = p;
    return QMOE_OK;
}

int qmoe_ep_peer_destroy(qmoe_ep_peer *p) {
    if (!p) return QMOE_OK;
    DeviceGuard g(p->ctx->device);
    for (int r = 0; r < p->d.world; ++r)
        if (p->opened[r]) cudaIpcCloseMemHandle(p->d.base[r]);
    if (p->mem) cudaFree(p->mem);
    delete p;
    return QMOE_OK;
}

int qmoe_ep_peer_handle(qmoe_ep_peer *p, void *handle) {
    if (!p || !handle) return fail(QMOE_ERR_INVALID, "NULL argument");
    std::memcpy(handle, &p->handle, QMOE_EP_HANDLE_BYTES);
    return QMOE_OK;
}

int qmoe_ep_peer_connect(qmoe_ep_peer *p, const void *handles) {
    if (!p || !handles) return fail(QMOE_ERR_INVALID, "NULL argument");
    DeviceGuard g(p->ctx->device);
    for (int r = 0; r < p->d.world; ++r) {
        if (r == p->d.rank || p->opened[r]) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)r * QMOE_EP_HANDLE_BYTES,
                    QMOE_EP_HANDLE_BYTES);
        void *ptr = nullptr;
        QTRY_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        p->d.base[r] = static_cast<uint8_t *>(ptr);
        p->opened[r] = true;
    }
    return QMOE_OK;
}

int qmoe_ep_peer_buffers(qmoe_ep_peer *p, void **recv_rows, int32_t **recv_meta, void **back_rows) {
    if (!p) return fail(QMOE_ERR_INVALID, "NULL argument");
    if (recv_rows) *recv_rows = p->mem + p->d.off_rows;
    if (recv_meta) *recv_meta = reinterpret_cast<int32_t *>(p->mem + p->d.off_meta);
    if (back_rows) *back_rows = p->mem + p->d.off_back;
    return QMOE_OK;
}

static int ep_ready(const qmoe_ep_peer *p) {
    for (int r = 0; r < p->d.world; ++r)
        if (!p->d.base[r]) return fail(QMOE_ERR_INVALID, "exchange not connected (rank %d)", r);
    return QMOE_OK;
}

int qmoe_ep_dispatch(qmoe_ep_peer *p, const void *x, int64_t T, const int32_t *send_counts,
                     const int32_t *send_tok, const int32_t *send_meta) {
    if (!p || !send_counts || !send_tok || !send_meta || (T > 0 && !x))
        return fail(QMOE_ERR_INVALID, "NULL argument");
    if (T < 0 || T > p->d.C) return fail(QMOE_ERR_INVALID, "T %lld outside 0 .. capacity %lld",
                                         (long long)T, (long long)p->d.C);
    QTRY(ep_ready(p));
    if (T > 0) QTRY(check_align(x, QMOE_PTR_DEVICE, "x"));
    DeviceGuard g(p->ctx->device);
    QTRY_CUDA(launch_ep_dispatch(p->d, x, T, send_counts, send_tok, send_meta, p->ctx->stream));
    return QMOE_OK;
}

int qmoe_ep_wait(qmoe_ep_peer *p, int phase) {
    if (!p) return fail(QMOE_ERR_INVALID, "NULL argument");
    if (phase != 0 && phase != 1) return fail(QMOE_ERR_INVALID, "phase %d (0 dispatch, 1 return)", phase);
    QTRY(ep_ready(p));
    DeviceGuard g(p->ctx->device);
    QTRY_CUDA(launch_ep_wait(p->d, phase, p->ctx->stream));
    return QMOE_OK;
}

int qmoe_ep_return(qmoe_ep_peer *p, const void *y) {
    if (!p || !y) return fail(QMOE_ERR_INVALID, "NULL argument");
    QTRY(ep_ready(p));
    QTRY(check_align(y, QMOE_PTR_DEVICE, "y"));
    DeviceGuard g(p->ctx->device);
    QTRY_CUDA(launch_ep_return(p->d, y, p->ctx->stream));
    return QMOE_OK;
}

int qmoe_layer_forward_ep_return(qmoe_layer *L, qmoe_ep_peer *p, const void *x, int dtype, int64_t R,
                                 const int32_t *meta, int64_t shared_row0, void *y) {
    if (!L || !p) return fail(QMOE_ERR_INVALID, "NULL layer or exchange");
    if (L->e_count == 0) return fail(QMOE_ERR_INVALID, "the layer has no routed experts");
    QTRY(check_dtype(dtype));
    QTRY(ep_ready(p));
    const int64_t GC = (int64_t)p->d.world * p->d.C;
    if (R < GC || shared_row0 != GC || R > GC + p->d.C)
        return fail(QMOE_ERR_INVALID, "rows R %lld / shared_row0 %lld do not match the exchange (%lld received)",
                    (long long)R, (long long)shared_row0, (long long)GC);
    if ((int64_t)dtype_size(dtype) != p->d.esize || p->d.H != L->cfg.hidden_dim || p->d.K != L->cfg.top_k)
        return fail(QMOE_ERR_INVALID, "exchange dtype / hidden / top_k differ from the layer's");
    if (!x || !meta || !y) return fail(QMOE_ERR_INVALID, "NULL argument");
    QTRY(check_align(x, QMOE_PTR_DEVICE, "x"));
    QTRY(check_align(y, QMOE_PTR_DEVICE, "y"));
    DeviceGuard g(L->ctx->device);
    QTRY(layer_reserve(L, R));
    const int K = L->cfg.top_k;
    ExpertsArgs a;
    a.topk_idx = meta;
    a.topk_w = reinterpret_cast<const float *>(meta + K);
    a.topk_ld = 2 * K;
    a.shared_row0 = shared_row0;
    a.shared_count = L->has_shared ? R - shared_row0 : 0;
    bool returned = false;
    a.ep_ret = &p->d;
    a.returned = &returned;
    a.wait_dispatch = true;
    QTRY(run_experts(L, x, dtype, R, a, y, 0));
    if (!returned) QTRY_CUDA(launch_ep_return(p->d, y, p->ctx->stream));
    return QMOE_OK;
}

int qmoe_ep_finish(qmoe_ep_peer *p, const int32_t *slot_pos, int64_t T, const void *extra, void *out) {
    if (!p || (T > 0 && (!slot_pos || !out))) return fail(QMOE_ERR_INVALID, "NULL argument");
    if (T < 0 || T > p->d.C) return fail(QMOE_ERR_INVALID, "T %lld outside 0 .. capacity %lld",
                                         (long long)T, (long long)p->d.C);
    QTRY(ep_ready(p));
    if (T == 0) return qmoe_ep_wait(p, 1);
    QTRY(check_align(out, QMOE_PTR_DEVICE, "out"));
    if (extra) QTRY(check_align(extra, QMOE_PTR_DEVICE, "extra"));
    DeviceGuard g(p->ctx->device);
    QTRY_CUDA(launch_ep_finish(p->d, slot_pos, T, extra, out, p->ctx->stream));
    return QMOE_OK;
}

int qmoe_layer_set_norm(qmoe_layer *L, const float *weight, const float *bias, float eps, int ptr_kind) {
    if (!L || !weight || !bias) return fail(QMOE_ERR_INVALID, "NULL argument");
    QTRY(check_ptr_kind(ptr_kind));
    if (!(eps >= 0.0f)) return fail(QMOE_ERR_INVALID, "eps must be >= 0");
    DeviceGuard g(L->ctx->device);
    const size_t nb = sizeof(float) * L->cfg.hidden_dim;
    if (!L->ln_w) QTRY_CUDA(cudaMalloc((void **)&L->ln_w, nb));
    if (!L->ln_b) QTRY_CUDA(cudaMalloc((void **)&L->ln_b, nb));
    QTRY_CUDA(cudaMemcpyAsync(L->ln_w, weight, nb, kind_in(ptr_kind), L->ctx->stream));
    QTRY_CUDA(cudaMemcpyAsync(L->ln_b, bias, nb, kind_in(ptr_kind), L->ctx->stream));
    QTRY_CUDA(cudaStreamSynchronize(L->ctx->stream));
    L->ln_eps = eps;
    return QMOE_OK;
}

// The block's device work on the layer's stream: LayerNorm of xd into the
// layer's rows, the router and experts on them, the combine adding the
// residual xd into outd.  Needs layer_reserve(L, T) and L->xn grown to the
// rows' bytes; allocates nothing itself (so a chain of blocks can be
// captured into a CUDA graph).
static int block_enqueue(qmoe_layer *L, const void *xd, int dtype, int64_t T, void *outd, bool want_routing) {
    cudaStream_t st = L->ctx->stream;
    const qmoe_moe_config &c = L->cfg;
    const size_t xbytes = dtype_size(dtype) * T * c.hidden_dim;
    // post_attention_layernorm (src/model.rs:401-403) into the block's rows
    NormParams np{xd, dtype, T, c.hidden_dim, L->ln_w, L->ln_b, L->ln_eps, L->xn.p};
    QTRY_CUDA(launch_layernorm(np, st));
    const void *xn = L->xn.p;
    ExpertsArgs a;
    a.residual = xd;                          // residual + (moe + shared), src/model.rs:409-412
    if (L->e_count == 0) {
        // no routed experts (src/moe.rs:46-48): x + shared(LN(x)), or x
        const size_t kb = sizeof(int32_t) * T * c.top_k;
        if (want_routing) {
            QTRY_CUDA(cudaMemsetAsync(L->topk_idx.p, 0xff, kb, st));
            QTRY_CUDA(cudaMemsetAsync(L->topk_w.p, 0, kb, st));
        }
        if (L->has_shared) {
            qmoe_moe_config saved = L->cfg;
            L->cfg.top_k = 0;
            a.shared_count = T;
            const int rc = run_experts(L, xn, dtype, T, a, outd, 0);
            L->cfg = saved;
            return rc;
        }
        QTRY_CUDA(cudaMemcpyAsync(outd, xd, xbytes, cudaMemcpyDeviceToDevice, st));
        return QMOE_OK;
    }
    a.topk_idx = L->topk_idx.as<int32_t>();
    a.topk_w = L->topk_w.as<float>();
    a.topk_ld = c.top_k;
    a.shared_count = L->has_shared ? T : 0;
    const bool front = router_tail_ok(T, c.num_experts, c.top_k);
    bool prefill = false;
    QTRY(choose_prefill(L, dtype, T, c.top_k, &prefill));
    if (front) {
        QTRY(run_front(L, xn, dtype, T, prefill));
        a.permuted = true;
    } else {
        QTRY(run_router(L, xn, dtype, T));
    }
    return run_experts(L, xn, dtype, T, a, outd, 0);
}

static int check_block_layer(const qmoe_layer *L) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    if (!L->ln_w) return fail(QMOE_ERR_INVALID, "no LayerNorm set (qmoe_layer_set_norm)");
    if (L->e_count > 0 && (L->e_begin != 0 || L->e_count != L->cfg.num_experts))
        return fail(QMOE_ERR_INVALID, "a block forward needs all experts local");
    return QMOE_OK;
}

int qmoe_layer_forward_block(qmoe_layer *L, const void *x, int dtype, int64_t T, void *out,
                             int32_t *topk_idx, float *topk_w, int ptr_kind) {
    QTRY(check_block_layer(L));
    QTRY(check_ptr_kind(ptr_kind));
    QTRY(check_dtype(dtype));
    if (T < 0) return fail(QMOE_ERR_INVALID, "T < 0");
    if (T > 0 && (!x || !out)) return fail(QMOE_ERR_INVALID, "NULL x or out");
    if (T == 0) return QMOE_OK;
    QTRY(check_align(x, ptr_kind, "x"));
    QTRY(check_align(out, ptr_kind, "out"));
    DeviceGuard g(L->ctx->device);
    cudaStream_t st = L->ctx->stream;
    QTRY(layer_reserve(L, T));
    const qmoe_moe_config &c = L->cfg;
    const size_t xbytes = dtype_size(dtype) * T * c.hidden_dim;
    const void *xd;
    QTRY(stage_in(L->x_in, x, xbytes, ptr_kind, st, &xd));
    void *outd = out;
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(grow(L->io_out, xbytes));
        outd = L->io_out.p;
    }
    QTRY(grow(L->xn, xbytes));
    QTRY(block_enqueue(L, xd, dtype, T, outd, topk_idx || topk_w));
    const size_t kb = sizeof(int32_t) * T * c.top_k;
    const cudaMemcpyKind k = ptr_kind == QMOE_PTR_HOST ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    if (topk_idx) QTRY_CUDA(cudaMemcpyAsync(topk_idx, L->topk_idx.p, kb, k, st));
    if (topk_w) QTRY_CUDA(cudaMemcpyAsync(topk_w, L->topk_w.p, kb, k, st));
    QTRY(finish_out(L, out, outd, xbytes, ptr_kind));
    if (ptr_kind == QMOE_PTR_HOST) QTRY(sync_and_check(st));
    return QMOE_OK;
}

// ---------------------------------------------------------------------------
// chain of blocks
// ---------------------------------------------------------------------------

struct qmoe_chain {
    qmoe_ctx *ctx = nullptr;
    std::vector<qmoe_layer *> layers;
    int64_t H = 0;
    DevBuf ping[2], in, out;
    // the captured launch sequence and what it was captured for: the input
    // and output rows, T, dtype, and every buffer of every layer it touches
    struct Key {
        const void *xd = nullptr, *outd = nullptr;
        int64_t T = -1;
        int dtype = -1;
        std::vector<const void *> bufs;
        std::vector<int64_t> caps;
        std::vector<int> paths;
    } key;
    cudaGraphExec_t exec = nullptr;
};

static void chain_key(const qmoe_chain *C, const void *xd, const void *outd, int64_t T, int dtype,
                      qmoe_chain::Key &k) {
    k.xd = xd;
    k.outd = outd;
    k.T = T;
    k.dtype = dtype;
    k.bufs.clear();
    k.caps.clear();
    k.paths.clear();
    k.bufs.push_back(C->ping[0].p);
    k.bufs.push_back(C->ping[1].p);
    for (const qmoe_layer *L : C->layers) {
        k.bufs.push_back(L->xn.p);
        k.caps.push_back(L->cap);
        k.paths.push_back(L->path);
    }
}

static bool same_key(const qmoe_chain::Key &a, const qmoe_chain::Key &b) {
    return a.xd == b.xd && a.outd == b.outd && a.T == b.T && a.dtype == b.dtype && a.bufs == b.bufs &&
           a.caps == b.caps && a.paths == b.paths;
}

int qmoe_chain_create(qmoe_layer *const *layers, int n_layers, qmoe_chain **out) {
    if (!layers || !out || n_layers < 1) return fail(QMOE_ERR_INVALID, "need at least one layer");
    *out = nullptr;
    for (int l = 0; l < n_layers; ++l) {
        QTRY(check_block_layer(layers[l]));
        if (layers[l]->ctx != layers[0]->ctx)
            return fail(QMOE_ERR_INVALID, "the layers of a chain must share one context");
        if (layers[l]->cfg.hidden_dim != layers[0]->cfg.hidden_dim)
            return fail(QMOE_ERR_INVALID, "the layers of a chain must share hidden_dim");
    }
    qmoe_chain *C = new (std::nothrow) qmoe_chain;
    if (!C) return fail(QMOE_ERR_NOMEM, "host allocation failed");
    C->ctx = layers[0]->ctx;
    C->layers.assign(layers, layers + n_layers);
    C->H = layers[0]->cfg.hidden_dim;
    *out = C;
    return QMOE_OK;
}

int qmoe_chain_destroy(qmoe_chain *C) {
    if (!C) return QMOE_OK;
    DeviceGuard g(C->ctx->device);
    if (C->exec) cudaGraphExecDestroy(C->exec);
    for (DevBuf *b : {&C->ping[0], &C->ping[1], &C->in, &C->out}) release(*b);
    delete C;
    return QMOE_OK;
}

int qmoe_chain_forward(qmoe_chain *C, const void *x, int dtype, int64_t T, void *out, int ptr_kind) {
    if (!C) return fail(QMOE_ERR_INVALID, "chain is NULL");
    QTRY(check_ptr_kind(ptr_kind));
    QTRY(check_dtype(dtype));
    if (T < 0) return fail(QMOE_ERR_INVALID, "T < 0");
    if (T > 0 && (!x || !out)) return fail(QMOE_ERR_INVALID, "NULL x or out");
    if (T == 0) return QMOE_OK;
    QTRY(check_align(x, ptr_kind, "x"));
    QTRY(check_align(out, ptr_kind, "out"));
    DeviceGuard g(C->ctx->device);
    cudaStream_t st = C->ctx->stream;
    const size_t xbytes = dtype_size(dtype) * T * C->H;
    // every buffer of the sequence exists before it is enqueued or captured
    const int n = (int)C->layers.size();
    for (qmoe_layer *L : C->layers) {
        QTRY(layer_reserve(L, T));
        QTRY(grow(L->xn, xbytes));
    }
    if (n > 1) QTRY(grow(C->ping[0], xbytes));
    if (n > 2) QTRY(grow(C->ping[1], xbytes));
    const void *xd = x;
    void *outd = out;
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY(grow(C->in, xbytes));
        QTRY(grow(C->out, xbytes));
        QTRY_CUDA(cudaMemcpyAsync(C->in.p, x, xbytes, cudaMemcpyHostToDevice, st));
        xd = C->in.p;
        outd = C->out.p;
    }
    auto enqueue = [&]() -> int {
        const void *cur = xd;
        for (int l = 0; l < n; ++l) {
            void *dst = l == n - 1 ? outd : C->ping[l & 1].p;
            QTRY(block_enqueue(C->layers[l], cur, dtype, T, dst, false));
            cur = dst;
        }
        return QMOE_OK;
    };
    bool profiling = false;
    for (const qmoe_layer *L : C->layers) profiling |= L->profiling;
    qmoe_chain::Key k;
    chain_key(C, xd, outd, T, dtype, k);
    if (!profiling && !(C->exec && same_key(k, C->key))) {
        if (C->exec) cudaGraphExecDestroy(C->exec);
        C->exec = nullptr;
        cudaGraph_t graph = nullptr;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int rc = enqueue();
            const cudaError_t ec = cudaStreamEndCapture(st, &graph);
            if (rc == QMOE_OK && ec == cudaSuccess && graph &&
                cudaGraphInstantiate(&C->exec, graph, 0) != cudaSuccess)
                C->exec = nullptr;
            if (graph) cudaGraphDestroy(graph);
            cudaGetLastError();
            if (rc != QMOE_OK) return rc;
            if (C->exec) C->key = k;
        } else {
            cudaGetLastError();   // e.g. the legacy default stream, which cannot be captured
        }
    }
    if (C->exec && !profiling) {
        QTRY_CUDA(cudaGraphLaunch(C->exec, st));
    } else {
        QTRY(enqueue());
    }
    if (ptr_kind == QMOE_PTR_HOST) {
        QTRY_CUDA(cudaMemcpyAsync(out, outd, xbytes, cudaMemcpyDeviceToHost, st));
        QTRY(sync_and_check(st));
    }
    return QMOE_OK;
}

int qmoe_layer_set_path(qmoe_layer *L, int path) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    if (path != QMOE_PATH_AUTO && path != QMOE_PATH_DECODE && path != QMOE_PATH_PREFILL &&
        path != QMOE_PATH_DECODE_SPLIT)
        return fail(QMOE_ERR_INVALID, "unknown path %d", path);
    if (path == QMOE_PATH_PREFILL && !L->prefill_ok)
        return fail(QMOE_ERR_UNSUPPORTED,
                    "the prefill path needs hidden %% 128 == 0 and intermediate dims %% 64 == 0");
    L->path = path;
    return QMOE_OK;
}

int qmoe_layer_set_profiling(qmoe_layer *L, int enable) {
    if (!L) return fail(QMOE_ERR_INVALID, "layer is NULL");
    DeviceGuard g(L->ctx->device);
    if (enable && !L->ev[0])
        for (cudaEvent_t &e : L->ev) QTRY_CUDA(cudaEventCreate(&e));
    L->profiling = enable != 0;
    return QMOE_OK;
}

int qmoe_layer_stage_times(qmoe_layer *L, float *ms, int capacity, int *count) {
    if (!L || !ms || capacity < 0) return fail(QMOE_ERR_INVALID, "bad argument");
    if (!L->ev[0]) return fail(QMOE_ERR_INVALID, "profiling was never enabled");
    DeviceGuard g(L->ctx->device);
    QTRY_CUDA(cudaEventSynchronize(L->ev[kStages]));
    const int n = capacity < kStages ? capacity : kStages;
    for (int i = 0; i < n; ++i) QTRY_CUDA(cudaEventElapsedTime(&ms[i], L->ev[i], L->ev[i + 1]));
    if (count) *count = n;
    return QMOE_OK;
}

}  // extern "C"

namespace qmoe {
void set_last_error_message(const char *msg) { g_err = msg ? msg : ""; }
}  // namespace qmoe
