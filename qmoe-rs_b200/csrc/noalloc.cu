// noalloc.cu -- the packed-matrix GEMV for callers that must not allocate.
//
// Some callers cannot allocate device memory at call time: a host program
// that hands the whole HBM budget to its own pool at start-up (a serving
// engine that reserves everything left for its KV cache, say) and gives a
// plugin nothing but the input and output buffers of each call; or a
// latency-critical path where cudaMalloc's implicit device-wide
// synchronisation and unbounded cost are not acceptable.  qmoe_packed_forward
// keeps its work list in memory it allocates on first use; the entry point in
// this file computes the same product with that work list in a fixed-size,
// file-scope device array instead, and calls no allocating routine at all.
//
// The array below is loaded with the library and held by every GPU that loads
// it until the process exits (about 52 KB per device).  Host code must not
// pass the array's name to a kernel (on the host it is only a stand-in for
// the symbol): its device address is fetched once per device with
// cudaGetSymbolAddress, with that device current, and passed as a pointer.
#include <mutex>

#include "../../include/qmoe_b200.h"
#include "kernels.h"

namespace qmoe {
namespace {

// The work list: 16 bytes of counters (two group counts and the one
// segment's two offsets), then one int4 descriptor per group of
// kQgemvTokens rows.
constexpr int64_t kMaxBatch = QMOE_NOALLOC_MAX_BATCH;
constexpr int64_t kMaxGroups = (kMaxBatch + kQgemvTokens - 1) / kQgemvTokens;
constexpr size_t kCounterBytes = 16;
constexpr size_t kScratchBytes = kCounterBytes + sizeof(int4) * kMaxGroups;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;

struct DeviceSetup {
    bool ready = false;
    void *scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int grid = 0;             // persistent GEMV grid, sized for the largest row
};

std::mutex g_setup_mu;
DeviceSetup g_setup[kMaxDevices];

// Errors are reported like every other entry point: a status code, and the
// message through qmoe_last_error().
int set_error(int code, const char *msg) {
    set_last_error_message(msg);
    return code;
}

// Once per device, with that device current: check the architecture, look
// up the scratch array's device address and size the GEMV grid.
int setup_device(int device, void **scratch, int *grid) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    DeviceSetup &s = g_setup[device];
    if (!s.ready) {
        cudaDeviceProp prop;
        cudaError_t e = cudaGetDeviceProperties(&prop, device);
        if (e != cudaSuccess) return set_error(QMOE_ERR_CUDA, cudaGetErrorString(e));
        if (prop.major != 10 || prop.minor != 0)
            return set_error(QMOE_ERR_UNSUPPORTED, "device is not sm_100 (B200)");
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return set_error(QMOE_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch) failed");
        s.scratch = p;
        s.grid = qgemv_max_grid(1, QMOE_NOALLOC_MAX_IN_FEATURES);
        s.ready = true;
    }
    *scratch = s.scratch;
    *grid = s.grid;
    return QMOE_OK;
}

}  // namespace
}  // namespace qmoe

using namespace qmoe;

extern "C" int qmoe_packed_forward_noalloc(int device, void *stream, const uint8_t *packed,
                                           const float *scales, int64_t out_features,
                                           int64_t in_features, const float *x,
                                           int64_t batch, float *y) {
    if (device < 0 || device >= kMaxDevices)
        return set_error(QMOE_ERR_INVALID, "device index out of range");
    if (!packed || !scales || (batch > 0 && (!x || !y)))
        return set_error(QMOE_ERR_INVALID, "NULL pointer argument");
    if (out_features <= 0 || out_features > (1LL << 30))
        return set_error(QMOE_ERR_INVALID, "out_features must be in 1 .. 2^30");
    if (in_features <= 0 || in_features % 64 != 0 ||
        in_features > QMOE_NOALLOC_MAX_IN_FEATURES)
        return set_error(QMOE_ERR_INVALID,
                         "in_features must be a positive multiple of 64 and at most "
                         "QMOE_NOALLOC_MAX_IN_FEATURES (8192)");
    if (batch < 0 || batch > QMOE_NOALLOC_MAX_BATCH)
        return set_error(QMOE_ERR_INVALID,
                         "batch must be in 0 .. QMOE_NOALLOC_MAX_BATCH (16384): the work "
                         "list of this entry point has a fixed size");
    if ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(x)) & 15u)
        return set_error(QMOE_ERR_INVALID, "packed and x must be 16-byte aligned device pointers");
    if (batch == 0) return QMOE_OK;

    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device) {
        cudaError_t e = cudaSetDevice(device);
        if (e != cudaSuccess) return set_error(QMOE_ERR_CUDA, cudaGetErrorString(e));
    }
    int rc = QMOE_OK;
    void *scratch = nullptr;
    int grid = 0;
    rc = setup_device(device, &scratch, &grid);
    if (rc == QMOE_OK) {
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        int32_t *counters = static_cast<int32_t *>(scratch);
        int4 *groups = reinterpret_cast<int4 *>(static_cast<unsigned char *>(scratch) + kCounterBytes);
        // Every call rewrites all of the work list its GEMV reads (both group
        // counts, the segment offsets and each descriptor up to the count), so
        // nothing has to be cleared between calls.
        PermuteParams pp{};
        pp.topk_idx = nullptr;
        pp.T = batch;
        pp.K = 0;
        pp.e_begin = 0;
        pp.e_count = 1;
        pp.chunk = kQgemvTokens;
        pp.shared_count = batch;
        pp.seg_off = counters + 2;
        pp.assign_pos = nullptr;
        pp.pos_tok = nullptr;
        pp.groups = groups;
        pp.n_groups = counters;
        cudaError_t e = launch_permute(pp, st);
        if (e == cudaSuccess) {
            QgemvParams q{};
            q.groups = groups;
            q.n_groups = counters;
            q.rows = 0;
            q.K = (int)in_features;
            q.ws[0] = packed;
            q.ss[0] = scales;
            q.rows_s = (int)out_features;
            q.K_s = (int)in_features;
            q.act = x;
            q.act_dtype = 0;
            q.act_ld = in_features;
            q.pos_tok = nullptr;
            q.shared_base = 0;
            q.out = y;
            q.out_ld = out_features;
            e = launch_qgemv(1, q, grid, st);
        }
        if (e != cudaSuccess) rc = set_error(QMOE_ERR_CUDA, cudaGetErrorString(e));
    }
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    return rc;
}
