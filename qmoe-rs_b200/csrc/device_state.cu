// device_state.cu -- per-device state the launchers share.
//
// The device-side error word: a tensor-core kernel whose bounded wait gives
// up sets a bit here (and returns instead of hanging); the host reads it back
// in qmoe_ctx_synchronize and after every call that returns host data, and
// reports QMOE_ERR_CUDA.  Every GPU holds its own copy of the word, so its
// device address is looked up (and cached) per device.
//
// The dynamic shared-memory opt-in of each kernel: a per-device attribute
// that the launchers only ever raise, so one launcher's setting for a small
// case never lowers what another launcher of the same kernel relies on.
#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "kernels.h"

namespace qmoe {

__device__ int g_device_error;

namespace {
constexpr int kMaxDevices = 64;
std::atomic<int *> g_error_addr[kMaxDevices];
}  // namespace

int *device_error_flag() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    if (dev >= 0 && dev < kMaxDevices) {
        int *p = g_error_addr[dev].load(std::memory_order_acquire);
        if (p) return p;
    }
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    if (dev >= 0 && dev < kMaxDevices) g_error_addr[dev].store(static_cast<int *>(p), std::memory_order_release);
    return static_cast<int *>(p);
}

int device_sm_count() {
    static std::atomic<int> cached[kMaxDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev >= 0 && dev < kMaxDevices) {
        const int c = cached[dev].load(std::memory_order_relaxed);
        if (c > 0) return c;
    }
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    if (dev >= 0 && dev < kMaxDevices) cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

cudaError_t ensure_dyn_smem(const void *func, size_t bytes) {
    // (no shortcut below 48 KB: a kernel's static shared memory counts
    // against the default limit too, so a launch with less dynamic memory
    // than that can still need the opt-in)
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, size_t> raised;
    std::lock_guard<std::mutex> lock(mu);
    size_t &cur = raised[{func, dev}];
    if (bytes <= cur) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) cur = bytes;
    return e;
}

}  // namespace qmoe
