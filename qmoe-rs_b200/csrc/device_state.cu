// device_state.cu -- the device-side error word.  A tensor-core kernel whose
// bounded wait gives up sets a bit here (and returns instead of hanging); the
// host reads it back in qmoe_ctx_synchronize and after every call that
// returns host data, and reports QMOE_ERR_CUDA.
#include "kernels.h"

namespace qmoe {

__device__ int g_device_error;

int *device_error_flag() {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    return static_cast<int *>(p);
}

}  // namespace qmoe
