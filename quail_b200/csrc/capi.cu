// Library-wide entry points: version, error messages, device status word.
#include <stdarg.h>
#include <string.h>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

// Set by the tcgen05 kernels when a bounded wait gives up; read by
// qb_kernel_status. One word per device that loaded the library.
__device__ uint32_t qb_device_status;

namespace qb {

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

uint32_t* device_status_ptr() {
    // cudaGetSymbolAddress is per device; cache the address per device id.
    static uint32_t* cache[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (cache[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, qb_device_status) != cudaSuccess) return nullptr;
        cache[dev] = static_cast<uint32_t*>(p);
    }
    return cache[dev];
}

int launch_status(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: %s", what, cudaGetErrorString(e));
        return QB_ERR_CUDA;
    }
    return QB_OK;
}

}  // namespace qb

extern "C" int qb_version(void) { return (0 << 16) | (1 << 8) | 0; }

extern "C" const char* qb_last_error(void) { return g_last_error; }

extern "C" int qb_kernel_status(int device, uint32_t* status_out) {
    if (status_out == nullptr) return qb::invalid("qb_kernel_status: status_out is NULL");
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return qb::launch_status("qb_kernel_status: cudaSetDevice");
    uint32_t zero = 0, value = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&value, qb_device_status, sizeof(value));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(qb_device_status, &zero, sizeof(zero));
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        qb::set_error("qb_kernel_status: %s", cudaGetErrorString(e));
        return QB_ERR_CUDA;
    }
    *status_out = value;
    return QB_OK;
}
