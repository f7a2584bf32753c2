// Library-wide entry points: version, error messages, device status word.
#include <stdarg.h>
#include <stddef.h>
#include <string.h>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

// Per device that loaded the library: the status word the kernels set when
// a bounded wait gives up (read by qb_kernel_status), and the limit of those
// waits in ns (qb_set_wait_limit). Kernels get the address of `status` and
// read the limit as the 64-bit word 8 bytes after it (qb::tc::wait_limit_ns).
struct DeviceHealth {
    uint32_t status;
    uint32_t pad;
    uint64_t wait_limit_ns;
};
static_assert(offsetof(DeviceHealth, wait_limit_ns) == 8, "kernels read the limit at status + 2");
constexpr uint64_t DEFAULT_WAIT_LIMIT_NS = 1000000000ull;
__device__ DeviceHealth qb_device_health = {0u, 0u, DEFAULT_WAIT_LIMIT_NS};

namespace qb {

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

uint32_t* device_status_ptr() {
    // cudaGetSymbolAddress is per device; the address is cached per device
    // id (host threads that race here store the same value).
    static std::atomic<uint32_t*> cache[MAX_DEVICES];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return nullptr;
    uint32_t* got = cache[dev].load(std::memory_order_acquire);
    if (got == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, qb_device_health) != cudaSuccess) return nullptr;
        got = static_cast<uint32_t*>(p);
        cache[dev].store(got, std::memory_order_release);
    }
    return got;
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

namespace {
// Where status_exchange_kernel leaves the word it took.
__device__ uint32_t qb_status_taken;

// Takes the status word and leaves 0 in one atomic step, so a bit that
// another stream's kernel sets meanwhile is either taken here or stays.
__global__ void status_exchange_kernel() {
    qb_status_taken = atomicExch(&qb_device_health.status, 0u);
}
}  // namespace

extern "C" int qb_kernel_status(int device, uint32_t* status_out) {
    if (status_out == nullptr) return qb::invalid("qb_kernel_status: status_out is NULL");
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return qb::launch_status("qb_kernel_status: cudaSetDevice");
    uint32_t value = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) {
        status_exchange_kernel<<<1, 1>>>();
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&value, qb_status_taken, sizeof(value));
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        qb::set_error("qb_kernel_status: %s", cudaGetErrorString(e));
        return QB_ERR_CUDA;
    }
    *status_out = value;
    return QB_OK;
}

extern "C" int qb_set_wait_limit(int device, uint64_t limit_ns) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return qb::launch_status("qb_set_wait_limit: cudaSetDevice");
    const uint64_t v = limit_ns ? limit_ns : DEFAULT_WAIT_LIMIT_NS;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess)
        e = cudaMemcpyToSymbol(qb_device_health, &v, sizeof(v), offsetof(DeviceHealth, wait_limit_ns));
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        qb::set_error("qb_set_wait_limit: %s", cudaGetErrorString(e));
        return QB_ERR_CUDA;
    }
    return QB_OK;
}
