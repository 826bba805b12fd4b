// Per-device sticky status word and cached device properties.
#include <mutex>

#include "common.cuh"
#include "engine.h"

namespace spmmb {

// One status word per device (a __device__ variable is instantiated on every
// device that loads this module).
__device__ DevStatus g_dev_status;

namespace {
constexpr int kMaxDevices = 64;
DevStatus *g_status_ptr[kMaxDevices];
int g_sm_count[kMaxDevices];
std::mutex g_mu;
}  // namespace

DevStatus *device_status_ptr(cudaError_t *err)
{
    int dev = 0;
    *err = cudaGetDevice(&dev);
    if (*err != cudaSuccess) return nullptr;
    if (dev < 0 || dev >= kMaxDevices) {
        *err = cudaErrorInvalidDevice;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_status_ptr[dev]) {
        void *p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_dev_status);
        if (*err != cudaSuccess) return nullptr;
        g_status_ptr[dev] = static_cast<DevStatus *>(p);
    }
    return g_status_ptr[dev];
}

int device_sm_count()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_sm_count[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

}  // namespace spmmb
