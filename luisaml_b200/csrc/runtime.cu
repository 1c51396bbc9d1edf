// Library state behind the C ABI: thread-local error text, device checks,
// the device error word and the launch counter.
#include <cstring>
#include <mutex>
#include <vector>

#include "lcml_device.cuh"
#include "lcml_internal.h"

namespace lcml {

namespace {
__device__ int g_device_error = 0;
}

std::atomic<uint64_t> g_launches{0};

namespace {
thread_local char t_error[1024] = "";
}

int set_error(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_error, sizeof(t_error), fmt, ap);
    va_end(ap);
    return status;
}

void clear_error() { t_error[0] = '\0'; }

int sm_count() {
    static std::mutex mu;
    static std::vector<int> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lk(mu);
    if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

int *device_error_word() {
    static std::mutex mu;
    static std::vector<int *> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, nullptr);
    if (cache[dev] == nullptr) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) cache[dev] = static_cast<int *>(p);
        else cudaGetLastError();
    }
    return cache[dev];
}

}// namespace lcml

extern "C" {

const char *lcml_last_error(void) { return lcml::t_error; }

int lcml_abi_version(void) { return 1; }

int lcml_device_check(void) {
    int dev = 0, n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return lcml::set_error(LCML_ERR_NO_DEVICE, "no CUDA device visible");
    }
    if (cudaGetDevice(&dev) != cudaSuccess) return lcml::set_error(LCML_ERR_NO_DEVICE, "cudaGetDevice failed");
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
        return lcml::set_error(LCML_ERR_NO_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                               major, minor);
    return LCML_OK;
}

int lcml_device_error(int *code) {
    LCML_CHECK_ARG(code != nullptr, "lcml_device_error: code is NULL");
    LCML_CUDA(cudaDeviceSynchronize());
    int v = 0, zero = 0;
    LCML_CUDA(cudaMemcpyFromSymbol(&v, lcml::g_device_error, sizeof(int)));
    LCML_CUDA(cudaMemcpyToSymbol(lcml::g_device_error, &zero, sizeof(int)));
    *code = v;
    if (v != 0) return lcml::set_error(LCML_ERR_DEVICE_TIMEOUT, "a kernel abandoned a bounded wait (code %d)", v);
    return LCML_OK;
}

uint64_t lcml_launch_count(void) { return lcml::g_launches.load(std::memory_order_relaxed); }

}// extern "C"
