// Library state behind the C ABI: thread-local error text, device checks,
// the device error word and the launch counter.
#include <cstring>
#include <mutex>
#include <set>
#include <tuple>
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

int ensure_max_smem(const void *kernel, int bytes, const char *what) {
    static std::mutex mu;
    static std::set<std::tuple<const void *, int, int>> done;  // (kernel, device, bytes)
    int dev = 0;
    LCML_CUDA(cudaGetDevice(&dev));
    const auto key = std::make_tuple(kernel, dev, bytes);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (done.count(key)) return LCML_OK;
    }
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess)
        return set_error(LCML_ERR_CUDA, "%s: cudaFuncSetAttribute(smem=%d) on device %d failed: %s", what, bytes, dev,
                         cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(mu);
    done.insert(key);
    return LCML_OK;
}

}// namespace lcml

extern "C" {

const char *lcml_last_error(void) { return lcml::t_error; }

int lcml_abi_version(void) { return 2; }

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

extern "C" {

int lcml_device_alloc(size_t bytes, void **ptr) {
    LCML_CHECK_ARG(ptr != nullptr, "lcml_device_alloc: ptr is NULL");
    *ptr = nullptr;
    if (bytes == 0) return LCML_OK;
    LCML_CUDA(cudaMalloc(ptr, bytes));
    return LCML_OK;
}

int lcml_device_free(void *ptr) {
    if (ptr) LCML_CUDA(cudaFree(ptr));
    return LCML_OK;
}

int lcml_memcpy_async(void *dst, const void *src, size_t bytes, int kind, lcml_stream_t stream) {
    if (bytes == 0) return LCML_OK;
    LCML_CHECK_ARG(dst && src, "lcml_memcpy_async: null pointer");
    cudaMemcpyKind k;
    switch (kind) {
        case 1: k = cudaMemcpyHostToDevice; break;
        case 2: k = cudaMemcpyDeviceToHost; break;
        case 3: k = cudaMemcpyDeviceToDevice; break;
        default: return lcml::set_error(LCML_ERR_INVALID_ARGUMENT, "lcml_memcpy_async: kind %d", kind);
    }
    LCML_CUDA(cudaMemcpyAsync(dst, src, bytes, k, lcml::to_cuda(stream)));
    return LCML_OK;
}

int lcml_memset_async(void *dst, int value, size_t bytes, lcml_stream_t stream) {
    if (bytes == 0) return LCML_OK;
    LCML_CHECK_ARG(dst != nullptr, "lcml_memset_async: null pointer");
    LCML_CUDA(cudaMemsetAsync(dst, value, bytes, lcml::to_cuda(stream)));
    return LCML_OK;
}

int lcml_stream_synchronize(lcml_stream_t stream) {
    LCML_CUDA(cudaStreamSynchronize(lcml::to_cuda(stream)));
    return LCML_OK;
}

int lcml_stream_create(lcml_stream_t *stream) {
    LCML_CHECK_ARG(stream != nullptr, "lcml_stream_create: stream is NULL");
    cudaStream_t s = nullptr;
    LCML_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *stream = reinterpret_cast<lcml_stream_t>(s);
    return LCML_OK;
}

int lcml_stream_destroy(lcml_stream_t stream) {
    if (stream) LCML_CUDA(cudaStreamDestroy(lcml::to_cuda(stream)));
    return LCML_OK;
}

int lcml_event_create(lcml_event_t *event) {
    LCML_CHECK_ARG(event != nullptr, "lcml_event_create: event is NULL");
    cudaEvent_t e = nullptr;
    LCML_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    *event = reinterpret_cast<lcml_event_t>(e);
    return LCML_OK;
}

int lcml_event_destroy(lcml_event_t event) {
    if (event) LCML_CUDA(cudaEventDestroy(reinterpret_cast<cudaEvent_t>(event)));
    return LCML_OK;
}

int lcml_event_record(lcml_event_t event, lcml_stream_t stream) {
    LCML_CHECK_ARG(event != nullptr, "lcml_event_record: event is NULL");
    LCML_CUDA(cudaEventRecord(reinterpret_cast<cudaEvent_t>(event), lcml::to_cuda(stream)));
    return LCML_OK;
}

int lcml_stream_wait_event(lcml_stream_t stream, lcml_event_t event) {
    LCML_CHECK_ARG(event != nullptr, "lcml_stream_wait_event: event is NULL");
    LCML_CUDA(cudaStreamWaitEvent(lcml::to_cuda(stream), reinterpret_cast<cudaEvent_t>(event), 0));
    return LCML_OK;
}

}// extern "C"

extern "C" {

int lcml_ipc_get_handle(void *device_ptr, void *handle_out) {
    LCML_CHECK_ARG(device_ptr && handle_out, "lcml_ipc_get_handle: null pointer");
    static_assert(sizeof(cudaIpcMemHandle_t) == LCML_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    LCML_CUDA(cudaIpcGetMemHandle(&h, device_ptr));
    std::memcpy(handle_out, &h, sizeof(h));
    return LCML_OK;
}

int lcml_ipc_open(const void *handle, void **device_ptr) {
    LCML_CHECK_ARG(handle && device_ptr, "lcml_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    LCML_CUDA(cudaIpcOpenMemHandle(device_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return LCML_OK;
}

int lcml_ipc_close(void *device_ptr) {
    if (device_ptr) LCML_CUDA(cudaIpcCloseMemHandle(device_ptr));
    return LCML_OK;
}

int lcml_enable_peer_access(int peer_device) {
    const cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return LCML_OK;
    }
    if (e != cudaSuccess) return lcml::set_error(LCML_ERR_CUDA, "cudaDeviceEnablePeerAccess(%d): %s", peer_device,
                                                 cudaGetErrorString(e));
    return LCML_OK;
}

}// extern "C"
