// Host-side helpers shared by the C-ABI translation units: error reporting,
// argument checks and the launch counter. Internal to liblcml_fp8.so.
#pragma once

#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include <cuda_runtime.h>

#include "../../include/lcml_fp8.h"

namespace lcml {

int set_error(int status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

// Kernels launched by this library (lcml_launch_count()).
extern std::atomic<uint64_t> g_launches;

inline cudaStream_t to_cuda(lcml_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int sm_count();

// Device address of the error word on the current device (nullptr if unavailable).
int *device_error_word();

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current
// device, once per (kernel, device): the attribute belongs to the device that
// is current when it is set, so a process driving several GPUs sets it on
// each. Returns an lcml_status (the message names `what`).
int ensure_max_smem(const void *kernel, int bytes, const char *what);

__host__ __device__ inline bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Geometry of an implicit-GEMM convolution: the GEMM's A operand (rows =
// output pixels (n, oh, ow), K = (kh, kw, c) with c fastest) is loaded from
// the NHWC activation by TMA im2col copies in the GEMM kernel instead of
// being materialized by an im2col pass. 32-bit extents (the caller checks).
struct ConvGeom {
    const uint8_t *x;  // NHWC e4m3 activation, C channels, C % 64 == 0, 16-byte aligned
    int N, H, W, C, oH, oW, kH, kW, sH, sW, pH, pW, dH, dW;
    int ktaps;         // kH * kW * C (the GEMM's K)
};

// lcml_fp8_gemm whose A is gathered through `geo` (d->A and d->lda unused;
// d->M = N * oH * oW, d->K = the packed K of the weights).
int fp8_gemm_implicit_conv(const lcml_fp8_gemm_desc *d, const ConvGeom &geo, cudaStream_t st);

// lcml_fp8_conv for group > 1: the direct grouped kernel (conv_direct.cu);
// Kp / Cp are the packed K and channels per tap of C / group channels.
int fp8_conv_grouped(const lcml_fp8_conv_desc *d, int64_t Kp, int64_t Cp, cudaStream_t st);

}// namespace lcml

#define LCML_CHECK_ARG(cond, ...)                                                  \
    do {                                                                           \
        if (!(cond)) return ::lcml::set_error(LCML_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
    } while (0)

// Reports the launch error (if any) of the kernel just enqueued.
#define LCML_LAUNCHED(name)                                                                        \
    do {                                                                                           \
        ::lcml::g_launches.fetch_add(1, std::memory_order_relaxed);                                \
        cudaError_t e_ = cudaGetLastError();                                                       \
        if (e_ != cudaSuccess)                                                                     \
            return ::lcml::set_error(LCML_ERR_CUDA, "%s launch failed: %s", name, cudaGetErrorString(e_)); \
    } while (0)

#define LCML_CUDA(call)                                                                           \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess)                                                                    \
            return ::lcml::set_error(LCML_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)
