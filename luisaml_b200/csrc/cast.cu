// Cast (src/onnx/operators/cast.cpp:10-162) between fp32, fp16, bf16 and the
// quantized storage types FLOAT8E4M3FN, FLOAT8E5M2 and FLOAT4E2M1 (two codes
// per byte, element 2i in the low nibble of byte i, as the reference's
// FP4Data packs them, include/onnx/dynamic_array/fp4_data.h).
//
// Semantics follow the reference's Cast::apply:
//   * to FP8 / FP4 from any floating type: from_float(half(x)) — the value is
//     first rounded to half (cast.cpp:63-67: `fp8_from(input[i].cast<half>())`),
//     then encoded with the reference's CPU codec (fp_quantized.h), so a value
//     can be rounded twice;
//   * from FP8 / FP4: decode, then convert to the destination type
//     (cast.cpp:44-48); every FP8 / FP4 value is exact in half, float and bf16;
//   * between fp32 / fp16 / bf16: one round-to-nearest-even conversion;
//   * FP8 / FP4 to another FP8 / FP4 type: decode, encode (the decoded value is
//     already a half, so no double rounding).
// The `saturate` attribute does not change FP8 results, as in the reference
// (its FP8 encoders saturate e4m3 / e2m1 and overflow e5m2 to inf regardless).
//
// One thread converts groups of 8 elements with one vector load and one
// vector store per operand where both pointers allow it (HBM-bound: bytes in
// + bytes out per element); the last partial group is done by one thread, so
// no byte of a packed FP4 output is written by two threads.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "lcml_device.cuh"
#include "lcml_internal.h"

namespace lcml {
namespace {

constexpr int kThreads = 256;
constexpr int kGroup = 8;  // elements per thread and step

enum CastType : int { kF32 = 0, kF16 = 1, kBF16 = 2, kE4M3 = 3, kE5M2 = 4, kE2M1 = 5 };

int cast_type(int onnx_dtype) {
    switch (onnx_dtype) {
        case LCML_DTYPE_FLOAT: return kF32;
        case LCML_DTYPE_FLOAT16: return kF16;
        case LCML_DTYPE_BFLOAT16: return kBF16;
        case LCML_DTYPE_FLOAT8E4M3FN: return kE4M3;
        case LCML_DTYPE_FLOAT8E5M2: return kE5M2;
        case LCML_DTYPE_FLOAT4E2M1: return kE2M1;
        default: return -1;
    }
}

// Bytes of one group of kGroup elements.
constexpr int group_bytes(int t) { return t == kF32 ? 32 : (t == kF16 || t == kBF16) ? 16 : t == kE2M1 ? 4 : 8; }

__host__ __device__ constexpr bool is_quantized(int t) { return t >= kE4M3; }

template <int T>
__device__ __forceinline__ float decode1(const uint8_t *p, int64_t i) {
    if (T == kF32) return reinterpret_cast<const float *>(p)[i];
    if (T == kF16) return __half2float(reinterpret_cast<const __half *>(p)[i]);
    if (T == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    if (T == kE4M3) return e4m3_decode(p[i]);
    if (T == kE5M2) return e5m2_decode(p[i]);
    return e2m1_decode((p[i >> 1] >> ((i & 1) * 4)) & 0xfu);
}

// The value `v` (of source type SRC) converted to destination DST's bits.
template <int SRC, int DST>
__device__ __forceinline__ uint32_t convert1(float v) {
    if (DST == kF32) return __float_as_uint(v);
    if (DST == kF16) return __half_as_ushort(__float2half_rn(v));
    if (DST == kBF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
    // quantized destination: the value rounded to half first (a no-op for a
    // half or quantized source, whose values are halves already)
    if (SRC == kF32 || SRC == kBF16) v = __half2float(__float2half_rn(v));
    if (DST == kE4M3) return e4m3_encode(v);
    if (DST == kE5M2) return e5m2_encode(v);
    return e2m1_encode(v);
}

// Loads group g (elements 8g .. 8g+7) of x as floats.
template <int T, bool VEC>
__device__ __forceinline__ void load_group(const uint8_t *x, int64_t g, float (&v)[kGroup]) {
    if (VEC) {
        const uint8_t *p = x + g * group_bytes(T);
        if (T == kF32) {
            const float4 a = __ldcs(reinterpret_cast<const float4 *>(p)), b = __ldcs(reinterpret_cast<const float4 *>(p) + 1);
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        } else if (T == kF16 || T == kBF16) {
            const uint4 w = __ldcs(reinterpret_cast<const uint4 *>(p));
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (T == kF16) {
                    v[2 * k] = __half2float(__ushort_as_half(static_cast<unsigned short>(ws[k] & 0xffffu)));
                    v[2 * k + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(ws[k] >> 16)));
                } else {
                    v[2 * k] = __uint_as_float(ws[k] << 16);
                    v[2 * k + 1] = __uint_as_float(ws[k] & 0xffff0000u);
                }
            }
        } else if (T == kE2M1) {
            const uint32_t w = __ldcs(reinterpret_cast<const unsigned int *>(p));
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = e2m1_decode((w >> (4 * k)) & 0xfu);
        } else {
            const uint2 w = __ldcs(reinterpret_cast<const uint2 *>(p));
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t b = ((k < 4 ? w.x : w.y) >> (8 * (k & 3))) & 0xffu;
                v[k] = T == kE4M3 ? e4m3_decode(b) : e5m2_decode(b);
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < kGroup; ++k) v[k] = decode1<T>(x, g * kGroup + k);
    }
}

template <int T, bool VEC>
__device__ __forceinline__ void store_group(uint8_t *y, int64_t g, const uint32_t (&b)[kGroup]) {
    uint8_t *p = y + g * group_bytes(T);
    if (T == kF32) {
        if (VEC) {
            __stcs(reinterpret_cast<uint4 *>(p), make_uint4(b[0], b[1], b[2], b[3]));
            __stcs(reinterpret_cast<uint4 *>(p) + 1, make_uint4(b[4], b[5], b[6], b[7]));
        } else {
#pragma unroll
            for (int k = 0; k < kGroup; ++k) reinterpret_cast<uint32_t *>(p)[k] = b[k];
        }
    } else if (T == kF16 || T == kBF16) {
        if (VEC) {
            __stcs(reinterpret_cast<uint4 *>(p),
                   make_uint4(b[0] | b[1] << 16, b[2] | b[3] << 16, b[4] | b[5] << 16, b[6] | b[7] << 16));
        } else {
#pragma unroll
            for (int k = 0; k < kGroup; ++k) reinterpret_cast<unsigned short *>(p)[k] = static_cast<unsigned short>(b[k]);
        }
    } else if (T == kE2M1) {
        uint32_t w = 0;
#pragma unroll
        for (int k = 0; k < kGroup; ++k) w |= b[k] << (4 * k);
        if (VEC) __stcs(reinterpret_cast<unsigned int *>(p), w);
        else
#pragma unroll
            for (int k = 0; k < 4; ++k) p[k] = static_cast<uint8_t>(w >> (8 * k));
    } else {
        if (VEC) {
            __stcs(reinterpret_cast<uint2 *>(p),
                   make_uint2(b[0] | b[1] << 8 | b[2] << 16 | b[3] << 24, b[4] | b[5] << 8 | b[6] << 16 | b[7] << 24));
        } else {
#pragma unroll
            for (int k = 0; k < kGroup; ++k) p[k] = static_cast<uint8_t>(b[k]);
        }
    }
}

template <int SRC, int DST, bool VEC>
__global__ void __launch_bounds__(kThreads) k_cast(const uint8_t *__restrict__ x, uint8_t *__restrict__ y, int64_t n) {
    const int64_t groups = n / kGroup;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nt = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t g = tid; g < groups; g += nt) {
        float v[kGroup];
        load_group<SRC, VEC>(x, g, v);
        uint32_t b[kGroup];
#pragma unroll
        for (int k = 0; k < kGroup; ++k) b[k] = convert1<SRC, DST>(v[k]);
        store_group<DST, VEC>(y, g, b);
    }
    // the last partial group: one thread, element by element
    if (tid == 0 && groups * kGroup < n) {
        const int64_t i0 = groups * kGroup;
        uint8_t nib = 0;
        for (int64_t i = i0; i < n; ++i) {
            const uint32_t b = convert1<SRC, DST>(decode1<SRC>(x, i));
            if (DST == kF32) reinterpret_cast<uint32_t *>(y)[i] = b;
            else if (DST == kF16 || DST == kBF16) reinterpret_cast<unsigned short *>(y)[i] = static_cast<unsigned short>(b);
            else if (DST == kE2M1) {
                // byte i/2 holds elements i (low nibble, i even) and i+1; a
                // lone last element leaves the high nibble zero
                if ((i & 1) == 0) nib = static_cast<uint8_t>(b);
                else y[i >> 1] = static_cast<uint8_t>(nib | (b << 4));
                if ((i & 1) == 0 && i + 1 == n) y[i >> 1] = nib;
            } else y[i] = static_cast<uint8_t>(b);
        }
    }
}

int grid_for(int64_t items) {
    const int64_t per_wave = static_cast<int64_t>(sm_count()) * (2048 / kThreads);
    int64_t b = (items + kThreads - 1) / kThreads;
    if (b > per_wave) b = per_wave;
    return static_cast<int>(b < 1 ? 1 : b);
}

template <int SRC, int DST>
int launch_cast(const void *x, void *y, int64_t n, cudaStream_t st) {
    const bool vec = aligned(x, group_bytes(SRC)) && aligned(y, group_bytes(DST));
    const int grid = grid_for((n + kGroup - 1) / kGroup);
    if (vec) k_cast<SRC, DST, true><<<grid, kThreads, 0, st>>>(static_cast<const uint8_t *>(x), static_cast<uint8_t *>(y), n);
    else k_cast<SRC, DST, false><<<grid, kThreads, 0, st>>>(static_cast<const uint8_t *>(x), static_cast<uint8_t *>(y), n);
    LCML_LAUNCHED("cast");
    return LCML_OK;
}

template <int SRC>
int dispatch_dst(int dst, const void *x, void *y, int64_t n, cudaStream_t st) {
    switch (dst) {
        case kF32: return launch_cast<SRC, kF32>(x, y, n, st);
        case kF16: return launch_cast<SRC, kF16>(x, y, n, st);
        case kBF16: return launch_cast<SRC, kBF16>(x, y, n, st);
        case kE4M3: return launch_cast<SRC, kE4M3>(x, y, n, st);
        case kE5M2: return launch_cast<SRC, kE5M2>(x, y, n, st);
        default: return launch_cast<SRC, kE2M1>(x, y, n, st);
    }
}

}// namespace
}// namespace lcml

extern "C" int lcml_cast(const void *x, int x_dtype, void *y, int y_dtype, int64_t n, lcml_stream_t stream) {
    using namespace lcml;
    LCML_CHECK_ARG(n >= 0, "lcml_cast: negative n");
    const int src = cast_type(x_dtype), dst = cast_type(y_dtype);
    if (src < 0 || dst < 0)
        return set_error(LCML_ERR_UNSUPPORTED, "lcml_cast: %d -> %d unsupported (FLOAT, FLOAT16, BFLOAT16, "
                                               "FLOAT8E4M3FN, FLOAT8E5M2, FLOAT4E2M1)", x_dtype, y_dtype);
    if (n == 0) return LCML_OK;
    LCML_CHECK_ARG(x && y, "lcml_cast: null pointer");
    LCML_CHECK_ARG(src != dst, "lcml_cast: same source and destination type (a copy)");
    // element alignment (the kernel's scalar path loads and stores whole elements)
    auto elem_align = [](int t) -> uintptr_t { return t == kF32 ? 4 : (t == kF16 || t == kBF16) ? 2 : 1; };
    LCML_CHECK_ARG(aligned(x, elem_align(src)) && aligned(y, elem_align(dst)),
                   "lcml_cast: x / y not aligned to their element size");
    cudaStream_t st = to_cuda(stream);
    switch (src) {
        case kF32: return dispatch_dst<kF32>(dst, x, y, n, st);
        case kF16: return dispatch_dst<kF16>(dst, x, y, n, st);
        case kBF16: return dispatch_dst<kBF16>(dst, x, y, n, st);
        case kE4M3: return dispatch_dst<kE4M3>(dst, x, y, n, st);
        case kE5M2: return dispatch_dst<kE5M2>(dst, x, y, n, st);
        default: return dispatch_dst<kE2M1>(dst, x, y, n, st);
    }
}
