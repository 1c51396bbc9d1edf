// QuantizeLinear / DequantizeLinear / dynamic-scale kernels for the e4m3 path.
//
// All of these are HBM-bound streaming kernels: 16 elements per thread per
// step (four 16-byte fp32 loads, one 16-byte e4m3 store), grid sized as a
// multiple of the SM count, grid-stride loops. Algorithmic traffic:
// 4 B read + 1 B written per element (+ one 4 B re-read per element for
// two-pass dynamic per-tensor scales).
#include <cuda_bf16.h>

#include "lcml_device.cuh"
#include "lcml_internal.h"

namespace lcml {
namespace {

constexpr int kThreads = 256;

enum ScaleKind : int {
    kScaleTensor = 0,   // one scale
    kScaleGroup16 = 1,  // per-axis, inner % 16 == 0: constant over each 16-element group
    kScaleInner1 = 2,   // per-axis, inner == 1, axis_len % 16 == 0: 16 consecutive scales
    kScaleGeneric = 3,  // per-axis, anything else: per-element index arithmetic
};

__device__ __forceinline__ float load_scale(const float *__restrict__ sc, int64_t idx, bool from_amax) {
    float v = __ldg(sc + idx);
    return from_amax ? scale_from_amax(v) : v;
}

// A scale with its correctly rounded reciprocal, for quantize2_fast().
struct Scale {
    float s, r;
    bool ok;
};

__device__ __forceinline__ Scale make_scale(float v) {
    Scale sc;
    sc.s = v;
    sc.r = __frcp_rn(v);
    sc.ok = scale_fast_ok(v, sc.r);
    return sc;
}

__device__ __forceinline__ uint4 pack16(float4 a, float4 b, float4 c, float4 d, const Scale &sc) {
    const float v[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
    uint32_t w[4];
    quantize_block_fast<16>(v, sc.s, sc.r, sc.ok, w);
    return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint32_t pack4v(float4 v, const float *s) {
    const Scale s0 = make_scale(s[0]), s1 = make_scale(s[1]), s2 = make_scale(s[2]), s3 = make_scale(s[3]);
    return (quantize2_fast(v.x, v.x, s0.s, s0.r, s0.ok) & 0xffu) | ((quantize2_fast(v.y, v.y, s1.s, s1.r, s1.ok) & 0xffu) << 8) |
           ((quantize2_fast(v.z, v.z, s2.s, s2.r, s2.ok) & 0xffu) << 16) | ((quantize2_fast(v.w, v.w, s3.s, s3.r, s3.ok) & 0xffu) << 24);
}

template <int KIND, bool FROM_AMAX>
__global__ void __launch_bounds__(kThreads) k_quantize(const float *__restrict__ x, int64_t n, int64_t axis_len,
                                                       int64_t inner, const float *__restrict__ sc,
                                                       float *__restrict__ scale_out, uint8_t *__restrict__ y) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t n16 = n >> 4;
    float s_tensor = 0.0f;
    if (KIND == kScaleTensor) s_tensor = load_scale(sc, 0, FROM_AMAX);
    const Scale st = make_scale(s_tensor);
    int64_t g = tid;
    if (KIND == kScaleTensor) {
        // two 16-element groups per thread per iteration: 8 loads in flight
        for (; g + nthreads < n16; g += 2 * nthreads) {
            const float4 *xa = reinterpret_cast<const float4 *>(x) + g * 4;
            const float4 *xb = reinterpret_cast<const float4 *>(x) + (g + nthreads) * 4;
            const float4 a0 = __ldcs(xa), a1 = __ldcs(xa + 1), a2 = __ldcs(xa + 2), a3 = __ldcs(xa + 3);
            const float4 b0 = __ldcs(xb), b1 = __ldcs(xb + 1), b2 = __ldcs(xb + 2), b3 = __ldcs(xb + 3);
            __stcs(reinterpret_cast<uint4 *>(y) + g, pack16(a0, a1, a2, a3, st));
            __stcs(reinterpret_cast<uint4 *>(y) + g + nthreads, pack16(b0, b1, b2, b3, st));
        }
    }
    for (; g < n16; g += nthreads) {
        const float4 *xp = reinterpret_cast<const float4 *>(x) + g * 4;
        const float4 v0 = __ldcs(xp), v1 = __ldcs(xp + 1), v2 = __ldcs(xp + 2), v3 = __ldcs(xp + 3);
        uint4 out;
        if (KIND == kScaleTensor) {
            out = pack16(v0, v1, v2, v3, st);
        } else if (KIND == kScaleGroup16) {
            out = pack16(v0, v1, v2, v3, make_scale(load_scale(sc, ((g << 4) / inner) % axis_len, FROM_AMAX)));
        } else {
            float s[16];
            if (KIND == kScaleInner1) {
                const int64_t base = (g << 4) % axis_len;
#pragma unroll
                for (int j = 0; j < 16; ++j) s[j] = load_scale(sc, base + j, FROM_AMAX);
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) s[j] = load_scale(sc, (((g << 4) + j) / inner) % axis_len, FROM_AMAX);
            }
            out.x = pack4v(v0, s);
            out.y = pack4v(v1, s + 4);
            out.z = pack4v(v2, s + 8);
            out.w = pack4v(v3, s + 12);
        }
        __stcs(reinterpret_cast<uint4 *>(y) + g, out);
    }
    // ragged tail (n % 16 elements)
    const int64_t t = (n16 << 4) + tid;
    if (t < n) {
        const float s = (KIND == kScaleTensor) ? s_tensor : load_scale(sc, (t / inner) % axis_len, FROM_AMAX);
        y[t] = static_cast<uint8_t>(quantize1(x[t], s));
    }
    if (FROM_AMAX && scale_out != nullptr) {
        const int64_t ns = (KIND == kScaleTensor) ? 1 : axis_len;
        for (int64_t i = tid; i < ns; i += nthreads) scale_out[i] = load_scale(sc, i, true);
    }
}

// Unaligned fallback: one element per thread-iteration.
template <bool FROM_AMAX>
__global__ void __launch_bounds__(kThreads) k_quantize_scalar(const float *__restrict__ x, int64_t n,
                                                              int64_t axis_len, int64_t inner,
                                                              const float *__restrict__ sc, int per_axis,
                                                              float *__restrict__ scale_out,
                                                              uint8_t *__restrict__ y) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = tid; i < n; i += nthreads) {
        const float s = load_scale(sc, per_axis ? (i / inner) % axis_len : 0, FROM_AMAX);
        y[i] = static_cast<uint8_t>(quantize1(x[i], s));
    }
    if (FROM_AMAX && scale_out != nullptr) {
        const int64_t ns = per_axis ? axis_len : 1;
        for (int64_t i = tid; i < ns; i += nthreads) scale_out[i] = load_scale(sc, i, true);
    }
}

// ---------------------------------------------------------------------------
// Reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide max of v (all threads get the result). `red` is >= 32 words of smem.
__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, uint32_t *red) {
    v = warp_max_u32(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    uint32_t r = (l < static_cast<int>(blockDim.x >> 5)) ? red[l] : 0u;
    r = warp_max_u32(r);
    return r;
}

__global__ void __launch_bounds__(kThreads) k_amax(const float *__restrict__ x, int64_t n, int vec_ok,
                                                   uint32_t *__restrict__ out) {
    __shared__ uint32_t red[32];
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    uint32_t m = 0;
    int64_t done = 0;
    if (vec_ok) {
        const int64_t n4 = n >> 2;
        for (int64_t i = tid; i < n4; i += nthreads) {
            const float4 v = __ldcs(reinterpret_cast<const float4 *>(x) + i);
            m = max(m, max(max(abs_bits_nan0(v.x), abs_bits_nan0(v.y)), max(abs_bits_nan0(v.z), abs_bits_nan0(v.w))));
        }
        done = n4 << 2;
    }
    for (int64_t i = done + tid; i < n; i += nthreads) m = max(m, abs_bits_nan0(x[i]));
    m = block_max_u32(m, red);
    if (threadIdx.x == 0) atomicMax(out, m);
}

// Dynamic per-tensor quantization, pass 1: block b's max |x| (as ordered
// bits, NaN ignored) into partial[b], so nothing needs zeroing first. x is
// read front to back with normal caching: the last ~100 MB stay in the L2
// for pass 2, which walks the tensor back to front.
constexpr int kMaxAmaxParts = 1024;  // LCML_FP8_TENSOR_DYNAMIC_WORKSPACE_BYTES / 4

__global__ void __launch_bounds__(kThreads) k_amax_partial(const float *__restrict__ x, int64_t n,
                                                           uint32_t *__restrict__ partial) {
    __shared__ uint32_t red[32];
    griddep_launch_dependents();  // pass 2 may start its set-up
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    uint32_t m = 0;
    const int64_t n4 = n >> 2;
    auto max4 = [](uint32_t a, const float4 &v) {
        return max(a, max(max(abs_bits_nan0(v.x), abs_bits_nan0(v.y)), max(abs_bits_nan0(v.z), abs_bits_nan0(v.w))));
    };
    // four independent 16-byte loads in flight per thread per step
    int64_t i = tid;
    for (; i + 3 * nthreads < n4; i += 4 * nthreads) {
        const float4 *p = reinterpret_cast<const float4 *>(x) + i;
        const float4 v0 = __ldg(p), v1 = __ldg(p + nthreads), v2 = __ldg(p + 2 * nthreads), v3 = __ldg(p + 3 * nthreads);
        m = max4(max4(m, v0), v1);
        m = max4(max4(m, v2), v3);
    }
    for (; i < n4; i += nthreads) m = max4(m, __ldg(reinterpret_cast<const float4 *>(x) + i));
    for (int64_t j = (n4 << 2) + tid; j < n; j += nthreads) m = max(m, abs_bits_nan0(x[j]));
    m = block_max_u32(m, red);
    if (threadIdx.x == 0) partial[blockIdx.x] = m;
}

// Pass 2 (launched with programmatic serialization after pass 1): every
// block reduces the partial maxima (an L2-resident read), s = amax / 448
// (1 for an all-zero tensor), and quantizes its share of x back to front.
__global__ void __launch_bounds__(kThreads) k_quantize_tensor_dynamic(const float *__restrict__ x, int64_t n,
                                                                      const uint32_t *__restrict__ partial,
                                                                      int nparts, float *__restrict__ scale_out,
                                                                      uint8_t *__restrict__ y) {
    __shared__ uint32_t red[32];
    griddep_wait();  // pass 1 has completed and its partials are visible
    uint32_t m = 0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) m = max(m, partial[i]);
    m = block_max_u32(m, red);
    const float s = scale_from_amax(__uint_as_float(m));
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
    griddep_launch_dependents();  // the next GEMM may start its set-up
    const Scale st = make_scale(s);
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t n16 = n >> 4;
    for (int64_t g = tid; g < n16; g += nthreads) {
        const int64_t gg = n16 - 1 - g;  // back to front: the tail pass 1 left in L2 first
        const float4 *xp = reinterpret_cast<const float4 *>(x) + gg * 4;
        const float4 v0 = __ldcs(xp), v1 = __ldcs(xp + 1), v2 = __ldcs(xp + 2), v3 = __ldcs(xp + 3);
        __stcs(reinterpret_cast<uint4 *>(y) + gg, pack16(v0, v1, v2, v3, st));
    }
    const int64_t t = (n16 << 4) + tid;
    if (t < n) y[t] = static_cast<uint8_t>(quantize1(x[t], s));
}

// One CTA per row; the row stays in registers between the amax and the
// quantize pass (VPT float4 per thread, so cols <= VPT * 4 * kThreads).
template <int VPT>
__global__ void __launch_bounds__(kThreads) k_quantize_rows_dynamic(const float *__restrict__ x, int64_t cols,
                                                                    int64_t ldx, float *__restrict__ scale_out,
                                                                    uint8_t *__restrict__ y) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    __shared__ uint32_t red[32];
    const int64_t r = blockIdx.x;
    const float4 *xr = reinterpret_cast<const float4 *>(x + r * ldx);
    const int64_t c4 = cols >> 2;
    float4 v[VPT];
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int64_t i = threadIdx.x + static_cast<int64_t>(j) * kThreads;
        if (i < c4) {
            v[j] = __ldcs(xr + i);
            m = max(m, max(max(abs_bits_nan0(v[j].x), abs_bits_nan0(v[j].y)),
                           max(abs_bits_nan0(v[j].z), abs_bits_nan0(v[j].w))));
        }
    }
    m = block_max_u32(m, red);
    const float s_row = scale_from_amax(__uint_as_float(m));
    if (threadIdx.x == 0) scale_out[r] = s_row;
    const Scale s = make_scale(s_row);
    uint32_t *yr = reinterpret_cast<uint32_t *>(y + r * cols);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
        const int64_t i = threadIdx.x + static_cast<int64_t>(j) * kThreads;
        if (i < c4) {
            const float q4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
            uint32_t w;
            quantize_block_fast<4>(q4, s.s, s.r, s.ok, &w);
            __stcs(yr + i, w);
        }
    }
}

// Rows of any width/alignment: amax pass, then quantize pass (the second read
// of the row is served from L1/L2).
__global__ void __launch_bounds__(kThreads) k_quantize_rows_dynamic_generic(const float *__restrict__ x,
                                                                            int64_t cols, int64_t ldx,
                                                                            float *__restrict__ scale_out,
                                                                            uint8_t *__restrict__ y) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    __shared__ uint32_t red[32];
    const int64_t r = blockIdx.x;
    const float *xr = x + r * ldx;
    uint32_t m = 0;
    for (int64_t c = threadIdx.x; c < cols; c += kThreads) m = max(m, abs_bits_nan0(xr[c]));
    m = block_max_u32(m, red);
    const float s = scale_from_amax(__uint_as_float(m));
    if (threadIdx.x == 0) scale_out[r] = s;
    for (int64_t c = threadIdx.x; c < cols; c += kThreads) y[r * cols + c] = static_cast<uint8_t>(quantize1(xr[c], s));
}

// ---------------------------------------------------------------------------
// DequantizeLinear
// ---------------------------------------------------------------------------
template <bool BF16>
__global__ void __launch_bounds__(kThreads) k_dequantize(const uint8_t *__restrict__ q, int64_t n, int64_t axis_len,
                                                         int64_t inner, const float *__restrict__ sc, int per_axis,
                                                         int vec_ok, void *__restrict__ yv) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const float s0 = __ldg(sc);
    int64_t done = 0;
    if (vec_ok) {
        const int64_t n16 = n >> 4;
        for (int64_t g = tid; g < n16; g += nthreads) {
            const uint4 w = __ldcs(reinterpret_cast<const uint4 *>(q) + g);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int64_t i = (g << 4) + j;
                const float s = per_axis ? __ldg(sc + (i / inner) % axis_len) : s0;
                o[j] = e4m3_decode((ws[j >> 2] >> ((j & 3) * 8)) & 0xffu) * s;
            }
            if (BF16) {
                uint32_t p[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * j], o[2 * j + 1]);
                    p[j] = *reinterpret_cast<uint32_t *>(&h);
                }
                uint4 *yp = reinterpret_cast<uint4 *>(yv) + g * 2;
                __stcs(yp, make_uint4(p[0], p[1], p[2], p[3]));
                __stcs(yp + 1, make_uint4(p[4], p[5], p[6], p[7]));
            } else {
                float4 *yp = reinterpret_cast<float4 *>(yv) + g * 4;
#pragma unroll
                for (int j = 0; j < 4; ++j) __stcs(yp + j, make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]));
            }
        }
        done = n16 << 4;
    }
    for (int64_t i = done + tid; i < n; i += nthreads) {
        const float s = per_axis ? __ldg(sc + (i / inner) % axis_len) : s0;
        const float v = e4m3_decode(q[i]) * s;
        if (BF16) reinterpret_cast<__nv_bfloat16 *>(yv)[i] = __float2bfloat16_rn(v);
        else reinterpret_cast<float *>(yv)[i] = v;
    }
}

// ---------------------------------------------------------------------------
// e4m3 transpose [rows, cols] -> [cols, rows], 64x64 tiles through smem.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_transpose_u8(const uint8_t *__restrict__ src, int64_t rows, int64_t cols,
                                                      uint8_t *__restrict__ dst) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    __shared__ uint8_t tile[64][65];
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 64, c0 = static_cast<int64_t>(blockIdx.x) * 64;
    for (int i = threadIdx.x; i < 64 * 64; i += 256) {
        const int rr = i / 64, cc = i % 64;
        const int64_t r = r0 + rr, c = c0 + cc;
        tile[rr][cc] = (r < rows && c < cols) ? src[r * cols + c] : 0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 64; i += 256) {
        const int cc = i / 64, rr = i % 64;
        const int64_t r = r0 + rr, c = c0 + cc;
        if (r < rows && c < cols) dst[c * rows + r] = tile[rr][cc];
    }
}

int grid_for(int64_t work_items) {
    const int64_t per_wave = static_cast<int64_t>(sm_count()) * (2048 / kThreads);
    int64_t blocks = (work_items + kThreads - 1) / kThreads;
    if (blocks > per_wave) blocks = per_wave;
    if (blocks < 1) blocks = 1;
    return static_cast<int>(blocks);
}

template <bool FROM_AMAX>
int launch_quantize(const float *x, int64_t outer, int64_t axis_len, int64_t inner, const float *sc, int per_axis,
                    float *scale_out, uint8_t *y, cudaStream_t st) {
    const int64_t n = outer * axis_len * inner;
    if (n == 0) return LCML_OK;
    const bool vec = aligned(x, 16) && aligned(y, 16);
    if (!vec) {
        k_quantize_scalar<FROM_AMAX><<<grid_for(n), kThreads, 0, st>>>(x, n, axis_len, inner, sc, per_axis, scale_out, y);
        LCML_LAUNCHED("quantize_scalar");
        return LCML_OK;
    }
    const int g = grid_for((n >> 4) > 0 ? (n >> 4) : 1);
    if (!per_axis) {
        k_quantize<kScaleTensor, FROM_AMAX><<<g, kThreads, 0, st>>>(x, n, 1, 1, sc, scale_out, y);
    } else if (inner % 16 == 0) {
        k_quantize<kScaleGroup16, FROM_AMAX><<<g, kThreads, 0, st>>>(x, n, axis_len, inner, sc, scale_out, y);
    } else if (inner == 1 && axis_len % 16 == 0) {
        k_quantize<kScaleInner1, FROM_AMAX><<<g, kThreads, 0, st>>>(x, n, axis_len, inner, sc, scale_out, y);
    } else {
        k_quantize<kScaleGeneric, FROM_AMAX><<<g, kThreads, 0, st>>>(x, n, axis_len, inner, sc, scale_out, y);
    }
    LCML_LAUNCHED("quantize");
    return LCML_OK;
}

}// namespace
}// namespace lcml

using namespace lcml;

extern "C" {

int lcml_fp8_quantize(const float *x, int64_t outer, int64_t axis_len, int64_t inner, const float *scale,
                      int scale_mode, uint8_t *y, lcml_stream_t stream) {
    LCML_CHECK_ARG(outer >= 0 && axis_len >= 0 && inner >= 0, "lcml_fp8_quantize: negative extent");
    LCML_CHECK_ARG(scale_mode == LCML_SCALE_TENSOR || scale_mode == LCML_SCALE_AXIS,
                   "lcml_fp8_quantize: scale_mode %d is not TENSOR or AXIS", scale_mode);
    if (outer * axis_len * inner == 0) return LCML_OK;
    LCML_CHECK_ARG(x && y && scale, "lcml_fp8_quantize: null pointer");
    return launch_quantize<false>(x, outer, axis_len, inner, scale, scale_mode == LCML_SCALE_AXIS, nullptr, y,
                                  to_cuda(stream));
}

int lcml_fp8_quantize_from_amax(const float *x, int64_t outer, int64_t axis_len, int64_t inner, const float *amax,
                                float *scale_out, uint8_t *y, lcml_stream_t stream) {
    LCML_CHECK_ARG(outer >= 0 && axis_len >= 0 && inner >= 0, "lcml_fp8_quantize_from_amax: negative extent");
    if (outer * axis_len * inner == 0) return LCML_OK;
    LCML_CHECK_ARG(x && y && amax, "lcml_fp8_quantize_from_amax: null pointer");
    return launch_quantize<true>(x, outer, axis_len, inner, amax, axis_len > 1 ? 1 : 0, scale_out, y,
                                 to_cuda(stream));
}

int lcml_fp8_quantize_rows_dynamic(const float *x, int64_t rows, int64_t cols, int64_t ldx, float *scale_out,
                                   uint8_t *y, lcml_stream_t stream) {
    LCML_CHECK_ARG(rows >= 0 && cols >= 0, "lcml_fp8_quantize_rows_dynamic: negative extent");
    if (rows == 0 || cols == 0) return LCML_OK;
    LCML_CHECK_ARG(x && y && scale_out, "lcml_fp8_quantize_rows_dynamic: null pointer");
    LCML_CHECK_ARG(ldx >= cols, "lcml_fp8_quantize_rows_dynamic: ldx %lld < cols %lld", (long long)ldx,
                   (long long)cols);
    LCML_CHECK_ARG(rows <= 0x7fffffff, "lcml_fp8_quantize_rows_dynamic: too many rows");
    cudaStream_t st = to_cuda(stream);
    const bool vec = aligned(x, 16) && (ldx % 4 == 0) && (cols % 4 == 0) && aligned(y, 4);
    const dim3 grid(static_cast<unsigned>(rows));
    if (vec && cols <= 4 * 4 * kThreads) {
        k_quantize_rows_dynamic<4><<<grid, kThreads, 0, st>>>(x, cols, ldx, scale_out, y);
    } else if (vec && cols <= 8 * 4 * kThreads) {
        k_quantize_rows_dynamic<8><<<grid, kThreads, 0, st>>>(x, cols, ldx, scale_out, y);
    } else if (vec && cols <= 12 * 4 * kThreads) {
        k_quantize_rows_dynamic<12><<<grid, kThreads, 0, st>>>(x, cols, ldx, scale_out, y);
    } else {
        k_quantize_rows_dynamic_generic<<<grid, kThreads, 0, st>>>(x, cols, ldx, scale_out, y);
    }
    LCML_LAUNCHED("quantize_rows_dynamic");
    return LCML_OK;
}

int lcml_amax(const float *x, int64_t n, float *amax_out, lcml_stream_t stream) {
    LCML_CHECK_ARG(n >= 0, "lcml_amax: negative n");
    LCML_CHECK_ARG(amax_out != nullptr, "lcml_amax: null output");
    cudaStream_t st = to_cuda(stream);
    LCML_CUDA(cudaMemsetAsync(amax_out, 0, sizeof(float), st));
    if (n == 0) return LCML_OK;
    LCML_CHECK_ARG(x != nullptr, "lcml_amax: null input");
    const int vec = aligned(x, 16) ? 1 : 0;
    k_amax<<<grid_for((n >> 2) + 1), kThreads, 0, st>>>(x, n, vec, reinterpret_cast<uint32_t *>(amax_out));
    LCML_LAUNCHED("amax");
    return LCML_OK;
}

int lcml_fp8_quantize_tensor_dynamic(const float *x, int64_t n, float *scale_out, uint8_t *y, float *workspace,
                                     lcml_stream_t stream) {
    LCML_CHECK_ARG(n >= 0, "lcml_fp8_quantize_tensor_dynamic: negative n");
    LCML_CHECK_ARG(scale_out && workspace, "lcml_fp8_quantize_tensor_dynamic: null scale_out/workspace");
    LCML_CHECK_ARG(n == 0 || (x && y), "lcml_fp8_quantize_tensor_dynamic: null pointer");
    if (n > 0 && aligned(x, 16) && aligned(y, 16)) {
        // two kernels, no memset: per-block partial maxima, then the quantize
        // pass (programmatic dependent launch, back to front over the L2-warm tail)
        cudaStream_t st = to_cuda(stream);
        int parts = grid_for((n >> 2) + 1);
        if (parts > kMaxAmaxParts) parts = kMaxAmaxParts;
        uint32_t *partial = reinterpret_cast<uint32_t *>(workspace);
        k_amax_partial<<<parts, kThreads, 0, st>>>(x, n, partial);
        LCML_LAUNCHED("amax_partial");
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(grid_for((n >> 4) > 0 ? (n >> 4) : 1)), 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, k_quantize_tensor_dynamic, x, n,
                                                 static_cast<const uint32_t *>(partial), parts, scale_out, y);
        g_launches.fetch_add(1, std::memory_order_relaxed);
        if (e != cudaSuccess)
            return set_error(LCML_ERR_CUDA, "quantize_tensor_dynamic launch failed: %s", cudaGetErrorString(e));
        return LCML_OK;
    }
    int rc = lcml_amax(x, n, workspace, stream);
    if (rc != LCML_OK) return rc;
    if (n == 0) {
        // empty tensor: scale of an all-zero tensor
        const float one = 1.0f;
        LCML_CUDA(cudaMemcpyAsync(scale_out, &one, sizeof(float), cudaMemcpyHostToDevice, to_cuda(stream)));
        return LCML_OK;
    }
    return launch_quantize<true>(x, 1, 1, n, workspace, 0, scale_out, y, to_cuda(stream));
}

int lcml_fp8_dequantize(const uint8_t *q, int64_t outer, int64_t axis_len, int64_t inner, const float *scale,
                        int scale_mode, void *y, int y_dtype, lcml_stream_t stream) {
    LCML_CHECK_ARG(outer >= 0 && axis_len >= 0 && inner >= 0, "lcml_fp8_dequantize: negative extent");
    LCML_CHECK_ARG(scale_mode == LCML_SCALE_TENSOR || scale_mode == LCML_SCALE_AXIS,
                   "lcml_fp8_dequantize: scale_mode %d is not TENSOR or AXIS", scale_mode);
    LCML_CHECK_ARG(y_dtype == LCML_DTYPE_FLOAT || y_dtype == LCML_DTYPE_BFLOAT16,
                   "lcml_fp8_dequantize: y_dtype %d unsupported", y_dtype);
    const int64_t n = outer * axis_len * inner;
    if (n == 0) return LCML_OK;
    LCML_CHECK_ARG(q && y && scale, "lcml_fp8_dequantize: null pointer");
    cudaStream_t st = to_cuda(stream);
    const int vec = (aligned(q, 16) && aligned(y, 16)) ? 1 : 0;
    const int per_axis = scale_mode == LCML_SCALE_AXIS;
    const int g = grid_for((n >> 4) + 1);
    if (y_dtype == LCML_DTYPE_BFLOAT16)
        k_dequantize<true><<<g, kThreads, 0, st>>>(q, n, axis_len, inner, scale, per_axis, vec, y);
    else
        k_dequantize<false><<<g, kThreads, 0, st>>>(q, n, axis_len, inner, scale, per_axis, vec, y);
    LCML_LAUNCHED("dequantize");
    return LCML_OK;
}

int lcml_fp8_transpose(const uint8_t *src, int64_t rows, int64_t cols, uint8_t *dst, lcml_stream_t stream) {
    LCML_CHECK_ARG(rows >= 0 && cols >= 0, "lcml_fp8_transpose: negative extent");
    if (rows == 0 || cols == 0) return LCML_OK;
    LCML_CHECK_ARG(src && dst, "lcml_fp8_transpose: null pointer");
    LCML_CHECK_ARG((rows + 63) / 64 <= 65535, "lcml_fp8_transpose: too many rows");
    dim3 grid(static_cast<unsigned>((cols + 63) / 64), static_cast<unsigned>((rows + 63) / 64));
    k_transpose_u8<<<grid, 256, 0, to_cuda(stream)>>>(src, rows, cols, dst);
    LCML_LAUNCHED("transpose_u8");
    return LCML_OK;
}

}// extern "C"
