// Memory-bound operators around the FP8 GEMMs: Relu / Sigmoid / Abs,
// Add / Sub / Mul / Div with trailing broadcast, ReduceMax over the last axis,
// Softmax over the last axis, MaxPool and GlobalAveragePool (Cast: cast.cu).
// Coalesced 16-byte accesses where the layout allows, grid-stride loops,
// grids sized from the SM count. Each kernel's HBM bound is its bytes moved:
// unary/cast 8 B/elem (fp32 in + out), binary 12 B/elem, reduce/softmax
// 4-8 B/elem, pools read each input once.
#include <cuda_bf16.h>

#include "lcml_device.cuh"
#include "lcml_internal.h"

namespace lcml {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t items) {
    const int64_t per_wave = static_cast<int64_t>(sm_count()) * (2048 / kThreads);
    int64_t b = (items + kThreads - 1) / kThreads;
    if (b > per_wave) b = per_wave;
    return static_cast<int>(b < 1 ? 1 : b);
}

__device__ __forceinline__ float sigmoid1(float x) {
    const float e = expf(-fabsf(x));
    return x >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
}

template <int OP>
__device__ __forceinline__ float unary1(float x) {
    if (OP == 0) return x > 0.0f ? x : 0.0f;
    if (OP == 1) return sigmoid1(x);
    return fabsf(x);
}

template <int OP>
__global__ void __launch_bounds__(kThreads) k_unary(const float *__restrict__ x, float *__restrict__ y, int64_t n,
                                                    int vec) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nt = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t done = 0;
    if (vec) {
        const int64_t n4 = n >> 2;
        for (int64_t i = tid; i < n4; i += nt) {
            float4 v = __ldcs(reinterpret_cast<const float4 *>(x) + i);
            v.x = unary1<OP>(v.x);
            v.y = unary1<OP>(v.y);
            v.z = unary1<OP>(v.z);
            v.w = unary1<OP>(v.w);
            __stcs(reinterpret_cast<float4 *>(y) + i, v);
        }
        done = n4 << 2;
    }
    for (int64_t i = done + tid; i < n; i += nt) y[i] = unary1<OP>(x[i]);
}

template <int OP>
__device__ __forceinline__ float binary1(float a, float b) {
    if (OP == 0) return a + b;
    if (OP == 1) return a - b;
    if (OP == 2) return a * b;
    return a / b;
}

template <int OP>
__global__ void __launch_bounds__(kThreads) k_binary(const float *__restrict__ a, const float *__restrict__ b,
                                                     float *__restrict__ y, int64_t n, int64_t bn, int vec) {
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nt = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t done = 0;
    if (vec) {  // bn % 4 == 0 (or bn == 1) and all pointers 16-byte aligned
        const int64_t n4 = n >> 2;
        for (int64_t i = tid; i < n4; i += nt) {
            const float4 va = __ldcs(reinterpret_cast<const float4 *>(a) + i);
            float4 vb;
            if (bn == 1) {
                const float s = __ldg(b);
                vb = make_float4(s, s, s, s);
            } else {
                vb = __ldg(reinterpret_cast<const float4 *>(b) + (i % (bn >> 2)));
            }
            __stcs(reinterpret_cast<float4 *>(y) + i,
                   make_float4(binary1<OP>(va.x, vb.x), binary1<OP>(va.y, vb.y), binary1<OP>(va.z, vb.z),
                               binary1<OP>(va.w, vb.w)));
        }
        done = n4 << 2;
    }
    for (int64_t i = done + tid; i < n; i += nt) y[i] = binary1<OP>(a[i], b[i % bn]);
}

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float *red) {
    v = MAX ? warp_max_f(v) : warp_sum_f(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float r = (l < static_cast<int>(blockDim.x >> 5)) ? red[l] : (MAX ? -INFINITY : 0.0f);
    return MAX ? warp_max_f(r) : warp_sum_f(r);
}

// ReduceMax over the last axis, one CTA per row. The reference's ReduceMax
// uses max(); NaN inputs follow fmaxf (ignored) here.
__global__ void __launch_bounds__(kThreads) k_reduce_max_rows(const float *__restrict__ x, int64_t cols, int abs_first,
                                                              float *__restrict__ y) {
    __shared__ float red[32];
    const float *xr = x + static_cast<int64_t>(blockIdx.x) * cols;
    float m = -INFINITY;
    for (int64_t c = threadIdx.x; c < cols; c += kThreads) {
        const float v = abs_first ? fabsf(xr[c]) : xr[c];
        m = fmaxf(m, v);
    }
    m = block_reduce<true>(m, red);
    if (threadIdx.x == 0) y[blockIdx.x] = m;
}

// Softmax over the last axis: max, sum of exp(x - max), then exp(x - max) / sum.
__global__ void __launch_bounds__(kThreads) k_softmax_rows(const float *__restrict__ x, int64_t cols,
                                                           float *__restrict__ y) {
    __shared__ float red[32];
    const int64_t r = blockIdx.x;
    const float *xr = x + r * cols;
    float m = -INFINITY;
    for (int64_t c = threadIdx.x; c < cols; c += kThreads) m = fmaxf(m, xr[c]);
    m = block_reduce<true>(m, red);
    float s = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += kThreads) s += expf(xr[c] - m);
    s = block_reduce<false>(s, red);
    for (int64_t c = threadIdx.x; c < cols; c += kThreads) y[r * cols + c] = expf(xr[c] - m) / s;
}

// ---------------------------------------------------------------------------
// FP8-typed tensors (FLOAT8E4M3FN / FLOAT8E5M2 values without a scale) in
// Add / Sub / Mul / Div and Softmax: the reference decodes to half, computes
// and re-encodes (binary.cpp:185-283, softmax.cpp:245-280).
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ float fp8_decode(uint32_t b) {
    return DT == LCML_DTYPE_FLOAT8E5M2 ? e5m2_decode(b) : e4m3_decode(b);
}

template <int DT>
__device__ __forceinline__ uint32_t fp8_encode(float v) {
    return DT == LCML_DTYPE_FLOAT8E5M2 ? e5m2_encode(v) : e4m3_encode(v);
}

// Binary: both operands decoded (exactly) to half, the op in IEEE half
// arithmetic (correctly rounded), the half result encoded with the codec.
template <int OP, int DT>
__global__ void __launch_bounds__(kThreads) k_binary_fp8(const uint8_t *__restrict__ a, const uint8_t *__restrict__ b,
                                                         uint8_t *__restrict__ y, int64_t n, int64_t bn) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const __half va = __float2half_rn(fp8_decode<DT>(a[i]));
        const __half vb = __float2half_rn(fp8_decode<DT>(b[bn == n ? i : i % bn]));
        const __half r = OP == 0 ? __hadd(va, vb) : OP == 1 ? __hsub(va, vb) : OP == 2 ? __hmul(va, vb) : __hdiv(va, vb);
        y[i] = static_cast<uint8_t>(fp8_encode<DT>(__half2float(r)));
    }
}

// Softmax of an FP8 row: decoded values, max, sum of exp(x - max) and the
// quotient in fp32 (the reference's half arithmetic and half exp are not
// reproduced), the result rounded to half and encoded, as the reference
// encodes a half value.
template <int DT>
__global__ void __launch_bounds__(kThreads) k_softmax_rows_fp8(const uint8_t *__restrict__ x, int64_t cols,
                                                               uint8_t *__restrict__ y) {
    __shared__ float red[32];
    const int64_t r = blockIdx.x;
    const uint8_t *xr = x + r * cols;
    float m = -INFINITY;
    for (int64_t c = threadIdx.x; c < cols; c += kThreads) m = fmaxf(m, fp8_decode<DT>(xr[c]));
    m = block_reduce<true>(m, red);
    float s = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += kThreads) s += expf(fp8_decode<DT>(xr[c]) - m);
    s = block_reduce<false>(s, red);
    for (int64_t c = threadIdx.x; c < cols; c += kThreads)
        y[r * cols + c] = static_cast<uint8_t>(
            fp8_encode<DT>(__half2float(__float2half_rn(expf(fp8_decode<DT>(xr[c]) - m) / s))));
}

// MaxPool 2-D, begin pads, padded taps skipped. E4M3: the code
// QuantizeLinear gives (at the same positive scale) for the max of the decoded
// values, i.e. the winning input byte, with -0 written as 0x00; NaN taps lose
// to everything (a window of NaNs gives the -inf result, saturated to 0xfe).
template <bool E4M3, bool NHWC>
__global__ void __launch_bounds__(kThreads) k_maxpool(const void *__restrict__ xv, int64_t NC, int64_t C, int64_t H,
                                                      int64_t W, int kH, int kW, int sH, int sW, int pH, int pW,
                                                      int64_t oH, int64_t oW, void *__restrict__ yv) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    const int64_t total = NC * oH * oW;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nt = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t o = tid; o < total; o += nt) {
        int64_t p, oh, ow, n = 0, c = 0;
        if (NHWC) {  // o = ((n * oH + oh) * oW + ow) * C + c
            c = o % C;
            int64_t t = o / C;
            ow = t % oW;
            t /= oW;
            oh = t % oH;
            n = t / oH;
            p = n * C + c;
        } else {
            ow = o % oW;
            int64_t t = o / oW;
            oh = t % oH;
            p = t / oH;
        }
        float best = -INFINITY;
        uint8_t best_b = 0xfe;
        for (int kh = 0; kh < kH; ++kh) {
            const int64_t ih = oh * sH + kh - pH;
            if (ih < 0 || ih >= H) continue;
            for (int kw = 0; kw < kW; ++kw) {
                const int64_t iw = ow * sW + kw - pW;
                if (iw < 0 || iw >= W) continue;
                const int64_t idx = NHWC ? ((n * H + ih) * W + iw) * C + c : (p * H + ih) * W + iw;
                if (E4M3) {
                    const uint8_t b = reinterpret_cast<const uint8_t *>(xv)[idx];
                    const float v = e4m3_decode(b);
                    if (v > best) {
                        best = v;
                        best_b = b;
                    }
                } else {
                    best = fmaxf(best, reinterpret_cast<const float *>(xv)[idx]);
                }
            }
        }
        if (E4M3) reinterpret_cast<uint8_t *>(yv)[o] = best_b == 0x80 ? 0 : best_b;
        else reinterpret_cast<float *>(yv)[o] = best;
    }
}

// Max of e4m3 codes through f16x2: every e4m3 value, -0 and NaN included, is
// exact in f16 (the hardware conversions both ways are exact for them), and
// max.f16x2 returns the other operand when one is NaN, so NaN taps drop out
// as MaxPool of the dequantized values ignores them. The running max starts
// at -448 (code 0xfe), which is also the result of a window that holds only
// NaN codes or lies outside the image. A 16-byte vector is 8 f16x2 words.
constexpr uint32_t kF16x2Neg448 = 0xDF00DF00u;  // two f16 -448.0

__device__ __forceinline__ void e4m3x4_to_f16x2(uint32_t w, uint32_t &lo, uint32_t &hi) {
    asm("{\n\t.reg .b16 a, b;\n\t"
        "mov.b32 {a, b}, %2;\n\t"
        "cvt.rn.f16x2.e4m3x2 %0, a;\n\t"
        "cvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
        : "=r"(lo), "=r"(hi)
        : "r"(w));
}

// -0 -> +0 (adding +0 under round-to-nearest), then back to four codes.
__device__ __forceinline__ uint32_t f16x2_to_e4m3x4(uint32_t lo, uint32_t hi) {
    uint32_t out;
    asm("{\n\t.reg .b16 a, b;\n\t.reg .b32 l, h, z;\n\t"
        "mov.b32 z, 0;\n\t"
        "add.rn.f16x2 l, %1, z;\n\t"
        "add.rn.f16x2 h, %2, z;\n\t"
        "cvt.rn.satfinite.e4m3x2.f16x2 a, l;\n\t"
        "cvt.rn.satfinite.e4m3x2.f16x2 b, h;\n\t"
        "mov.b32 %0, {a, b};\n\t}"
        : "=r"(out)
        : "r"(lo), "r"(hi));
    return out;
}

__device__ __forceinline__ uint32_t hmax2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// acc[8] (f16x2) = max(acc, the 16 codes of v)
__device__ __forceinline__ void max_codes16(uint32_t (&acc)[8], const uint4 &v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t lo, hi;
        e4m3x4_to_f16x2(w[j], lo, hi);
        acc[2 * j] = hmax2_bits(acc[2 * j], lo);
        acc[2 * j + 1] = hmax2_bits(acc[2 * j + 1], hi);
    }
}

// e4m3 NHWC MaxPool with C a multiple of 16: one thread per (output pixel,
// 16 channels), 16-byte loads, the max taken in f16x2 (above). Same results
// as k_maxpool<true, true>. I is the index type. KH x KW > 0 fixes the window
// at compile time: every tap's load is issued before the first max (a tap
// outside the image reads as code 0xfe, which changes no max), so a thread
// has the whole window in flight; 0 x 0 reads kH x kW at run time.
template <typename I, int KH, int KW>
__global__ void __launch_bounds__(kThreads) k_maxpool_e4m3_nhwc16(const uint8_t *__restrict__ x, I N, I C, I H, I W,
                                                                  int kH, int kW, int sH, int sW, int pH, int pW, I oH,
                                                                  I oW, uint8_t *__restrict__ y) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    const I groups = C / 16;
    const I total = N * oH * oW * groups;
    for (I o = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; o < total;
         o += static_cast<I>(gridDim.x) * blockDim.x) {
        const I pix = o / groups, g = o - pix * groups;
        const I t = pix / oW, ow = pix - t * oW, n = t / oH, oh = t - n * oH;
        uint32_t acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = kF16x2Neg448;
        if constexpr (KH > 0) {
            constexpr uint32_t kNeg = 0xfefefefeu;  // four codes of -448
            uint4 v[KH * KW];
#pragma unroll
            for (int kh = 0; kh < KH; ++kh) {
                const I ih = oh * sH + kh - pH;
#pragma unroll
                for (int kw = 0; kw < KW; ++kw) {
                    const I iw = ow * sW + kw - pW;
                    const bool in = ih >= 0 && ih < H && iw >= 0 && iw < W;
                    v[kh * KW + kw] = in ? __ldg(reinterpret_cast<const uint4 *>(x + ((n * H + ih) * W + iw) * C) + g)
                                         : make_uint4(kNeg, kNeg, kNeg, kNeg);
                }
            }
#pragma unroll
            for (int k = 0; k < KH * KW; ++k) max_codes16(acc, v[k]);
        } else {
            for (int kh = 0; kh < kH; ++kh) {
                const I ih = oh * sH + kh - pH;
                if (ih < 0 || ih >= H) continue;
                for (int kw = 0; kw < kW; ++kw) {
                    const I iw = ow * sW + kw - pW;
                    if (iw < 0 || iw >= W) continue;
                    max_codes16(acc, __ldg(reinterpret_cast<const uint4 *>(x + ((n * H + ih) * W + iw) * C) + g));
                }
            }
        }
        reinterpret_cast<uint4 *>(y)[o] = make_uint4(f16x2_to_e4m3x4(acc[0], acc[1]), f16x2_to_e4m3x4(acc[2], acc[3]),
                                                     f16x2_to_e4m3x4(acc[4], acc[5]), f16x2_to_e4m3x4(acc[6], acc[7]));
    }
}

template <int DT>
__device__ __forceinline__ float load_elem(const void *x, int64_t i) {
    if (DT == LCML_DTYPE_FLOAT) return reinterpret_cast<const float *>(x)[i];
    if (DT == LCML_DTYPE_BFLOAT16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(x)[i]);
    return e4m3_decode(reinterpret_cast<const uint8_t *>(x)[i]);
}

// GlobalAveragePool: NCHW -> one CTA per (n, c) plane; NHWC -> one thread per (n, c), strided over HW.
template <int DT>
__global__ void __launch_bounds__(kThreads) k_gap_nchw(const void *__restrict__ x, const float *__restrict__ xs,
                                                       int64_t HW, float *__restrict__ y) {
    __shared__ float red[32];
    const int64_t p = blockIdx.x;
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < HW; i += kThreads) s += load_elem<DT>(x, p * HW + i);
    s = block_reduce<false>(s, red);
    const float scale = (DT == LCML_DTYPE_FLOAT8E4M3FN) ? __ldg(xs) : 1.0f;
    if (threadIdx.x == 0) y[p] = (s * scale) / static_cast<float>(HW);
}

// Four consecutive channels of element i (i a multiple of 4, the tensor
// aligned to four elements) as floats, with one vector load.
template <int DT>
__device__ __forceinline__ void load_elem4(const void *x, int64_t i, float (&v)[4]) {
    if (DT == LCML_DTYPE_FLOAT) {
        const float4 f = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(x) + i));
        v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
    } else if (DT == LCML_DTYPE_BFLOAT16) {
        const uint2 w = __ldg(reinterpret_cast<const uint2 *>(static_cast<const __nv_bfloat16 *>(x) + i));
        v[0] = __uint_as_float(w.x << 16), v[1] = __uint_as_float(w.x & 0xffff0000u);
        v[2] = __uint_as_float(w.y << 16), v[3] = __uint_as_float(w.y & 0xffff0000u);
    } else {
        const uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(static_cast<const uint8_t *>(x) + i));
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = e4m3_decode(static_cast<uint8_t>(w >> (8 * k)));
    }
}

// NHWC GlobalAveragePool: one thread per (n, CPT channels), each channel
// summed over HW in pixel order (the order of global_average_pool.cpp's
// loop). CPT = 4 reads the four channels with one vector load and issues the
// loads of 8 pixels before adding them, so a thread keeps 8 loads in flight
// instead of one.
template <int DT, int CPT>
__global__ void __launch_bounds__(kThreads) k_gap_nhwc(const void *__restrict__ x, const float *__restrict__ xs,
                                                       int64_t N, int64_t C, int64_t HW, float *__restrict__ y) {
    const int64_t groups = C / CPT;
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (tid >= N * groups) return;
    const int64_t n = tid / groups, c = (tid - n * groups) * CPT;
    const float scale = (DT == LCML_DTYPE_FLOAT8E4M3FN) ? __ldg(xs) : 1.0f;
    if constexpr (CPT == 1) {
        float s = 0.0f;
        for (int64_t i = 0; i < HW; ++i) s += load_elem<DT>(x, (n * HW + i) * C + c);
        y[tid] = (s * scale) / static_cast<float>(HW);
    } else if (DT == LCML_DTYPE_FLOAT8E4M3FN && HW <= 64) {
        // e4m3 with at most 64 pixels (the ResNet head: 7 x 7): every pixel's
        // 4-code word is loaded before the first add, so the whole sum waits
        // on one memory latency; the adds then run in pixel order
        uint32_t w[64];
        const uint32_t *px = reinterpret_cast<const uint32_t *>(static_cast<const uint8_t *>(x) + n * HW * C + c);
        const int64_t cw = C / 4;  // words per pixel
#pragma unroll
        for (int i = 0; i < 64; ++i) w[i] = i < HW ? __ldg(px + i * cw) : 0u;
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < 64; ++i)
            if (i < HW) {  // hardware decode through f16x2 (exact for every code)
                float d[4];
                e4m3x2_decode(w[i], d[0], d[1]);
                e4m3x2_decode(w[i] >> 16, d[2], d[3]);
#pragma unroll
                for (int k = 0; k < 4; ++k) s[k] += d[k];
            }
#pragma unroll
        for (int k = 0; k < 4; ++k) y[n * C + c + k] = (s[k] * scale) / static_cast<float>(HW);
    } else {
        constexpr int U = 8;
        float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        int64_t i = 0;
        for (; i + U <= HW; i += U) {
            float v[U][4];
#pragma unroll
            for (int u = 0; u < U; ++u) load_elem4<DT>(x, (n * HW + i + u) * C + c, v[u]);
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int k = 0; k < 4; ++k) s[k] += v[u][k];
        }
        for (; i < HW; ++i) {
            float v[4];
            load_elem4<DT>(x, (n * HW + i) * C + c, v);
#pragma unroll
            for (int k = 0; k < 4; ++k) s[k] += v[k];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) y[n * C + c + k] = (s[k] * scale) / static_cast<float>(HW);
    }
}

}// namespace
}// namespace lcml

using namespace lcml;

extern "C" {

int lcml_unary_f32(int op, const float *x, float *y, int64_t n, lcml_stream_t stream) {
    LCML_CHECK_ARG(op >= 0 && op <= 2, "lcml_unary_f32: op %d unknown", op);
    LCML_CHECK_ARG(n >= 0, "lcml_unary_f32: negative n");
    if (n == 0) return LCML_OK;
    LCML_CHECK_ARG(x && y, "lcml_unary_f32: null pointer");
    const int vec = aligned(x, 16) && aligned(y, 16);
    const int g = grid_for((n >> 2) + 1);
    cudaStream_t st = to_cuda(stream);
    if (op == 0) k_unary<0><<<g, kThreads, 0, st>>>(x, y, n, vec);
    else if (op == 1) k_unary<1><<<g, kThreads, 0, st>>>(x, y, n, vec);
    else k_unary<2><<<g, kThreads, 0, st>>>(x, y, n, vec);
    LCML_LAUNCHED("unary");
    return LCML_OK;
}

int lcml_binary_f32(int op, const float *a, const float *b, int64_t n, int64_t b_n, float *y, lcml_stream_t stream) {
    LCML_CHECK_ARG(op >= 0 && op <= 3, "lcml_binary_f32: op %d unknown", op);
    LCML_CHECK_ARG(n >= 0 && b_n >= 1, "lcml_binary_f32: bad extents");
    if (n == 0) return LCML_OK;
    LCML_CHECK_ARG(n % b_n == 0, "lcml_binary_f32: b (%lld) does not broadcast over a (%lld)", (long long)b_n,
                   (long long)n);
    LCML_CHECK_ARG(a && b && y, "lcml_binary_f32: null pointer");
    const int vec = aligned(a, 16) && aligned(b, 16) && aligned(y, 16) && (b_n == 1 || b_n % 4 == 0);
    const int g = grid_for((n >> 2) + 1);
    cudaStream_t st = to_cuda(stream);
    switch (op) {
        case 0: k_binary<0><<<g, kThreads, 0, st>>>(a, b, y, n, b_n, vec); break;
        case 1: k_binary<1><<<g, kThreads, 0, st>>>(a, b, y, n, b_n, vec); break;
        case 2: k_binary<2><<<g, kThreads, 0, st>>>(a, b, y, n, b_n, vec); break;
        default: k_binary<3><<<g, kThreads, 0, st>>>(a, b, y, n, b_n, vec); break;
    }
    LCML_LAUNCHED("binary");
    return LCML_OK;
}

int lcml_reduce_max_rows(const float *x, int64_t rows, int64_t cols, int abs_first, float *y, lcml_stream_t stream) {
    LCML_CHECK_ARG(rows >= 0 && cols >= 1, "lcml_reduce_max_rows: bad extents");
    if (rows == 0) return LCML_OK;
    LCML_CHECK_ARG(rows <= 0x7fffffff, "lcml_reduce_max_rows: too many rows");
    LCML_CHECK_ARG(x && y, "lcml_reduce_max_rows: null pointer");
    k_reduce_max_rows<<<static_cast<unsigned>(rows), kThreads, 0, to_cuda(stream)>>>(x, cols, abs_first, y);
    LCML_LAUNCHED("reduce_max_rows");
    return LCML_OK;
}

int lcml_binary_fp8(int op, const uint8_t *a, const uint8_t *b, int64_t n, int64_t b_n, uint8_t *y, int dtype,
                    lcml_stream_t stream) {
    LCML_CHECK_ARG(op >= 0 && op <= 3, "lcml_binary_fp8: op %d unknown", op);
    LCML_CHECK_ARG(dtype == LCML_DTYPE_FLOAT8E4M3FN || dtype == LCML_DTYPE_FLOAT8E5M2,
                   "lcml_binary_fp8: dtype %d (FLOAT8E4M3FN or FLOAT8E5M2)", dtype);
    LCML_CHECK_ARG(n >= 0 && b_n >= 1, "lcml_binary_fp8: bad extents");
    if (n == 0) return LCML_OK;
    LCML_CHECK_ARG(n % b_n == 0, "lcml_binary_fp8: b (%lld) does not broadcast over a (%lld)", (long long)b_n,
                   (long long)n);
    LCML_CHECK_ARG(a && b && y, "lcml_binary_fp8: null pointer");
    const int g = grid_for(n);
    cudaStream_t st = to_cuda(stream);
    if (dtype == LCML_DTYPE_FLOAT8E4M3FN) {
        switch (op) {
            case 0: k_binary_fp8<0, LCML_DTYPE_FLOAT8E4M3FN><<<g, kThreads, 0, st>>>(a, b, y, n, b_n); break;
            case 1: k_binary_fp8<1, LCML_DTYPE_FLOAT8E4M3FN><<<g, kThreads, 0, st>>>(a, b, y, n, b_n); break;
            case 2: k_binary_fp8<2, LCML_DTYPE_FLOAT8E4M3FN><<<g, kThreads, 0, st>>>(a, b, y, n, b_n); break;
            default: k_binary_fp8<3, LCML_DTYPE_FLOAT8E4M3FN><<<g, kThreads, 0, st>>>(a, b, y, n, b_n); break;
        }
    } else {
        switch (op) {
            case 0: k_binary_fp8<0, LCML_DTYPE_FLOAT8E5M2><<<g, kThreads, 0, st>>>(a, b, y, n, b_n); break;
            case 1: k_binary_fp8<1, LCML_DTYPE_FLOAT8E5M2><<<g, kThreads, 0, st>>>(a, b, y, n, b_n); break;
            case 2: k_binary_fp8<2, LCML_DTYPE_FLOAT8E5M2><<<g, kThreads, 0, st>>>(a, b, y, n, b_n); break;
            default: k_binary_fp8<3, LCML_DTYPE_FLOAT8E5M2><<<g, kThreads, 0, st>>>(a, b, y, n, b_n); break;
        }
    }
    LCML_LAUNCHED("binary_fp8");
    return LCML_OK;
}

int lcml_softmax_rows_fp8(const uint8_t *x, int64_t rows, int64_t cols, uint8_t *y, int dtype, lcml_stream_t stream) {
    LCML_CHECK_ARG(dtype == LCML_DTYPE_FLOAT8E4M3FN || dtype == LCML_DTYPE_FLOAT8E5M2,
                   "lcml_softmax_rows_fp8: dtype %d (FLOAT8E4M3FN or FLOAT8E5M2)", dtype);
    LCML_CHECK_ARG(rows >= 0 && cols >= 1, "lcml_softmax_rows_fp8: bad extents");
    if (rows == 0) return LCML_OK;
    LCML_CHECK_ARG(rows <= 0x7fffffff, "lcml_softmax_rows_fp8: too many rows");
    LCML_CHECK_ARG(x && y, "lcml_softmax_rows_fp8: null pointer");
    if (dtype == LCML_DTYPE_FLOAT8E4M3FN)
        k_softmax_rows_fp8<LCML_DTYPE_FLOAT8E4M3FN><<<static_cast<unsigned>(rows), kThreads, 0, to_cuda(stream)>>>(x, cols, y);
    else
        k_softmax_rows_fp8<LCML_DTYPE_FLOAT8E5M2><<<static_cast<unsigned>(rows), kThreads, 0, to_cuda(stream)>>>(x, cols, y);
    LCML_LAUNCHED("softmax_rows_fp8");
    return LCML_OK;
}

int lcml_softmax_rows(const float *x, int64_t rows, int64_t cols, float *y, lcml_stream_t stream) {
    LCML_CHECK_ARG(rows >= 0 && cols >= 1, "lcml_softmax_rows: bad extents");
    if (rows == 0) return LCML_OK;
    LCML_CHECK_ARG(rows <= 0x7fffffff, "lcml_softmax_rows: too many rows");
    LCML_CHECK_ARG(x && y, "lcml_softmax_rows: null pointer");
    k_softmax_rows<<<static_cast<unsigned>(rows), kThreads, 0, to_cuda(stream)>>>(x, cols, y);
    LCML_LAUNCHED("softmax_rows");
    return LCML_OK;
}

int lcml_maxpool2d(const void *x, int elem_dtype, int64_t NC, int64_t H, int64_t W, int kH, int kW, int sH, int sW,
                   int pH, int pW, int64_t oH, int64_t oW, void *y, int x_nhwc, int64_t C, lcml_stream_t stream) {
    LCML_CHECK_ARG(elem_dtype == LCML_DTYPE_FLOAT || elem_dtype == LCML_DTYPE_FLOAT8E4M3FN,
                   "lcml_maxpool2d: dtype %d unsupported", elem_dtype);
    LCML_CHECK_ARG(NC >= 0 && H > 0 && W > 0 && kH > 0 && kW > 0 && sH > 0 && sW > 0 && oH >= 0 && oW >= 0,
                   "lcml_maxpool2d: bad geometry");
    LCML_CHECK_ARG(!x_nhwc || (C > 0 && NC % C == 0), "lcml_maxpool2d: NHWC needs C dividing NC");
    const int64_t total = NC * oH * oW;
    if (total == 0) return LCML_OK;
    LCML_CHECK_ARG(x && y, "lcml_maxpool2d: null pointer");
    const int g = grid_for(total);
    cudaStream_t st = to_cuda(stream);
    const bool e4 = elem_dtype == LCML_DTYPE_FLOAT8E4M3FN;
    if (e4 && x_nhwc && C % 16 == 0 && aligned(x, 16) && aligned(y, 16)) {
        const int64_t N = NC / C;
        const int gv = grid_for(total / 16);
        const bool w3 = kH == 3 && kW == 3;
        if (N * H * W * C < (int64_t(1) << 31)) {
            auto kern = w3 ? k_maxpool_e4m3_nhwc16<int32_t, 3, 3> : k_maxpool_e4m3_nhwc16<int32_t, 0, 0>;
            kern<<<gv, kThreads, 0, st>>>(static_cast<const uint8_t *>(x), static_cast<int32_t>(N),
                                          static_cast<int32_t>(C), static_cast<int32_t>(H), static_cast<int32_t>(W), kH,
                                          kW, sH, sW, pH, pW, static_cast<int32_t>(oH), static_cast<int32_t>(oW),
                                          static_cast<uint8_t *>(y));
        } else {
            auto kern = w3 ? k_maxpool_e4m3_nhwc16<int64_t, 3, 3> : k_maxpool_e4m3_nhwc16<int64_t, 0, 0>;
            kern<<<gv, kThreads, 0, st>>>(static_cast<const uint8_t *>(x), N, C, H, W, kH, kW, sH, sW, pH, pW, oH, oW,
                                          static_cast<uint8_t *>(y));
        }
    } else if (e4 && x_nhwc) k_maxpool<true, true><<<g, kThreads, 0, st>>>(x, NC, C, H, W, kH, kW, sH, sW, pH, pW, oH, oW, y);
    else if (e4) k_maxpool<true, false><<<g, kThreads, 0, st>>>(x, NC, C, H, W, kH, kW, sH, sW, pH, pW, oH, oW, y);
    else if (x_nhwc) k_maxpool<false, true><<<g, kThreads, 0, st>>>(x, NC, C, H, W, kH, kW, sH, sW, pH, pW, oH, oW, y);
    else k_maxpool<false, false><<<g, kThreads, 0, st>>>(x, NC, C, H, W, kH, kW, sH, sW, pH, pW, oH, oW, y);
    LCML_LAUNCHED("maxpool2d");
    return LCML_OK;
}

int lcml_global_avgpool(const void *x, int elem_dtype, const float *x_scale, int64_t N, int64_t C, int64_t HW,
                        int x_nhwc, float *y, lcml_stream_t stream) {
    LCML_CHECK_ARG(elem_dtype == LCML_DTYPE_FLOAT || elem_dtype == LCML_DTYPE_BFLOAT16 ||
                       elem_dtype == LCML_DTYPE_FLOAT8E4M3FN,
                   "lcml_global_avgpool: dtype %d unsupported", elem_dtype);
    LCML_CHECK_ARG(N >= 0 && C >= 0 && HW > 0, "lcml_global_avgpool: bad extents");
    LCML_CHECK_ARG(elem_dtype != LCML_DTYPE_FLOAT8E4M3FN || x_scale, "lcml_global_avgpool: e4m3 input needs x_scale");
    if (N * C == 0) return LCML_OK;
    LCML_CHECK_ARG(x && y, "lcml_global_avgpool: null pointer");
    cudaStream_t st = to_cuda(stream);
    if (!x_nhwc) {
        LCML_CHECK_ARG(N * C <= 0x7fffffff, "lcml_global_avgpool: too many planes");
        const unsigned g = static_cast<unsigned>(N * C);
        if (elem_dtype == LCML_DTYPE_FLOAT) k_gap_nchw<LCML_DTYPE_FLOAT><<<g, kThreads, 0, st>>>(x, x_scale, HW, y);
        else if (elem_dtype == LCML_DTYPE_BFLOAT16) k_gap_nchw<LCML_DTYPE_BFLOAT16><<<g, kThreads, 0, st>>>(x, x_scale, HW, y);
        else k_gap_nchw<LCML_DTYPE_FLOAT8E4M3FN><<<g, kThreads, 0, st>>>(x, x_scale, HW, y);
    } else {
        const int es = elem_dtype == LCML_DTYPE_FLOAT ? 4 : (elem_dtype == LCML_DTYPE_BFLOAT16 ? 2 : 1);
        const bool v4 = C % 4 == 0 && aligned(x, 4 * es);
        const unsigned g = static_cast<unsigned>((N * (v4 ? C / 4 : C) + kThreads - 1) / kThreads);
        if (v4) {
            if (elem_dtype == LCML_DTYPE_FLOAT) k_gap_nhwc<LCML_DTYPE_FLOAT, 4><<<g, kThreads, 0, st>>>(x, x_scale, N, C, HW, y);
            else if (elem_dtype == LCML_DTYPE_BFLOAT16) k_gap_nhwc<LCML_DTYPE_BFLOAT16, 4><<<g, kThreads, 0, st>>>(x, x_scale, N, C, HW, y);
            else k_gap_nhwc<LCML_DTYPE_FLOAT8E4M3FN, 4><<<g, kThreads, 0, st>>>(x, x_scale, N, C, HW, y);
        } else {
            if (elem_dtype == LCML_DTYPE_FLOAT) k_gap_nhwc<LCML_DTYPE_FLOAT, 1><<<g, kThreads, 0, st>>>(x, x_scale, N, C, HW, y);
            else if (elem_dtype == LCML_DTYPE_BFLOAT16) k_gap_nhwc<LCML_DTYPE_BFLOAT16, 1><<<g, kThreads, 0, st>>>(x, x_scale, N, C, HW, y);
            else k_gap_nhwc<LCML_DTYPE_FLOAT8E4M3FN, 1><<<g, kThreads, 0, st>>>(x, x_scale, N, C, HW, y);
        }
    }
    LCML_LAUNCHED("global_avgpool");
    return LCML_OK;
}

}// extern "C"
