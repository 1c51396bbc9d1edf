// Direct convolutions on the CUDA cores, for the convs the tensor-core
// implicit GEMM does not take:
//
//  * lcml_conv2d_f32: the reference's fp32 Conv (src/onnx/operators/conv.cpp:
//    115-207): NCHW input, weights [M, C/group, kH, kW], optional bias,
//    strides / begin pads / dilations / group, NCHW output. Each output sums
//    its taps in (kh, kw) order; within a tap the channels of the group go
//    four at a time into four lane sums (fma), added as ((x + y) + z) + w to
//    the running sum, the last C/group % 4 channels by fma into the running
//    sum (conv.cpp:150-191); then + bias (conv.cpp:195-198).
//  * grouped FP8 convolution (group > 1, e.g. depthwise): the fused QDQ conv
//    of lcml_fp8_conv with e4m3 input (NCHW or NHWC) and packed weights, exact
//    e4m3 products accumulated in fp32 in (kh, kw, c) order, then the fused
//    GEMM's epilogue arithmetic (scales, bias, residual, Relu, output type).
//
// Grouped and depthwise convs have little reuse per output (C/group channels
// per tap): they are memory-bound, so one thread computes one output with
// coalesced stores along the fastest output dimension.
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

// One output per thread, ow fastest (consecutive threads read consecutive iw
// and share the weights of (m, tap)).
__global__ void __launch_bounds__(kThreads) k_conv2d_f32(const float *__restrict__ X, const float *__restrict__ W,
                                                         const float *__restrict__ B, int64_t N, int64_t C, int64_t H,
                                                         int64_t Wd, int64_t M, int64_t kH, int64_t kW, int64_t oH,
                                                         int64_t oW, int sH, int sW, int pH, int pW, int dH, int dW,
                                                         int64_t Cg, int64_t Mg, float *__restrict__ Y) {
    const int64_t total = N * M * oH * oW;
    const int64_t c4 = (Cg / 4) * 4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t ow = i % oW;
        int64_t t = i / oW;
        const int64_t oh = t % oH;
        t /= oH;
        const int64_t m = t % M, n = t / M;
        const int64_t g = m / Mg;
        const float *xg = X + (n * C + g * Cg) * H * Wd;
        const float *wm = W + m * Cg * kH * kW;
        float sum = 0.0f;
        for (int64_t kh = 0; kh < kH; ++kh) {
            const int64_t ih = oh * sH + kh * dH - pH;
            if (ih < 0 || ih >= H) continue;
            for (int64_t kw = 0; kw < kW; ++kw) {
                const int64_t iw = ow * sW + kw * dW - pW;
                if (iw < 0 || iw >= Wd) continue;
                const float *xp = xg + ih * Wd + iw;
                const float *wp = wm + kh * kW + kw;
                if (c4 > 0) {
                    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                    for (int64_t c = 0; c < c4; c += 4) {
                        a0 = fmaf(__ldg(xp + (c + 0) * H * Wd), __ldg(wp + (c + 0) * kH * kW), a0);
                        a1 = fmaf(__ldg(xp + (c + 1) * H * Wd), __ldg(wp + (c + 1) * kH * kW), a1);
                        a2 = fmaf(__ldg(xp + (c + 2) * H * Wd), __ldg(wp + (c + 2) * kH * kW), a2);
                        a3 = fmaf(__ldg(xp + (c + 3) * H * Wd), __ldg(wp + (c + 3) * kH * kW), a3);
                    }
                    sum += ((a0 + a1) + a2) + a3;
                }
                for (int64_t c = c4; c < Cg; ++c) sum = fmaf(__ldg(xp + c * H * Wd), __ldg(wp + c * kH * kW), sum);
            }
        }
        if (B) sum += __ldg(B + m);
        Y[i] = sum;
    }
}

// ConvTranspose (conv_transpose.cpp) as a gather: output (n, m, oh, ow) sums
// X[n, g*Cg + c, ih, iw] * W[g*Cg + c, m % Mg, kh, kw] over the taps with
// ih = (oh + pH - kh*dH) / sH exact and in range (likewise iw), in the
// reference's order: taps (kh, kw), within a tap four lane sums over c added
// as ((x + y) + z) + w, the C/group % 4 tail by fma; then + bias.
__global__ void __launch_bounds__(kThreads)
    k_conv_transpose2d_f32(const float *__restrict__ X, const float *__restrict__ W, const float *__restrict__ B,
                           int64_t N, int64_t C, int64_t H, int64_t Wd, int64_t M, int64_t kH, int64_t kW, int64_t oH,
                           int64_t oW, int sH, int sW, int pH, int pW, int dH, int dW, int64_t Cg, int64_t Mg,
                           float *__restrict__ Y) {
    const int64_t total = N * M * oH * oW;
    const int64_t c4 = (Cg / 4) * 4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t ow = i % oW;
        int64_t t = i / oW;
        const int64_t oh = t % oH;
        t /= oH;
        const int64_t m = t % M, n = t / M;
        const int64_t g = m / Mg, mg = m % Mg;
        const float *xg = X + (n * C + g * Cg) * H * Wd;
        const float *wg = W + (g * Cg * Mg + mg) * kH * kW;  // W[g*Cg + c, mg, kh, kw] at wg + c * Mg*kH*kW
        float sum = 0.0f;
        for (int64_t kh = 0; kh < kH; ++kh) {
            const int64_t ihs = oh + pH - kh * dH;
            if (ihs < 0 || ihs % sH != 0 || ihs / sH >= H) continue;
            const int64_t ih = ihs / sH;
            for (int64_t kw = 0; kw < kW; ++kw) {
                const int64_t iws = ow + pW - kw * dW;
                if (iws < 0 || iws % sW != 0 || iws / sW >= Wd) continue;
                const int64_t iw = iws / sW;
                const float *xp = xg + ih * Wd + iw;
                const float *wp = wg + kh * kW + kw;
                const int64_t wcs = Mg * kH * kW;  // weight stride between input channels
                if (c4 > 0) {
                    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                    for (int64_t c = 0; c < c4; c += 4) {
                        a0 = fmaf(__ldg(xp + (c + 0) * H * Wd), __ldg(wp + (c + 0) * wcs), a0);
                        a1 = fmaf(__ldg(xp + (c + 1) * H * Wd), __ldg(wp + (c + 1) * wcs), a1);
                        a2 = fmaf(__ldg(xp + (c + 2) * H * Wd), __ldg(wp + (c + 2) * wcs), a2);
                        a3 = fmaf(__ldg(xp + (c + 3) * H * Wd), __ldg(wp + (c + 3) * wcs), a3);
                    }
                    sum += ((a0 + a1) + a2) + a3;
                }
                for (int64_t c = c4; c < Cg; ++c) sum = fmaf(__ldg(xp + c * H * Wd), __ldg(wp + c * wcs), sum);
            }
        }
        if (B) sum += __ldg(B + m);
        Y[i] = sum;
    }
}

// Grouped FP8 conv: one output (pixel p = (n, oh, ow), channel m) per thread,
// m fastest (NHWC output rows). Packed weights Wp[m, (kh * kW + kw) * Cp + c].
template <int OUT, bool RELU>
__global__ void __launch_bounds__(kThreads)
    k_conv_fp8_grouped(const uint8_t *__restrict__ X, int x_nhwc, int64_t N, int64_t C, int64_t H, int64_t Wd,
                       const uint8_t *__restrict__ Wp, int64_t Kp, int64_t Cp, int64_t M, int64_t kH, int64_t kW,
                       int64_t oH, int64_t oW, int sH, int sW, int pH, int pW, int dH, int dW, int64_t Cg, int64_t Mg,
                       const float *__restrict__ sx, const float *__restrict__ sw, int sw_per_channel,
                       const float *__restrict__ bias, const uint8_t *__restrict__ res8, const float *__restrict__ res32,
                       const float *__restrict__ res_scale, void *__restrict__ Y, const float *__restrict__ y_scale) {
    const int64_t total = N * oH * oW * M;
    const float xs = __ldg(sx);
    float ys = 1.0f, yr = 1.0f;
    bool s_ok = false;
    if (OUT == 2) {
        ys = __ldg(y_scale);
        yr = __frcp_rn(ys);
        s_ok = scale_fast_ok(ys, yr);
    }
    const float rs = res_scale ? __ldg(res_scale) : 1.0f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t m = i % M, p = i / M;
        const int64_t ow = p % oW;
        const int64_t t = p / oW;
        const int64_t oh = t % oH, n = t / oH;
        const int64_t g = m / Mg;
        const uint8_t *wm = Wp + m * Kp;
        float acc = 0.0f;
        for (int64_t kh = 0; kh < kH; ++kh) {
            const int64_t ih = oh * sH + kh * dH - pH;
            if (ih < 0 || ih >= H) continue;
            for (int64_t kw = 0; kw < kW; ++kw) {
                const int64_t iw = ow * sW + kw * dW - pW;
                if (iw < 0 || iw >= Wd) continue;
                const uint8_t *wt = wm + (kh * kW + kw) * Cp;
                for (int64_t c = 0; c < Cg; ++c) {
                    const int64_t ch = g * Cg + c;
                    const uint8_t xb = x_nhwc ? X[((n * H + ih) * Wd + iw) * C + ch] : X[((n * C + ch) * H + ih) * Wd + iw];
                    acc = fmaf(e4m3_decode(xb), e4m3_decode(wt[c]), acc);
                }
            }
        }
        // the fused GEMM epilogue: acc * (sx * sw[m]) + bias, + residual, Relu, output
        const float f = (sw_per_channel ? __ldg(sw + m) : __ldg(sw)) * xs;
        float v = fmaf(acc, f, bias ? __ldg(bias + m) : 0.0f);
        if (res8) v = fmaf(e4m3_decode(res8[i]), rs, v);
        else if (res32) v += __ldg(res32 + i);
        if (RELU) v = fmaxf(v, 0.0f);
        if (OUT == 0) reinterpret_cast<float *>(Y)[i] = v;
        else if (OUT == 1) reinterpret_cast<__nv_bfloat16 *>(Y)[i] = __float2bfloat16_rn(v);
        else reinterpret_cast<uint8_t *>(Y)[i] = static_cast<uint8_t>(s_ok ? quantize_rcp1(v, yr) : quantize1(v, ys));
    }
}

template <int OUT, bool RELU>
void launch_grouped(const lcml_fp8_conv_desc *d, int64_t Kp, int64_t Cp, cudaStream_t st) {
    const int64_t total = d->N * d->oH * d->oW * d->M;
    const bool r8 = d->residual && d->residual_dtype == LCML_DTYPE_FLOAT8E4M3FN;
    k_conv_fp8_grouped<OUT, RELU><<<grid_for(total), kThreads, 0, st>>>(
        d->X, d->x_nhwc, d->N, d->C, d->H, d->W, d->Wp, Kp, Cp, d->M, d->kH, d->kW, d->oH, d->oW, d->sH, d->sW, d->pH,
        d->pW, d->dH, d->dW, d->C / d->group, d->M / d->group, d->scale_x, d->scale_w,
        d->scale_w_mode == LCML_SCALE_AXIS ? 1 : 0, d->bias, r8 ? static_cast<const uint8_t *>(d->residual) : nullptr,
        (!r8 && d->residual) ? static_cast<const float *>(d->residual) : nullptr, r8 ? d->residual_scale : nullptr, d->Y,
        d->y_scale);
}

}// namespace

// The grouped path of lcml_fp8_conv (called from conv.cu for group > 1).
int fp8_conv_grouped(const lcml_fp8_conv_desc *d, int64_t Kp, int64_t Cp, cudaStream_t st) {
    const bool relu = d->epilogue == LCML_EPI_RELU;
    const int out = d->y_dtype == LCML_DTYPE_FLOAT ? 0 : (d->y_dtype == LCML_DTYPE_BFLOAT16 ? 1 : 2);
    if (out == 0) relu ? launch_grouped<0, true>(d, Kp, Cp, st) : launch_grouped<0, false>(d, Kp, Cp, st);
    else if (out == 1) relu ? launch_grouped<1, true>(d, Kp, Cp, st) : launch_grouped<1, false>(d, Kp, Cp, st);
    else relu ? launch_grouped<2, true>(d, Kp, Cp, st) : launch_grouped<2, false>(d, Kp, Cp, st);
    LCML_LAUNCHED("conv_fp8_grouped");
    return LCML_OK;
}

}// namespace lcml

extern "C" int lcml_conv2d_f32(const float *X, const float *W, const float *B, int64_t N, int64_t C, int64_t H,
                               int64_t Wd, int64_t M, int64_t kH, int64_t kW, int64_t oH, int64_t oW, int sH, int sW,
                               int pH, int pW, int dH, int dW, int group, float *Y, lcml_stream_t stream) {
    using namespace lcml;
    LCML_CHECK_ARG(N >= 0 && C > 0 && H > 0 && Wd > 0 && M > 0 && kH > 0 && kW > 0 && oH >= 0 && oW >= 0 && sH > 0 &&
                       sW > 0 && dH > 0 && dW > 0 && pH >= 0 && pW >= 0 && group > 0,
                   "lcml_conv2d_f32: bad geometry");
    LCML_CHECK_ARG(C % group == 0 && M % group == 0, "lcml_conv2d_f32: C and M must be multiples of group");
    if (N == 0 || oH == 0 || oW == 0) return LCML_OK;
    LCML_CHECK_ARG(X && W && Y, "lcml_conv2d_f32: null pointer");
    const int64_t total = N * M * oH * oW;
    k_conv2d_f32<<<grid_for(total), kThreads, 0, to_cuda(stream)>>>(X, W, B, N, C, H, Wd, M, kH, kW, oH, oW, sH, sW, pH,
                                                                     pW, dH, dW, C / group, M / group, Y);
    LCML_LAUNCHED("conv2d_f32");
    return LCML_OK;
}

extern "C" int lcml_conv_transpose2d_f32(const float *X, const float *W, const float *B, int64_t N, int64_t C,
                                         int64_t H, int64_t Wd, int64_t M, int64_t kH, int64_t kW, int64_t oH,
                                         int64_t oW, int sH, int sW, int pH, int pW, int dH, int dW, int group,
                                         float *Y, lcml_stream_t stream) {
    using namespace lcml;
    LCML_CHECK_ARG(N >= 0 && C > 0 && H > 0 && Wd > 0 && M > 0 && kH > 0 && kW > 0 && oH >= 0 && oW >= 0 && sH > 0 &&
                       sW > 0 && dH > 0 && dW > 0 && pH >= 0 && pW >= 0 && group > 0,
                   "lcml_conv_transpose2d_f32: bad geometry");
    LCML_CHECK_ARG(C % group == 0 && M % group == 0, "lcml_conv_transpose2d_f32: C and M must be multiples of group");
    if (N == 0 || oH == 0 || oW == 0) return LCML_OK;
    LCML_CHECK_ARG(X && W && Y, "lcml_conv_transpose2d_f32: null pointer");
    const int64_t total = N * M * oH * oW;
    k_conv_transpose2d_f32<<<grid_for(total), kThreads, 0, to_cuda(stream)>>>(
        X, W, B, N, C, H, Wd, M, kH, kW, oH, oW, sH, sW, pH, pW, dH, dW, C / group, M / group, Y);
    LCML_LAUNCHED("conv_transpose2d_f32");
    return LCML_OK;
}
