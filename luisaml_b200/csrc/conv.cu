// FP8 convolution lowered to the tensor-core GEMM (gemm_fp8.cu):
//   rows = output pixels (n, oh, ow), columns = output channels,
//   K = (kh, kw, c) with c fastest, zero-padded to a multiple of 16.
// NHWC activations make every (pixel, tap) a contiguous run of C bytes, so the
// im2col gather moves 16-byte vectors; a 1x1 / stride-1 / unpadded conv needs
// no gather at all (X is already the GEMM's A). The epilogue fuses the
// per-tensor x scale, per-channel w scale, bias, residual, Relu and the
// requantization of the output.
#include "lcml_device.cuh"
#include "lcml_internal.h"

namespace lcml {
namespace {

constexpr int kThreads = 256;

int64_t packed_k(int64_t cg, int64_t kh, int64_t kw) { return ((cg * kh * kw + 15) / 16) * 16; }

bool direct_path(const lcml_fp8_conv_desc *d) {
    return d->kH == 1 && d->kW == 1 && d->sH == 1 && d->sW == 1 && d->pH == 0 && d->pW == 0 && d->x_nhwc &&
           d->C % 16 == 0 && d->oH == d->H && d->oW == d->W;
}

// Wp[m, (kh*kW + kw)*Cg + c] = W[m, c, kh, kw]; zero beyond kH*kW*Cg.
__global__ void __launch_bounds__(kThreads) k_pack_weight(const uint8_t *__restrict__ W, int64_t M, int64_t Cg,
                                                          int64_t kH, int64_t kW, int64_t Kp, uint8_t *__restrict__ Wp) {
    const int64_t total = M * Kp;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t m = i / Kp, k = i % Kp;
        uint8_t v = 0;
        if (k < kH * kW * Cg) {
            const int64_t tap = k / Cg, c = k % Cg;
            const int64_t kh = tap / kW, kw = tap % kW;
            v = W[((m * Cg + c) * kH + kh) * kW + kw];
        }
        Wp[i] = v;
    }
}

// NHWC im2col, C % 16 == 0: one 16-byte vector per (pixel, 16-channel chunk of a tap).
__global__ void __launch_bounds__(kThreads) k_im2col_nhwc16(const uint8_t *__restrict__ X, int64_t N, int64_t C,
                                                            int64_t H, int64_t W, int64_t kH, int64_t kW, int64_t oH,
                                                            int64_t oW, int sH, int sW, int pH, int pW, int dH, int dW,
                                                            int64_t Kp, uint8_t *__restrict__ A) {
    const int64_t chunks = Kp / 16, taps_chunks = kH * kW * (C / 16);
    const int64_t total = N * oH * oW * chunks;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = i / chunks, ch = i % chunks;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (ch < taps_chunks) {
            const int64_t tap = ch / (C / 16), c16 = ch % (C / 16);
            const int64_t kh = tap / kW, kw = tap % kW;
            const int64_t ow = p % oW, t = p / oW, oh = t % oH, n = t / oH;
            const int64_t ih = oh * sH + kh * dH - pH, iw = ow * sW + kw * dW - pW;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                v = __ldg(reinterpret_cast<const uint4 *>(X + ((n * H + ih) * W + iw) * C) + c16);
        }
        reinterpret_cast<uint4 *>(A)[i] = v;
    }
}

// Generic im2col (any C, NHWC or NCHW input): one byte per thread-iteration.
template <bool NHWC>
__global__ void __launch_bounds__(kThreads) k_im2col_bytes(const uint8_t *__restrict__ X, int64_t N, int64_t C,
                                                           int64_t H, int64_t W, int64_t kH, int64_t kW, int64_t oH,
                                                           int64_t oW, int sH, int sW, int pH, int pW, int dH, int dW,
                                                           int64_t Kp, uint8_t *__restrict__ A) {
    const int64_t total = N * oH * oW * Kp;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = i / Kp, k = i % Kp;
        uint8_t v = 0;
        if (k < kH * kW * C) {
            const int64_t tap = k / C, c = k % C;
            const int64_t kh = tap / kW, kw = tap % kW;
            const int64_t ow = p % oW, t = p / oW, oh = t % oH, n = t / oH;
            const int64_t ih = oh * sH + kh * dH - pH, iw = ow * sW + kw * dW - pW;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                v = NHWC ? X[((n * H + ih) * W + iw) * C + c] : X[((n * C + c) * H + ih) * W + iw];
        }
        A[i] = v;
    }
}

int grid_for(int64_t items) {
    const int64_t per_wave = static_cast<int64_t>(sm_count()) * (2048 / kThreads);
    int64_t b = (items + kThreads - 1) / kThreads;
    if (b > per_wave) b = per_wave;
    return static_cast<int>(b < 1 ? 1 : b);
}

}// namespace
}// namespace lcml

using namespace lcml;

extern "C" {

int64_t lcml_fp8_conv_packed_k(int64_t Cg, int64_t kH, int64_t kW) { return packed_k(Cg, kH, kW); }

int64_t lcml_fp8_conv_workspace_size(const lcml_fp8_conv_desc *d) {
    if (!d) return -1;
    if (direct_path(d)) return 0;
    return d->N * d->oH * d->oW * packed_k(d->C / (d->group > 0 ? d->group : 1), d->kH, d->kW);
}

int lcml_fp8_conv_pack_weight(const uint8_t *W, int64_t M, int64_t Cg, int64_t kH, int64_t kW, uint8_t *Wp,
                              lcml_stream_t stream) {
    LCML_CHECK_ARG(M > 0 && Cg > 0 && kH > 0 && kW > 0, "lcml_fp8_conv_pack_weight: bad extents");
    LCML_CHECK_ARG(W && Wp, "lcml_fp8_conv_pack_weight: null pointer");
    const int64_t Kp = packed_k(Cg, kH, kW);
    k_pack_weight<<<grid_for(M * Kp), kThreads, 0, to_cuda(stream)>>>(W, M, Cg, kH, kW, Kp, Wp);
    LCML_LAUNCHED("conv_pack_weight");
    return LCML_OK;
}

int lcml_fp8_conv(const lcml_fp8_conv_desc *d, lcml_stream_t stream) {
    LCML_CHECK_ARG(d != nullptr, "lcml_fp8_conv: desc is NULL");
    LCML_CHECK_ARG(d->N > 0 && d->C > 0 && d->H > 0 && d->W > 0 && d->M > 0 && d->kH > 0 && d->kW > 0 && d->oH > 0 &&
                       d->oW > 0 && d->sH > 0 && d->sW > 0 && d->dH > 0 && d->dW > 0 && d->pH >= 0 && d->pW >= 0,
                   "lcml_fp8_conv: bad geometry");
    if (d->group != 1) return set_error(LCML_ERR_UNSUPPORTED, "lcml_fp8_conv: group %d (only 1 is built)", d->group);
    LCML_CHECK_ARG((d->oH - 1) * d->sH + (d->kH - 1) * d->dH - d->pH < d->H + d->pH + d->kH &&
                       (d->oW - 1) * d->sW + (d->kW - 1) * d->dW - d->pW < d->W + d->pW + d->kW,
                   "lcml_fp8_conv: output extent inconsistent with the input");
    LCML_CHECK_ARG(d->X && d->Wp && d->Y && d->scale_x && d->scale_w, "lcml_fp8_conv: null operand");
    LCML_CHECK_ARG(d->epilogue == LCML_EPI_NONE || d->epilogue == LCML_EPI_RELU, "lcml_fp8_conv: epilogue %d", d->epilogue);
    LCML_CHECK_ARG(!d->residual || d->residual_dtype == LCML_DTYPE_FLOAT ||
                       (d->residual_dtype == LCML_DTYPE_FLOAT8E4M3FN && d->residual_scale),
                   "lcml_fp8_conv: residual must be FLOAT or FLOAT8E4M3FN with residual_scale");
    const int64_t P = d->N * d->oH * d->oW;
    const int64_t Kp = packed_k(d->C, d->kH, d->kW);
    cudaStream_t st = to_cuda(stream);
    const uint8_t *A = d->X;
    int64_t K = d->C;
    if (!direct_path(d)) {
        LCML_CHECK_ARG(d->workspace != nullptr, "lcml_fp8_conv: this conv needs a workspace of %lld bytes",
                       static_cast<long long>(P * Kp));
        uint8_t *ws = static_cast<uint8_t *>(d->workspace);
        if (d->x_nhwc && d->C % 16 == 0 && aligned(d->X, 16) && aligned(ws, 16)) {
            k_im2col_nhwc16<<<grid_for(P * (Kp / 16)), kThreads, 0, st>>>(d->X, d->N, d->C, d->H, d->W, d->kH, d->kW,
                                                                         d->oH, d->oW, d->sH, d->sW, d->pH, d->pW,
                                                                         d->dH, d->dW, Kp, ws);
        } else if (d->x_nhwc) {
            k_im2col_bytes<true><<<grid_for(P * Kp), kThreads, 0, st>>>(d->X, d->N, d->C, d->H, d->W, d->kH, d->kW,
                                                                       d->oH, d->oW, d->sH, d->sW, d->pH, d->pW,
                                                                       d->dH, d->dW, Kp, ws);
        } else {
            k_im2col_bytes<false><<<grid_for(P * Kp), kThreads, 0, st>>>(d->X, d->N, d->C, d->H, d->W, d->kH, d->kW,
                                                                        d->oH, d->oW, d->sH, d->sW, d->pH, d->pW,
                                                                        d->dH, d->dW, Kp, ws);
        }
        LCML_LAUNCHED("conv_im2col");
        A = ws;
        K = Kp;
    }
    lcml_fp8_gemm_desc g{};
    g.M = P;
    g.N = d->M;
    g.K = K;
    g.A = A;
    g.lda = K;
    g.B = d->Wp;
    g.ldb = Kp;
    g.b_kmajor = 1;
    g.scale_a = d->scale_x;
    g.scale_a_mode = LCML_SCALE_TENSOR;
    g.scale_b = d->scale_w;
    g.scale_b_mode = d->scale_w_mode == LCML_SCALE_AXIS ? LCML_SCALE_COL : LCML_SCALE_TENSOR;
    g.alpha = 1.0f;
    g.beta = 1.0f;
    if (d->bias) {
        g.c_vec = d->bias;
        g.c_vec_mode = LCML_SCALE_COL;
    }
    if (d->residual) {
        g.c_mat = d->residual;
        g.c_mat_dtype = d->residual_dtype;
        g.c_mat_scale = d->residual_scale;
        g.ldc = d->M;
    }
    g.epilogue = d->epilogue;
    g.Y = d->Y;
    g.y_dtype = d->y_dtype;
    g.ldy = d->M;
    g.y_scale = d->y_scale;
    return lcml_fp8_gemm(&g, stream);
}

}// extern "C"
