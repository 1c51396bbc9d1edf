// Plain fp32 Gemm for graphs without QDQ nodes (Gemm::apply,
// src/onnx/operators/gemm.cpp:28-325): 64x64 output tile per 256-thread CTA,
// 4x4 outputs per thread, K staged through shared memory in steps of 16,
// fp32 fma accumulation, then alpha, then + beta * C with ONNX broadcasting.
#include "lcml_internal.h"

namespace {

__global__ void __launch_bounds__(256) k_gemm_f32(const float *__restrict__ A, const float *__restrict__ B,
                                                  const float *__restrict__ C, int64_t M, int64_t N, int64_t K,
                                                  int transA, int transB, float alpha, float beta, int c_ndim,
                                                  int64_t c_d0, int64_t c_d1, float *__restrict__ Y) {
    __shared__ float sA[16][65];
    __shared__ float sB[16][65];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * 64, n0 = static_cast<int64_t>(blockIdx.x) * 64;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int r = i / 16, kk = i % 16;
            const int64_t m = m0 + r, k = k0 + kk;
            sA[kk][r] = (m < M && k < K) ? (transA ? A[k * M + m] : A[m * K + k]) : 0.0f;
            const int64_t n = n0 + r;
            sB[kk][r] = (n < N && k < K) ? (transB ? B[n * K + k] : B[k * N + n]) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(sA[kk][ty * 4 + i], sB[kk][tx * 4 + j], acc[i][j]);
        __syncthreads();
    }
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + ty * 4 + i;
        if (m >= M) continue;
        for (int j = 0; j < 4; ++j) {
            const int64_t n = n0 + tx * 4 + j;
            if (n >= N) continue;
            float v = acc[i][j];
            if (alpha != 1.0f) v *= alpha;
            if (C && c_ndim >= 0 && beta != 0.0f) {
                float c;
                if (c_ndim == 0 || (c_ndim == 1 && c_d0 == 1)) c = C[0];
                else if (c_ndim == 1) c = (c_d0 == N) ? C[n] : C[m];
                else c = C[((c_d0 == 1) ? 0 : m) * c_d1 + ((c_d1 == 1) ? 0 : n)];
                v = (beta == 1.0f) ? v + c : v + beta * c;
            }
            Y[m * N + n] = v;
        }
    }
}

}// namespace

extern "C" int lcml_gemm_f32(const float *A, const float *B, const float *C, int64_t M, int64_t N, int64_t K,
                             int transA, int transB, float alpha, float beta, int c_ndim, int64_t c_d0,
                             int64_t c_d1, float *Y, lcml_stream_t stream) {
    LCML_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "lcml_gemm_f32: negative extent");
    if (M == 0 || N == 0) return LCML_OK;
    LCML_CHECK_ARG(A && B && Y, "lcml_gemm_f32: null operand");
    LCML_CHECK_ARG(c_ndim < 0 || C != nullptr, "lcml_gemm_f32: c_ndim set but C is NULL");
    LCML_CHECK_ARG((M + 63) / 64 <= 65535, "lcml_gemm_f32: M too large");
    dim3 grid(static_cast<unsigned>((N + 63) / 64), static_cast<unsigned>((M + 63) / 64));
    k_gemm_f32<<<grid, 256, 0, lcml::to_cuda(stream)>>>(A, B, C, M, N, K, transA, transB, alpha, beta, c_ndim, c_d0,
                                                         c_d1, Y);
    LCML_LAUNCHED("gemm_f32");
    return LCML_OK;
}
