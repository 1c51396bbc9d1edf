// Plain fp32 Gemm for graphs without QDQ nodes (Gemm::apply,
// src/onnx/operators/gemm.cpp:28-325): 64x64 output tile per 256-thread CTA,
// 4x4 outputs per thread, K staged through shared memory in steps of 16,
// fp32 fma accumulation, then alpha, then + beta * C with ONNX broadcasting.
#include <mutex>

#include "lcml_internal.h"

namespace {

template <bool RELU>
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
            if (RELU) v = v > 0.0f ? v : 0.0f;  // the Relu operator's formula
            Y[m * N + n] = v;
        }
    }
}

// Small-M variant (few 64x64 tiles: decode-sized batches, the MLP): one
// output per thread, 8 rows x 32 columns per 256-thread CTA, so a 32 x 512
// output runs on 64 CTAs instead of 8. K is staged through shared memory in
// steps of 64; each output is still one fmaf chain in K order from 0, then
// alpha, then + beta * C, so the result is bit-identical to k_gemm_f32.
constexpr int kSmTM = 8, kSmTN = 32, kSmTK = 64;

template <bool RELU>
__global__ void __launch_bounds__(256) k_gemm_f32_small(const float *__restrict__ A, const float *__restrict__ B,
                                                        const float *__restrict__ C, int64_t M, int64_t N, int64_t K,
                                                        int transA, int transB, float alpha, float beta, int c_ndim,
                                                        int64_t c_d0, int64_t c_d1, float *__restrict__ Y) {
    __shared__ float sA[kSmTM][kSmTK + 1];
    __shared__ float sB[kSmTN][kSmTK + 1];
    const int tn = threadIdx.x & 31, tm = threadIdx.x >> 5;  // a warp = 32 columns of one row
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kSmTM, n0 = static_cast<int64_t>(blockIdx.x) * kSmTN;
    float acc = 0.0f;
    for (int64_t k0 = 0; k0 < K; k0 += kSmTK) {
        for (int i = threadIdx.x; i < kSmTM * kSmTK; i += 256) {
            const int r = i / kSmTK, kk = i % kSmTK;
            const int64_t m = m0 + r, k = k0 + kk;
            sA[r][kk] = (m < M && k < K) ? (transA ? A[k * M + m] : A[m * K + k]) : 0.0f;
        }
        for (int i = threadIdx.x; i < kSmTN * kSmTK; i += 256) {
            const int r = i / kSmTK, kk = i % kSmTK;
            const int64_t n = n0 + r, k = k0 + kk;
            sB[r][kk] = (n < N && k < K) ? (transB ? B[n * K + k] : B[k * N + n]) : 0.0f;
        }
        __syncthreads();
        const int kn = K - k0 < kSmTK ? static_cast<int>(K - k0) : kSmTK;
        if (kn == kSmTK) {
#pragma unroll 16
            for (int kk = 0; kk < kSmTK; ++kk) acc = fmaf(sA[tm][kk], sB[tn][kk], acc);
        } else {
            for (int kk = 0; kk < kn; ++kk) acc = fmaf(sA[tm][kk], sB[tn][kk], acc);
        }
        __syncthreads();
    }
    const int64_t m = m0 + tm, n = n0 + tn;
    if (m >= M || n >= N) return;
    float v = acc;
    if (alpha != 1.0f) v *= alpha;
    if (C && c_ndim >= 0 && beta != 0.0f) {
        float c;
        if (c_ndim == 0 || (c_ndim == 1 && c_d0 == 1)) c = C[0];
        else if (c_ndim == 1) c = (c_d0 == N) ? C[n] : C[m];
        else c = C[((c_d0 == 1) ? 0 : m) * c_d1 + ((c_d1 == 1) ? 0 : n)];
        v = (beta == 1.0f) ? v + c : v + beta * c;
    }
    if (RELU) v = v > 0.0f ? v : 0.0f;
    Y[m * N + n] = v;
}

// Whole-K variant of the small-M kernel (K up to ~1250): the CTA's 8 rows of
// A and 32 rows of B^T for all of K are loaded into shared memory at once
// (one round of global-load latency instead of one per 64-wide K step), then
// each thread runs its fmaf chain in K order, reading both operands as
// float4 (rows kst floats apart, kst % 32 == 4).
template <bool RELU>
__global__ void __launch_bounds__(256) k_gemm_f32_small_wk(const float *__restrict__ A, const float *__restrict__ B,
                                                           const float *__restrict__ C, int64_t M, int64_t N,
                                                           int64_t K, int kst, int transA, int transB, float alpha,
                                                           float beta, int c_ndim, int64_t c_d0, int64_t c_d1,
                                                           float *__restrict__ Y) {
    extern __shared__ float sm[];
    float *sA = sm, *sB = sm + kSmTM * kst;
    const int tn = threadIdx.x & 31, tm = threadIdx.x >> 5;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kSmTM, n0 = static_cast<int64_t>(blockIdx.x) * kSmTN;
    const int k32 = static_cast<int>(K);
    // staging, row by row (8 rows of A, then 32 rows of B^T): float4 loads
    // along K when the rows are contiguous and 16-byte aligned
    const bool vecA = !transA && (K % 4 == 0) && (reinterpret_cast<uintptr_t>(A) % 16 == 0);
    const bool vecB = transB && (K % 4 == 0) && (reinterpret_cast<uintptr_t>(B) % 16 == 0);
#pragma unroll 4
    for (int r = 0; r < kSmTM + kSmTN; ++r) {
        const bool isA = r < kSmTM;
        const int64_t row = isA ? m0 + r : n0 + (r - kSmTM);
        const bool valid = isA ? row < M : row < N;
        float *dst = sm + r * kst;
        if (isA ? vecA : vecB) {
            // asynchronous 16-byte copies: every row of the tile in flight at once
            const float *src = (isA ? A : B) + (valid ? row : 0) * K;
            const uint32_t d0 = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
            for (int q = threadIdx.x; q < k32 / 4; q += 256)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d0 + 16u * q), "l"(src + 4 * q),
                             "r"(valid ? 16u : 0u)
                             : "memory");
        } else {
            for (int kk = threadIdx.x; kk < k32; kk += 256) {
                float v = 0.0f;
                if (valid) v = isA ? (transA ? A[kk * M + row] : A[row * K + kk]) : (transB ? B[row * K + kk] : B[kk * N + row]);
                dst[kk] = v;
            }
        }
    }
    // rows are 16-byte aligned (kst % 4 == 0) and kst % 32 == 4, so the float4
    // reads of 8 lanes (one shared-memory phase) hit 8 different bank quads
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    const float4 *a4 = reinterpret_cast<const float4 *>(sA + tm * kst);
    const float4 *b4 = reinterpret_cast<const float4 *>(sB + tn * kst);
    float acc = 0.0f;
    const int kq = k32 / 4;
#pragma unroll 4
    for (int q = 0; q < kq; ++q) {
        const float4 av = a4[q], bv = b4[q];
        acc = fmaf(av.x, bv.x, acc);
        acc = fmaf(av.y, bv.y, acc);
        acc = fmaf(av.z, bv.z, acc);
        acc = fmaf(av.w, bv.w, acc);
    }
    for (int kk = 4 * kq; kk < k32; ++kk) acc = fmaf(sA[tm * kst + kk], sB[tn * kst + kk], acc);
    const int64_t m = m0 + tm, n = n0 + tn;
    if (m >= M || n >= N) return;
    float v = acc;
    if (alpha != 1.0f) v *= alpha;
    if (C && c_ndim >= 0 && beta != 0.0f) {
        float c;
        if (c_ndim == 0 || (c_ndim == 1 && c_d0 == 1)) c = C[0];
        else if (c_ndim == 1) c = (c_d0 == N) ? C[n] : C[m];
        else c = C[((c_d0 == 1) ? 0 : m) * c_d1 + ((c_d1 == 1) ? 0 : n)];
        v = (beta == 1.0f) ? v + c : v + beta * c;
    }
    if (RELU) v = v > 0.0f ? v : 0.0f;
    Y[m * N + n] = v;
}

constexpr int kWholeKSmem = 200 * 1024;

}// namespace

namespace {
template <bool RELU>
int gemm_f32(const float *A, const float *B, const float *C, int64_t M, int64_t N, int64_t K, int transA, int transB,
             float alpha, float beta, int c_ndim, int64_t c_d0, int64_t c_d1, float *Y, lcml_stream_t stream) {
    LCML_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "lcml_gemm_f32: negative extent");
    if (M == 0 || N == 0) return LCML_OK;
    LCML_CHECK_ARG(A && B && Y, "lcml_gemm_f32: null operand");
    LCML_CHECK_ARG(c_ndim < 0 || C != nullptr, "lcml_gemm_f32: c_ndim set but C is NULL");
    LCML_CHECK_ARG((M + 63) / 64 <= 65535, "lcml_gemm_f32: M too large");
    const int64_t tiles64 = ((N + 63) / 64) * ((M + 63) / 64);
    if (tiles64 < lcml::sm_count() && (M + kSmTM - 1) / kSmTM <= 65535) {
        // too few 64 x 64 tiles to fill the GPU: one output per thread
        dim3 grid(static_cast<unsigned>((N + kSmTN - 1) / kSmTN), static_cast<unsigned>((M + kSmTM - 1) / kSmTM));
        const int64_t kst = ((K + 31) / 32) * 32 + 4;  // row stride in floats
        const int64_t smem = (kSmTM + kSmTN) * kst * 4;
        if (K > 0 && smem <= kWholeKSmem) {
            auto kern = k_gemm_f32_small_wk<RELU>;
            if (const int rc = lcml::ensure_max_smem(reinterpret_cast<const void *>(kern), kWholeKSmem, "gemm_f32_small"))
                return rc;
            kern<<<grid, 256, static_cast<size_t>(smem), lcml::to_cuda(stream)>>>(
                A, B, C, M, N, K, static_cast<int>(kst), transA, transB, alpha, beta, c_ndim, c_d0, c_d1, Y);
            LCML_LAUNCHED("gemm_f32_small");
            return LCML_OK;
        }
        k_gemm_f32_small<RELU><<<grid, 256, 0, lcml::to_cuda(stream)>>>(A, B, C, M, N, K, transA, transB, alpha,
                                                                        beta, c_ndim, c_d0, c_d1, Y);
        LCML_LAUNCHED("gemm_f32_small");
        return LCML_OK;
    }
    dim3 grid(static_cast<unsigned>((N + 63) / 64), static_cast<unsigned>((M + 63) / 64));
    k_gemm_f32<RELU><<<grid, 256, 0, lcml::to_cuda(stream)>>>(A, B, C, M, N, K, transA, transB, alpha, beta, c_ndim,
                                                               c_d0, c_d1, Y);
    LCML_LAUNCHED("gemm_f32");
    return LCML_OK;
}
}// namespace

extern "C" int lcml_gemm_f32(const float *A, const float *B, const float *C, int64_t M, int64_t N, int64_t K,
                             int transA, int transB, float alpha, float beta, int c_ndim, int64_t c_d0,
                             int64_t c_d1, float *Y, lcml_stream_t stream) {
    return gemm_f32<false>(A, B, C, M, N, K, transA, transB, alpha, beta, c_ndim, c_d0, c_d1, Y, stream);
}

extern "C" int lcml_gemm_f32_relu(const float *A, const float *B, const float *C, int64_t M, int64_t N, int64_t K,
                                  int transA, int transB, float alpha, float beta, int c_ndim, int64_t c_d0,
                                  int64_t c_d1, float *Y, lcml_stream_t stream) {
    return gemm_f32<true>(A, B, C, M, N, K, transA, transB, alpha, beta, c_ndim, c_d0, c_d1, Y, stream);
}
