// FP8 convolution lowered to the tensor-core GEMM (gemm_fp8.cu):
//   rows = output pixels (n, oh, ow), columns = output channels,
//   K = (kh, kw, c) with c fastest, zero-padded to a multiple of 16.
// NHWC activations make every (pixel, tap) a contiguous run of C bytes, so the
// im2col gather moves 16-byte vectors; a 1x1 / stride-1 / unpadded conv needs
// no gather at all (X is already the GEMM's A). The epilogue fuses the
// per-tensor x scale, per-channel w scale, bias, residual, Relu and the
// requantization of the output.
#include <type_traits>

#include "lcml_device.cuh"
#include "lcml_internal.h"

namespace lcml {
namespace {

constexpr int kThreads = 256;

// Channels per tap in the packed K order: C itself when it is a multiple of
// 16 (every tap is whole 16-byte vectors), else C padded to 4, 8 or the next
// multiple of 16 so that each tap is one 4-, 8- or 16-byte vector.
int64_t packed_c(int64_t c) { return c % 16 == 0 ? c : (c <= 4 ? 4 : (c <= 8 ? 8 : ((c + 15) / 16) * 16)); }

int64_t packed_k(int64_t cg, int64_t kh, int64_t kw) { return ((packed_c(cg) * kh * kw + 15) / 16) * 16; }

bool direct_path(const lcml_fp8_conv_desc *d) {
    return d->kH == 1 && d->kW == 1 && d->sH == 1 && d->sW == 1 && d->pH == 0 && d->pW == 0 && d->x_nhwc &&
           d->C % 16 == 0 && d->oH == d->H && d->oW == d->W;
}

// The input is gathered straight from X (NHWC, C a multiple of 16) or from a
// channel-padded NHWC copy of it in the workspace.
bool needs_repack(const lcml_fp8_conv_desc *d) { return !(d->x_nhwc && d->C % 16 == 0); }

// Convs the GEMM can run as an implicit GEMM (TMA im2col loads of the NHWC
// activation; C % 64 == 0; with two spatial dims the im2col bounding-box
// corners must lie in [-128, 127], the tap offsets in [0, 255], the traversal
// strides in 1..8): no im2col pass, no workspace.
bool implicit_ok(const lcml_fp8_conv_desc *d) {
    const int64_t up_w = (d->oW - 1) * d->sW + 1 - d->W - d->pW, up_h = (d->oH - 1) * d->sH + 1 - d->H - d->pH;
    return !direct_path(d) && d->x_nhwc && d->C % 64 == 0 && d->N * d->H * d->W * d->C < (int64_t(1) << 31) &&
           d->N * d->oH * d->oW < (int64_t(1) << 31) && d->pH <= 128 && d->pW <= 128 && up_w >= -128 && up_w <= 127 &&
           up_h >= -128 && up_h <= 127 && d->sH <= 8 && d->sW <= 8 && (d->kH - 1) * d->dH <= 255 &&
           (d->kW - 1) * d->dW <= 255 && d->kH * d->kW * d->C < (int64_t(1) << 31);
}

int64_t repack_bytes(const lcml_fp8_conv_desc *d) {
    return needs_repack(d) ? ((d->N * d->H * d->W * packed_c(d->C) + 255) / 256) * 256 : 0;
}

// Wp[m, (kh*kW + kw)*Cp + c] = W[m, c, kh, kw] for c < Cg; zero for the
// padding channels and beyond kH*kW*Cp.
__global__ void __launch_bounds__(kThreads) k_pack_weight(const uint8_t *__restrict__ W, int64_t M, int64_t Cg,
                                                          int64_t Cp, int64_t kH, int64_t kW, int64_t Kp,
                                                          uint8_t *__restrict__ Wp) {
    const int64_t total = M * Kp;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t m = i / Kp, k = i % Kp;
        uint8_t v = 0;
        if (k < kH * kW * Cp) {
            const int64_t tap = k / Cp, c = k % Cp;
            const int64_t kh = tap / kW, kw = tap % kW;
            if (c < Cg) v = W[((m * Cg + c) * kH + kh) * kW + kw];
        }
        Wp[i] = v;
    }
}

// X (NCHW, or NHWC with C not a multiple of 16) -> Xc NHWC with Cp channels,
// the padding channels zero. One thread per pixel; I is the index type.
template <typename I, bool NHWC_IN>
__global__ void __launch_bounds__(kThreads) k_repack_nhwc(const uint8_t *__restrict__ X, I N, I C, I HW, I Cp,
                                                          uint8_t *__restrict__ Xc) {
    const I total = N * HW;
    for (I pix = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; pix < total;
         pix += static_cast<I>(gridDim.x) * blockDim.x) {
        const I n = pix / HW, hw = pix - n * HW;
        for (I c0 = 0; c0 < Cp; c0 += 4) {
            uint32_t w = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const I c = c0 + j;
                if (c < C) {
                    const uint32_t b = NHWC_IN ? X[pix * C + c] : X[(n * C + c) * HW + hw];
                    w |= b << (8 * j);
                }
            }
            *reinterpret_cast<uint32_t *>(Xc + pix * Cp + c0) = w;
        }
    }
}

// NCHW with C <= 4 -> NHWC with 4 channels (the stem's image): one thread per
// 4 consecutive pixels of one image (HW % 4 == 0, X 4-byte aligned), one
// 4-byte load per channel plane and one 16-byte store, instead of a byte load
// per (pixel, channel). Same bytes as k_repack_nhwc<I, false> with Cp = 4.
__global__ void __launch_bounds__(kThreads) k_repack_nchw_c4(const uint8_t *__restrict__ X, int64_t N, int C,
                                                             int64_t HW, uint8_t *__restrict__ Xc) {
    const int64_t quads = HW / 4, total = N * quads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t n = i / quads, hw = (i - n * quads) * 4;
        uint32_t plane[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (c < C) plane[c] = __ldg(reinterpret_cast<const uint32_t *>(X + (n * C + c) * HW + hw));
        uint32_t px[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)  // pixel j: byte c = channel c
            px[j] = ((plane[0] >> (8 * j)) & 0xffu) | (((plane[1] >> (8 * j)) & 0xffu) << 8) |
                    (((plane[2] >> (8 * j)) & 0xffu) << 16) | (((plane[3] >> (8 * j)) & 0xffu) << 24);
        reinterpret_cast<uint4 *>(Xc)[i] = make_uint4(px[0], px[1], px[2], px[3]);
    }
}

// im2col from NHWC with C a multiple of 16: one 16-byte vector per (pixel,
// 16-channel piece of a tap). I is the index type (32-bit when it fits).
template <typename I>
__global__ void __launch_bounds__(kThreads) k_im2col_nhwc16(const uint8_t *__restrict__ X, I N, I C, I H, I W, I kH,
                                                            I kW, I oH, I oW, I sH, I sW, I pH, I pW, I dH, I dW, I Kp,
                                                            uint8_t *__restrict__ A) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    const I chunks = Kp / 16, cpt = C / 16, taps_chunks = kH * kW * cpt;
    const I total = N * oH * oW * chunks;
    for (I i = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<I>(gridDim.x) * blockDim.x) {
        const I p = i / chunks, ch = i - p * chunks;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (ch < taps_chunks) {
            const I tap = ch / cpt, c16 = ch - tap * cpt;
            const I kh = tap / kW, kw = tap - kh * kW;
            const I t = p / oW, ow = p - t * oW, n = t / oH, oh = t - n * oH;
            const I ih = oh * sH + kh * dH - pH, iw = ow * sW + kw * dW - pW;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                v = __ldg(reinterpret_cast<const uint4 *>(X + ((n * H + ih) * W + iw) * C) + c16);
        }
        reinterpret_cast<uint4 *>(A)[i] = v;
    }
}

// im2col from NHWC with VW (4 or 8) channels: one 16-byte output vector holds
// 16 / VW whole taps, each one VW-byte load.
template <typename I, int VW>
__global__ void __launch_bounds__(kThreads) k_im2col_narrow(const uint8_t *__restrict__ X, I N, I H, I W, I kH, I kW,
                                                            I oH, I oW, I sH, I sW, I pH, I pW, I dH, I dW, I Kp,
                                                            uint8_t *__restrict__ A) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    using V = typename std::conditional<VW == 4, uint32_t, uint2>::type;
    constexpr int TPC = 16 / VW;  // taps per 16-byte chunk
    const I chunks = Kp / 16, taps = kH * kW;
    const I total = N * oH * oW * chunks;
    for (I i = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<I>(gridDim.x) * blockDim.x) {
        const I p = i / chunks, ch = i - p * chunks;
        const I t = p / oW, ow = p - t * oW, n = t / oH, oh = t - n * oH;
        V v[TPC];
#pragma unroll
        for (int j = 0; j < TPC; ++j) {
            const I tap = ch * TPC + j;
            v[j] = V{};
            if (tap < taps) {
                const I kh = tap / kW, kw = tap - kh * kW;
                const I ih = oh * sH + kh * dH - pH, iw = ow * sW + kw * dW - pW;
                if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                    v[j] = __ldg(reinterpret_cast<const V *>(X + ((n * H + ih) * W + iw) * VW));
            }
        }
        *reinterpret_cast<uint4 *>(A + static_cast<int64_t>(i) * 16) = *reinterpret_cast<const uint4 *>(v);
    }
}

// im2col from NHWC with VW (4 or 8) channels, one output pixel per thread:
// the thread walks its kH x kW taps with running indices (no per-tap
// division), packs 16 / VW taps per 16-byte vector into its row of a
// shared-memory tile, and the block then writes its rows, which are
// contiguous in A, with coalesced 16-byte stores. A row is Kp bytes (a
// multiple of 16), so the tile is kRowThreads * Kp bytes of dynamic shared
// memory.
constexpr int kRowThreads = 128;

// A KH x KW window with dilation 1 over 4-byte pixels (4 channels: the ResNet
// stem's 7 x 7): the KW taps of one window row are KW consecutive input
// pixels, so each is a 4-byte load at an immediate offset from one row
// address, and tap t lands in word t of the patch row (K = (kh, kw, c), c
// fastest). Every load of the row is issued before the first store, with a
// few integer operations per tap (the generic kernel spends most of its
// instructions on per-tap index arithmetic). The patch row is staged in
// shared memory and written out with coalesced 16-byte stores.
template <int KH, int KW>
__global__ void __launch_bounds__(kRowThreads) k_im2col_rows_w4(const uint8_t *__restrict__ X, int H, int W, int oH,
                                                                 int oW, int sH, int sW, int pH, int pW, int64_t P,
                                                                 uint8_t *__restrict__ A) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    constexpr int kTaps = KH * KW;
    constexpr int kChunks = (kTaps + 3) / 4;  // Kp / 16
    extern __shared__ uint4 tile[];
    for (int64_t p0 = static_cast<int64_t>(blockIdx.x) * kRowThreads; p0 < P;
         p0 += static_cast<int64_t>(gridDim.x) * kRowThreads) {
        const int64_t p = p0 + threadIdx.x;
        if (p < P) {
            const int64_t t = p / oW;
            const int ow = static_cast<int>(p - t * oW);
            const int64_t n = t / oH;
            const int oh = static_cast<int>(t - n * oH);
            const int ih0 = oh * sH - pH, iw0 = ow * sW - pW;
            const uint32_t *xn = reinterpret_cast<const uint32_t *>(X) + n * H * W;
            uint32_t v[kChunks * 4];
#pragma unroll
            for (int kh = 0; kh < KH; ++kh) {
                const int ih = ih0 + kh;
                const bool row_in = static_cast<unsigned>(ih) < static_cast<unsigned>(H);
                const uint32_t *xr = xn + static_cast<int64_t>(row_in ? ih : 0) * W;
#pragma unroll
                for (int kw = 0; kw < KW; ++kw) {
                    const int iw = iw0 + kw;
                    v[kh * KW + kw] = (row_in && static_cast<unsigned>(iw) < static_cast<unsigned>(W)) ? __ldg(xr + iw) : 0u;
                }
            }
#pragma unroll
            for (int k = kTaps; k < kChunks * 4; ++k) v[k] = 0u;
            uint4 *row = tile + threadIdx.x * kChunks;
#pragma unroll
            for (int c = 0; c < kChunks; ++c) row[c] = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        }
        __syncthreads();
        const int64_t rows = P - p0 < kRowThreads ? P - p0 : kRowThreads;
        uint4 *dst = reinterpret_cast<uint4 *>(A + p0 * kChunks * 16);
        const int64_t vecs = rows * kChunks;
        for (int64_t i = threadIdx.x; i < vecs; i += kRowThreads) dst[i] = tile[i];
        __syncthreads();
    }
}

// MAXCH > 0: the chunk loop is unrolled over at most MAXCH chunks (Kp <=
// 16 * MAXCH), so every tap load of the row is issued before the first one is
// stored (the ResNet stem, Kp = 208: 49 loads in flight per thread instead of
// 4); MAXCH = 0 loops over any Kp.
template <int VW, int MAXCH>
__global__ void __launch_bounds__(kRowThreads) k_im2col_rows(const uint8_t *__restrict__ X, int H, int W, int kH,
                                                              int kW, int oH, int oW, int sH, int sW, int pH, int pW,
                                                              int dH, int dW, int Kp, int64_t P,
                                                              uint8_t *__restrict__ A) {
    griddep_launch_dependents();  // the next GEMM may start its set-up
    using V = typename std::conditional<VW == 4, uint32_t, uint2>::type;
    constexpr int TPC = 16 / VW;  // taps per 16-byte vector
    extern __shared__ uint4 tile[];
    const int chunks = Kp / 16, taps = kH * kW;
    for (int64_t p0 = static_cast<int64_t>(blockIdx.x) * kRowThreads; p0 < P;
         p0 += static_cast<int64_t>(gridDim.x) * kRowThreads) {
        const int64_t p = p0 + threadIdx.x;
        if (p < P) {
            const int64_t t = p / oW;
            const int ow = static_cast<int>(p - t * oW);
            const int64_t n = t / oH;
            const int oh = static_cast<int>(t - n * oH);
            const int ih0 = oh * sH - pH, iw0 = ow * sW - pW;
            const uint8_t *xn = X + n * H * W * VW;
            uint4 *row = tile + threadIdx.x * chunks;
            int kh = 0, kw = 0, tap = 0;
            // the taps of one 16-byte chunk (zero past the last tap and outside the image)
            auto gather = [&](V (&v)[TPC]) {
#pragma unroll
                for (int j = 0; j < TPC; ++j) {
                    v[j] = V{};
                    if (tap < taps) {
                        const int ih = ih0 + kh * dH, iw = iw0 + kw * dW;
                        if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                            v[j] = __ldg(reinterpret_cast<const V *>(xn + (static_cast<int64_t>(ih) * W + iw) * VW));
                        ++tap;
                        if (++kw == kW) {
                            kw = 0;
                            ++kh;
                        }
                    }
                }
            };
            if constexpr (MAXCH > 0) {
                V v[MAXCH][TPC];
#pragma unroll
                for (int c = 0; c < MAXCH; ++c)
                    if (c < chunks) gather(v[c]);
#pragma unroll
                for (int c = 0; c < MAXCH; ++c)
                    if (c < chunks) row[c] = *reinterpret_cast<const uint4 *>(v[c]);
            } else {
                for (int c = 0; c < chunks; ++c) {
                    V v[TPC];
                    gather(v);
                    row[c] = *reinterpret_cast<const uint4 *>(v);
                }
            }
        }
        __syncthreads();
        const int64_t rows = P - p0 < kRowThreads ? P - p0 : kRowThreads;
        uint4 *dst = reinterpret_cast<uint4 *>(A + p0 * Kp);
        const int64_t vecs = rows * chunks;
        for (int64_t i = threadIdx.x; i < vecs; i += kRowThreads) dst[i] = tile[i];
        __syncthreads();
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
    if (d->group > 1) return 0;  // the grouped direct kernel reads X and the packed weights as they are
    if (direct_path(d) || (implicit_ok(d) && !(d->variant & 1))) return 0;
    return d->N * d->oH * d->oW * packed_k(d->C / (d->group > 0 ? d->group : 1), d->kH, d->kW) + repack_bytes(d);
}

int lcml_fp8_conv_pack_weight(const uint8_t *W, int64_t M, int64_t Cg, int64_t kH, int64_t kW, uint8_t *Wp,
                              lcml_stream_t stream) {
    LCML_CHECK_ARG(M > 0 && Cg > 0 && kH > 0 && kW > 0, "lcml_fp8_conv_pack_weight: bad extents");
    LCML_CHECK_ARG(W && Wp, "lcml_fp8_conv_pack_weight: null pointer");
    const int64_t Kp = packed_k(Cg, kH, kW);
    k_pack_weight<<<grid_for(M * Kp), kThreads, 0, to_cuda(stream)>>>(W, M, Cg, packed_c(Cg), kH, kW, Kp, Wp);
    LCML_LAUNCHED("conv_pack_weight");
    return LCML_OK;
}

}// extern "C"

namespace {
template <typename I>
int launch_im2col(const lcml_fp8_conv_desc *d, const uint8_t *X, int64_t Cp, int64_t Kp, uint8_t *A, cudaStream_t st) {
    const int64_t P = d->N * d->oH * d->oW;
    const int grid = grid_for(P * (Kp / 16));
    const int64_t row_smem = static_cast<int64_t>(kRowThreads) * Kp;
    if ((Cp == 4 || Cp == 8) && row_smem <= 96 * 1024 && d->H * d->W * Cp < (int64_t(1) << 31)) {
        // one pixel per thread through a shared-memory row tile (<= 96 KB: two blocks per SM)
        int64_t blocks = (P + kRowThreads - 1) / kRowThreads;
        const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
        if (blocks > cap) blocks = cap;
        if (Cp == 4 && d->kH == 7 && d->kW == 7 && d->dH == 1 && d->dW == 1) {  // the stem
            auto k77 = k_im2col_rows_w4<7, 7>;
            if (const int rc = ensure_max_smem(reinterpret_cast<const void *>(k77), 96 * 1024, "im2col_rows_w4"))
                return rc;
            k77<<<static_cast<int>(blocks), kRowThreads, static_cast<size_t>(row_smem), st>>>(
                X, static_cast<int>(d->H), static_cast<int>(d->W), static_cast<int>(d->oH), static_cast<int>(d->oW),
                d->sH, d->sW, d->pH, d->pW, P, A);
            return LCML_OK;
        }
        const bool unrolled = Kp <= 16 * 16;  // up to 16 chunks: the whole row's loads in flight
        auto kern = Cp == 4 ? (unrolled ? k_im2col_rows<4, 16> : k_im2col_rows<4, 0>)
                            : (unrolled ? k_im2col_rows<8, 16> : k_im2col_rows<8, 0>);
        if (const int rc = ensure_max_smem(reinterpret_cast<const void *>(kern), 96 * 1024, "im2col_rows")) return rc;
        kern<<<static_cast<int>(blocks), kRowThreads, static_cast<size_t>(row_smem), st>>>(
            X, static_cast<int>(d->H), static_cast<int>(d->W), static_cast<int>(d->kH), static_cast<int>(d->kW),
            static_cast<int>(d->oH), static_cast<int>(d->oW), d->sH, d->sW, d->pH, d->pW, d->dH, d->dW,
            static_cast<int>(Kp), P, A);
        return LCML_OK;
    }
    if (Cp == 4)
        k_im2col_narrow<I, 4><<<grid, kThreads, 0, st>>>(X, d->N, d->H, d->W, d->kH, d->kW, d->oH, d->oW, d->sH, d->sW,
                                                         d->pH, d->pW, d->dH, d->dW, Kp, A);
    else if (Cp == 8)
        k_im2col_narrow<I, 8><<<grid, kThreads, 0, st>>>(X, d->N, d->H, d->W, d->kH, d->kW, d->oH, d->oW, d->sH, d->sW,
                                                         d->pH, d->pW, d->dH, d->dW, Kp, A);
    else
        k_im2col_nhwc16<I><<<grid, kThreads, 0, st>>>(X, d->N, Cp, d->H, d->W, d->kH, d->kW, d->oH, d->oW, d->sH, d->sW,
                                                      d->pH, d->pW, d->dH, d->dW, Kp, A);
    return LCML_OK;
}

template <typename I>
void launch_repack(const lcml_fp8_conv_desc *d, int64_t Cp, uint8_t *Xc, cudaStream_t st) {
    const int64_t HW = d->H * d->W;
    if (!d->x_nhwc && Cp == 4 && HW % 4 == 0 && aligned(d->X, 4)) {
        // every thread's four plane loads in flight at once: up to 32 blocks of 256 per SM
        const int64_t items = d->N * (HW / 4);
        int64_t blocks = (items + kThreads - 1) / kThreads;
        const int64_t cap = static_cast<int64_t>(sm_count()) * 32;
        if (blocks > cap) blocks = cap;
        k_repack_nchw_c4<<<static_cast<int>(blocks), kThreads, 0, st>>>(d->X, d->N, static_cast<int>(d->C), HW, Xc);
        return;
    }
    const int grid = grid_for(d->N * d->H * d->W);
    if (d->x_nhwc)
        k_repack_nhwc<I, true><<<grid, kThreads, 0, st>>>(d->X, d->N, d->C, d->H * d->W, Cp, Xc);
    else
        k_repack_nhwc<I, false><<<grid, kThreads, 0, st>>>(d->X, d->N, d->C, d->H * d->W, Cp, Xc);
}
}// namespace

extern "C" {

int lcml_fp8_conv(const lcml_fp8_conv_desc *d, lcml_stream_t stream) {
    LCML_CHECK_ARG(d != nullptr, "lcml_fp8_conv: desc is NULL");
    LCML_CHECK_ARG(d->N > 0 && d->C > 0 && d->H > 0 && d->W > 0 && d->M > 0 && d->kH > 0 && d->kW > 0 && d->oH > 0 &&
                       d->oW > 0 && d->sH > 0 && d->sW > 0 && d->dH > 0 && d->dW > 0 && d->pH >= 0 && d->pW >= 0,
                   "lcml_fp8_conv: bad geometry");
    LCML_CHECK_ARG(d->group >= 1 && d->C % d->group == 0 && d->M % d->group == 0,
                   "lcml_fp8_conv: group %d must divide C = %lld and M = %lld", d->group, (long long)d->C,
                   (long long)d->M);
    LCML_CHECK_ARG((d->oH - 1) * d->sH + (d->kH - 1) * d->dH - d->pH < d->H + d->pH + d->kH &&
                       (d->oW - 1) * d->sW + (d->kW - 1) * d->dW - d->pW < d->W + d->pW + d->kW,
                   "lcml_fp8_conv: output extent inconsistent with the input");
    LCML_CHECK_ARG(d->X && d->Wp && d->Y && d->scale_x && d->scale_w, "lcml_fp8_conv: null operand");
    LCML_CHECK_ARG((d->variant & ~0x701) == 0, "lcml_fp8_conv: variant 0x%x unknown", d->variant);
    LCML_CHECK_ARG(d->epilogue == LCML_EPI_NONE || d->epilogue == LCML_EPI_RELU, "lcml_fp8_conv: epilogue %d", d->epilogue);
    LCML_CHECK_ARG(!d->residual || d->residual_dtype == LCML_DTYPE_FLOAT ||
                       (d->residual_dtype == LCML_DTYPE_FLOAT8E4M3FN && d->residual_scale),
                   "lcml_fp8_conv: residual must be FLOAT or FLOAT8E4M3FN with residual_scale");
    cudaStream_t st = to_cuda(stream);
    if (d->group > 1) {  // grouped / depthwise: memory-bound direct kernel on the CUDA cores
        LCML_CHECK_ARG(d->y_dtype == LCML_DTYPE_FLOAT || d->y_dtype == LCML_DTYPE_BFLOAT16 ||
                           (d->y_dtype == LCML_DTYPE_FLOAT8E4M3FN && d->y_scale),
                       "lcml_fp8_conv: y_dtype %d (FLOAT, BFLOAT16 or FLOAT8E4M3FN with y_scale)", d->y_dtype);
        const int64_t cg = d->C / d->group;
        return fp8_conv_grouped(d, packed_k(cg, d->kH, d->kW), packed_c(cg), st);
    }
    const int64_t P = d->N * d->oH * d->oW;
    const int64_t Cp = packed_c(d->C);
    const int64_t Kp = packed_k(d->C, d->kH, d->kW);
    const uint8_t *A = d->X;
    int64_t K = d->C;
    // Implicit GEMM where the geometry allows it (no im2col pass, no
    // workspace); the materialized lowering otherwise, or when the caller asks.
    const bool implicit = implicit_ok(d) && aligned(d->X, 16) && !(d->variant & 1);
    if (implicit) {
        A = nullptr;
        K = Kp;
    } else if (!direct_path(d)) {
        LCML_CHECK_ARG(d->workspace != nullptr && aligned(d->workspace, 256),
                       "lcml_fp8_conv: this conv needs a 256-byte aligned workspace of %lld bytes",
                       static_cast<long long>(lcml_fp8_conv_workspace_size(d)));
        LCML_CHECK_ARG(aligned(d->X, 16) || needs_repack(d), "lcml_fp8_conv: X must be 16-byte aligned");
        uint8_t *ws = static_cast<uint8_t *>(d->workspace);
        const uint8_t *src = d->X;
        const bool small = d->N * d->H * d->W * Cp < (int64_t(1) << 31) && P * Kp < (int64_t(1) << 31);
        if (needs_repack(d)) {
            uint8_t *xc = ws + P * Kp;  // after the im2col matrix (256-byte aligned below)
            xc = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(xc) + 255) & ~uintptr_t(255));
            if (small) launch_repack<int32_t>(d, Cp, xc, st);
            else launch_repack<int64_t>(d, Cp, xc, st);
            LCML_LAUNCHED("conv_repack");
            src = xc;
        }
        const int rc = small ? launch_im2col<int32_t>(d, src, Cp, Kp, ws, st) : launch_im2col<int64_t>(d, src, Cp, Kp, ws, st);
        if (rc != LCML_OK) return rc;
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
    g.variant = (d->variant >> 8) & 7;
    if (implicit) {
        ConvGeom geo;
        geo.x = d->X;
        geo.N = static_cast<int>(d->N);
        geo.H = static_cast<int>(d->H);
        geo.W = static_cast<int>(d->W);
        geo.C = static_cast<int>(d->C);
        geo.oH = static_cast<int>(d->oH);
        geo.oW = static_cast<int>(d->oW);
        geo.kH = static_cast<int>(d->kH);
        geo.kW = static_cast<int>(d->kW);
        geo.sH = d->sH;
        geo.sW = d->sW;
        geo.pH = d->pH;
        geo.pW = d->pW;
        geo.dH = d->dH;
        geo.dW = d->dW;
        geo.ktaps = geo.kH * geo.kW * geo.C;
        return fp8_gemm_implicit_conv(&g, geo, st);
    }
    return lcml_fp8_gemm(&g, stream);
}

}// extern "C"
