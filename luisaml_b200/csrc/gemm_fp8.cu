// FP8 e4m3 GEMM with a fused QDQ epilogue on sm_100a tensor cores.
//
// Persistent, warp-specialised kernel (192 threads, one CTA per SM):
//   warp 0      TMA producer: A [BM x 128 B] and B [BN x 128 B] K-major tiles,
//               128-byte swizzle, into a STAGES-deep shared-memory ring
//               (mbarrier full/empty pairs, expect-tx byte counts);
//   warp 1      allocates TMEM, one elected thread issues
//               tcgen05.mma.cta_group::1.kind::f8f6f4 (M=128, N=BN, K=32) and
//               tcgen05.commit to release ring stages / publish accumulators;
//   warps 2..5  epilogue: tcgen05.ld 32x32b rows out of TMEM, scale
//               (alpha * sa * sb), + beta*C, Relu or SiLU*up, store fp32/bf16/e4m3,
//               optional per-row amax for the next dynamic quantization.
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the mainloop of tile i+1.
//
// A SIMT kernel (exact same epilogue) covers what TMA cannot address
// (K or leading dimensions that are not 16-byte multiples, MN-major B).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <utility>

#include "lcml_device.cuh"
#include "lcml_internal.h"

namespace lcml {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 128;     // bytes == e4m3 elements per k-block (one 128-byte swizzle atom)
constexpr int UMMA_K = 32;  // K per tcgen05.mma for 8-bit inputs
constexpr int kSmemLimit = 232448;  // dynamic shared memory per CTA on sm_100
constexpr int GROUP_M = 16; // tile rasterisation band height (in BM tiles)

enum OutType : int { kOutF32 = 0, kOutBF16 = 1, kOutE4M3 = 2 };

struct EpiParams {
    int64_t M, N;          // GEMM extents (N counts B rows, i.e. gate+up for SILU_MUL)
    const float *sa;
    int sa_row;
    const float *sb;
    int sb_col;
    float alpha, beta;
    const float *c_vec;
    int c_vec_mode;        // 0 none, 1 tensor, 2 row, 3 col
    const void *c_mat;
    int c_mat_kind;  // 0 fp32, 1 bf16, 2 e4m3 (times c_mat_scale)
    const float *c_mat_scale;
    int64_t ldc;
    void *y;
    int64_t ldy;
    const float *y_scale;
    float *row_amax;
    int64_t y_col_offset;
    void *const *y_peers;
    int y_num_peers;
    int tma_store;  // output written by TMA stores through the kernel's output tensor map
};

__device__ __forceinline__ float silu_mul(float g, float u) {
    const float e = __expf(-fabsf(g));
    const float sig = g >= 0.0f ? __fdividef(1.0f, 1.0f + e) : __fdividef(e, 1.0f + e);
    return (g * sig) * u;
}

__device__ __forceinline__ float load_cmat(const EpiParams &ep, int64_t row, int64_t col) {
    if (ep.c_mat_kind == 1) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(ep.c_mat)[row * ep.ldc + col]);
    if (ep.c_mat_kind == 2)
        return e4m3_decode(reinterpret_cast<const uint8_t *>(ep.c_mat)[row * ep.ldc + col]) * __ldg(ep.c_mat_scale);
    return reinterpret_cast<const float *>(ep.c_mat)[row * ep.ldc + col];
}

// Output quantization constants of one launch: y_scale, RN(1 / y_scale) and
// whether the multiply-by-reciprocal rule (quantize_block_rcp) applies; for
// unusual scales (subnormal, or a reciprocal that is not a normal float)
// every element takes the exact divide of quantize1.
struct OutQuant {
    float ys, r;
    bool s_ok;
};

template <int OUT>
__device__ __forceinline__ OutQuant make_out_quant(const EpiParams &ep) {
    OutQuant q{1.0f, 1.0f, false};
    if (OUT == kOutE4M3) {
        q.ys = __ldg(ep.y_scale);
        q.r = __frcp_rn(q.ys);
        q.s_ok = scale_fast_ok(q.ys, q.r);
    }
    return q;
}

template <int OUT>
__device__ __forceinline__ void store_out(void *y, int64_t ldy, int64_t row, int64_t col, float v, const OutQuant &q) {
    if (OUT == kOutF32) reinterpret_cast<float *>(y)[row * ldy + col] = v;
    else if (OUT == kOutBF16) reinterpret_cast<__nv_bfloat16 *>(y)[row * ldy + col] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<uint8_t *>(y)[row * ldy + col] =
            static_cast<uint8_t>(q.s_ok ? quantize_rcp1(v, q.r) : quantize1(v, q.ys));
}

// Per-column factors of 32 consecutive gemm columns [n0, n0+32): the B scale
// and beta * C broadcast along N. Loaded once per chunk as broadcast vector
// loads (every lane reads the same addresses).
struct ColFactors {
    float scale[32];
    float add[32];
};

__device__ __forceinline__ void load_col_factors(const EpiParams &ep, int64_t n0, ColFactors &f) {
    const bool in_range = n0 + 32 <= ep.N;
    if (ep.sb_col) {
        if (in_range && aligned(ep.sb + n0, 16)) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 v = __ldg(reinterpret_cast<const float4 *>(ep.sb + n0) + j);
                f.scale[4 * j] = v.x;
                f.scale[4 * j + 1] = v.y;
                f.scale[4 * j + 2] = v.z;
                f.scale[4 * j + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) f.scale[j] = (n0 + j < ep.N) ? __ldg(ep.sb + n0 + j) : 0.0f;
        }
    } else {
        const float s = __ldg(ep.sb);
#pragma unroll
        for (int j = 0; j < 32; ++j) f.scale[j] = s;
    }
    if (ep.c_vec_mode == 3) {  // C along N
        if (in_range && aligned(ep.c_vec + n0, 16)) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 v = __ldg(reinterpret_cast<const float4 *>(ep.c_vec + n0) + j);
                f.add[4 * j] = v.x;
                f.add[4 * j + 1] = v.y;
                f.add[4 * j + 2] = v.z;
                f.add[4 * j + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) f.add[j] = (n0 + j < ep.N) ? __ldg(ep.c_vec + n0 + j) : 0.0f;
        }
        if (ep.beta != 1.0f) {
#pragma unroll
            for (int j = 0; j < 32; ++j) f.add[j] *= ep.beta;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) f.add[j] = 0.0f;
    }
}

// beta * C[row, col0 .. col0+32) of the full C matrix (residual), into r[].
__device__ __forceinline__ void load_cmat32(const EpiParams &ep, int64_t row, int64_t col0, int64_t n_out, float (&r)[32]) {
    const bool full = col0 + 32 <= n_out;
    if (ep.c_mat_kind == 2) {
        const uint8_t *cp = reinterpret_cast<const uint8_t *>(ep.c_mat) + row * ep.ldc + col0;
        const float cs = __ldg(ep.c_mat_scale);
        if (full && aligned(cp, 16)) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint4 w = *reinterpret_cast<const uint4 *>(cp + 16 * j);
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float lo, hi;
                    e4m3x2_decode(ws[k >> 1] >> ((k & 1) * 16), lo, hi);
                    r[16 * j + 2 * k] = lo * cs;
                    r[16 * j + 2 * k + 1] = hi * cs;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = (col0 + j < n_out) ? e4m3_decode(cp[j]) * cs : 0.0f;
        }
    } else if (ep.c_mat_kind == 1) {
        const __nv_bfloat16 *cp = reinterpret_cast<const __nv_bfloat16 *>(ep.c_mat) + row * ep.ldc + col0;
        if (full && aligned(cp, 16)) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint4 w = *reinterpret_cast<const uint4 *>(cp + 8 * j);
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    r[8 * j + 2 * k] = __uint_as_float(ws[k] << 16);
                    r[8 * j + 2 * k + 1] = __uint_as_float(ws[k] & 0xffff0000u);
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = (col0 + j < n_out) ? __bfloat162float(cp[j]) : 0.0f;
        }
    } else {
        const float *cp = reinterpret_cast<const float *>(ep.c_mat) + row * ep.ldc + col0;
        if (full && aligned(cp, 16)) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 v = *reinterpret_cast<const float4 *>(cp + 4 * j);
                r[4 * j] = v.x;
                r[4 * j + 1] = v.y;
                r[4 * j + 2] = v.z;
                r[4 * j + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = (col0 + j < n_out) ? cp[j] : 0.0f;
        }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] *= ep.beta;
}

constexpr int out_es(int out) { return out == kOutF32 ? 4 : (out == kOutBF16 ? 2 : 1); }

// 32 values -> the output's bytes as 8 * element-size little-endian words
// (e4m3 by the epilogue quantization rule of quantize_block_rcp). RELU: the
// values have not been through Relu yet (e4m3 output only: Relu is folded
// into the conversion); NONNEG: they have.
template <int OUT, bool NONNEG = false, bool RELU = false>
__device__ __forceinline__ void pack32(const float (&v)[32], const OutQuant &q, uint32_t (&w)[8 * out_es(OUT)]) {
    static_assert(!RELU || OUT == kOutE4M3, "Relu is folded into the conversion for e4m3 outputs only");
    if (OUT == kOutF32) {
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(v[j]);
    } else if (OUT == kOutBF16) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
            w[j] = *reinterpret_cast<uint32_t *>(&h);
        }
    } else if (q.s_ok) {
        quantize_block_rcp<32, NONNEG, RELU>(v, q.r, w);
    } else {
        auto rl = [](float x) { return RELU ? fmaxf(x, 0.0f) : x; };
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = quantize1(rl(v[4 * j]), q.ys) | (quantize1(rl(v[4 * j + 1]), q.ys) << 8) |
                   (quantize1(rl(v[4 * j + 2]), q.ys) << 16) | (quantize1(rl(v[4 * j + 3]), q.ys) << 24);
    }
}

// Stores 32 consecutive output values of one row (vector stores when the row
// segment is in range and 16-byte aligned).
template <int OUT>
__device__ __forceinline__ void store_row32_to(const EpiParams &ep, void *ybase, int64_t row, int64_t col0, int64_t n_out,
                                               const float (&v)[32], const OutQuant &q) {
    constexpr int ES = out_es(OUT);
    const int64_t ocol0 = col0 + ep.y_col_offset;
    uint8_t *yp = reinterpret_cast<uint8_t *>(ybase) + (row * ep.ldy + ocol0) * ES;
    if (col0 + 32 <= n_out && aligned(yp, 16)) {
        uint32_t w[8 * ES];
        pack32<OUT>(v, q, w);
#pragma unroll
        for (int p = 0; p < 2 * ES; ++p)
            reinterpret_cast<uint4 *>(yp)[p] = make_uint4(w[4 * p], w[4 * p + 1], w[4 * p + 2], w[4 * p + 3]);
        return;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j)
        if (col0 + j < n_out) store_out<OUT>(ybase, ep.ldy, row, ocol0 + j, v[j], q);
}

// Warp-cooperative store of a 32-row x 32-column chunk through shared memory
// to the local output and every peer's: lane l holds row (row0 + l); after a
// swizzled transpose each store instruction writes whole 16-byte pieces of
// (32 / P) consecutive rows, i.e. (32 / P) contiguous row segments, instead of
// 32 scattered 16-byte pieces (NVLink write efficiency depends on contiguous
// segments). `stage` holds 32 x 32 elements for this warp. All 32 lanes call it.
template <int OUT>
__device__ __forceinline__ void store_chunk_peers(const EpiParams &ep, uint8_t *stage, int64_t row0, int64_t col0,
                                                  const uint32_t (&w)[8 * out_es(OUT)]) {
    constexpr int ES = out_es(OUT);
    constexpr int RB = 32 * ES;      // bytes of one chunk row
    constexpr int P = RB / 16;       // 16-byte pieces per row
    constexpr int LPG = 8 / P;       // lanes sharing one swizzle phase (8 lanes per shared-memory wavefront)
    const int lane = static_cast<int>(threadIdx.x & 31);
    const int fw = (lane / LPG) % P;
#pragma unroll
    for (int p = 0; p < P; ++p)
        *reinterpret_cast<uint4 *>(stage + lane * RB + ((p ^ fw) * 16)) =
            make_uint4(w[4 * p], w[4 * p + 1], w[4 * p + 2], w[4 * p + 3]);
    __syncwarp();
    const int qq = lane % P;
#pragma unroll
    for (int k = 0; k < P; ++k) {
        const int r = lane / P + k * (32 / P);
        const uint4 d = *reinterpret_cast<const uint4 *>(stage + r * RB + ((qq ^ ((r / LPG) % P)) * 16));
        const int64_t row = row0 + r;
        if (row < ep.M) {
            const int64_t off = (row * ep.ldy + ep.y_col_offset + col0) * ES + qq * 16;
            *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(ep.y) + off) = d;
            for (int pr = 0; pr < ep.y_num_peers; ++pr)
                *reinterpret_cast<uint4 *>(static_cast<uint8_t *>(ep.y_peers[pr]) + off) = d;
        }
    }
    __syncwarp();
}

// Per-warp staging for TMA stores: two buffers of 32 rows x 32 output
// elements (double-buffered so the bulk copy of chunk i overlaps chunk i+1;
// four buffers for e4m3 outputs measured 3 % slower on the short-K convs).
// The row layout matches the output tensor map's swizzle (32B / 64B / 128B
// for 1 / 2 / 4-byte elements: 16-byte piece p of row r sits at p ^ ((r * RB
// / 128) mod P)), which also makes the 16-byte shared stores conflict-free.
template <int OUT>
constexpr int stage_bytes_per_warp() { return 2 * 32 * 32 * out_es(OUT); }

// In the single-CTA kernel each warp's column factors of its current chunk
// (gate scale, gate add, up scale, up add: 4 x 32 floats) sit in a slot after
// all staging buffers (which keep the alignment their swizzle needs); the
// CTA-pair kernel (long K, shared memory full) keeps them in registers.
constexpr int kFacSlotBytes = 4 * 32 * 4;

// Column-factor table of the single-CTA kernel: for GEMMs with N <= kTabMaxN
// (every convolution of ResNet-50) the epilogue warps load each column's
// factors (B scale times the per-tensor A scale and alpha; beta * C along N)
// into shared memory once per CTA, so no chunk waits on a global load for
// them. SILU_MUL GEMMs (the FFN's 22016 columns) keep the per-chunk slots.
constexpr int kTabMaxN = 2048;


// Epilogue warps per CTA: 8 (two per TMEM lane quarter, each taking every
// other 32-column chunk, so one warp's TMEM and memory latency hides behind
// the other's math) except for SILU_MUL, whose register footprint allows 4.
template <int EPI>
constexpr int epi_warps() { return EPI == LCML_EPI_SILU_MUL ? 4 : 8; }
template <int EPI>
constexpr int threads_for() { return 64 + 32 * epi_warps<EPI>(); }
// Single-CTA kernel: epilogue warps as in the pair kernel.
template <int EPI, int OUT>
constexpr int sc_epi_warps() { return EPI == LCML_EPI_SILU_MUL ? 4 : 8; }
// The fast-epilogue kernel without a residual (FAST = 1) fits in 128
// registers, the cap of a 14-warp CTA, and runs 12 epilogue warps: three
// per TMEM lane quarter.
template <int EPI, int OUT, int FAST>
constexpr int sc_epi_warps_f() { return FAST == 1 ? 12 : sc_epi_warps<EPI, OUT>(); }
template <int EPI, int OUT>
constexpr int sc_threads() { return 64 + 32 * sc_epi_warps<EPI, OUT>(); }
template <int EPI, int OUT, int FAST>
constexpr int sc_threads_f() { return 64 + 32 * sc_epi_warps_f<EPI, OUT, FAST>(); }
constexpr int kGatherRowsPerWarp = 64;

template <int OUT>
__device__ __forceinline__ void store_chunk_tma(const CUtensorMap *tmY, uint8_t *stage, uint32_t &seq, int64_t row0,
                                                int64_t col0, const uint32_t (&w)[8 * out_es(OUT)]) {
    constexpr int ES = out_es(OUT);
    constexpr int RB = 32 * ES;
    constexpr int P = RB / 16;
    const int lane = static_cast<int>(threadIdx.x & 31);
    uint8_t *buf = stage + (seq & 1u) * (32 * RB);
    if (lane == 0) bulk_wait_group_read<1>();  // the copy that last read `buf` (two chunks ago) is done
    __syncwarp();
    const int sw = (lane * RB / 128) % P;
#pragma unroll
    for (int p = 0; p < P; ++p)
        *reinterpret_cast<uint4 *>(buf + lane * RB + ((p ^ sw) * 16)) =
            make_uint4(w[4 * p], w[4 * p + 1], w[4 * p + 2], w[4 * p + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(tmY, buf, static_cast<int>(col0), static_cast<int>(row0));
        bulk_commit_group();
    }
    ++seq;
}

// Values of 32 output columns [col0, col0+32) of one row: scale, beta*C,
// SiLU*up, residual, Relu, running |max|. g holds the accumulators of gemm
// columns ng0.. (for SILU_MUL the gate columns; u the up columns nu0..), fg
// their column factors. Parameter-dependent branches are per chunk; the
// element loops are branch-free.
// Raw bytes of the 32 residual values of one row segment, loaded ahead of
// the TMEM wait when the residual is e4m3 and the segment is whole and
// 16-byte aligned (the common conv case); `ok` says the bytes are valid.
struct ResidualRaw {
    uint4 w[2];
    float scale;  // beta * the residual's DequantizeLinear scale
    bool ok;
};

__device__ __forceinline__ void prefetch_residual(const EpiParams &ep, int64_t row, bool row_ok, int64_t col0,
                                                  int64_t n_out, float scale, ResidualRaw &rr) {
    rr.ok = false;
    rr.scale = scale;
    if (!ep.c_mat || ep.c_mat_kind != 2 || !row_ok || col0 + 32 > n_out) return;
    const uint8_t *cp = reinterpret_cast<const uint8_t *>(ep.c_mat) + row * ep.ldc + col0;
    if (!aligned(cp, 16)) return;
    rr.w[0] = __ldg(reinterpret_cast<const uint4 *>(cp));
    rr.w[1] = __ldg(reinterpret_cast<const uint4 *>(cp) + 1);
    rr.ok = true;
}

// Values of 32 output columns [col0, col0+32) of one row: scale, beta*C,
// SiLU*up, residual, Relu, running |max|. g holds the accumulators of gemm
// columns ng0.. (for SILU_MUL the gate columns; u the up columns nu0..), fg
// their column factors, rr the prefetched residual (else it is loaded here).
// Parameter-dependent branches are per chunk; the element loops are
// branch-free.
// RELU_LATER: Relu is left to the output conversion (pack32<..., RELU>), so
// the values come back before Relu (the row |max| still takes Relu into account).
template <int EPI, bool VEC, bool RELU_LATER = false>
__device__ __forceinline__ void epi_values(const EpiParams &ep, int64_t row, bool row_ok, int64_t col0, int64_t nu0,
                                           int64_t n_out, const uint32_t (&g)[32], const uint32_t (&u)[32],
                                           const float *fs, const float *fa, const float *fsu, const float *fau,
                                           const ResidualRaw &rr, float row_scale, float row_add, float &amax,
                                           float (&v)[32]) {
    // fs / fa: B scale and beta * C along N of the 32 (gate) columns (VEC:
    // 16-byte aligned shared memory, read as float4); fsu / fau the same for
    // the up columns
    if (VEC && row_scale == 1.0f && row_add == 0.0f) {  // row scale folded into fs
        const float4 *fs4 = reinterpret_cast<const float4 *>(fs), *fa4 = reinterpret_cast<const float4 *>(fa);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 sc = fs4[j], ad = fa4[j];
            fma2(v[4 * j], v[4 * j + 1], __uint_as_float(g[4 * j]), __uint_as_float(g[4 * j + 1]), sc.x, sc.y, ad.x,
                 ad.y);
            fma2(v[4 * j + 2], v[4 * j + 3], __uint_as_float(g[4 * j + 2]), __uint_as_float(g[4 * j + 3]), sc.z, sc.w,
                 ad.z, ad.w);
        }
    } else if (row_scale == 1.0f && row_add == 0.0f) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaf(__uint_as_float(g[j]), fs[j], fa[j]);
    } else if (row_add == 0.0f) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaf(__uint_as_float(g[j]) * row_scale, fs[j], fa[j]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaf(__uint_as_float(g[j]) * row_scale, fs[j], fa[j] + row_add);
    }
    if (EPI == LCML_EPI_SILU_MUL) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float up = fmaf(__uint_as_float(u[j]) * row_scale, fsu[j], fau[j] + row_add);
            v[j] = silu_mul(v[j], up);
        }
    }
    if (rr.ok) {
        const float cs = rr.scale;
        const uint32_t ws[8] = {rr.w[0].x, rr.w[0].y, rr.w[0].z, rr.w[0].w, rr.w[1].x, rr.w[1].y, rr.w[1].z, rr.w[1].w};
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            float lo, hi;
            e4m3x2_decode(ws[k >> 1] >> ((k & 1) * 16), lo, hi);
            fma2(v[2 * k], v[2 * k + 1], lo, hi, cs, cs, v[2 * k], v[2 * k + 1]);
        }
    } else if (ep.c_mat && row_ok) {
        float r[32];
        load_cmat32(ep, row, col0, n_out, r);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += r[j];
    }
    if (EPI == LCML_EPI_RELU && !RELU_LATER) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
    }
    if (ep.row_amax) {
        // |Relu(v)| = max(v, 0) (NaN ignored either way) when Relu is applied later
#pragma unroll
        for (int j = 0; j < 32; ++j)
            amax = (col0 + j < n_out) ? fmaxf(amax, (EPI == LCML_EPI_RELU && RELU_LATER) ? v[j] : fabsf(v[j])) : amax;
    }
}

__device__ __forceinline__ void atomic_max_abs(float *p, float v) {
    if (!(v > 0.0f)) return;  // also skips NaN
    atomicMax(reinterpret_cast<unsigned int *>(p), __float_as_uint(v));
}

// beta * the DequantizeLinear scale of an e4m3 residual (0 without one).
__device__ __forceinline__ float residual_scale(const EpiParams &ep) {
    return (ep.c_mat && ep.c_mat_kind == 2) ? __ldg(ep.c_mat_scale) * ep.beta : 0.0f;
}

// One output tile's epilogue for the calling warp: TMEM lanes of rows
// [row0, row0+32) (lane l = row row0 + l) of the accumulator at `taddr` (BN
// fp32 columns), gemm column block `tn`, 32-column chunks c_first,
// c_first + c_step, ... Chunks past the last output column are skipped; a
// warp whose rows are all past M does nothing. `stage` is the warp's staging
// area (its two TMA buffers), `seq` its running chunk count (TMA buffer
// parity). Column factors by FAC: kFacTable, the CTA's shared-memory table
// `facw` of every column (scale with the per-tensor A scale folded in at
// [n], beta * C at [kTabMaxN + n]), read as broadcasts; kFacSlot, the warp's
// slot `facw` (gate scale, gate add, up scale, up add), each lane loading
// those of one column one chunk ahead; kFacLoad, every lane loads them as
// broadcast vector loads.
enum FacMode : int { kFacLoad = 0, kFacSlot = 1, kFacTable = 2 };

template <int BN, int EPI, int OUT, int FAC>
__device__ __forceinline__ void epilogue_tile(const EpiParams &ep, const CUtensorMap *tmY, uint32_t taddr, int64_t row0,
                                              int tn, int split, const OutQuant &oq, uint8_t *stage, uint32_t &seq,
                                              int c_first, int c_step, float *facw, float res_scale) {
    constexpr bool FACSLOT = FAC == kFacSlot;
    if (row0 >= ep.M) return;
    const int64_t n_out = (EPI == LCML_EPI_SILU_MUL) ? ep.N / 2 : ep.N;
    const int64_t row = row0 + static_cast<int64_t>(threadIdx.x & 31);
    const bool row_ok = row < ep.M;
    // alpha * the A scale of this row; a per-tensor A scale is folded into the
    // table's column scales (kFacTable), so nothing is loaded for it here
    float row_scale = 1.0f;
    if (ep.sa_row) row_scale = ep.alpha * (row_ok ? __ldg(ep.sa + row) : 0.0f);
    else if (FAC != kFacTable) row_scale = ep.alpha * __ldg(ep.sa);
    float row_add = 0.0f;  // beta * C broadcast as a scalar or along M
    if (ep.c_vec_mode == 1) row_add = ep.beta * __ldg(ep.c_vec);
    else if (ep.c_vec_mode == 2 && row_ok) row_add = ep.beta * __ldg(ep.c_vec + row);
    float amax = 0.0f;
    constexpr int kChunks = (EPI == LCML_EPI_SILU_MUL) ? BN / 64 : BN / 32;
    // a split item (split 0 / 1, never for SILU_MUL) is the first / last BN/2
    // columns of tile column tn, its accumulator in the buffer's first BN/2
    // TMEM columns
    const int nchunks = split < 0 ? kChunks : kChunks / 2;
    const int64_t gbase = static_cast<int64_t>(tn) * BN + (split < 0 ? 0 : split * (BN / 2));  // gemm column of chunk 0
    // SILU_MUL: BN columns = BN/2 gate columns followed by BN/2 up columns
    auto col_of = [&](int c) {
        return (EPI == LCML_EPI_SILU_MUL) ? static_cast<int64_t>(tn) * (BN / 2) + c * 32 : gbase + c * 32;
    };
    const int lane = static_cast<int>(threadIdx.x & 31);
    // this lane's column factors of chunk c: gemm column gbase + c*32 + lane (and its up column);
    // a per-tensor A scale (times alpha) is folded into the slot's column scale
    const float fold_scale = ep.sa_row ? 1.0f : row_scale;
    auto load_fac = [&](int c, float (&f)[4]) {
        const int64_t n = gbase + c * 32 + lane;
#pragma unroll
        for (int h = 0; h < (EPI == LCML_EPI_SILU_MUL ? 2 : 1); ++h) {
            const int64_t nn = n + h * (BN / 2);
            f[2 * h] = (ep.sb_col ? (nn < ep.N ? __ldg(ep.sb + nn) : 0.0f) : __ldg(ep.sb)) * fold_scale;
            f[2 * h + 1] = (ep.c_vec_mode == 3 && nn < ep.N) ? ep.beta * __ldg(ep.c_vec + nn) : 0.0f;
        }
    };
    // Relu of an e4m3 output is folded into the conversion (pack32)
    constexpr bool kReluInPack = EPI == LCML_EPI_RELU && OUT == kOutE4M3;
    // the residual and the factors of the next chunk are loaded while this one is processed
    // (res_scale: beta * the e4m3 residual's scale, loaded once per kernel)
    ResidualRaw rr_next;
    prefetch_residual(ep, row, row_ok, col_of(c_first), n_out, res_scale, rr_next);
    float fnext[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (FACSLOT && c_first < nchunks) load_fac(c_first, fnext);
#pragma unroll 1
    for (int c = c_first; c < nchunks; c += c_step) {
        const int64_t ng0 = gbase + c * 32;
        const int64_t col0 = col_of(c);
        if (col0 >= n_out) break;  // warp-uniform
        uint32_t g[32], u[32];
        tmem_ld_32x32b_x32(taddr + c * 32, g);
        if (EPI == LCML_EPI_SILU_MUL) tmem_ld_32x32b_x32(taddr + BN / 2 + c * 32, u);
        const ResidualRaw rr = rr_next;
        float v[32];
        if (FAC == kFacTable) {
            if (c + c_step < nchunks) prefetch_residual(ep, row, row_ok, col_of(c + c_step), n_out, res_scale, rr_next);
            tmem_wait_ld();
            epi_values<EPI, true, kReluInPack>(ep, row, row_ok, col0, ng0 + BN / 2, n_out, g, g, facw + ng0,
                                               facw + kTabMaxN + ng0, facw, facw, rr, row_scale, row_add, amax, v);
        } else if (FACSLOT) {
            facw[lane] = fnext[0];
            facw[32 + lane] = fnext[1];
            if (EPI == LCML_EPI_SILU_MUL) {
                facw[64 + lane] = fnext[2];
                facw[96 + lane] = fnext[3];
            }
            if (c + c_step < nchunks) {
                prefetch_residual(ep, row, row_ok, col_of(c + c_step), n_out, res_scale, rr_next);
                load_fac(c + c_step, fnext);
            }
            __syncwarp();
            tmem_wait_ld();
            epi_values<EPI, true, kReluInPack>(ep, row, row_ok, col0, ng0 + BN / 2, n_out, g,
                                               EPI == LCML_EPI_SILU_MUL ? u : g, facw, facw + 32, facw + 64, facw + 96,
                                               rr, ep.sa_row ? row_scale : 1.0f, row_add, amax, v);
            __syncwarp();  // every lane has read facw before the next chunk rewrites it
        } else {
            ColFactors fg, fu;
            load_col_factors(ep, ng0, fg);  // global loads overlap the TMEM load
            if (EPI == LCML_EPI_SILU_MUL) load_col_factors(ep, ng0 + BN / 2, fu);
            if (c + c_step < nchunks)
                prefetch_residual(ep, row, row_ok, col_of(c + c_step), n_out, res_scale, rr_next);
            tmem_wait_ld();
            epi_values<EPI, false, kReluInPack>(ep, row, row_ok, col0, ng0 + BN / 2, n_out, g,
                                                EPI == LCML_EPI_SILU_MUL ? u : g, fg.scale, fg.add, fu.scale, fu.add, rr,
                                                row_scale, row_add, amax, v);
        }
        constexpr int ES = out_es(OUT);
        constexpr bool kNonNeg = EPI == LCML_EPI_RELU && !kReluInPack;
        if (ep.tma_store) {
            uint32_t w[8 * ES];
            pack32<OUT, kNonNeg, kReluInPack>(v, oq, w);
            store_chunk_tma<OUT>(tmY, stage, seq, row0, col0, w);
        } else if (ep.y_num_peers > 0 && col0 + 32 <= n_out && ((ep.ldy * ES) % 16 == 0) &&
                   (((ep.y_col_offset + col0) * ES) % 16 == 0)) {
            uint32_t w[8 * ES];
            pack32<OUT, kNonNeg, kReluInPack>(v, oq, w);
            store_chunk_peers<OUT>(ep, stage, row0, col0, w);
        } else if (row_ok) {
            if (kReluInPack) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
            }
            store_row32_to<OUT>(ep, ep.y, row, col0, n_out, v, oq);
            for (int p = 0; p < ep.y_num_peers; ++p) store_row32_to<OUT>(ep, ep.y_peers[p], row, col0, n_out, v, oq);
        }
    }
    if (ep.row_amax && row_ok) atomic_max_abs(ep.row_amax + row, amax);
}

// Fast path of the single-CTA epilogue for the common convolution case,
// compiled as its own kernels (FAST = 1, 2) that the host picks: column factors
// from the shared table (per-tensor A scale and alpha folded in, beta * C
// along N or none), e4m3 output through TMA stores by the reciprocal rule,
// no row |max|, no peers, N a multiple of 32, and either no residual (RES =
// false) or an e4m3 residual with 16-byte aligned rows (RES = true). With
// those decided at compile time the chunk loop carries no per-chunk tests
// besides the last-column one and the output scale's (pack32), and the
// kernel holds no generic epilogue beside it; the same arithmetic as
// epilogue_tile (fma2 by the table's factors, the residual's fma2, the
// block conversion). S warps share a TMEM lane quarter (two, or three in
// the 12-warp kernels), each taking every S-th chunk from c_first. Rows
// past M read row M - 1's residual; the TMA store drops their outputs.
template <int BN, int EPI, bool RES, int S>
__device__ __forceinline__ void epilogue_tile_fast(const EpiParams &ep, const CUtensorMap *tmY, uint32_t taddr,
                                                   int64_t row0, int tn, const OutQuant &oq, uint8_t *stage,
                                                   uint32_t &seq, int c_first, const float *tab, float res_scale) {
    constexpr int kChunks = BN / 32;  // S warps share the tile's chunks: c_first, c_first + S, ...
    if (row0 >= ep.M) return;
    const int lane = static_cast<int>(threadIdx.x & 31);
    int64_t row = row0 + lane;
    if (row >= ep.M) row = ep.M - 1;
    const int64_t colt = static_cast<int64_t>(tn) * BN;
    const uint8_t *res_row = RES ? reinterpret_cast<const uint8_t *>(ep.c_mat) + row * ep.ldc : nullptr;
    uint4 rn0 = make_uint4(0, 0, 0, 0), rn1 = rn0;
    if (RES && c_first < kChunks && colt + c_first * 32 < ep.N) {
        const uint4 *p = reinterpret_cast<const uint4 *>(res_row + colt + c_first * 32);
        rn0 = __ldg(p);
        rn1 = __ldg(p + 1);
    }
#pragma unroll 1
    for (int c = c_first; c < kChunks; c += S) {
        const int64_t col0 = colt + c * 32;
        if (col0 >= ep.N) break;  // warp-uniform
        uint32_t g[32];
        tmem_ld_32x32b_x32(taddr + c * 32, g);
        const uint4 r0 = rn0, r1 = rn1;
        if (RES && c + S < kChunks && col0 + 32 * S < ep.N) {  // the residual of this warp's next chunk
            const uint4 *p = reinterpret_cast<const uint4 *>(res_row + col0 + 32 * S);
            rn0 = __ldg(p);
            rn1 = __ldg(p + 1);
        }
        tmem_wait_ld();
        float v[32];
        const float4 *fs4 = reinterpret_cast<const float4 *>(tab + col0);
        const float4 *fa4 = reinterpret_cast<const float4 *>(tab + kTabMaxN + col0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 sc = fs4[j], ad = fa4[j];
            fma2(v[4 * j], v[4 * j + 1], __uint_as_float(g[4 * j]), __uint_as_float(g[4 * j + 1]), sc.x, sc.y, ad.x,
                 ad.y);
            fma2(v[4 * j + 2], v[4 * j + 3], __uint_as_float(g[4 * j + 2]), __uint_as_float(g[4 * j + 3]), sc.z, sc.w,
                 ad.z, ad.w);
        }
        if (RES) {
            const uint32_t ws[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                float lo, hi;
                e4m3x2_decode(ws[k >> 1] >> ((k & 1) * 16), lo, hi);
                fma2(v[2 * k], v[2 * k + 1], lo, hi, res_scale, res_scale, v[2 * k], v[2 * k + 1]);
            }
        }
        uint32_t w[8];
        pack32<kOutE4M3, false, EPI == LCML_EPI_RELU>(v, oq, w);
        store_chunk_tma<kOutE4M3>(tmY, stage, seq, row0, col0, w);
    }
}

// Tile index -> (m tile, n tile), banded so that CTAs running at the same time
// share A rows and B columns in L2.
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int &tm, int &tn) {
    const int per_group = GROUP_M * num_n;
    const int group = tile / per_group;
    const int first_m = group * GROUP_M;
    const int gsize = min(num_m - first_m, GROUP_M);
    const int in_group = tile - group * per_group;
    tm = first_m + in_group % gsize;
    tn = in_group / gsize;
}

// Bytes of the column-factor table: none for SILU_MUL, and none where it
// would leave fewer than three operand stages (BN = 256 with fp32 output).
template <int BN, int EPI, int OUT, int BKB, int FAST = 0>
constexpr int tab_bytes() {
    const int room = kSmemLimit - 2048 - sc_epi_warps_f<EPI, OUT, FAST>() * (stage_bytes_per_warp<OUT>() + kFacSlotBytes) -
                     2 * kTabMaxN * 4;
    return (EPI != LCML_EPI_SILU_MUL && room / (BM * BKB + BN * BKB) >= 3) ? 2 * kTabMaxN * 4 : 0;
}

template <int BN, int STAGES, int EPI, int OUT, int BKB = BK, int FAST = 0>
struct Layout {
    static constexpr int kABytes = BM * BKB;
    static constexpr int kBBytes = BN * BKB;
    static constexpr int kStageBytes = kABytes + kBBytes;
    // fp32 accumulators in TMEM: 4 buffers for BN <= 128 (the MMA can run up to
    // three tiles ahead of the slowest epilogue warp), 2 for BN = 256
    static constexpr int kAcc = BN <= 128 ? 4 : 2;
    static constexpr int kTmemCols = kAcc * BN;
    static constexpr int kBarOffset = STAGES * kStageBytes;
    static constexpr int kEpiOffset = kBarOffset + 1024;     // epilogue warps' output staging
    static constexpr int kFacOffset = kEpiOffset + sc_epi_warps_f<EPI, OUT, FAST>() * stage_bytes_per_warp<OUT>();  // factor slots
    static constexpr int kTabOffset = kFacOffset + sc_epi_warps_f<EPI, OUT, FAST>() * kFacSlotBytes;  // column-factor table
    static constexpr int kSmemBytes = kTabOffset + tab_bytes<BN, EPI, OUT, BKB, FAST>() + 1024;  // +1024 alignment
};

// The deepest operand ring (at most 8 stages) that fits beside the staging
// and the column-factor table.
template <int BN, int EPI, int OUT, int BKB = BK, int FAST = 0>
constexpr int stages_for() {
    const int room = kSmemLimit - 2048 - sc_epi_warps_f<EPI, OUT, FAST>() * (stage_bytes_per_warp<OUT>() + kFacSlotBytes) -
                     tab_bytes<BN, EPI, OUT, BKB, FAST>();
    const int s = room / (BM * BKB + BN * BKB);
    return s > 8 ? 8 : s;
}

// Work item j of the CTA-pair kernel's persistent schedule -> (tile, half):
// items below n_whole are whole 256 x 256 tiles (half = -1); each tile from
// n_whole on is split into two 256 x 128 items (half 0 and 1: its first and
// last 128 columns). The host splits the tiles of a last wave that would
// leave at least half of the pairs idle, so that wave takes half a tile's
// time.
__device__ __forceinline__ int split_item_tile(int j, int n_whole, int &half) {
    if (j < n_whole) {
        half = -1;
        return j;
    }
    half = (j - n_whole) & 1;
    return n_whole + ((j - n_whole) >> 1);
}

// IM2COL: tmA is an im2col tensor map of the NHWC activation described by
// `geo` (implicit-GEMM convolution): per K-block the producer loads, with one
// TMA im2col copy, the tile's 128 output positions x BKB channels of one
// filter tap (zero outside the image), exactly the K-major A tile the MMA
// reads. BKB = 128 needs C % 128 == 0, BKB = 64 (64-byte rows, 64-byte
// swizzle) C % 64 == 0.
template <int BN, int STAGES, int EPI, int OUT, bool IM2COL, int BKB = BK, int FAST = 0>
__global__ void __launch_bounds__(sc_threads_f<EPI, OUT, FAST>(), 1)
    k_gemm_fp8_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmY, int M, int N, int K, EpiParams ep, ConvGeom geo,
                  int *err) {
    using L = Layout<BN, STAGES, EPI, OUT, BKB, FAST>;
    constexpr int kEW = sc_epi_warps_f<EPI, OUT, FAST>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBarOffset);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + L::kAcc;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + L::kAcc);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_m = (M + BM - 1) / BM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int kblocks = (K + BKB - 1) / BKB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < L::kAcc; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kEW);
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_wait();  // operands, scales and residuals may come from the previous kernel

    if (IM2COL && warp == 0) {
        // ---------------- TMA im2col producer (implicit-GEMM convolution) ----------------
        if (elect_one()) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            const int ohw = geo.oH * geo.oW;
            const int cblocks = geo.C / BKB;  // K-blocks per filter tap
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                int tm, tn;
                tile_coords(tile, num_m, num_n, tm, tn);
                // first output position of the tile -> its input corner (rows past M read zeros: image N)
                const int m0 = tm * BM;
                const int n0 = m0 / ohw, rem = m0 - n0 * ohw;
                const int oh0 = rem / geo.oW, ow0 = rem - oh0 * geo.oW;
                const int w0 = ow0 * geo.sW - geo.pW, h0 = oh0 * geo.sH - geo.pH;
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err, kDevTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + stage * L::kStageBytes;
                    uint8_t *sb = sa + L::kABytes;
                    const int tap = kb / cblocks, c0 = (kb - tap * cblocks) * BKB;
                    const int kh = tap / geo.kW, kw = tap - kh * geo.kW;
                    mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
                    tma_load_im2col_4d(&tmA, &full[stage], sa, c0, w0, h0, n0, static_cast<uint16_t>(kw * geo.dW),
                                       static_cast<uint16_t>(kh * geo.dH));
                    tma_load_2d(&tmB, &full[stage], sb, kb * BKB, tn * BN);
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            const int pending = issued < STAGES ? issued : STAGES;
            for (int i = 0; i < pending; ++i) {
                if (--stage < 0) {
                    stage = STAGES - 1;
                    phase ^= 1u;
                }
                mbar_wait(&full[stage], phase, err, kDevTimeoutDrain);
            }
        }
    } else if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (elect_one()) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                int tm, tn;
                tile_coords(tile, num_m, num_n, tm, tn);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err, kDevTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + stage * L::kStageBytes;
                    uint8_t *sb = sa + L::kABytes;
                    mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
                    tma_load_2d(&tmA, &full[stage], sa, kb * BKB, tm * BM);
                    tma_load_2d(&tmB, &full[stage], sb, kb * BKB, tn * BN);
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Drain: the last min(STAGES, issued) loads must land before the CTA
            // can retire (bounded; normally already complete).
            const int pending = issued < STAGES ? issued : STAGES;
            for (int i = 0; i < pending; ++i) {
                if (--stage < 0) {
                    stage = STAGES - 1;
                    phase ^= 1u;
                }
                mbar_wait(&full[stage], phase, err, kDevTimeoutDrain);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_e4m3_f32(BM, BN, 0);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err, kDevTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, err, kDevTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
                    const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
                    for (int k = 0; k < BKB / UMMA_K; ++k) {
                        const uint64_t adesc = sdesc_kmajor<BKB>(a_addr + k * UMMA_K);
                        const uint64_t bdesc = sdesc_kmajor<BKB>(b_addr + k * UMMA_K);
                        umma_f8f6f4(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                if (++acc == L::kAcc) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
    } else {
        // ---------------- epilogue warps ----------------
        const int quarter = warp & 3;    // TMEM lanes [32*quarter, 32*quarter+32)
        const int e = warp - 2;          // epilogue warp index
        const int phase_c = e >> 2;      // this warp takes chunks phase_c, phase_c + kEW/4, ...
        const OutQuant oq = make_out_quant<OUT>(ep);
        uint8_t *stage = smem + L::kEpiOffset + e * stage_bytes_per_warp<OUT>();
        float *facw = reinterpret_cast<float *>(smem + L::kFacOffset + e * kFacSlotBytes);
        float *tab = reinterpret_cast<float *>(smem + L::kTabOffset);
        // every column's factors into the shared table once (N <= kTabMaxN; zero past N up to the chunk edge)
        constexpr bool kHasTable = tab_bytes<BN, EPI, OUT, BKB, FAST>() > 0;
        const bool use_table = kHasTable && N <= kTabMaxN;
        if (use_table) {
            const float fold = ep.sa_row ? 1.0f : ep.alpha * __ldg(ep.sa);
            const int nfill = ((N + 31) / 32) * 32;
            for (int n = e * 32 + lane; n < nfill; n += kEW * 32) {
                const bool ok = n < N;
                tab[n] = ok ? (ep.sb_col ? __ldg(ep.sb + n) : __ldg(ep.sb)) * fold : 0.0f;
                tab[kTabMaxN + n] = (ok && ep.c_vec_mode == 3) ? ep.beta * __ldg(ep.c_vec + n) : 0.0f;
            }
            named_barrier_sync(1, kEW * 32);  // the epilogue warps only
        }
        uint32_t seq = 0;
        if (ep.tma_store && lane == 0) tma_prefetch_desc(&tmY);
        const float res_scale = residual_scale(ep);
        static_assert(FAST == 0 || (kHasTable && OUT == kOutE4M3 && EPI != LCML_EPI_SILU_MUL && kEW % 4 == 0),
                      "the fast epilogue needs the column-factor table and e4m3 output");
        int acc = 0;
        uint32_t acc_phase = 0;
        int tile_iter = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++tile_iter) {
            int tm, tn;
            tile_coords(tile, num_m, num_n, tm, tn);
            if (!mbar_wait(&tfull[acc], acc_phase, err, kDevTimeoutEpilogue)) break;
            tc_fence_after();
            const int64_t row0 = static_cast<int64_t>(tm) * BM + quarter * 32;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
            if constexpr (FAST != 0) {  // the host checked epilogue_tile_fast's conditions
                // three warps per quarter: the chunk rotation moves on by one each tile, so no warp
                // always takes the extra chunk of a tile whose chunk count three does not divide
                const int first = kEW == 12 ? (phase_c + tile_iter) % 3 : phase_c;
                epilogue_tile_fast<BN, EPI, FAST == 2, kEW / 4>(ep, &tmY, taddr, row0, tn, oq, stage, seq, first, tab,
                                                                res_scale);
            } else if constexpr (kHasTable) {
                if (use_table)
                    epilogue_tile<BN, EPI, OUT, kFacTable>(ep, &tmY, taddr, row0, tn, -1, oq, stage, seq, phase_c,
                                                           kEW / 4, tab, res_scale);
                else
                    epilogue_tile<BN, EPI, OUT, kFacSlot>(ep, &tmY, taddr, row0, tn, -1, oq, stage, seq, phase_c,
                                                          kEW / 4, facw, res_scale);
            } else {
                epilogue_tile<BN, EPI, OUT, kFacSlot>(ep, &tmY, taddr, row0, tn, -1, oq, stage, seq, phase_c, kEW / 4,
                                                      facw, res_scale);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            if (++acc == L::kAcc) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_group_all();  // TMA stores done before the staging memory goes away
        // this warp's peer stores ordered before the kernel's completion: once
        // per kernel, not per tile (a system fence waits for the NVLink stores)
        if (ep.y_num_peers > 0) __threadfence_system();
    }

    griddep_launch_dependents();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (cluster of 2, tcgen05.mma.cta_group::2): a 256 x 256 tile
// per pair. Each CTA stages its 128 rows of A and 128 rows of B (32 KB per
// k-block), so six stages fit and every staged byte feeds twice the MMA work
// of the single-CTA kernel. The even CTA ("leader") arms the full barrier for
// both halves and issues the MMAs; commits multicast to both CTAs' barriers;
// both CTAs run an epilogue over their own 128 TMEM lanes. No TMA multicast.
// ---------------------------------------------------------------------------

template <int STAGES, int EPI, int OUT>
struct PairLayout {
    static constexpr int kHalfBytes = 128 * BK;           // 16 KB: A half or B half
    static constexpr int kStageBytes = 2 * kHalfBytes;    // per CTA
    static constexpr int kTmemCols = 512;                 // 2 x 256 fp32 accumulators
    static constexpr int kBarOffset = STAGES * kStageBytes;
    static constexpr int kEpiOffset = kBarOffset + 1024;     // epilogue warps' output staging
    static constexpr int kSmemBytes = kEpiOffset + epi_warps<EPI>() * stage_bytes_per_warp<OUT>() + 1024;
};

template <int EPI, int OUT>
constexpr int pair_stages_for() {
    const int s = (kSmemLimit - 2048 - epi_warps<EPI>() * stage_bytes_per_warp<OUT>()) / (2 * 128 * BK);
    return s > 8 ? 8 : s;
}

// tmB2: B with 64-row boxes, for the split tiles (each CTA supplies 64 of
// the 128 columns); n_split: tiles split in two at the end of the schedule.
template <int STAGES, int EPI, int OUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads_for<EPI>(), 1)
    k_gemm_fp8_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmY, int M, int N,
                   int K, int n_split, EpiParams ep, int *err) {
    using L = PairLayout<STAGES, EPI, OUT>;
    constexpr int BN = 256;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBarOffset);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;
    const int num_m = (M + 255) / 256;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int n_whole = num_tiles - n_split;
    const int num_items = num_tiles + n_split;
    const int kblocks = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 2 * epi_warps<EPI>());  // the epilogue warps of both CTAs
        }
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, L::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // barrier inits and TMEM allocation visible to the peer
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_wait();  // operands, scales and residuals may come from the previous kernel

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (elect_one()) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            for (int item = pair; item < num_items && ok; item += npairs) {
                int half, tm, tn;
                tile_coords(split_item_tile(item, n_whole, half), num_m, num_n, tm, tn);
                const int arow = tm * 256 + static_cast<int>(rank) * 128;
                // a split tile's 128 columns: 64 B rows from each CTA
                const int brow = half < 0 ? tn * BN + static_cast<int>(rank) * 128
                                          : tn * BN + half * 128 + static_cast<int>(rank) * 64;
                const CUtensorMap *tb = half < 0 ? &tmB : &tmB2;
                const uint32_t tx = half < 0 ? 2 * L::kStageBytes : 2 * (L::kHalfBytes + L::kHalfBytes / 2);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err, kDevTimeoutProducer)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + stage * L::kStageBytes;
                    uint8_t *sb = sa + L::kHalfBytes;
                    if (rank == 0) mbar_arrive_expect_tx(&full[stage], tx);
                    const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
                    tma_load_2d_pair(&tmA, bar, sa, kb * BK, arow);
                    tma_load_2d_pair(tb, bar, sb, kb * BK, brow);
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (rank == 0) {
                // drain: the last loads (both halves land on the leader's barriers)
                const int pending = issued < STAGES ? issued : STAGES;
                for (int i = 0; i < pending; ++i) {
                    if (--stage < 0) {
                        stage = STAGES - 1;
                        phase ^= 1u;
                    }
                    mbar_wait(&full[stage], phase, err, kDevTimeoutDrain);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader CTA only) ----------------
        if (rank == 0 && elect_one()) {
            constexpr uint32_t idesc_whole = idesc_e4m3_f32(256, BN, 0);
            constexpr uint32_t idesc_split = idesc_e4m3_f32(256, BN / 2, 0);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int item = pair; item < num_items && ok; item += npairs) {
                const uint32_t idesc = item < n_whole ? idesc_whole : idesc_split;
                if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, err, kDevTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < kblocks; ++kb) {
                    if (!mbar_wait(&full[stage], phase, err, kDevTimeoutMma)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
                    const uint32_t b_addr = a_addr + L::kHalfBytes;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k) {
                        umma_f8f6f4_pair(d_tmem, sdesc_kmajor_sw128(a_addr + k * UMMA_K),
                                         sdesc_kmajor_sw128(b_addr + k * UMMA_K), idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    umma_commit_pair_mc(&empty[stage], 0x3);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair_mc(&tfull[acc], 0x3);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
    } else {
        // ---------------- epilogue warps (both CTAs) ----------------
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const OutQuant oq = make_out_quant<OUT>(ep);
        uint8_t *stage = smem + L::kEpiOffset + (warp - 2) * stage_bytes_per_warp<OUT>();
        uint32_t seq = 0;
        if (ep.tma_store && lane == 0) tma_prefetch_desc(&tmY);
        const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[0]), 0);
        const float res_scale = residual_scale(ep);
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int item = pair; item < num_items; item += npairs) {
            int split, tm, tn;
            tile_coords(split_item_tile(item, n_whole, split), num_m, num_n, tm, tn);
            if (!mbar_wait(&tfull[acc], acc_phase, err, kDevTimeoutEpilogue)) break;
            tc_fence_after();
            const int64_t row0 = static_cast<int64_t>(tm) * 256 + rank * 128 + quarter * 32;
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
            // split: -1 for a whole tile, else which 128-column half of tile column tn
            epilogue_tile<BN, EPI, OUT, kFacLoad>(ep, &tmY, taddr, row0, tn, split, oq, stage, seq, half,
                                                  epi_warps<EPI>() / 4, nullptr, res_scale);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader + 8u * static_cast<uint32_t>(acc));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (lane == 0) bulk_wait_group_all();  // TMA stores done before the staging memory goes away
        // this warp's peer stores ordered before the kernel's completion: once
        // per kernel, not per tile (a system fence waits for the NVLink stores)
        if (ep.y_num_peers > 0) __threadfence_system();
    }

    griddep_launch_dependents();
    tc_fence_before();
    cluster_sync_all();  // every MMA consumed, every accumulator read, in both CTAs
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, L::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// SIMT fallback: 64x64 output tile per 256-thread CTA, operands decoded to
// fp32 in shared memory, same epilogue semantics (per element).
// ---------------------------------------------------------------------------
// Scale + C for one accumulator value (SIMT fallback path, per element).
__device__ __forceinline__ float simt_pre(float acc, float row_scale, int64_t row, int64_t n, const EpiParams &ep) {
    const float sb = ep.sb_col ? __ldg(ep.sb + n) : __ldg(ep.sb);
    float v = acc * row_scale * sb;
    if (ep.c_vec_mode) {
        const float c = ep.c_vec_mode == 1 ? __ldg(ep.c_vec) : (ep.c_vec_mode == 2 ? __ldg(ep.c_vec + row) : __ldg(ep.c_vec + n));
        v = fmaf(ep.beta, c, v);
    }
    return v;
}

// ---------------------------------------------------------------------------
// Split-K kernel for GEMMs with too few 128 x 128 output tiles to fill the
// GPU (skinny M: decode-sized batches, classifier heads). A cluster of S CTAs
// shares one tile; CTA r accumulates K-blocks [r*kb/S, (r+1)*kb/S) in its
// own TMEM and writes the fp32 partial (valid rows) to its shared memory.
// After a cluster barrier CTA r reduces rows [r*R, (r+1)*R) of the tile over
// the S partials through distributed shared memory (ld.shared::cluster, in
// rank order: deterministic), applies the epilogue (scales, beta*C,
// residual, Relu, row |max|, output conversion) and stores; a second cluster
// barrier keeps every partial alive until all of them have been read. Every
// thread of every CTA reaches both barriers, also after a timed-out wait.
// ---------------------------------------------------------------------------
constexpr int kSplitBN = 128;
constexpr int kSplitStages = 7;
constexpr int kSplitThreads = 192;  // warp 0 TMA producer, warp 1 MMA issuer, warps 2-5 TMEM readers
constexpr int kSplitMax = 8;        // portable cluster size
constexpr int kRedBatch = 2;        // items per thread whose remote loads are in flight together

struct SplitLayout {
    static constexpr int kABytes = BM * BK;
    static constexpr int kBBytes = kSplitBN * BK;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kPartStride = kSplitBN + 4;  // floats per partial row: 16-byte skew, conflict-free rows
    // the partial reuses the operand ring: it is written only after the MMAs
    // have committed, i.e. after every stage has been loaded and read
    static constexpr int kPartOffset = 0;
    static constexpr int kBarOffset = kSplitStages * kStageBytes;
    static constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // barriers, TMEM slot, +1024 alignment
    static_assert(BM * kPartStride * 4 <= kBarOffset, "partial tile must fit in the operand ring");
};

template <int EPI, int OUT>
__global__ void __launch_bounds__(kSplitThreads, 1)
    k_gemm_fp8_splitk(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                      int K, int splits, EpiParams ep, int *err) {
    using L = SplitLayout;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::kBarOffset);
    uint64_t *empty = full + kSplitStages;
    uint64_t *tfull = empty + kSplitStages;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfull + 1);
    float *part = reinterpret_cast<float *>(smem + L::kPartOffset);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rank = static_cast<int>(blockIdx.x) % splits;  // the cluster rank (1-D clusters of `splits` CTAs)
    const int tile = static_cast<int>(blockIdx.x) / splits;
    const int num_n = (N + kSplitBN - 1) / kSplitBN;
    const int tm = tile / num_n, tn = tile - tm * num_n;
    const int kblocks = (K + BK - 1) / BK;
    const int kb0 = static_cast<int>(static_cast<int64_t>(rank) * kblocks / splits);
    const int kb1 = static_cast<int>(static_cast<int64_t>(rank + 1) * kblocks / splits);
    const int mv = min(BM, M - tm * BM);  // valid rows of the tile

    if (threadIdx.x == 0) {
        for (int st = 0; st < kSplitStages; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], 1);
        }
        mbar_init(tfull, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kSplitBN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_wait();  // operands, scales and residuals may come from the previous kernel

    if (warp == 0) {
        if (elect_one()) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            int stage = 0, issued = 0;
            uint32_t phase = 0;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, err, kDevTimeoutProducer)) break;
                uint8_t *sa = smem + stage * L::kStageBytes;
                mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
                tma_load_2d(&tmA, &full[stage], sa, kb * BK, tm * BM);
                tma_load_2d(&tmB, &full[stage], sa + L::kABytes, kb * BK, tn * kSplitBN);
                ++issued;
                if (++stage == kSplitStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            const int pending = issued < kSplitStages ? issued : kSplitStages;
            for (int i = 0; i < pending; ++i) {
                if (--stage < 0) {
                    stage = kSplitStages - 1;
                    phase ^= 1u;
                }
                mbar_wait(&full[stage], phase, err, kDevTimeoutDrain);
            }
        }
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_e4m3_f32(BM, kSplitBN, 0);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(&full[stage], phase, err, kDevTimeoutMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
                const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
                for (int k = 0; k < BK / UMMA_K; ++k)
                    umma_f8f6f4(tmem_base, sdesc_kmajor<BK>(a_addr + k * UMMA_K), sdesc_kmajor<BK>(b_addr + k * UMMA_K),
                                idesc, (kb > kb0 || k > 0) ? 1u : 0u);
                umma_commit(&empty[stage]);
                if (++stage == kSplitStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (ok) umma_commit(tfull);
        }
    } else {
        // TMEM -> this CTA's partial (rows of lane quarter warp & 3)
        const int quarter = warp & 3;
        const bool ok = mbar_wait(tfull, 0, err, kDevTimeoutEpilogue);
        tc_fence_after();
        if (32 * quarter < mv) {  // warp-uniform
            const int r = 32 * quarter + lane;
#pragma unroll 1
            for (int c = 0; c < kSplitBN / 32; ++c) {
                uint32_t g[32];
                tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(32 * quarter) << 16) + c * 32, g);
                tmem_wait_ld();
                if (r < mv) {
                    float4 *dst = reinterpret_cast<float4 *>(part + r * L::kPartStride + c * 32);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        dst[j] = ok ? make_float4(__uint_as_float(g[4 * j]), __uint_as_float(g[4 * j + 1]),
                                                  __uint_as_float(g[4 * j + 2]), __uint_as_float(g[4 * j + 3]))
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
            }
        }
    }
    tc_fence_before();
    cluster_sync_all();  // every partial of the cluster is written

    // reduce rows [r0, r1) of the tile over the cluster's partials, epilogue, store
    const OutQuant oq = make_out_quant<OUT>(ep);
    const int64_t n_out = ep.N;
    const int per = (mv + splits - 1) / splits;
    const int r0 = rank * per, r1 = min(mv, r0 + per);
    const int items = r1 > r0 ? (r1 - r0) * (kSplitBN / 4) : 0;
    const uint32_t part_base = smem_u32(part);
    // A thread takes kRedBatch items at a time and issues every remote load of
    // the batch (kRedBatch x splits) before the first add, so it waits for the
    // distributed-shared-memory latency once per batch, not once per load.
    // Each item's sum still runs over the partials in rank order.
    for (int it0 = threadIdx.x; it0 < items; it0 += kSplitThreads * kRedBatch) {
        float4 pv[kRedBatch][kSplitMax];
#pragma unroll
        for (int u = 0; u < kRedBatch; ++u) {
            const int iu = it0 + u * kSplitThreads < items ? it0 + u * kSplitThreads : it0;  // past the end: reload item it0
            const uint32_t off = part_base + static_cast<uint32_t>(((r0 + iu / (kSplitBN / 4)) * L::kPartStride +
                                                                    (iu % (kSplitBN / 4)) * 4) * 4);
#pragma unroll
            for (int sp = 0; sp < kSplitMax; ++sp)
                if (sp < splits) pv[u][sp] = ld_shared_cluster_f4(mapa_shared(off, static_cast<uint32_t>(sp)));
        }
#pragma unroll
        for (int u = 0; u < kRedBatch; ++u) {
            const int it = it0 + u * kSplitThreads;
            if (it >= items) break;
            const int rr = r0 + it / (kSplitBN / 4), c4 = it % (kSplitBN / 4);
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int sp = 0; sp < kSplitMax; ++sp) {
                if (sp < splits) {
                    acc.x += pv[u][sp].x;
                    acc.y += pv[u][sp].y;
                    acc.z += pv[u][sp].z;
                    acc.w += pv[u][sp].w;
                }
            }
            const int64_t row = static_cast<int64_t>(tm) * BM + rr;
            const int64_t col = static_cast<int64_t>(tn) * kSplitBN + c4 * 4;
            const float rs = ep.alpha * (ep.sa_row ? __ldg(ep.sa + row) : __ldg(ep.sa));
            const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
            float amax = 0.0f;
            constexpr int ES = out_es(OUT);
            uint8_t *yp = static_cast<uint8_t *>(ep.y) + (row * ep.ldy + col + ep.y_col_offset) * ES;
            if (col + 4 <= n_out && !ep.c_mat && aligned(yp, 4 * ES) && (!ep.sb_col || aligned(ep.sb + col, 16)) &&
                (ep.c_vec_mode != 3 || aligned(ep.c_vec + col, 16))) {
                // four whole columns: vector loads of the factors, one vector store (same arithmetic as simt_pre)
                const float4 sb4 = ep.sb_col ? __ldg(reinterpret_cast<const float4 *>(ep.sb + col))
                                             : make_float4(__ldg(ep.sb), __ldg(ep.sb), __ldg(ep.sb), __ldg(ep.sb));
                float4 c4v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (ep.c_vec_mode == 3) c4v = __ldg(reinterpret_cast<const float4 *>(ep.c_vec + col));
                else if (ep.c_vec_mode == 1) c4v = make_float4(__ldg(ep.c_vec), __ldg(ep.c_vec), __ldg(ep.c_vec), __ldg(ep.c_vec));
                else if (ep.c_vec_mode == 2) {
                    const float c = __ldg(ep.c_vec + row);
                    c4v = make_float4(c, c, c, c);
                }
                const float sbs[4] = {sb4.x, sb4.y, sb4.z, sb4.w}, cs[4] = {c4v.x, c4v.y, c4v.z, c4v.w};
                float v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v[j] = a4[j] * rs * sbs[j];
                    if (ep.c_vec_mode) v[j] = fmaf(ep.beta, cs[j], v[j]);
                    if (EPI == LCML_EPI_RELU) v[j] = fmaxf(v[j], 0.0f);
                    amax = fmaxf(amax, fabsf(v[j]));
                }
                if (OUT == kOutF32) {
                    *reinterpret_cast<float4 *>(yp) = make_float4(v[0], v[1], v[2], v[3]);
                } else if (OUT == kOutBF16) {
                    __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
                    *reinterpret_cast<uint2 *>(yp) =
                        make_uint2(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1));
                } else {
                    uint32_t w = 0;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        w |= (oq.s_ok ? quantize_rcp1(v[j], oq.r) : quantize1(v[j], oq.ys)) << (8 * j);
                    *reinterpret_cast<uint32_t *>(yp) = w;
                }
                if (ep.row_amax) atomic_max_abs(ep.row_amax + row, amax);
                continue;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t n = col + j;
                if (n >= n_out) break;
                float v = simt_pre(a4[j], rs, row, n, ep);
                if (ep.c_mat) v += ep.beta * load_cmat(ep, row, n);
                if (EPI == LCML_EPI_RELU) v = fmaxf(v, 0.0f);
                amax = fmaxf(amax, fabsf(v));
                store_out<OUT>(ep.y, ep.ldy, row, n + ep.y_col_offset, v, oq);
            }
            if (ep.row_amax) atomic_max_abs(ep.row_amax + row, amax);
        }
    }
    griddep_launch_dependents();
    cluster_sync_all();  // no CTA exits while another may still read its partial
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, kSplitBN);
    }
}

// ---------------------------------------------------------------------------
// Decode-sized GEMM (M <= 4 rows of A): a streaming GEMV on the CUDA cores.
// With one to four rows the work is one read of B (N x K e4m3 bytes); a
// 128-row tensor-core tile would be 1-3 % used, and split-K adds two cluster
// barriers and a reduction through distributed shared memory to the stream.
// Each CTA stages A as floats in shared memory, laid out [row][q][chunk] so
// that lanes reading consecutive 16-byte chunks of B read consecutive float4s
// of A (no bank conflicts). A warp owns kGemvRows rows of B at a time; every
// lane issues all of its 16-byte loads of a step before the first FMA,
// decodes the codes exactly through f16x2 and accumulates the products in
// fp32; a fixed warp-shuffle tree sums the lanes (deterministic). Lane 0 runs
// the per-element epilogue of the other kernels (scales, beta*C, residual,
// Relu, row |max|, output conversion).
// ---------------------------------------------------------------------------
constexpr int kGemvMaxM = 4;
constexpr int kGemvThreads = 256;
constexpr int kGemvRows = 2;     // rows of B per warp in flight
constexpr int kGemvChunks = 8;   // 16-byte chunks per lane per row and step: 4 KB of a row per warp step
constexpr int kGemvSmemMax = 48 * 1024;

// QuantizeLinear of an fp32 A with a dynamic per-tensor scale fused into the
// GEMV (QA kernels): A is at most kGemvMaxM rows, so every CTA takes max|A|
// over all of it (an L2-resident read), derives s = amax / 448 (1 for an
// all-zero A) exactly as the quantize kernels do, and quantizes A with the
// bit-exact block quantizer while staging it; CTA 0 also writes s and the
// codes. One launch instead of the two quantize passes and the GEMV.
struct GemvQuantA {
    const float *a;    // [M, K] fp32, row stride lda (elements, a multiple of 4), 16-byte aligned
    int64_t lda;
    float *scale_out;  // s (one float)
    uint8_t *aq_out;   // the codes [M, K] (row stride K), or nullptr
};

template <int MR, int EPI, int OUT, bool QA = false>
__global__ void __launch_bounds__(kGemvThreads) k_gemv_fp8(const uint8_t *__restrict__ A, int64_t lda,
                                                           const uint8_t *__restrict__ B, int64_t ldb, int M, int N,
                                                           int K, EpiParams ep, GemvQuantA qa) {
    extern __shared__ float4 sA4[];  // [MR][4][K/16]: float4 q of chunk c of row m at m*(K/4) + q*(K/16) + c
    const int kc = K / 16;           // 16-byte chunks per row (K % 16 == 0)
    const int lane = threadIdx.x & 31;
    const int gw = static_cast<int>(blockIdx.x) * (kGemvThreads / 32) + (threadIdx.x >> 5);
    const int nw = static_cast<int>(gridDim.x) * (kGemvThreads / 32);
    // start the DRAM reads of this warp's first rows of B (first 4 KB of each)
    // before staging A, so the two latencies overlap
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
        if (gw * kGemvRows + r < N && lane * 128 < K)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(B + static_cast<int64_t>(gw * kGemvRows + r) * ldb + lane * 128));
    griddep_wait();  // A, the scales and a residual may come from the previous kernel
    griddep_launch_dependents();
    float s_a = 0.0f;  // QA: the per-tensor scale of A derived here
    if constexpr (QA) {
        __shared__ uint32_t red[kGemvThreads / 32];
        uint32_t mx = 0;
        for (int i = threadIdx.x; i < M * (K / 4); i += kGemvThreads) {
            const int m = i / (K / 4), k4 = i - m * (K / 4);
            const float4 v = __ldg(reinterpret_cast<const float4 *>(qa.a + m * qa.lda) + k4);
            mx = max(mx, max(max(abs_bits_nan0(v.x), abs_bits_nan0(v.y)), max(abs_bits_nan0(v.z), abs_bits_nan0(v.w))));
        }
        mx = __reduce_max_sync(0xffffffffu, mx);
        if (lane == 0) red[threadIdx.x >> 5] = mx;
        __syncthreads();
        mx = 0;
#pragma unroll
        for (int w = 0; w < kGemvThreads / 32; ++w) mx = max(mx, red[w]);
        s_a = scale_from_amax(__uint_as_float(mx));
        const float r = __frcp_rn(s_a);
        const bool s_ok = scale_fast_ok(s_a, r);
        for (int i = threadIdx.x; i < MR * kc; i += kGemvThreads) {  // 16 elements per step
            const int m = i / kc, c = i - m * kc;
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            if (m < M) {
                const float4 *p = reinterpret_cast<const float4 *>(qa.a + m * qa.lda) + 4 * c;
                const float4 v0 = __ldg(p), v1 = __ldg(p + 1), v2 = __ldg(p + 2), v3 = __ldg(p + 3);
                const float v[16] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w,
                                     v2.x, v2.y, v2.z, v2.w, v3.x, v3.y, v3.z, v3.w};
                quantize_block_fast<16>(v, s_a, r, s_ok, w);
                if (blockIdx.x == 0 && qa.aq_out)
                    *reinterpret_cast<uint4 *>(qa.aq_out + static_cast<int64_t>(m) * K + 16 * c) =
                        make_uint4(w[0], w[1], w[2], w[3]);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {  // word q = elements 16c + 4q .. +3: float4 q of chunk c
                float d[4];
                e4m3x2_decode(w[q] & 0xffffu, d[0], d[1]);
                e4m3x2_decode(w[q] >> 16, d[2], d[3]);
                sA4[m * (K / 4) + q * kc + c] = make_float4(d[0], d[1], d[2], d[3]);
            }
        }
        if (blockIdx.x == 0 && threadIdx.x == 0) *qa.scale_out = s_a;
    } else {
        for (int i = threadIdx.x; i < MR * (K / 4); i += kGemvThreads) {
            const int m = i / (K / 4), k4 = i - m * (K / 4);
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (m < M) {
                const uint32_t w = *reinterpret_cast<const uint32_t *>(A + m * lda + 4 * k4);
                e4m3x2_decode(w & 0xffffu, v[0], v[1]);
                e4m3x2_decode(w >> 16, v[2], v[3]);
            }
            sA4[m * (K / 4) + (k4 & 3) * kc + (k4 >> 2)] = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
    __syncthreads();

    const OutQuant oq = make_out_quant<OUT>(ep);
    // 64-bit row index: N may come within one grid stride of INT_MAX
    for (int64_t n0 = static_cast<int64_t>(gw) * kGemvRows; n0 < N; n0 += static_cast<int64_t>(nw) * kGemvRows) {
        float acc[kGemvRows][MR];
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
            for (int m = 0; m < MR; ++m) acc[r][m] = 0.0f;
        for (int c0 = 0; c0 < kc; c0 += 32 * kGemvChunks) {
            uint4 bv[kGemvRows][kGemvChunks];
#pragma unroll
            for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
                for (int j = 0; j < kGemvChunks; ++j) {
                    const int c = c0 + j * 32 + lane;
                    bv[r][j] = (n0 + r < N && c < kc) ? __ldcs(reinterpret_cast<const uint4 *>(B + (n0 + r) * ldb) + c)
                                                      : make_uint4(0u, 0u, 0u, 0u);
                }
#pragma unroll
            for (int j = 0; j < kGemvChunks; ++j) {
                const int c = c0 + j * 32 + lane;
                if (c < kc) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        float4 a[MR];
#pragma unroll
                        for (int m = 0; m < MR; ++m) a[m] = sA4[m * (K / 4) + q * kc + c];
#pragma unroll
                        for (int r = 0; r < kGemvRows; ++r) {
                            const uint32_t w = q == 0 ? bv[r][j].x : (q == 1 ? bv[r][j].y : (q == 2 ? bv[r][j].z : bv[r][j].w));
                            float b0, b1, b2, b3;
                            e4m3x2_decode(w & 0xffffu, b0, b1);
                            e4m3x2_decode(w >> 16, b2, b3);
#pragma unroll
                            for (int m = 0; m < MR; ++m) {
                                acc[r][m] = fmaf(a[m].x, b0, acc[r][m]);
                                acc[r][m] = fmaf(a[m].y, b1, acc[r][m]);
                                acc[r][m] = fmaf(a[m].z, b2, acc[r][m]);
                                acc[r][m] = fmaf(a[m].w, b3, acc[r][m]);
                            }
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
            for (int m = 0; m < MR; ++m)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < kGemvRows; ++r) {
                const int64_t col = n0 + r;
                if (col >= N) continue;
#pragma unroll
                for (int m = 0; m < MR; ++m) {
                    if (m >= M) continue;
                    const float rs = ep.alpha * (QA ? s_a : (ep.sa_row ? __ldg(ep.sa + m) : __ldg(ep.sa)));
                    float v = simt_pre(acc[r][m], rs, m, col, ep);
                    if (ep.c_mat) v += ep.beta * load_cmat(ep, m, col);
                    if (EPI == LCML_EPI_RELU) v = fmaxf(v, 0.0f);
                    store_out<OUT>(ep.y, ep.ldy, m, col + ep.y_col_offset, v, oq);
                    if (ep.row_amax) atomic_max_abs(ep.row_amax + m, fabsf(v));
                }
            }
        }
    }
}

template <int EPI, int OUT>
__global__ void __launch_bounds__(256) k_gemm_fp8_simt(const uint8_t *__restrict__ A, int64_t lda,
                                                       const uint8_t *__restrict__ B, int64_t ldb, int b_kmajor,
                                                       int64_t M, int64_t N, int64_t K, EpiParams ep) {
    __shared__ float sA[32][65];
    __shared__ float sB[32][65];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * 64, n0 = static_cast<int64_t>(blockIdx.x) * 64;
    // For SILU the CTA covers 64 output columns = gemm columns gate(n) and up(n).
    float accg[4][4] = {}, accu[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += 32) {
        for (int i = threadIdx.x; i < 64 * 32; i += 256) {
            const int r = i / 32, kk = i % 32;
            const int64_t m = m0 + r, k = k0 + kk;
            sA[kk][r] = (m < M && k < K) ? e4m3_decode(A[m * lda + k]) : 0.0f;
        }
        for (int pass = 0; pass < (EPI == LCML_EPI_SILU_MUL ? 2 : 1); ++pass) {
            __syncthreads();
            for (int i = threadIdx.x; i < 64 * 32; i += 256) {
                const int c = i / 32, kk = i % 32;
                int64_t n = n0 + c;
                if (EPI == LCML_EPI_SILU_MUL) n = (n / 128) * 256 + (n % 128) + pass * 128;
                const int64_t k = k0 + kk;
                float v = 0.0f;
                if (n < N && k < K) v = e4m3_decode(b_kmajor ? B[n * ldb + k] : B[k * ldb + n]);
                sB[kk][c] = v;
            }
            __syncthreads();
            for (int kk = 0; kk < 32; ++kk) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float p = sA[kk][ty * 4 + i] * sB[kk][tx * 4 + j];
                        if (pass == 0) accg[i][j] += p;
                        else accu[i][j] += p;
                    }
            }
        }
        __syncthreads();
    }
    const OutQuant oq = make_out_quant<OUT>(ep);
    const int64_t n_out = (EPI == LCML_EPI_SILU_MUL) ? N / 2 : N;
    for (int i = 0; i < 4; ++i) {
        const int64_t row = m0 + ty * 4 + i;
        if (row >= M) continue;
        const float rs = ep.alpha * (ep.sa_row ? __ldg(ep.sa + row) : __ldg(ep.sa));
        float amax = 0.0f;
        for (int j = 0; j < 4; ++j) {
            const int64_t col = n0 + tx * 4 + j;
            if (col >= n_out) continue;
            float a;
            if (EPI == LCML_EPI_SILU_MUL) {
                const int64_t ng = (col / 128) * 256 + (col % 128);
                a = silu_mul(simt_pre(accg[i][j], rs, row, ng, ep), simt_pre(accu[i][j], rs, row, ng + 128, ep));
            } else {
                a = simt_pre(accg[i][j], rs, row, col, ep);
            }
            if (ep.c_mat) a += ep.beta * load_cmat(ep, row, col);
            if (EPI == LCML_EPI_RELU) a = fmaxf(a, 0.0f);
            amax = fmaxf(amax, fabsf(a));
            store_out<OUT>(ep.y, ep.ldy, row, col + ep.y_col_offset, a, oq);
            for (int p = 0; p < ep.y_num_peers; ++p) store_out<OUT>(ep.y_peers[p], ep.ldy, row, col + ep.y_col_offset, a, oq);
        }
        if (ep.row_amax) atomic_max_abs(ep.row_amax + row, amax);
    }
    if (ep.y_num_peers > 0) __threadfence_system();  // peer stores ordered before the kernel's completion
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D e4m3 K-major operand: `rows` rows of `k` bytes, row stride `ld` bytes,
// box = [box_rows x 128 B] with the 128-byte swizzle.
int make_tmap(CUtensorMap *map, const void *ptr, int64_t k, int64_t rows, int64_t ld, int box_rows, int bkb = BK) {
    auto fn = encode_fn();
    if (!fn) return set_error(LCML_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(bkb), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, bkb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(LCML_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return LCML_OK;
}

// im2col tensor map of the NHWC e4m3 activation of `g`: boxes of 128 output
// positions x bkb channels. The bounding box runs from -pad to the last
// position a filter tap 0 reads ({w, h} order), traversed with the conv
// strides; positions outside the image load zeros.
int make_tmap_im2col(CUtensorMap *map, const ConvGeom &g, int bkb) {
    using Fn = PFN_cuTensorMapEncodeIm2col_v12000;
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeIm2col", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(p);
    });
    if (!fn) return set_error(LCML_ERR_CUDA, "cuTensorMapEncodeIm2col is not available from the driver");
    const uint64_t C = g.C, W = g.W, H = g.H, N = g.N;
    cuuint64_t dims[4] = {C, W, H, N};
    cuuint64_t strides[3] = {C, W * C, H * W * C};
    int lower[2] = {-g.pW, -g.pH};
    int upper[2] = {(g.oW - 1) * g.sW + 1 - g.W - g.pW, (g.oH - 1) * g.sH + 1 - g.H - g.pH};
    cuuint32_t estr[4] = {1, static_cast<cuuint32_t>(g.sW), static_cast<cuuint32_t>(g.sH), 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t *>(g.x), dims, strides, lower, upper,
                    static_cast<cuuint32_t>(bkb), BM, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    bkb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(LCML_ERR_CUDA, "cuTensorMapEncodeIm2col failed (%d)", static_cast<int>(r));
    // Drivers up to 13.1 mis-encode one field of im2col maps over tensors
    // smaller than 128 KiB; CUTLASS clears that bit (bit 21 of word 1) for them.
    int drv = 0;
    if (cudaDriverGetVersion(&drv) == cudaSuccess && drv <= 13010 && N * H * W * C < 131072)
        reinterpret_cast<uint64_t *>(map)[1] &= ~(uint64_t(1) << 21);
    return LCML_OK;
}

// Output tensor map for the TMA-store epilogue: `rows` x `cols` elements of
// `es` bytes starting at `ptr`, row pitch `ld_bytes`, box 32 x 32 with the
// swizzle whose span equals one box row (32 * es bytes).
int make_tmap_out(CUtensorMap *map, void *ptr, int64_t cols, int64_t rows, int64_t ld_bytes, int es) {
    auto fn = encode_fn();
    if (!fn) return set_error(LCML_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_bytes)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt =
        es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : (es == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8);
    const CUtensorMapSwizzle sw =
        es == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : (es == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    CUresult r = fn(map, dt, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(LCML_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", static_cast<int>(r));
    return LCML_OK;
}

// The output map when the epilogue stores through TMA, else an unused zero map.
template <int EPI, int OUT>
int output_tmap(const lcml_fp8_gemm_desc *d, const EpiParams &ep, CUtensorMap *ty) {
    memset(ty, 0, sizeof(*ty));
    if (!ep.tma_store) return LCML_OK;
    constexpr int ES = out_es(OUT);
    const int64_t n_out = (EPI == LCML_EPI_SILU_MUL) ? d->N / 2 : d->N;
    return make_tmap_out(ty, static_cast<uint8_t *>(d->Y) + d->y_col_offset * ES, n_out, d->M, d->ldy * ES, ES);
}

// Every GEMM kernel is launched with programmatic stream serialization (its
// set-up overlaps the tail of the previous kernel on the stream; the kernel
// reads nothing that kernel wrote before griddep_wait), and with a cluster
// shape when cluster_x > 0 (kernels with compile-time cluster dimensions
// pass 0).
template <typename... Params, typename... Args>
int launch_gemm_kernel(void (*kern)(Params...), unsigned grid, unsigned threads, size_t smem, cudaStream_t st,
                       unsigned cluster_x, const char *name, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (cluster_x > 0) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cluster_x;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (e != cudaSuccess) return set_error(LCML_ERR_CUDA, "%s launch failed: %s", name, cudaGetErrorString(e));
    return LCML_OK;
}

// Tiles of the CTA-pair schedule to split into two 256 x 128 items: the
// tiles of a last wave that would leave at least half of the pairs idle
// (with fewer tiles than pairs, every tile), so the pairs that would wait
// take half a tile each (4096^3 on B200: 49.4 vs 54.8 us). None for
// SILU_MUL (a tile's gate and up columns are its two halves). The
// single-CTA kernel does not split: its 128 x 128 halves gained nothing
// measurable on the ResNet-50 convs, and the extra schedule state cost its
// epilogue registers.
int split_tiles(int64_t tiles, int64_t pairs, bool silu_mul) {
    if (silu_mul || pairs < 2) return 0;
    const int64_t rem = tiles % pairs;
    return (rem > 0 && 2 * rem <= pairs) ? static_cast<int>(rem) : 0;
}

template <int BN, int EPI, int OUT, bool IM2COL = false, int BKB = BK, int FAST = 0>
int launch_tc_kernel(const lcml_fp8_gemm_desc *d, const EpiParams &ep, cudaStream_t st, const ConvGeom &geo) {
    constexpr int STAGES = stages_for<BN, EPI, OUT, BKB, FAST>();
    using L = Layout<BN, STAGES, EPI, OUT, BKB, FAST>;
    static_assert(STAGES >= 3 && L::kSmemBytes <= kSmemLimit, "shared memory layout does not fit");
    auto kern = k_gemm_fp8_tc<BN, STAGES, EPI, OUT, IM2COL, BKB, FAST>;
    if (const int rc = ensure_max_smem(reinterpret_cast<const void *>(kern), L::kSmemBytes, "gemm_fp8_tc")) return rc;
    CUtensorMap ta, tb;
    int rc = IM2COL ? make_tmap_im2col(&ta, geo, BKB) : make_tmap(&ta, d->A, d->K, d->M, d->lda, BM, BKB);
    if (rc) return rc;
    rc = make_tmap(&tb, d->B, d->K, d->N, d->ldb, BN, BKB);
    if (rc) return rc;
    CUtensorMap ty;
    rc = output_tmap<EPI, OUT>(d, ep, &ty);
    if (rc) return rc;
    const int64_t tiles = ((d->M + BM - 1) / BM) * ((d->N + BN - 1) / BN);
    const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
    return launch_gemm_kernel(kern, static_cast<unsigned>(grid), sc_threads_f<EPI, OUT, FAST>(), L::kSmemBytes, st, 0,
                              IM2COL ? "conv_implicit_gemm_fp8_tc" : "gemm_fp8_tc", ta, tb, ty, static_cast<int>(d->M),
                              static_cast<int>(d->N), static_cast<int>(d->K), ep, geo, device_error_word());
}

// Which single-CTA kernel serves a GEMM: the fast-epilogue ones (1 without
// a residual, 2 with an e4m3 residual) when every condition of
// epilogue_tile_fast holds, else the generic one (0).
template <int BN, int EPI, int OUT, int BKB>
int fast_kind(const lcml_fp8_gemm_desc *d, const EpiParams &ep) {
    if constexpr (OUT != kOutE4M3 || EPI == LCML_EPI_SILU_MUL || tab_bytes<BN, EPI, OUT, BKB>() == 0) {
        return 0;
    } else {
        if (d->N > kTabMaxN || d->N % 32 != 0 || !ep.tma_store || ep.y_num_peers != 0 || ep.row_amax || ep.sa_row ||
            (ep.c_vec_mode != 0 && ep.c_vec_mode != 3))
            return 0;
        if (!ep.c_mat) return 1;
        return (ep.c_mat_kind == 2 && ep.ldc % 16 == 0 && aligned(ep.c_mat, 16)) ? 2 : 0;
    }
}

template <int BN, int EPI, int OUT, bool IM2COL = false, int BKB = BK>
int launch_tc(const lcml_fp8_gemm_desc *d, const EpiParams &ep, cudaStream_t st, const ConvGeom &geo = ConvGeom{}) {
    if constexpr (OUT == kOutE4M3 && EPI != LCML_EPI_SILU_MUL && tab_bytes<BN, EPI, OUT, BKB>() > 0) {
        switch (fast_kind<BN, EPI, OUT, BKB>(d, ep)) {
            case 1: return launch_tc_kernel<BN, EPI, OUT, IM2COL, BKB, 1>(d, ep, st, geo);
            case 2: return launch_tc_kernel<BN, EPI, OUT, IM2COL, BKB, 2>(d, ep, st, geo);
            default: break;
        }
    }
    return launch_tc_kernel<BN, EPI, OUT, IM2COL, BKB, 0>(d, ep, st, geo);
}

template <int EPI, int OUT>
int launch_tc2(const lcml_fp8_gemm_desc *d, const EpiParams &ep, cudaStream_t st) {
    constexpr int STAGES = pair_stages_for<EPI, OUT>();
    using L = PairLayout<STAGES, EPI, OUT>;
    static_assert(STAGES >= 3 && L::kSmemBytes <= kSmemLimit, "shared memory layout does not fit");
    auto kern = k_gemm_fp8_tc2<STAGES, EPI, OUT>;
    if (const int rc = ensure_max_smem(reinterpret_cast<const void *>(kern), L::kSmemBytes, "gemm_fp8_tc2")) return rc;
    CUtensorMap ta, tb, tb2;
    int rc = make_tmap(&ta, d->A, d->K, d->M, d->lda, 128);
    if (rc) return rc;
    rc = make_tmap(&tb, d->B, d->K, d->N, d->ldb, 128);
    if (rc) return rc;
    const int64_t tiles = ((d->M + 255) / 256) * ((d->N + 255) / 256);
    const int64_t pairs = sm_count() / 2;
    const int n_split = split_tiles(tiles, pairs, EPI == LCML_EPI_SILU_MUL);
    if (n_split > 0) {
        rc = make_tmap(&tb2, d->B, d->K, d->N, d->ldb, 64);
        if (rc) return rc;
    } else {
        tb2 = tb;  // not read
    }
    CUtensorMap ty;
    rc = output_tmap<EPI, OUT>(d, ep, &ty);
    if (rc) return rc;
    const int64_t items = tiles + n_split;
    const int grid = static_cast<int>(2 * (items < pairs ? items : pairs));
    return launch_gemm_kernel(kern, static_cast<unsigned>(grid), threads_for<EPI>(), L::kSmemBytes, st, 0,
                              "gemm_fp8_tc2", ta, tb, tb2, ty, static_cast<int>(d->M), static_cast<int>(d->N),
                              static_cast<int>(d->K), n_split, ep, device_error_word());
}

// Split factor for a GEMM whose 128 x 128 tiles would leave most SMs idle:
// S CTAs per tile (S <= 8, at least two K-blocks each, S x tiles <= SMs);
// 0 when split-K does not apply. Only GEMMs with one row of tiles (M <= 128)
// split unless `any_m`: the partials cross distributed shared memory at a few
// tens of GB/s per SM, so once M spans two or more row tiles, one CTA per
// tile over the whole K is faster (1024^3: 12.5 vs 15.6 us; 256 x 1024 x
// 1024: 11.8 vs 14.1 us on B200).
int splitk_factor(const lcml_fp8_gemm_desc *d, const EpiParams &ep, bool any_m) {
    if (d->epilogue == LCML_EPI_SILU_MUL || ep.y_num_peers > 0 || d->M > 0x7fffffff || d->N > 0x7fffffff ||
        d->K > 0x7fffffff || (!any_m && d->M > BM))
        return 0;
    const int64_t tiles = ((d->M + BM - 1) / BM) * ((d->N + kSplitBN - 1) / kSplitBN);
    const int64_t kblocks = (d->K + BK - 1) / BK;
    const int64_t sms = sm_count();
    if (2 * tiles > sms || kblocks < 4) return 0;
    int64_t s = sms / tiles;
    if (s > kSplitMax) s = kSplitMax;
    if (s > kblocks / 2) s = kblocks / 2;
    return s >= 2 ? static_cast<int>(s) : 0;
}

template <int EPI, int OUT>
int launch_splitk(const lcml_fp8_gemm_desc *d, const EpiParams &ep, cudaStream_t st, int splits) {
    using L = SplitLayout;
    static_assert(L::kSmemBytes <= kSmemLimit, "shared memory layout does not fit");
    auto kern = k_gemm_fp8_splitk<EPI, OUT>;
    if (const int rc = ensure_max_smem(reinterpret_cast<const void *>(kern), L::kSmemBytes, "gemm_fp8_splitk")) return rc;
    CUtensorMap ta, tb;
    int rc = make_tmap(&ta, d->A, d->K, d->M, d->lda, BM);
    if (rc) return rc;
    rc = make_tmap(&tb, d->B, d->K, d->N, d->ldb, kSplitBN);
    if (rc) return rc;
    const int64_t tiles = ((d->M + BM - 1) / BM) * ((d->N + kSplitBN - 1) / kSplitBN);
    return launch_gemm_kernel(kern, static_cast<unsigned>(tiles * splits), kSplitThreads, L::kSmemBytes, st,
                              static_cast<unsigned>(splits), "gemm_fp8_splitk", ta, tb, static_cast<int>(d->M),
                              static_cast<int>(d->N), static_cast<int>(d->K), splits, ep, device_error_word());
}

// Rows of A held per GEMV instantiation for an M <= kGemvMaxM GEMM (0: not a GEMV shape).
int gemv_rows(const lcml_fp8_gemm_desc *d, const EpiParams &ep) {
    if (d->M < 1 || d->M > kGemvMaxM || d->epilogue == LCML_EPI_SILU_MUL || ep.y_num_peers > 0) return 0;
    const int mr = d->M == 1 ? 1 : (d->M == 2 ? 2 : 4);
    return static_cast<int64_t>(mr) * d->K * 4 <= kGemvSmemMax ? mr : 0;
}

template <int MR, int EPI, int OUT, bool QA = false>
int launch_gemv(const lcml_fp8_gemm_desc *d, const EpiParams &ep, cudaStream_t st, const GemvQuantA &qa = {}) {
    constexpr int rows_per_cta = (kGemvThreads / 32) * kGemvRows;
    const int64_t want = (d->N + rows_per_cta - 1) / rows_per_cta;
    const int64_t cap = 4LL * sm_count();
    const int grid = static_cast<int>(want < cap ? want : cap);
    const size_t smem = static_cast<size_t>(MR) * static_cast<size_t>(d->K) * 4;
    return launch_gemm_kernel(k_gemv_fp8<MR, EPI, OUT, QA>, static_cast<unsigned>(grid), kGemvThreads, smem, st, 0,
                              QA ? "gemv_fp8_quantize_a" : "gemv_fp8", d->A, d->lda, d->B, d->ldb,
                              static_cast<int>(d->M), static_cast<int>(d->N), static_cast<int>(d->K), ep, qa);
}

template <int EPI, int OUT>
int launch_simt(const lcml_fp8_gemm_desc *d, const EpiParams &ep, cudaStream_t st) {
    const int64_t n_out = (EPI == LCML_EPI_SILU_MUL) ? d->N / 2 : d->N;
    dim3 grid(static_cast<unsigned>((n_out + 63) / 64), static_cast<unsigned>((d->M + 63) / 64));
    if (grid.y > 65535) return set_error(LCML_ERR_UNSUPPORTED, "SIMT GEMM: M too large for the fallback grid");
    k_gemm_fp8_simt<EPI, OUT><<<grid, 256, 0, st>>>(d->A, d->lda, d->B, d->ldb, d->b_kmajor, d->M, d->N, d->K, ep);
    LCML_LAUNCHED("gemm_fp8_simt");
    return LCML_OK;
}

// 128 x 256 single-CTA tiles instead of 128 x 128 where they still give
// every SM two tiles or more: each epilogue warp then works through four
// chunks per tile instead of two, so the per-tile start-up (the first
// chunk's TMEM, factor and residual latency) is paid half as often. On the
// ResNet-50 1x1 convs (N = 256 / 512, epilogue-bound) this is 10-13 % faster.
bool wide_tiles(const lcml_fp8_gemm_desc *d) {
    const int64_t tiles256 = ((d->M + BM - 1) / BM) * ((d->N + 255) / 256);
    return d->N >= 256 && tiles256 >= 2 * static_cast<int64_t>(sm_count());
}

template <int EPI, int OUT>
int dispatch(const lcml_fp8_gemm_desc *d, const EpiParams &ep, cudaStream_t st, bool force_simt, const ConvGeom *geo,
             const GemvQuantA *qa) {
    if (qa) {  // fp32 A quantized inside the GEMV (the caller checked the GEMV conditions)
        if constexpr (EPI != LCML_EPI_SILU_MUL) {
            switch (gemv_rows(d, ep)) {
                case 1: return launch_gemv<1, EPI, OUT, true>(d, ep, st, *qa);
                case 2: return launch_gemv<2, EPI, OUT, true>(d, ep, st, *qa);
                case 4: return launch_gemv<4, EPI, OUT, true>(d, ep, st, *qa);
                default: break;
            }
        }
        return set_error(LCML_ERR_UNSUPPORTED, "fused A quantization: not a GEMV shape");
    }
    if (geo) {  // implicit-GEMM convolution: single-CTA tiles as wide as the output channels
        if constexpr (EPI == LCML_EPI_SILU_MUL) {
            return set_error(LCML_ERR_UNSUPPORTED, "implicit-GEMM convolution: SILU_MUL epilogue");
        } else {
            if (geo->C % 128 == 0) {
                if (d->N <= 64) return launch_tc<64, EPI, OUT, true, 128>(d, ep, st, *geo);
                if (d->N >= 2048 || wide_tiles(d)) return launch_tc<256, EPI, OUT, true, 128>(d, ep, st, *geo);
                return launch_tc<128, EPI, OUT, true, 128>(d, ep, st, *geo);
            }
            if (d->N <= 64) return launch_tc<64, EPI, OUT, true, 64>(d, ep, st, *geo);
            if (d->N >= 2048 || wide_tiles(d)) return launch_tc<256, EPI, OUT, true, 64>(d, ep, st, *geo);
            return launch_tc<128, EPI, OUT, true, 64>(d, ep, st, *geo);
        }
    }
    const bool tma_ok = !force_simt && d->b_kmajor && (d->K % 16 == 0) && (d->lda % 16 == 0) && (d->ldb % 16 == 0) &&
                        aligned(d->A, 16) && aligned(d->B, 16) && d->M <= 0x7fffffff && d->N <= 0x7fffffff &&
                        d->K <= 0x7fffffff;
    if (!tma_ok) return launch_simt<EPI, OUT>(d, ep, st);
    if constexpr (EPI != LCML_EPI_SILU_MUL) {
        const int mode = d->variant & 3;
        if (mode == 0) {  // decode-sized M: stream B once on the CUDA cores
            switch (gemv_rows(d, ep)) {
                case 1: return launch_gemv<1, EPI, OUT>(d, ep, st);
                case 2: return launch_gemv<2, EPI, OUT>(d, ep, st);
                case 4: return launch_gemv<4, EPI, OUT>(d, ep, st);
                default: break;
            }
        }
        const int splits = (mode == 0 || mode == 3) ? splitk_factor(d, ep, mode == 3) : 0;
        if (splits) return launch_splitk<EPI, OUT>(d, ep, st, splits);
    }
    // CTA pairs (256 x 256 tiles, half the staged bytes per MMA) pay off once
    // the mainloop is long: K >= 1024 with a tile for every SM, K >= 2048 with
    // a tile for every pair, K >= 4096 with a tile for every other pair (B200,
    // warm L2: 1024 x 8192 x 8192 49.9 vs 61.9 us single-CTA, 512 x 8192 x
    // 8192 27.9 vs 35.6, 3072^3 22.3 vs 23.2; but 2048^3, 64 tiles of K =
    // 2048, 12.8 vs 11.4, and ResNet-50's 1024 -> 256 1x1 convs, 98 tiles of
    // K = 1024, slower as pairs). Short-K and narrow GEMMs are epilogue-bound
    // and run single-CTA tiles as wide as N.
    const int64_t pair_tiles = ((d->M + 255) / 256) * ((d->N + 255) / 256);
    const int64_t pairs = sm_count() / 2;
    const bool pair = d->M >= 256 && d->N >= 256 && d->K >= 1024 &&
                      (pair_tiles >= 2 * pairs || (d->K >= 2048 && pair_tiles >= pairs) ||
                       (d->K >= 4096 && 2 * pair_tiles >= pairs));
    if ((d->variant & 3) != 1 && ((d->variant & 3) == 2 || pair)) return launch_tc2<EPI, OUT>(d, ep, st);
    if (EPI == LCML_EPI_SILU_MUL || d->N >= 2048 || wide_tiles(d)) return launch_tc<256, EPI, OUT>(d, ep, st);
    if (EPI != LCML_EPI_SILU_MUL && d->N <= 64) return launch_tc<64, EPI, OUT>(d, ep, st);
    return launch_tc<128, EPI, OUT>(d, ep, st);
}

template <int EPI>
int dispatch_out(const lcml_fp8_gemm_desc *d, const EpiParams &ep, cudaStream_t st, bool force_simt,
                 const ConvGeom *geo, const GemvQuantA *qa) {
    switch (d->y_dtype) {
        case LCML_DTYPE_FLOAT: return dispatch<EPI, kOutF32>(d, ep, st, force_simt, geo, qa);
        case LCML_DTYPE_BFLOAT16: return dispatch<EPI, kOutBF16>(d, ep, st, force_simt, geo, qa);
        case LCML_DTYPE_FLOAT8E4M3FN: return dispatch<EPI, kOutE4M3>(d, ep, st, force_simt, geo, qa);
        default: return set_error(LCML_ERR_INVALID_ARGUMENT, "lcml_fp8_gemm: y_dtype %d unsupported", d->y_dtype);
    }
}

int gemm_entry(const lcml_fp8_gemm_desc *d, lcml_stream_t stream, bool force_simt, const ConvGeom *geo = nullptr,
               const GemvQuantA *qa = nullptr) {
    LCML_CHECK_ARG(d != nullptr, "lcml_fp8_gemm: desc is NULL");
    LCML_CHECK_ARG(d->M >= 0 && d->N >= 0 && d->K >= 0, "lcml_fp8_gemm: negative extent");
    LCML_CHECK_ARG(d->epilogue >= LCML_EPI_NONE && d->epilogue <= LCML_EPI_SILU_MUL,
                   "lcml_fp8_gemm: epilogue %d unknown", d->epilogue);
    if (d->epilogue == LCML_EPI_SILU_MUL)
        LCML_CHECK_ARG(d->N % 256 == 0, "lcml_fp8_gemm: SILU_MUL needs N (gate+up) to be a multiple of 256, got %lld",
                       (long long)d->N);
    if (d->M == 0 || d->N == 0) return LCML_OK;
    LCML_CHECK_ARG((d->A || geo || qa) && d->B && d->Y && d->scale_a && d->scale_b, "lcml_fp8_gemm: null operand");
    LCML_CHECK_ARG(geo || qa || d->lda >= d->K, "lcml_fp8_gemm: lda < K");
    LCML_CHECK_ARG(d->b_kmajor ? d->ldb >= d->K : d->ldb >= d->N, "lcml_fp8_gemm: ldb too small");
    const int64_t n_out = d->epilogue == LCML_EPI_SILU_MUL ? d->N / 2 : d->N;
    LCML_CHECK_ARG(d->y_col_offset >= 0 && d->ldy >= n_out + d->y_col_offset, "lcml_fp8_gemm: ldy < y_col_offset + output columns");
    LCML_CHECK_ARG(d->y_num_peers >= 0 && (d->y_num_peers == 0 || d->y_peers), "lcml_fp8_gemm: y_peers missing");
    LCML_CHECK_ARG(d->scale_a_mode == LCML_SCALE_TENSOR || d->scale_a_mode == LCML_SCALE_ROW,
                   "lcml_fp8_gemm: scale_a_mode must be TENSOR or ROW");
    LCML_CHECK_ARG(d->scale_b_mode == LCML_SCALE_TENSOR || d->scale_b_mode == LCML_SCALE_COL,
                   "lcml_fp8_gemm: scale_b_mode must be TENSOR or COL");
    LCML_CHECK_ARG(d->y_dtype != LCML_DTYPE_FLOAT8E4M3FN || d->y_scale, "lcml_fp8_gemm: e4m3 output needs y_scale");
    LCML_CHECK_ARG(!d->c_mat || d->c_mat_dtype == LCML_DTYPE_FLOAT || d->c_mat_dtype == LCML_DTYPE_BFLOAT16 ||
                       (d->c_mat_dtype == LCML_DTYPE_FLOAT8E4M3FN && d->c_mat_scale),
                   "lcml_fp8_gemm: c_mat dtype must be FLOAT, BFLOAT16 or FLOAT8E4M3FN with c_mat_scale");
    LCML_CHECK_ARG(!d->c_vec || (d->c_vec_mode >= 0 && d->c_vec_mode <= 2), "lcml_fp8_gemm: bad c_vec_mode");
    LCML_CHECK_ARG(d->variant >= 0 && d->variant <= 7, "lcml_fp8_gemm: variant %d unknown", d->variant);
    EpiParams ep;
    ep.M = d->M;
    ep.N = d->N;
    ep.sa = d->scale_a;
    ep.sa_row = d->scale_a_mode == LCML_SCALE_ROW;
    ep.sb = d->scale_b;
    ep.sb_col = d->scale_b_mode == LCML_SCALE_COL;
    ep.alpha = d->alpha;
    ep.beta = d->beta;
    ep.c_vec = d->c_vec;
    // external modes TENSOR(0)/ROW(1)/COL(2) -> internal 1/2/3, 0 = none
    ep.c_vec_mode = d->c_vec ? (d->c_vec_mode == LCML_SCALE_TENSOR ? 1 : (d->c_vec_mode == LCML_SCALE_ROW ? 2 : 3)) : 0;
    ep.c_mat = d->c_mat;
    ep.c_mat_kind = d->c_mat_dtype == LCML_DTYPE_BFLOAT16 ? 1 : (d->c_mat_dtype == LCML_DTYPE_FLOAT8E4M3FN ? 2 : 0);
    ep.c_mat_scale = d->c_mat_scale;
    ep.ldc = d->ldc;
    ep.y = d->Y;
    ep.ldy = d->ldy;
    ep.y_scale = d->y_scale;
    ep.row_amax = d->row_amax;
    ep.y_col_offset = d->y_col_offset;
    ep.y_peers = d->y_peers;
    ep.y_num_peers = d->y_num_peers;
    {
        const int es = d->y_dtype == LCML_DTYPE_FLOAT ? 4 : (d->y_dtype == LCML_DTYPE_BFLOAT16 ? 2 : 1);
        ep.tma_store = !(d->variant & 4) && d->y_num_peers == 0 && n_out <= 0x7fffffff && d->M <= 0x7fffffff &&
                       aligned(static_cast<const uint8_t *>(d->Y) + d->y_col_offset * es, 16) &&
                       (d->ldy * es) % 16 == 0;
    }
    cudaStream_t st = to_cuda(stream);
    switch (d->epilogue) {
        case LCML_EPI_NONE: return dispatch_out<LCML_EPI_NONE>(d, ep, st, force_simt, geo, qa);
        case LCML_EPI_RELU: return dispatch_out<LCML_EPI_RELU>(d, ep, st, force_simt, geo, qa);
        default: return dispatch_out<LCML_EPI_SILU_MUL>(d, ep, st, force_simt, geo, qa);
    }
}

}// namespace gemm

int fp8_gemm_implicit_conv(const lcml_fp8_gemm_desc *d, const ConvGeom &geo, cudaStream_t st) {
    LCML_CHECK_ARG(d && d->b_kmajor && d->K % 16 == 0 && d->ldb % 16 == 0 && aligned(d->B, 16),
                   "implicit-GEMM convolution: packed weights must be K-major with 16-byte rows");
    LCML_CHECK_ARG(geo.x && aligned(geo.x, 16) && geo.C % 64 == 0 && geo.ktaps == geo.kH * geo.kW * geo.C &&
                       d->K == geo.ktaps && d->M == static_cast<int64_t>(geo.N) * geo.oH * geo.oW,
                   "implicit-GEMM convolution: inconsistent geometry");
    return gemm::gemm_entry(d, reinterpret_cast<lcml_stream_t>(st), false, &geo);
}

}// namespace lcml

extern "C" {

int lcml_fp8_gemm(const lcml_fp8_gemm_desc *desc, lcml_stream_t stream) {
    return lcml::gemm::gemm_entry(desc, stream, false);
}

int lcml_fp8_gemm_rowquant(const lcml_fp8_gemm_desc *desc, uint8_t *q, float *q_scale, float *workspace,
                           lcml_stream_t stream) {
    LCML_CHECK_ARG(desc != nullptr, "lcml_fp8_gemm_rowquant: desc is NULL");
    LCML_CHECK_ARG(desc->y_dtype == LCML_DTYPE_FLOAT, "lcml_fp8_gemm_rowquant: Y must be fp32");
    LCML_CHECK_ARG(desc->row_amax == nullptr, "lcml_fp8_gemm_rowquant: desc->row_amax must be NULL");
    const int64_t n_out = desc->epilogue == LCML_EPI_SILU_MUL ? desc->N / 2 : desc->N;
    LCML_CHECK_ARG(desc->ldy == n_out, "lcml_fp8_gemm_rowquant: Y must be dense (ldy == %lld)", (long long)n_out);
    if (desc->M == 0 || n_out == 0) return LCML_OK;
    LCML_CHECK_ARG(q && q_scale && workspace, "lcml_fp8_gemm_rowquant: null q / q_scale / workspace");
    cudaStream_t st = lcml::to_cuda(stream);
    LCML_CUDA(cudaMemsetAsync(workspace, 0, sizeof(float) * static_cast<size_t>(desc->M), st));
    lcml_fp8_gemm_desc d = *desc;
    d.row_amax = workspace;
    int rc = lcml::gemm::gemm_entry(&d, stream, false);
    if (rc != LCML_OK) return rc;
    return lcml_fp8_quantize_from_amax(static_cast<const float *>(d.Y), 1, d.M, n_out, workspace, q_scale, q, stream);
}

int lcml_fp8_gemm_quantize_a(const lcml_fp8_gemm_desc *desc, const float *a, int64_t lda, uint8_t *aq,
                             float *scale_a_out, float *workspace, lcml_stream_t stream) {
    LCML_CHECK_ARG(desc != nullptr, "lcml_fp8_gemm_quantize_a: desc is NULL");
    LCML_CHECK_ARG(desc->M >= 0 && desc->K >= 0 && lda >= desc->K, "lcml_fp8_gemm_quantize_a: bad extents / lda");
    if (desc->M == 0 || desc->N == 0) return LCML_OK;
    LCML_CHECK_ARG(a && scale_a_out, "lcml_fp8_gemm_quantize_a: null a / scale_a_out");
    lcml_fp8_gemm_desc d = *desc;
    d.A = aq;
    d.lda = desc->K;
    d.scale_a = scale_a_out;
    d.scale_a_mode = LCML_SCALE_TENSOR;
    // one fused kernel for decode-sized M on the GEMV path (its conditions as in dispatch: automatic kernel
    // choice, K-major 16-byte B rows, A rows of whole float4s)
    const bool fused = d.variant == 0 && d.M <= lcml::gemm::kGemvMaxM && d.epilogue != LCML_EPI_SILU_MUL &&
                       d.y_num_peers == 0 && d.b_kmajor && d.K % 16 == 0 && d.ldb % 16 == 0 && d.B &&
                       lcml::aligned(d.B, 16) && lda % 4 == 0 && lcml::aligned(a, 16) &&
                       static_cast<int64_t>(d.M == 1 ? 1 : (d.M == 2 ? 2 : 4)) * d.K * 4 <= lcml::gemm::kGemvSmemMax &&
                       d.N <= 0x7fffffff && d.K <= 0x7fffffff;
    if (fused) {
        const lcml::gemm::GemvQuantA qa{a, lda, scale_a_out, aq};
        return lcml::gemm::gemm_entry(&d, stream, false, nullptr, &qa);
    }
    LCML_CHECK_ARG(aq && workspace, "lcml_fp8_gemm_quantize_a: this shape needs aq and workspace");
    LCML_CHECK_ARG(lda == desc->K, "lcml_fp8_gemm_quantize_a: this shape needs a dense A (lda == K)");
    const int rc = lcml_fp8_quantize_tensor_dynamic(a, desc->M * desc->K, scale_a_out, aq, workspace, stream);
    if (rc != LCML_OK) return rc;
    return lcml::gemm::gemm_entry(&d, stream, false);
}

// Test hook (not in the public header): the SIMT kernel on the same
// descriptor, so tests can cross-check it against the tensor-core kernels.
int lcml_fp8_gemm_simt(const lcml_fp8_gemm_desc *desc, lcml_stream_t stream) {
    return lcml::gemm::gemm_entry(desc, stream, true);
}

}// extern "C"
