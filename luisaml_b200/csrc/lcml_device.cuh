// Device-side building blocks shared by every kernel of the FP8 operator path:
// the bit-exact e4m3 codec, bounded mbarrier waits, TMA and tcgen05 wrappers.
// sm_100a only.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace lcml {

// ---------------------------------------------------------------------------
// Device error word. A kernel that gives up on a bounded wait records the
// reason here and returns; the host reads and clears it via
// lcml_device_error(). Nothing in this library traps.
// ---------------------------------------------------------------------------
enum DeviceError : int {
    kDevOk = 0,
    kDevTimeoutProducer = 1,   // TMA producer waited too long for a free stage
    kDevTimeoutMma = 2,        // MMA issuer waited too long for a loaded stage
    kDevTimeoutEpilogue = 3,   // epilogue waited too long for an accumulator
    kDevTimeoutDrain = 4,      // final drain of in-flight copies timed out
    kDevTimeoutPeer = 5,       // a peer rank's slot did not reach the expected epoch in time
};

// The word lives in runtime.cu; kernels receive its device address as a
// parameter (lcml::device_error_word()), so no relocatable device code is needed.
__device__ __forceinline__ void record_device_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// ~2 s at the B200's 1.965 GHz boost clock: far above any legitimate wait in
// this library (the largest GEMM runs well under 100 ms).
constexpr long long kWaitLimitCycles = 4000000000LL;

// ---------------------------------------------------------------------------
// e4m3 codec (FP8 E4M3FN), bit-exact with the reference's CPU codec
// FP8E4M3FN::from_float / to_float (include/onnx/fp_quantized.h:149-249):
//   NaN -> 0x7f; +-0 -> 0x00; |v| > 448 (inf included) -> +-448;
//   round-to-nearest-even; a nonzero value that rounds to zero keeps its sign.
// Integer-only for normal results: adding 0x7ffff plus the lowest kept bit and
// shifting by 20 is RNE on 3 mantissa bits, and a carry moves into the
// exponent field by itself. Subnormal results are RNE(|v| * 2^9) in [0, 8],
// where 8 is exactly the smallest normal code 0x08.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e4m3_encode(float v) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t sign = (u >> 24) & 0x80u;
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return 0x7fu;              // NaN
    if (a == 0u) return 0u;                         // +-0 -> 0x00
    if (a > 0x43e00000u) return sign | 0x7eu;       // > 448 saturates
    uint32_t r;
    if (a >= 0x3c800000u) {                         // >= 2^-6: normal result
        r = ((a + 0x7ffffu + ((a >> 20) & 1u)) >> 20) - (120u << 3);
    } else {                                        // subnormal or zero result
        r = __float2uint_rn(__uint_as_float(a) * 512.0f);
    }
    return sign | r;
}

__device__ __forceinline__ float e4m3_decode(uint32_t b) {
    const uint32_t sign = (b & 0x80u) << 24;
    const uint32_t e = (b >> 3) & 0xfu;
    const uint32_t m = b & 0x7u;
    if ((b & 0x7fu) == 0x7fu) return __uint_as_float(0x7fc00000u);
    float v = (e == 0u) ? float(m) * 0.001953125f : __uint_as_float(((e + 120u) << 23) | (m << 20));
    return __uint_as_float(__float_as_uint(v) | sign);
}

// ---------------------------------------------------------------------------
// e5m2 (FP8 E5M2) and e2m1 (FP4 E2M1) codecs, bit-exact with the reference's
// FP8E5M2::from_float / to_float (include/onnx/fp_quantized.h:259-378) and
// FP4E2M1::from_float / to_float (:20-115), by the same integer RNE as
// e4m3_encode (round constant + lowest kept bit, shift; carries move into the
// exponent field) with each format's own edges:
//   e5m2: NaN -> 0x7f; +-0 -> 0x00; |v| > 57344 (inf included) -> +-inf
//         (0x7c / 0xfc: the reference does not saturate); subnormal grid 2^-16.
//   e2m1: +-0 -> 0x0; |v| > 6 (inf included) -> +-6 (0x7 / 0xf); subnormal
//         grid 0.5. NaN -> 0x0: the reference's encoder has no NaN case (the
//         value reaches a float -> uint8 conversion of NaN, which is undefined
//         in C++); 0x0 is what its x86-64 build returns.
// A nonzero value that rounds to zero keeps its sign in both (0x80 / 0x8).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e5m2_encode(float v) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t sign = (u >> 24) & 0x80u;
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return 0x7fu;              // NaN
    if (a == 0u) return 0u;                         // +-0 -> 0x00
    if (a > 0x47600000u) return sign | 0x7cu;       // > 57344 -> inf
    uint32_t r;
    if (a >= 0x38800000u) {                         // >= 2^-14: normal result
        r = ((a + 0xfffffu + ((a >> 21) & 1u)) >> 21) - (112u << 2);
    } else {                                        // RNE(|v| * 2^16) in [0, 4]; 4 is the smallest normal 0x04
        r = __float2uint_rn(__uint_as_float(a) * 65536.0f);
    }
    return sign | r;
}

// e5m2 is the high byte of an IEEE half: the decode is exact through f16.
// NaN codes give the canonical quiet NaN, as the reference's to_float does.
__device__ __forceinline__ float e5m2_decode(uint32_t b) {
    if ((b & 0x7cu) == 0x7cu && (b & 0x3u) != 0u) return __uint_as_float(0x7fc00000u);
    return __half2float(__ushort_as_half(static_cast<unsigned short>((b & 0xffu) << 8)));
}

__device__ __forceinline__ uint32_t e2m1_encode(float v) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u || a == 0u) return 0u;      // NaN, +-0
    const uint32_t sign = (u >> 28) & 0x8u;
    if (a > 0x40c00000u) return sign | 0x7u;        // > 6 saturates
    uint32_t r;
    if (a >= 0x3f800000u) {                         // >= 1: normal result
        r = ((a + 0x1fffffu + ((a >> 22) & 1u)) >> 22) - (126u << 1);
    } else {                                        // RNE(|v| * 2) in [0, 2]; 2 is the smallest normal 0x2
        r = __float2uint_rn(__uint_as_float(a) * 2.0f);
    }
    return sign | r;
}

__device__ __forceinline__ float e2m1_decode(uint32_t b) {
    // magnitudes of codes 0..7: 0, 0.5, 1, 1.5, 2, 3, 4, 6 (bias 1, one mantissa bit)
    const uint32_t m = b & 0x7u;
    const float mag = m < 2u ? 0.5f * static_cast<float>(m)
                             : __uint_as_float(((m >> 1) + 126u) << 23 | (m & 1u) << 22);
    return __uint_as_float(__float_as_uint(mag) | ((b & 0x8u) << 28));
}

// QuantizeLinear of one element: e4m3(x / s) with an IEEE round-to-nearest divide.
__device__ __forceinline__ uint32_t quantize1(float x, float s) {
    return e4m3_encode(__fdiv_rn(x, s));
}

// Fast QuantizeLinear of two elements, bit-identical to quantize1():
// q = x * r with r = RN(1/s) is within 2.5 fp32 ulps of RN(x / s). Every e4m3
// rounding boundary in the normal range (a midpoint between neighbouring e4m3
// values, incl. the binade steps) has low 20 mantissa bits 0x80000; in the
// subnormal range (|q| < 2^-6, grid 2^-9) the boundaries (2k+1) * 2^-10 have
// low 20 bits 0. So whenever q is finite and its low 20 bits are more than 3
// ulps away from the boundary pattern of its range, q and x / s round to the
// same e4m3 value, which the hardware cvt.rn.satfinite (RNE, |v| > 448 ->
// +-448, tiny values to a signed zero) produces. An exact +-0 input is 0x00
// (x / s is +-0 for a usable scale and the codec drops the sign of zero),
// which matters because Relu outputs are often half zeros. All other cases
// (NaN/inf, near-boundaries, a product that underflowed to zero, unusual
// scales) take the exact divide + integer encoder. `s_ok` says r is usable
// (s normal positive, r finite normal).
__device__ __forceinline__ bool needs_exact(float q, float x) {
    const uint32_t a = __float_as_uint(q) & 0x7fffffffu;
    const bool normal = a >= 0x3c800000u;
    const uint32_t d = normal ? (a & 0xfffffu) - 0x7fffdu : (a + 3u) & 0xfffffu;
    return (a >= 0x7f800000u) | ((d <= 6u) & (normal | (x != 0.0f)));
}

__device__ __forceinline__ uint32_t quantize2_fast(float x0, float x1, float s, float r, bool s_ok) {
    const float q0 = x0 * r, q1 = x1 * r;
    uint32_t out;
    asm("{\n\t.reg .b16 t;\n\t"
        "cvt.rn.satfinite.e4m3x2.f32 t, %2, %1;\n\t"
        "cvt.u32.u16 %0, t;\n\t}"
        : "=r"(out)
        : "f"(q0), "f"(q1));
    if (x0 == 0.0f) out &= 0xff00u;  // -0 -> 0x00
    if (x1 == 0.0f) out &= 0x00ffu;
    if (!s_ok || needs_exact(q0, x0) || needs_exact(q1, x1)) out = quantize1(x0, s) | (quantize1(x1, s) << 8);
    return out;
}

// Two e4m3 codes (low byte, high byte of `b`) -> floats, exactly as
// e4m3_decode: every e4m3 value, -0 and NaN included, is representable in
// f16, so the hardware conversion through f16x2 is exact.
__device__ __forceinline__ void e4m3x2_decode(uint32_t b, float &lo, float &hi) {
    asm("{\n\t.reg .b16 t, h0, h1;\n\t"
        "cvt.u16.u32 t, %2;\n\t"
        "{\n\t.reg .b32 p;\n\t"
        "cvt.rn.f16x2.e4m3x2 p, t;\n\t"
        "mov.b32 {h0, h1}, p;\n\t}\n\t"
        "cvt.f32.f16 %0, h0;\n\t"
        "cvt.f32.f16 %1, h1;\n\t}"
        : "=f"(lo), "=f"(hi)
        : "r"(b));
}

// Hardware conversion of two values to e4m3 (RNE, saturating), low byte from
// `lo`; no QuantizeLinear corner cases handled (see quantize2_fast).
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
    uint32_t out;
    asm("{\n\t.reg .b16 t;\n\t"
        "cvt.rn.satfinite.e4m3x2.f32 t, %2, %1;\n\t"
        "cvt.u32.u16 %0, t;\n\t}"
        : "=r"(out)
        : "f"(lo), "f"(hi));
    return out;
}

__device__ __forceinline__ bool scale_fast_ok(float s, float r) {
    return s >= 1.17549435e-38f && s < 3.0e38f && r >= 1.17549435e-38f && r < 3.0e38f;
}

// Branch-free QuantizeLinear of N values (N a multiple of 4) into N / 4
// little-endian words, bit-identical to quantize1. With r = RN(1/s),
// r_lo = RN(r (1 - 2^-21)) < 1/s < r_hi = RN(r (1 + 2^-21)), so for every v
// the real v/s lies between v·r_lo and v·r_hi, and RN (monotone) keeps
// RN(v/s) between RN(v·r_lo) and RN(v·r_hi). The hardware conversion
// cvt.rn.satfinite.e4m3x2.f32 is monotone too, so where the codes of the two
// bounds agree they are the code of RN(v/s) (saturation at 448 included).
// The fma with a +0 addend turns v = -0 into +0, which the codec writes as
// 0x00. One flag per block collects disagreeing bounds, NaN codes (the
// hardware may write 0xff where the codec writes 0x7f) and 0x80 codes (a
// quotient that rounds to -0 in fp32 is 0x00 for the codec); if it is set,
// the whole block takes the exact divide + integer encoder.
template <int N>
__device__ __forceinline__ void quantize_block_fast(const float *v, float s, float r, bool s_ok, uint32_t *w) {
    const float r_lo = r * 0.99999952316284180f;  // 1 - 2^-21
    const float r_hi = r * 1.00000047683715820f;  // 1 + 2^-21
    bool exact = !s_ok;
#pragma unroll
    for (int j = 0; j < N / 4; ++j) {
        float lo[4], hi[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            lo[k] = fmaf(v[4 * j + k], r_lo, 0.0f);
            hi[k] = fmaf(v[4 * j + k], r_hi, 0.0f);
        }
        const uint32_t wl = cvt_e4m3x2(lo[0], lo[1]) | (cvt_e4m3x2(lo[2], lo[3]) << 16);
        const uint32_t wh = cvt_e4m3x2(hi[0], hi[1]) | (cvt_e4m3x2(hi[2], hi[3]) << 16);
        exact |= (wl != wh) | (__vcmpeq4(wl | 0x80808080u, 0xffffffffu) != 0u) | (__vcmpeq4(wl, 0x80808080u) != 0u);
        w[j] = wl;
    }
    if (exact) {  // unrolled: a runtime index would move v and w to local memory
#pragma unroll
        for (int j = 0; j < N / 4; ++j)
            w[j] = quantize1(v[4 * j], s) | (quantize1(v[4 * j + 1], s) << 8) | (quantize1(v[4 * j + 2], s) << 16) |
                   (quantize1(v[4 * j + 3], s) << 24);
    }
}

// ---------------------------------------------------------------------------
// Packed fp32 pair arithmetic (sm_100 fma/mul .rn.f32x2: one instruction for
// two lanes, each lane rounded exactly like fmaf / __fmul_rn; subnormals kept).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fma2(float &d0, float &d1, float a0, float a1, float b0, float b1, float c0, float c1) {
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__device__ __forceinline__ void mul2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\t"
        "mov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\t"
        "mov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Hardware conversion of two values to e4m3 with Relu folded in (negative
// values become +0; RNE, saturating). NaN stays NaN (0x7f / 0xff), unlike
// fmaxf(NaN, 0) = 0: callers that need Relu's NaN -> 0 check for NaN codes.
__device__ __forceinline__ uint32_t cvt_e4m3x2_relu(float lo, float hi) {
    uint32_t out;
    asm("{\n\t.reg .b16 t;\n\t"
        "cvt.rn.satfinite.relu.e4m3x2.f32 t, %2, %1;\n\t"
        "cvt.u32.u16 %0, t;\n\t}"
        : "=r"(out)
        : "f"(lo), "f"(hi));
    return out;
}

// Bytes 0x80 and 0xff of four hardware-converted codes (bit 7 set in the
// result's byte): a = x & 0x7f7f7f7f; (a + 0x7f) sets bit 7 of a byte exactly
// when it is nonzero, (a + 1) exactly when it is 0x7f (no carry crosses a
// byte); the sign bit of x selects the negative ones.
__device__ __forceinline__ uint32_t e4m3_odd_bytes(uint32_t x) {
    const uint32_t a = x & 0x7f7f7f7fu;
    return (~((a + 0x7f7f7f7fu) | a) | (a + 0x01010101u)) & x & 0x80808080u;
}

// One value by the epilogue quantization rule below: the codec applied to
// the fp32 product q = RN(v * r) (+-0 -> 0x00, NaN -> 0x7f, else the RNE
// saturating conversion, which equals the codec on every other q).
__device__ __forceinline__ uint32_t quantize_rcp1(float v, float r) {
    const float q = __fmul_rn(v, r);
    if (q == 0.0f) return 0u;
    if (q != q) return 0x7fu;
    return cvt_e4m3x2(q, 0.0f) & 0xffu;
}

// Output quantization of the fused GEMM / conv epilogues: the codec applied
// to q = RN(v * r), r = RN(1 / y_scale). It equals QuantizeLinear of the
// epilogue's fp32 value v (RN(v / s), quantize1) except where v / s lies
// within 2.5 fp32 ulps of an e4m3 rounding boundary: the same order of
// difference as the fp32 accumulation order of the GEMM itself, whose outputs
// match the reference within a tolerance. The hardware conversion gives the
// codec's byte except for q = -0 (0x80 where the codec writes 0x00) and NaN
// (possibly 0xff where the codec writes 0x7f); a block holding either byte is
// redone element by element (both are rare: -0 needs v = -0 or an underflow).
// Used only when r is a normal float (scale_fast_ok); QuantizeLinear proper
// (quantize.cu) stays bit-exact.
// NONNEG: the values are known to be >= +0 or -0 (Relu outputs; fmaxf never
// returns NaN for a non-NaN bound), so the only possible odd byte is 0x80 and
// any set sign bit flags the block.
// RELU: v has not been through Relu yet; the rule is applied to Relu(v)
// (fmaxf(v, 0), so NaN -> 0), with Relu folded into the conversion
// (cvt ... .relu: q < 0 -> +0, and r > 0 keeps the sign of v): its only odd
// outputs are NaN codes (where Relu(v) = 0) and a possible 0x80, both flagged.
template <int N, bool NONNEG = false, bool RELU = false>
__device__ __forceinline__ void quantize_block_rcp(const float *v, float r, uint32_t *w) {
    uint32_t odd = 0;
#pragma unroll
    for (int j = 0; j < N / 4; ++j) {
        float q[4];
        mul2(q[0], q[1], v[4 * j], v[4 * j + 1], r, r);
        mul2(q[2], q[3], v[4 * j + 2], v[4 * j + 3], r, r);
        if (RELU) {
            w[j] = cvt_e4m3x2_relu(q[0], q[1]) | (cvt_e4m3x2_relu(q[2], q[3]) << 16);
            // bit 7 of a byte: a sign (0x80) or, after adding 1 to the low 7 bits, a NaN code (0x7f)
            odd |= w[j] | ((w[j] & 0x7f7f7f7fu) + 0x01010101u);
        } else {
            w[j] = cvt_e4m3x2(q[0], q[1]) | (cvt_e4m3x2(q[2], q[3]) << 16);
            odd |= NONNEG ? w[j] : e4m3_odd_bytes(w[j]);
        }
    }
    if (NONNEG || RELU) odd &= 0x80808080u;
    if (odd) {  // unrolled: a runtime index would move v and w to local memory
#pragma unroll
        for (int j = 0; j < N / 4; ++j) {
            float x[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) x[k] = RELU ? fmaxf(v[4 * j + k], 0.0f) : v[4 * j + k];
            w[j] = quantize_rcp1(x[0], r) | (quantize_rcp1(x[1], r) << 8) | (quantize_rcp1(x[2], r) << 16) |
                   (quantize_rcp1(x[3], r) << 24);
        }
    }
}

// amax -> scale for every dynamic mode: amax / 448, or 1 when amax is 0.
__device__ __forceinline__ float scale_from_amax(float amax) {
    return amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
}

// |x| as an integer that orders like the float; NaN maps to 0 (ignored).
__device__ __forceinline__ uint32_t abs_bits_nan0(float x) {
    uint32_t a = __float_as_uint(x) & 0x7fffffffu;
    return a > 0x7f800000u ? 0u : a;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch. The GEMM kernels are launched with
// programmatic stream serialization: their CTAs may be scheduled while the
// previous kernel on the stream is still running, run their set-up (barrier
// init, TMEM allocation, tensor-map prefetch) and then block in
// griddep_wait() until that kernel has completed and its memory writes are
// visible; nothing written by an earlier kernel is read before the wait.
// Producer kernels call griddep_launch_dependents() to let that happen as
// early as they like (without the call the dependent starts when the
// producer's last CTA exits). Both are no-ops for a kernel launched without
// the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Shared memory / mbarrier helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0u;
}

// Bounded wait for the phase with the given parity to complete. Returns false
// (and records `err` in *err_word) after kWaitLimitCycles instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err_word, int err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitLimitCycles) {
            record_device_error(err_word, err);
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(const void *tmap, uint64_t *bar, void *smem_dst, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// CTA-pair form: the copy lands in this CTA's shared memory but completes
// (complete_tx) on `bar_cluster`, a shared::cluster address that may name the
// peer CTA's mbarrier (used by the 2-SM GEMM to signal the leader's barrier).
__device__ __forceinline__ void tma_load_2d_pair(const void *tmap, uint32_t bar_cluster, void *smem_dst, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(smem_dst)),
        "l"(tmap), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}

// 16-byte cp.async global -> shared (L2 only), zero-filling the bytes past
// `src_bytes` (0 or 16): a padded tap reads nothing and writes zeros.
__device__ __forceinline__ void cp_async_16_zfill(uint32_t dst_smem, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst_smem), "l"(src), "r"(src_bytes)
                 : "memory");
}

// Arrives on `bar` once every cp.async issued so far by this thread has
// landed; the arrival counts against the barrier's expected count.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// TMA load in im2col mode from an NHWC activation: the box is `pixels`
// consecutive output positions (walked through the map's bounding box with
// its traversal strides, wrapping rows and images) x `channels` channels
// starting at channel c of input position (w, h) of image n, shifted by the
// filter tap (off_w, off_h); positions outside the image read zeros.
__device__ __forceinline__ void tma_load_im2col_4d(const void *tmap, uint64_t *bar, void *smem_dst, int c, int w, int h,
                                                   int n, uint16_t off_w, uint16_t off_h) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(smem_u32(smem_dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(c), "r"(w), "r"(h), "r"(n), "h"(off_w), "h"(off_h)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// TMA store of a 2-D box from this CTA's shared memory (bulk async-group
// completion). The smem writes it reads must be made visible to the async
// proxy first (fence_proxy_async_smem by every writing thread).
__device__ __forceinline__ void tma_store_2d(const void *tmap, const void *smem_src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N committed bulk groups of this thread still read their
// shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until every bulk group of this thread has completed (writes done).
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Barrier among `nthreads` threads (a multiple of 32) on hardware barrier `id` (1..15).
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Barrier among `nthreads` threads (a multiple of 32) on hardware barrier
// `id` (1..15; 0 is __syncthreads) that also ANDs a per-thread flag: all
// participants see the same result, so they can leave a loop together.
__device__ __forceinline__ bool named_barrier_and(int id, int nthreads, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.and.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0u;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Clusters (CTA pairs)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0u;
}

// Bounded wait with cluster-scope acquire (for barriers other CTAs arrive on).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, int *err_word, int err) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (clock64() - t0 > kWaitLimitCycles) {
            record_device_error(err_word, err);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// 16-byte load from the shared memory of a CTA of this cluster (an address
// from mapa_shared).
__device__ __forceinline__ float4 ld_shared_cluster_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in TMEM)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> f32, shape from `idesc`.
__device__ __forceinline__ void umma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// CTA-pair MMA (issued by the even CTA of the pair): A rows split across the
// two CTAs' shared memory (M = 256), B columns split likewise, D in both CTAs' TMEM.
__device__ __forceinline__ void umma_f8f6f4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on the mbarrier at `bar`'s offset in every CTA of `cta_mask`
// when the pair MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair_mc(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32-bit, 32 consecutive columns: thread i of the warp receives
// row (lane_base + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// Shared-memory matrix descriptor, K-major operand staged by TMA with the
// 128-byte swizzle: rows 128 B apart, 8-row groups 1024 B apart (SBO), tile
// base 1024-byte aligned. Fields: start>>4 [0,14), LBO>>4 [16,30) (unused for
// swizzled K-major, set to 1), SBO>>4 [32,46), version 1 [46,48),
// layout SWIZZLE_128B = 2 at [61,64).
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3ffffu) >> 4);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// The same for a K-major operand with 64-byte rows (64 e4m3 per K-block)
// staged with the 64-byte swizzle: 8-row groups 512 bytes apart, layout
// SWIZZLE_64B = 4.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw64(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3ffffu) >> 4);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(512u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(4u) << 61;
    return d;
}

template <int BKB>
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t smem_addr) {
    return BKB == 128 ? sdesc_kmajor_sw128(smem_addr) : sdesc_kmajor_sw64(smem_addr);
}

// Instruction descriptor for kind::f8f6f4: D f32 [4,6)=1, A/B e4m3 [7,10)=[10,13)=0,
// A K-major [15]=0, B major [16], N>>3 [17,23), M>>4 [24,29).
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(uint32_t M, uint32_t N, uint32_t b_mn_major) {
    return (1u << 4) | (b_mn_major << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0u;
}

}// namespace lcml
