/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the FP8 QDQ operator path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library, and only as the checker. The product (luisaml_b200/) never
 * links or calls it.
 *
 * Every function is a plain-C restatement of the reference algorithm it
 * names (paths are relative to the LuisaML source tree). The e4m3 codec is
 * pinned bit-for-bit against the reference's own compiled codec
 * (oracle/_ref, built from include/onnx/fp_quantized.h) and against the
 * committed golden vectors in tests/golden/.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* e4m3 codec                                                                 */
/* ------------------------------------------------------------------------- */

/*
 * fp32 -> FP8 E4M3FN byte. Restates FP8E4M3FN::from_float
 * (include/onnx/fp_quantized.h:149-223):
 *   NaN -> 0x7f (:151-153); +-0 -> 0x00 (:155-158);
 *   |v| > 448 (inf included) -> +-448 = 0x7e/0xfe (:166-171);
 *   otherwise round-to-nearest-even on 3 mantissa bits, subnormals in units of
 *   2^-9 (:174-205); a result that rounds to zero keeps the sign (0x80) (:213-216).
 */
ORC_EXPORT uint8_t orc_e4m3_from_float(float v) {
    if (isnan(v)) return 0x7f;
    if (v == 0.0f) return 0x00;
    uint8_t sign = signbit(v) ? 0x80 : 0x00;
    float a = fabsf(v);
    if (a > 448.0f) return (uint8_t)(sign | 0x7e);
    int ex;
    float fr = frexpf(a, &ex);      /* a = fr * 2^ex, fr in [0.5, 1) */
    int e = ex - 1 + 7;             /* e4m3 biased exponent of the leading bit */
    float units;                    /* a measured in units of the result's ulp */
    if (e <= 0) {
        e = 0;
        units = ldexpf(a, 9);       /* subnormal ulp is 2^-9 */
    } else {
        units = ldexpf(fr, 4);      /* [8, 16): implicit bit + 3 mantissa bits */
    }
    float fl = floorf(units);
    float rem = units - fl;         /* exact: units has at most 24 significant bits */
    uint32_t m = (uint32_t)fl;
    if (rem > 0.5f || (rem == 0.5f && (m & 1u))) m += 1u;
    if (e == 0) {
        /* m in [0, 8]; m == 8 is exactly the smallest normal 0x08 */
        if (m == 0) return sign;
        return (uint8_t)(sign | m);
    }
    /* m in [8, 16]; m == 16 carries into the exponent by plain addition */
    uint32_t code = ((uint32_t)e << 3) + (m - 8u);
    if (code > 0x7e) code = 0x7e;   /* unreachable for a <= 448; kept as the :207-211 clamp */
    return (uint8_t)(sign | code);
}

/*
 * FP8 E4M3FN byte -> fp32. Restates FP8E4M3FN::to_float
 * (include/onnx/fp_quantized.h:226-249): 0x7f/0xff -> NaN, 0x80 -> -0.0,
 * subnormal m * 2^-9, normal (1 + m/8) * 2^(e-7).
 */
ORC_EXPORT float orc_e4m3_to_float(uint8_t b) {
    int neg = (b & 0x80) != 0;
    int e = (b >> 3) & 0xf;
    int m = b & 0x7;
    float v;
    if (e == 15 && m == 7) return NAN;
    if (e == 0) v = ldexpf((float)m, -9);
    else v = ldexpf((float)(8 + m), e - 10);
    return neg ? -v : v;
}

ORC_EXPORT void orc_e4m3_encode_n(const float *x, uint8_t *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_e4m3_from_float(x[i]);
}

ORC_EXPORT void orc_e4m3_decode_n(const uint8_t *q, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_e4m3_to_float(q[i]);
}

/* ------------------------------------------------------------------------- */
/* e5m2 and e2m1 codecs                                                       */
/* ------------------------------------------------------------------------- */

/*
 * Round-to-nearest-even of a finite a > 0 onto a minifloat grid with `mbits`
 * mantissa bits, exponent bias `bias` and subnormal ulp 2^(1 - bias - mbits):
 * returns the code without sign (exponent field << mbits | mantissa); a carry
 * out of the mantissa moves into the exponent by plain addition.
 */
static uint32_t orc_minifloat_rne(float a, int mbits, int bias) {
    int ex;
    float fr = frexpf(a, &ex);      /* a = fr * 2^ex, fr in [0.5, 1) */
    int e = ex - 1 + bias;          /* biased exponent of the leading bit */
    float units;                    /* a in units of the result's ulp */
    if (e <= 0) {
        e = 0;
        units = ldexpf(a, bias - 1 + mbits);
    } else {
        units = ldexpf(fr, mbits + 1);  /* [2^mbits, 2^(mbits+1)): implicit bit + mantissa */
    }
    float fl = floorf(units);
    float rem = units - fl;
    uint32_t m = (uint32_t)fl;
    if (rem > 0.5f || (rem == 0.5f && (m & 1u))) m += 1u;
    if (e == 0) return m;           /* m == 2^mbits is exactly the smallest normal code */
    return ((uint32_t)e << mbits) + (m - (1u << mbits));
}

/*
 * fp32 -> FP8 E5M2 byte. Restates FP8E5M2::from_float
 * (include/onnx/fp_quantized.h:271-353): NaN -> 0x7f (:273-276); +-inf and
 * |v| > 57344 -> +-inf 0x7c/0xfc, no saturation (:277-294); +-0 -> 0x00
 * (:281-284); RNE on 2 mantissa bits, subnormal ulp 2^-16 (:296-327); a
 * result that rounds to zero keeps the sign (:337-341).
 */
ORC_EXPORT uint8_t orc_e5m2_from_float(float v) {
    if (isnan(v)) return 0x7f;
    if (v == 0.0f) return 0x00;
    uint8_t sign = signbit(v) ? 0x80 : 0x00;
    float a = fabsf(v);
    if (a > 57344.0f) return (uint8_t)(sign | 0x7c);
    return (uint8_t)(sign | orc_minifloat_rne(a, 2, 15));
}

/* FP8 E5M2 byte -> fp32 (fp_quantized.h:356-377): 0x7c/0xfc -> +-inf, other
 * exponent-31 codes NaN, subnormal m * 2^-16, normal (1 + m/4) * 2^(e-15). */
ORC_EXPORT float orc_e5m2_to_float(uint8_t b) {
    int neg = (b & 0x80) != 0;
    int e = (b >> 2) & 0x1f;
    int m = b & 0x3;
    float v;
    if (e == 31) {
        if (m != 0) return NAN;
        return neg ? -INFINITY : INFINITY;
    }
    if (e == 0) v = ldexpf((float)m, -16);
    else v = ldexpf((float)(4 + m), e - 17);
    return neg ? -v : v;
}

/*
 * fp32 -> FP4 E2M1 code (low nibble). Restates FP4E2M1::from_float
 * (include/onnx/fp_quantized.h:33-93): +-0 -> 0x0 (:34-36); |v| > 6 (inf
 * included) -> +-6 = 0x7/0xf (:43-46); RNE on 1 mantissa bit, subnormal ulp
 * 0.5 (:48-79); a result that rounds to zero keeps the sign (:87-89). The
 * reference has no NaN case (NaN reaches an undefined float -> uint8
 * conversion); its x86-64 build returns 0x0, which is the value used here.
 */
ORC_EXPORT uint8_t orc_e2m1_from_float(float v) {
    if (isnan(v) || v == 0.0f) return 0x0;
    uint8_t sign = signbit(v) ? 0x8 : 0x0;
    float a = fabsf(v);
    if (a > 6.0f) return (uint8_t)(sign | 0x7);
    return (uint8_t)(sign | orc_minifloat_rne(a, 1, 1));
}

/* FP4 E2M1 code -> fp32 (fp_quantized.h:96-114): subnormal m * 0.5, normal
 * (1 + m/2) * 2^(e-1), code 0x8 -> -0.0. */
ORC_EXPORT float orc_e2m1_to_float(uint8_t b) {
    int neg = (b & 0x8) != 0;
    int e = (b >> 1) & 0x3;
    int m = b & 0x1;
    float v = e == 0 ? 0.5f * (float)m : ldexpf((float)(2 + m), e - 2);
    return neg ? -v : v;
}

/*
 * Cast (src/onnx/operators/cast.cpp:10-162) of n elements. Type codes are the
 * ONNX numbers: 1 FLOAT, 10 FLOAT16, 16 BFLOAT16, 17 FLOAT8E4M3FN,
 * 19 FLOAT8E5M2, 23 FLOAT4E2M1 (packed, element 2i in the low nibble of byte
 * i). To an FP8 / FP4 type the value is first rounded to half and then
 * encoded (cast.cpp:58-72: `fp8_from(input[i].cast<half>())`); from FP8 / FP4
 * it is decoded (cast.cpp:39-53, exact in every floating type); between the
 * floating types one round-to-nearest-even conversion (_Float16 / bf16 RNE).
 */
static float orc_bf16_to_float(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static uint16_t orc_float_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  /* quiet NaN, sign kept */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float orc_load(const uint8_t *x, int t, int64_t i) {
    switch (t) {
        case 1: { float f; memcpy(&f, x + 4 * i, 4); return f; }
        case 10: { _Float16 h; memcpy(&h, x + 2 * i, 2); return (float)h; }
        case 16: { uint16_t h; memcpy(&h, x + 2 * i, 2); return orc_bf16_to_float(h); }
        case 17: return orc_e4m3_to_float(x[i]);
        case 19: return orc_e5m2_to_float(x[i]);
        default: return orc_e2m1_to_float((uint8_t)((x[i >> 1] >> ((i & 1) * 4)) & 0xf));
    }
}

static int orc_cast_type_ok(int t) { return t == 1 || t == 10 || t == 16 || t == 17 || t == 19 || t == 23; }

/* The destination bits of value v (already rounded to half where the Cast
 * semantics ask for it). */
static uint32_t orc_cast_bits(float v, int dst) {
    if (dst == 1) {
        uint32_t u;
        memcpy(&u, &v, 4);
        return u;
    }
    if (dst == 10) {
        _Float16 h = (_Float16)v;
        uint16_t u;
        memcpy(&u, &h, 2);
        return u;
    }
    if (dst == 16) return orc_float_to_bf16(v);
    if (dst == 17) return orc_e4m3_from_float(v);
    if (dst == 19) return orc_e5m2_from_float(v);
    return orc_e2m1_from_float(v);
}

/*
 * Add/Sub/Mul/Div of FP8-typed tensors (binary.cpp:185-283): both operands
 * decoded to half (exact), the op in half (_Float16 arithmetic: computed in
 * float and rounded to half, which is the correctly rounded half result for
 * these four ops since float carries more than 2 * 11 + 2 bits), the half
 * result encoded. dtype 17 (e4m3) or 19 (e5m2); b broadcast by b[i % bn].
 */
ORC_EXPORT void orc_binary_fp8(int op, const uint8_t *a, const uint8_t *b, int64_t n, int64_t bn, uint8_t *y,
                               int dtype) {
    for (int64_t i = 0; i < n; ++i) {
        float fa = dtype == 19 ? orc_e5m2_to_float(a[i]) : orc_e4m3_to_float(a[i]);
        float fb = dtype == 19 ? orc_e5m2_to_float(b[i % bn]) : orc_e4m3_to_float(b[i % bn]);
        _Float16 ha = (_Float16)fa, hb = (_Float16)fb, r;
        if (op == 0) r = ha + hb;
        else if (op == 1) r = ha - hb;
        else if (op == 2) r = ha * hb;
        else r = ha / hb;
        y[i] = dtype == 19 ? orc_e5m2_from_float((float)r) : orc_e4m3_from_float((float)r);
    }
}

ORC_EXPORT int orc_cast(const void *xv, int src, void *yv, int dst, int64_t n) {
    if (!orc_cast_type_ok(src) || !orc_cast_type_ok(dst)) return -1;
    const uint8_t *x = (const uint8_t *)xv;
    uint8_t *y = (uint8_t *)yv;
    const int quantized_dst = dst == 17 || dst == 19 || dst == 23;
    const int bytes = dst == 1 ? 4 : (dst == 10 || dst == 16) ? 2 : 1;
    if (dst == 23) memset(y, 0, (size_t)((n + 1) / 2));
    for (int64_t i = 0; i < n; ++i) {
        float v = orc_load(x, src, i);
        if (quantized_dst && (src == 1 || src == 16)) v = (float)(_Float16)v;  /* cast<half>() first */
        const uint32_t b = orc_cast_bits(v, dst);
        if (dst == 23) y[i >> 1] |= (uint8_t)(b << ((i & 1) * 4));
        else memcpy(y + bytes * i, &b, (size_t)bytes);  /* little-endian low bytes */
    }
    return 0;
}

/* ------------------------------------------------------------------------- */
/* QuantizeLinear / DequantizeLinear (ONNX semantics, float8e4m3fn, zp = 0,    */
/* saturate = 1). The reference registers neither op; the encoder is the      */
/* reference codec above applied to the fp32 quotient x / s.                  */
/* ------------------------------------------------------------------------- */

/* max |x| over finite and infinite values; NaN is ignored (treated as 0). */
ORC_EXPORT float orc_amax(const float *x, int64_t n) {
    float m = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        float a = fabsf(x[i]);
        if (a > m) m = a;           /* comparison with NaN is false: ignored */
    }
    return m;
}

/* Scale used by every dynamic mode: amax / 448 in fp32, or 1 for an all-zero
 * (or all-NaN) slice so that the quotient stays finite. */
ORC_EXPORT float orc_scale_from_amax(float amax) {
    return amax > 0.0f ? amax / 448.0f : 1.0f;
}

/*
 * x viewed as [outer, axis_len, inner]. per_axis == 0: one scale s[0];
 * per_axis == 1: s[a] for a in [0, axis_len) (ONNX per-axis QuantizeLinear).
 */
ORC_EXPORT void orc_quantize_axis(const float *x, int64_t outer, int64_t axis_len, int64_t inner,
                                  const float *s, int per_axis, uint8_t *y) {
    int64_t n = outer * axis_len * inner;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float sc = per_axis ? s[(i / inner) % axis_len] : s[0];
        y[i] = orc_e4m3_from_float(x[i] / sc);
    }
}

/* Dynamic per-row (per-token) quantization: s[r] = amax(row r) / 448. */
ORC_EXPORT void orc_quantize_dynamic_rows(const float *x, int64_t rows, int64_t cols,
                                          float *s_out, uint8_t *y) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * cols;
        float s = orc_scale_from_amax(orc_amax(xr, cols));
        s_out[r] = s;
        for (int64_t c = 0; c < cols; ++c) y[r * cols + c] = orc_e4m3_from_float(xr[c] / s);
    }
}

/* DequantizeLinear: y = to_float(q) * s (fp32 multiply). Same [outer, axis, inner] view. */
ORC_EXPORT void orc_dequantize_axis(const uint8_t *q, int64_t outer, int64_t axis_len, int64_t inner,
                                    const float *s, int per_axis, float *y) {
    int64_t n = outer * axis_len * inner;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float sc = per_axis ? s[(i / inner) % axis_len] : s[0];
        y[i] = orc_e4m3_to_float(q[i]) * sc;
    }
}

/* ------------------------------------------------------------------------- */
/* Gemm (src/onnx/operators/gemm.cpp)                                         */
/* ------------------------------------------------------------------------- */

/*
 * Y = alpha * op(A) * op(B) + beta * C in fp32.
 *   op(A) is [M,K] (A stored [M,K], or [K,M] when transA), op(B) is [K,N]
 *   (B stored [K,N], or [N,K] when transB)                 gemm.cpp:33-39
 *   sum = fma(a, b, sum) over k in order, starting at 0    gemm.cpp:113-119, :153-157
 *   sum *= alpha when alpha != 1                           gemm.cpp:106-110
 *   sum += C (beta == 1) or beta * C, C broadcast from a scalar, [N], [M],
 *   [1,N], [M,1] or [M,N]                                  gemm.cpp:78-103
 * c_ndim < 0 means no C. Rows [row0, row1) only (row1 <= M) so callers can
 * time a bounded sample of a large problem.
 */
/*
 * lanes == 4 restates the reference's vector path for byte-buffer operands
 * with unit stride along K (gemm.cpp:123-152): four lane accumulators, lane
 * l taking k = 4j + l with fma in j order, summed as ((x + y) + z) + w and
 * added to the running sum (starting at 0), then the K % 4 tail with fma in
 * order. lanes == 1 is the scalar loop (gemm.cpp:153-157).
 */
ORC_EXPORT void orc_gemm_f32_rows_lanes(const float *A, const float *B, const float *C,
                                        int64_t M, int64_t N, int64_t K, int transA, int transB,
                                        float alpha, float beta, int c_ndim, int64_t c_d0, int64_t c_d1,
                                        float *Y, int64_t row0, int64_t row1, int lanes) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t m = row0; m < row1; ++m) {
        for (int64_t n = 0; n < N; ++n) {
            float sum = 0.0f;
            int64_t k0 = 0;
            if (lanes == 4) {
                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (int64_t j = 0; j < K / 4; ++j)
                    for (int l = 0; l < 4; ++l) {
                        const int64_t k = 4 * j + l;
                        acc[l] = fmaf(transA ? A[k * M + m] : A[m * K + k], transB ? B[n * K + k] : B[k * N + n], acc[l]);
                    }
                sum += ((acc[0] + acc[1]) + acc[2]) + acc[3];
                k0 = (K / 4) * 4;
            }
            for (int64_t k = k0; k < K; ++k) {
                float a = transA ? A[k * M + m] : A[m * K + k];
                float b = transB ? B[n * K + k] : B[k * N + n];
                sum = fmaf(a, b, sum);
            }
            if (alpha != 1.0f) sum *= alpha;
            if (C && c_ndim >= 0 && beta != 0.0f) {
                float c;
                if (c_ndim == 0 || (c_ndim == 1 && c_d0 == 1)) c = C[0];
                else if (c_ndim == 1) c = (c_d0 == N) ? C[n] : C[m];
                else {
                    int64_t ci = (c_d0 == 1) ? 0 : m;
                    int64_t cj = (c_d1 == 1) ? 0 : n;
                    c = C[ci * c_d1 + cj];
                }
                if (beta == 1.0f) sum += c;
                else sum += beta * c;
            }
            Y[(m - row0) * N + n] = sum;
        }
    }
}

ORC_EXPORT void orc_gemm_f32_rows(const float *A, const float *B, const float *C,
                                  int64_t M, int64_t N, int64_t K, int transA, int transB,
                                  float alpha, float beta, int c_ndim, int64_t c_d0, int64_t c_d1,
                                  float *Y, int64_t row0, int64_t row1) {
    orc_gemm_f32_rows_lanes(A, B, C, M, N, K, transA, transB, alpha, beta, c_ndim, c_d0, c_d1, Y, row0, row1, 1);
}

/*
 * The same K-ordered fma dot for a *transposed-B* layout, reading the weights
 * directly from e4m3 bytes with their scales — the CPU baseline of the QDQ
 * Gemm (DequantizeLinear of both operands followed by gemm.cpp's loop).
 * sa: per-tensor (sa_mode 0) or per-row (1); sb: per-tensor (0) or per-col (1).
 * B is [N,K] (transB = 1) when b_kmajor, else [K,N]. Rows [row0,row1).
 */
ORC_EXPORT void orc_qdq_gemm_rows(const uint8_t *Aq, const float *sa, int sa_mode,
                                  const uint8_t *Bq, const float *sb, int sb_mode, int b_kmajor,
                                  const float *bias, int64_t M, int64_t N, int64_t K,
                                  float *Y, int64_t row0, int64_t row1) {
    (void)M;
    float lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = orc_e4m3_to_float((uint8_t)i);
#pragma omp parallel
    {
        float *arow = (float *)malloc(sizeof(float) * (size_t)K);
        float *bcol = b_kmajor ? NULL : (float *)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(dynamic, 1)
        for (int64_t m = row0; m < row1; ++m) {
            float s_a = sa_mode ? sa[m] : sa[0];
            for (int64_t k = 0; k < K; ++k) arow[k] = lut[Aq[m * K + k]] * s_a;
            for (int64_t n = 0; n < N; ++n) {
                float s_b = sb_mode ? sb[n] : sb[0];
                float sum = 0.0f;
                if (b_kmajor) {
                    const uint8_t *bn = Bq + n * K;
                    for (int64_t k = 0; k < K; ++k) sum = fmaf(arow[k], lut[bn[k]] * s_b, sum);
                } else {
                    for (int64_t k = 0; k < K; ++k) sum = fmaf(arow[k], lut[Bq[k * N + n]] * s_b, sum);
                }
                if (bias) sum += bias[n];
                Y[(m - row0) * N + n] = sum;
            }
        }
        free(arow);
        free(bcol);
    }
}

/* ------------------------------------------------------------------------- */
/* Conv (src/onnx/operators/conv.cpp:115-207), 2-D NCHW, fp32                 */
/* ------------------------------------------------------------------------- */

/*
 * Y[n,m,oh,ow] = bias[m] + sum_{kh,kw,c} X[n, g*Cg + c, ih, iw] * W[m, c, kh, kw]
 * with ih = oh*sH + kh*dH - pH, iw = ow*sW + kw*dW - pW (begin pads only,
 * conv.cpp:119-121), out-of-range taps skipped (conv.cpp:147), loop order
 * kh, kw, c with fma accumulation (conv.cpp:141-195), then + bias
 * (conv.cpp:197-200). Images [n0, n1) only.
 */
/*
 * lanes == 4 restates the reference's fp32 order (conv.cpp:150-191): per
 * tap, the group's channels four at a time into four lane sums (fma),
 * added as ((x + y) + z) + w to the running sum, the last Cg % 4 channels
 * by fma into the running sum. lanes == 1: one fma chain over (kh, kw, c).
 */
ORC_EXPORT void orc_conv2d_f32_lanes(const float *X, const float *W, const float *bias,
                                     int64_t N, int64_t C, int64_t H, int64_t Wd,
                                     int64_t M, int64_t kH, int64_t kW, int64_t oH, int64_t oW,
                                     int sH, int sW, int pH, int pW, int dH, int dW, int group,
                                     float *Y, int64_t n0, int64_t n1, int lanes) {
    (void)N;
    int64_t Cg = C / group, Mg = M / group;
    int64_t c4 = lanes == 4 ? (Cg / 4) * 4 : 0;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int64_t n = n0; n < n1; ++n) {
        for (int64_t m = 0; m < M; ++m) {
            int64_t g = m / Mg;
            for (int64_t oh = 0; oh < oH; ++oh) {
                for (int64_t ow = 0; ow < oW; ++ow) {
                    float sum = 0.0f;
                    for (int64_t kh = 0; kh < kH; ++kh) {
                        int64_t ih = oh * sH + kh * dH - pH;
                        if (ih < 0 || ih >= H) continue;
                        for (int64_t kw = 0; kw < kW; ++kw) {
                            int64_t iw = ow * sW + kw * dW - pW;
                            if (iw < 0 || iw >= Wd) continue;
                            if (c4 > 0) {
                                float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                                for (int64_t c = 0; c < c4; ++c)
                                    a[c & 3] = fmaf(X[((n * C + g * Cg + c) * H + ih) * Wd + iw],
                                                    W[((m * Cg + c) * kH + kh) * kW + kw], a[c & 3]);
                                sum += ((a[0] + a[1]) + a[2]) + a[3];
                            }
                            for (int64_t c = c4; c < Cg; ++c) {
                                float xv = X[((n * C + g * Cg + c) * H + ih) * Wd + iw];
                                float wv = W[((m * Cg + c) * kH + kh) * kW + kw];
                                sum = fmaf(xv, wv, sum);
                            }
                        }
                    }
                    if (bias) sum += bias[m];
                    Y[(((n - n0) * M + m) * oH + oh) * oW + ow] = sum;
                }
            }
        }
    }
}

/*
 * ConvTranspose (src/onnx/operators/conv_transpose.cpp), the reference's
 * gather loop: Y[n, m, oh, ow] = sum over taps (kh, kw) with
 * oh + pH - kh*dH = ih * sH, 0 <= ih < H (likewise w), of the group's
 * channels in four lane sums (conv_transpose.cpp:215-232), tail by fma, then
 * + bias (:270-273). W is [C, M/group, kH, kW].
 */
ORC_EXPORT void orc_conv_transpose2d_f32(const float *X, const float *W, const float *bias, int64_t N, int64_t C,
                                         int64_t H, int64_t Wd, int64_t M, int64_t kH, int64_t kW, int64_t oH,
                                         int64_t oW, int sH, int sW, int pH, int pW, int dH, int dW, int group,
                                         float *Y) {
    int64_t Cg = C / group, Mg = M / group, c4 = (Cg / 4) * 4;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t m = 0; m < M; ++m) {
            int64_t g = m / Mg, mg = m % Mg;
            for (int64_t oh = 0; oh < oH; ++oh) {
                for (int64_t ow = 0; ow < oW; ++ow) {
                    float sum = 0.0f;
                    for (int64_t kh = 0; kh < kH; ++kh) {
                        int64_t ihs = oh + pH - kh * dH;
                        if (ihs < 0 || ihs % sH != 0 || ihs / sH >= H) continue;
                        for (int64_t kw = 0; kw < kW; ++kw) {
                            int64_t iws = ow + pW - kw * dW;
                            if (iws < 0 || iws % sW != 0 || iws / sW >= Wd) continue;
                            int64_t ih = ihs / sH, iw = iws / sW;
#define XV(c) X[((n * C + g * Cg + (c)) * H + ih) * Wd + iw]
#define WV(c) W[(((g * Cg + (c)) * Mg + mg) * kH + kh) * kW + kw]
                            if (c4 > 0) {
                                float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                                for (int64_t c = 0; c < c4; ++c) a[c & 3] = fmaf(XV(c), WV(c), a[c & 3]);
                                sum += ((a[0] + a[1]) + a[2]) + a[3];
                            }
                            for (int64_t c = c4; c < Cg; ++c) sum = fmaf(XV(c), WV(c), sum);
#undef XV
#undef WV
                        }
                    }
                    if (bias) sum += bias[m];
                    Y[((n * M + m) * oH + oh) * oW + ow] = sum;
                }
            }
        }
    }
}

ORC_EXPORT void orc_conv2d_f32(const float *X, const float *W, const float *bias,
                               int64_t N, int64_t C, int64_t H, int64_t Wd,
                               int64_t M, int64_t kH, int64_t kW, int64_t oH, int64_t oW,
                               int sH, int sW, int pH, int pW, int dH, int dW, int group,
                               float *Y, int64_t n0, int64_t n1) {
    orc_conv2d_f32_lanes(X, W, bias, N, C, H, Wd, M, kH, kW, oH, oW, sH, sW, pH, pW, dH, dW, group, Y, n0, n1, 1);
}

/* ------------------------------------------------------------------------- */
/* Memory-bound ops around the GEMMs                                          */
/* ------------------------------------------------------------------------- */

/* Relu: max(0, x) (src/onnx/operators/unary.cpp:85). */
ORC_EXPORT void orc_relu(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

/* Sigmoid written with exp(-|x|) for stability (src/onnx/operators/unary.cpp:86-87). */
ORC_EXPORT float orc_sigmoid1(float x) {
    float e = expf(-fabsf(x));
    return x >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
}

ORC_EXPORT void orc_sigmoid(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_sigmoid1(x[i]);
}

/* SiLU(g) * u = (g * sigmoid(g)) * u, the Sigmoid -> Mul -> Mul chain
 * (unary.cpp:86-87, binary.cpp:347). */
ORC_EXPORT void orc_silu_mul(const float *g, const float *u, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = (g[i] * orc_sigmoid1(g[i])) * u[i];
}

/* Softmax over the last axis of [rows, cols]: exp(x - max) / sum
 * (src/onnx/operators/softmax.cpp:216-280). */
ORC_EXPORT void orc_softmax_rows(const float *x, float *y, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * cols;
        float mx = -INFINITY;
        for (int64_t c = 0; c < cols; ++c) mx = xr[c] > mx ? xr[c] : mx;
        float s = 0.0f;
        for (int64_t c = 0; c < cols; ++c) s += expf(xr[c] - mx);
        for (int64_t c = 0; c < cols; ++c) y[r * cols + c] = expf(xr[c] - mx) / s;
    }
}

/* MaxPool 2-D NCHW with begin pads; padded taps are skipped
 * (src/onnx/operators/max_pool.cpp:20-300). */
ORC_EXPORT void orc_maxpool2d(const float *x, float *y, int64_t NC, int64_t H, int64_t W,
                              int kH, int kW, int sH, int sW, int pH, int pW,
                              int64_t oH, int64_t oW) {
    for (int64_t p = 0; p < NC; ++p)
        for (int64_t oh = 0; oh < oH; ++oh)
            for (int64_t ow = 0; ow < oW; ++ow) {
                float m = -INFINITY;
                for (int kh = 0; kh < kH; ++kh) {
                    int64_t ih = oh * sH + kh - pH;
                    if (ih < 0 || ih >= H) continue;
                    for (int kw = 0; kw < kW; ++kw) {
                        int64_t iw = ow * sW + kw - pW;
                        if (iw < 0 || iw >= W) continue;
                        float v = x[(p * H + ih) * W + iw];
                        m = v > m ? v : m;
                    }
                }
                y[(p * oH + oh) * oW + ow] = m;
            }
}

/* GlobalAveragePool: mean over H*W per (n, c) (global_average_pool.cpp:40-150). */
ORC_EXPORT void orc_global_avgpool(const float *x, float *y, int64_t NC, int64_t HW) {
    for (int64_t p = 0; p < NC; ++p) {
        float s = 0.0f;
        for (int64_t i = 0; i < HW; ++i) s += x[p * HW + i];
        y[p] = s / (float)HW;
    }
}

ORC_EXPORT int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
