// TEST INFRASTRUCTURE ONLY — never linked into the product library.
//
// Exposes the reference's own CPU FP8 codec with a C ABI so the oracle
// restatement (oracle.c) and the golden fixtures can be pinned against it.
// The codec itself is NOT in this repository: the Makefile extracts the CPU
// half of the reference header (include/onnx/fp_quantized.h, everything above
// `namespace luisa::compute {`, i.e. lines 1-403) into oracle/_ref/ at build
// time and this file includes that extracted copy.
//
//   FP8E4M3FN::from_float   include/onnx/fp_quantized.h:149-223
//   FP8E4M3FN::to_float     include/onnx/fp_quantized.h:226-249
//   FP8E5M2 / FP4E2M1       include/onnx/fp_quantized.h:259-378, :20-115
#include <cstdint>
#include <cstddef>
#include "fp_quantized_cpu.h"

extern "C" {

uint8_t lcml_ref_e4m3_from_float(float v) { return FP8E4M3FN::from_float(v); }
float lcml_ref_e4m3_to_float(uint8_t b) { return FP8E4M3FN::to_float(b); }
uint8_t lcml_ref_e5m2_from_float(float v) { return FP8E5M2::from_float(v); }
float lcml_ref_e5m2_to_float(uint8_t b) { return FP8E5M2::to_float(b); }
uint8_t lcml_ref_e2m1_from_float(float v) { return FP4E2M1::from_float(v); }
float lcml_ref_e2m1_to_float(uint8_t b) { return FP4E2M1::to_float(b); }

// y[i] = from_float(x[i])
void lcml_ref_e4m3_encode_n(const float *x, uint8_t *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = FP8E4M3FN::from_float(x[i]);
}

// y[i] = to_float(q[i])
void lcml_ref_e4m3_decode_n(const uint8_t *q, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = FP8E4M3FN::to_float(q[i]);
}

// QuantizeLinear with one fp32 scale: y[i] = from_float(x[i] / s).
// The division is an IEEE fp32 divide, the same operation the CUDA path uses.
void lcml_ref_e4m3_quantize_tensor(const float *x, float s, uint8_t *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = FP8E4M3FN::from_float(x[i] / s);
}

// Counts encoder disagreements between a reference encoder and a candidate
// encoder over the fp32 bit patterns [lo, hi). Used by the exhaustive checks.
extern "C++" {
template <uint8_t (*REF)(float)>
static int64_t count_mismatch(uint8_t (*candidate)(float), uint64_t lo, uint64_t hi, uint32_t *first_bad) {
    int64_t bad = 0;
    for (uint64_t u = lo; u < hi; ++u) {
        uint32_t bits = static_cast<uint32_t>(u);
        float v;
        __builtin_memcpy(&v, &bits, 4);
        if (REF(v) != candidate(v)) {
            if (bad == 0 && first_bad) *first_bad = bits;
            ++bad;
        }
    }
    return bad;
}
}

int64_t lcml_ref_e4m3_count_mismatch(uint8_t (*candidate)(float), uint64_t lo, uint64_t hi, uint32_t *first_bad) {
    return count_mismatch<FP8E4M3FN::from_float>(candidate, lo, hi, first_bad);
}

int64_t lcml_ref_e5m2_count_mismatch(uint8_t (*candidate)(float), uint64_t lo, uint64_t hi, uint32_t *first_bad) {
    return count_mismatch<FP8E5M2::from_float>(candidate, lo, hi, first_bad);
}

int64_t lcml_ref_e2m1_count_mismatch(uint8_t (*candidate)(float), uint64_t lo, uint64_t hi, uint32_t *first_bad) {
    return count_mismatch<FP4E2M1::from_float>(candidate, lo, hi, first_bad);
}

}// extern "C"
