// FP8 implicit-GEMM convolution (NCHW / NHWC) on the tcgen05 GEMM mainloop.
#include "lcml_device.cuh"
#include "lcml_internal.h"

extern "C" {

int64_t lcml_fp8_conv_workspace_size(const lcml_fp8_conv_desc *desc) { return desc ? 0 : -1; }

int64_t lcml_fp8_conv_packed_weight_size(int64_t M, int64_t Cg, int64_t kH, int64_t kW) {
    return M * Cg * kH * kW;
}

int lcml_fp8_conv_pack_weight(const uint8_t *, int64_t, int64_t, int64_t, int64_t, uint8_t *, lcml_stream_t) {
    return lcml::set_error(LCML_ERR_UNSUPPORTED, "lcml_fp8_conv_pack_weight: not built yet");
}

int lcml_fp8_conv(const lcml_fp8_conv_desc *, lcml_stream_t) {
    return lcml::set_error(LCML_ERR_UNSUPPORTED, "lcml_fp8_conv: not built yet");
}

}// extern "C"
