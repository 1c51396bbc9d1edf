// Operator classes shared between the registry (operators.cpp) and the
// executor's fusion pass (network_instance.cpp).
#pragma once

#include "../../include/lcml_onnx.h"

namespace lcml::onnx {

// Base for operators that enqueue work on the owning NetworkInstance's stream.
class StreamOperator : public Operator {
protected:
    lcml_stream_t stream_ = nullptr;

public:
    using Operator::Operator;
    void set_environment(NetworkInstance &env, TensorTable &) override { stream_ = env.stream(); }
};

// One fused QDQ GEMM node group (built by the fusion pass, not registered):
//   inputs  [A_q e4m3 [M,K], s_a (1|M), B_q e4m3 ([N,K] when b_kmajor, else [K,N]), s_b (1|N),
//            (C), (y_scale)]
//   output  Y [M, N] (N/2 for SILU_MUL) in fp32 / bf16 / e4m3
class FusedQdqGemm : public StreamOperator {
public:
    int b_kmajor = 1;
    float alpha = 1.0f, beta = 1.0f;
    int epilogue = LCML_EPI_NONE;
    bool has_c = false;
    bool has_y_scale = false;
    // dynamic per-row quantization of the output (rowquant): extra outputs [q, s]
    bool row_quant = false;
    void *workspace = nullptr;  // M floats (row maxima) when row_quant

    FusedQdqGemm() : StreamOperator("FusedQdqGemm") {}
    void forward(std::span<std::reference_wrapper<ITensor>> in, std::span<std::reference_wrapper<ITensor>> out) override;
};

// Abs -> ReduceMax(last axis) -> Div(448) -> QuantizeLinear(axis 0) on a 2-D
// tensor, as one kernel (lcml_fp8_quantize_rows_dynamic):
//   inputs [x fp32 [rows, cols]]  outputs [q e4m3 [rows, cols], s fp32 [rows]]
class DynamicRowQuant : public StreamOperator {
public:
    DynamicRowQuant() : StreamOperator("DynamicRowQuant") {}
    void forward(std::span<std::reference_wrapper<ITensor>> in, std::span<std::reference_wrapper<ITensor>> out) override;
};

// One fused QDQ convolution group (built by the fusion pass, not registered):
// DequantizeLinear(x) / DequantizeLinear(W) -> Conv (+bias) -> (Add with a
// DequantizeLinear'd residual) -> (Relu) -> QuantizeLinear, as one implicit-
// GEMM kernel chain (lcml_fp8_conv):
//   inputs  [x e4m3 (NCHW or NHWC), s_x [1], W packed e4m3 [M, Kp], s_w (1|M),
//            (bias fp32 [M]), (residual e4m3 NHWC, s_r [1]), y_scale [1]]
//   output  y e4m3 NHWC [N, oH, oW, M] (shape() keeps the ONNX NCHW shape)
class FusedQdqConv : public StreamOperator {
public:
    lcml_fp8_conv_desc desc{};  // geometry and epilogue; pointers are bound per forward
    bool has_bias = false, has_residual = false;
    void *workspace = nullptr;  // shared by every fused conv of the instance

    FusedQdqConv() : StreamOperator("FusedQdqConv") {}
    void forward(std::span<std::reference_wrapper<ITensor>> in, std::span<std::reference_wrapper<ITensor>> out) override;
};

// DequantizeLinear -> MaxPool -> QuantizeLinear with the same per-tensor scale
// on both sides: the max commutes with the monotonic encoding, so the pool
// runs on the e4m3 codes directly.
//   inputs [x e4m3 (NCHW or NHWC)]  outputs [y e4m3, same layout]
class QdqMaxPool : public StreamOperator {
public:
    int kH = 1, kW = 1, sH = 1, sW = 1, pH = 0, pW = 0;
    bool nhwc = false;

    QdqMaxPool() : StreamOperator("QdqMaxPool") {}
    void forward(std::span<std::reference_wrapper<ITensor>> in, std::span<std::reference_wrapper<ITensor>> out) override;
};

// DequantizeLinear -> GlobalAveragePool: the mean of the decoded codes times
// the scale, read straight from the e4m3 tensor.
//   inputs [x e4m3 (NCHW or NHWC), s_x [1]]  outputs [y fp32 [N, C, 1, 1]]
class QdqGlobalAveragePool : public StreamOperator {
public:
    bool nhwc = false;

    QdqGlobalAveragePool() : StreamOperator("QdqGlobalAveragePool") {}
    void forward(std::span<std::reference_wrapper<ITensor>> in, std::span<std::reference_wrapper<ITensor>> out) override;
};

// An fp32 Gemm node (alpha, beta, transA, transB read from it) whose output
// goes through Relu in the same kernel (lcml_gemm_f32_relu): built by the
// fusion pass for a Gemm whose only reader is a Relu.
std::unique_ptr<Operator> make_gemm_f32_relu(const Node &gemm);

}// namespace lcml::onnx
