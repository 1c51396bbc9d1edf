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

}// namespace lcml::onnx
