// The operator library: one Operator subclass per ONNX op on the FP8 path,
// registered in the default opset under the ONNX names, each calling the C
// ABI of lcml_fp8.h from forward(). Reference operators they stand in for:
//   QuantizeLinear / DequantizeLinear  (not registered in the reference)
//   Gemm        src/onnx/operators/gemm.cpp:18-385
//   MatMul      src/onnx/operators/mat_mul.cpp:12-311
//   Conv        src/onnx/operators/conv.cpp:18-275
//   Relu/Sigmoid/Abs   unary.cpp:85-110; Add/Sub/Mul/Div binary.cpp:341-350
//   ReduceMax   reduce.cpp:431; Softmax softmax.cpp:443; MaxPool max_pool.cpp;
//   GlobalAveragePool global_average_pool.cpp:150; Flatten/Reshape/Identity;
//   Cast        cast.cpp:149
#include <cstring>

#include "operators.h"

namespace lcml::onnx {

namespace {

using Span = std::span<std::reference_wrapper<ITensor>>;

void require(bool cond, const std::string &msg) {
    if (!cond) throw Error(msg);
}

int64_t norm_axis(int64_t axis, int64_t ndim) { return axis < 0 ? axis + ndim : axis; }

void axis_view(const ITensor &t, int64_t axis, int64_t &outer, int64_t &alen, int64_t &inner) {
    const int64_t ax = norm_axis(axis, t.ndim());
    require(ax >= 0 && ax < t.ndim(), "axis out of range");
    outer = 1;
    inner = 1;
    for (int64_t i = 0; i < ax; ++i) outer *= t.shape(i);
    alen = t.shape(ax);
    for (int64_t i = ax + 1; i < t.ndim(); ++i) inner *= t.shape(i);
}

// zero point inputs must be all-zero constants (this path has no zero point)
void require_zero_point(Span in, size_t idx, const char *op) {
    if (in.size() <= idx) return;
    const ITensor &zp = in[idx].get();
    const std::string *h = zp.host_data();
    require(h != nullptr, std::string(op) + ": zero point must be a constant");
    for (char c : *h) require(c == 0, std::string(op) + ": nonzero zero point is not supported on the e4m3 path");
}

int64_t get_int(const Node &node, const char *name, int64_t dflt) {
    if (auto p = node.try_get_attr(name)) return p->get<AttributeType::INT>();
    return dflt;
}

float get_float(const Node &node, const char *name, float dflt) {
    if (auto p = node.try_get_attr(name)) return p->get<AttributeType::FLOAT>();
    return dflt;
}

std::vector<int64_t> get_ints(const Node &node, const char *name) {
    if (auto p = node.try_get_attr(name)) return p->get<AttributeType::INTS>();
    return {};
}

// ------------------------------------------------------------------ Q / DQ
class QuantizeLinear : public StreamOperator {
    int64_t axis_;

public:
    explicit QuantizeLinear(int64_t axis) : StreamOperator("QuantizeLinear"), axis_(axis) {}
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get(), &s = in[1].get();
        ITensor &y = out[0].get();
        require(x.dtype() == DataType::FLOAT && s.dtype() == DataType::FLOAT, "QuantizeLinear: x and scale must be FLOAT");
        require(y.dtype() == DataType::FLOAT8E4M3FN, "QuantizeLinear: output must be FLOAT8E4M3FN");
        require_zero_point(in, 2, "QuantizeLinear");
        int64_t outer = 1, alen = 1, inner = x.size();
        int mode = LCML_SCALE_TENSOR;
        if (s.size() > 1) {
            axis_view(x, axis_, outer, alen, inner);
            require(s.size() == alen, "QuantizeLinear: scale length does not match the axis");
            mode = LCML_SCALE_AXIS;
        }
        check_status(lcml_fp8_quantize(x.ptr<float>(), outer, alen, inner, s.ptr<float>(), mode, y.ptr<uint8_t>(), stream_),
                     "QuantizeLinear");
    }
};

class DequantizeLinear : public StreamOperator {
    int64_t axis_;

public:
    explicit DequantizeLinear(int64_t axis) : StreamOperator("DequantizeLinear"), axis_(axis) {}
    void forward(Span in, Span out) override {
        const ITensor &q = in[0].get(), &s = in[1].get();
        ITensor &y = out[0].get();
        require(q.dtype() == DataType::FLOAT8E4M3FN, "DequantizeLinear: input must be FLOAT8E4M3FN");
        require(y.dtype() == DataType::FLOAT || y.dtype() == DataType::BFLOAT16, "DequantizeLinear: output must be FLOAT or BFLOAT16");
        require_zero_point(in, 2, "DequantizeLinear");
        int64_t outer = 1, alen = 1, inner = q.size();
        int mode = LCML_SCALE_TENSOR;
        if (s.size() > 1) {
            axis_view(q, axis_, outer, alen, inner);
            require(s.size() == alen, "DequantizeLinear: scale length does not match the axis");
            mode = LCML_SCALE_AXIS;
        }
        check_status(lcml_fp8_dequantize(q.ptr<uint8_t>(), outer, alen, inner, s.ptr<float>(), mode, y.data(),
                                         static_cast<int>(y.dtype()), stream_),
                     "DequantizeLinear");
    }
};

// ------------------------------------------------------------------ Gemm / MatMul (fp32)
class Gemm : public StreamOperator {
public:
    float alpha, beta;
    int64_t transA, transB;
    bool relu = false;  // fused Relu (lcml_gemm_f32_relu)
    Gemm(float a, float b, int64_t ta, int64_t tb) : StreamOperator("Gemm"), alpha(a), beta(b), transA(ta), transB(tb) {}
    void forward(Span in, Span out) override {
        const ITensor &A = in[0].get(), &B = in[1].get();
        ITensor &Y = out[0].get();
        require(A.ndim() == 2 && B.ndim() == 2, "Gemm: A and B must be 2-D");
        require(A.dtype() == DataType::FLOAT && B.dtype() == DataType::FLOAT && Y.dtype() == DataType::FLOAT,
                "Gemm: unfused Gemm runs in FLOAT (FP8 Gemm comes from DequantizeLinear inputs)");
        const int64_t M = transA ? A.shape(1) : A.shape(0), K = transA ? A.shape(0) : A.shape(1);
        const int64_t K2 = transB ? B.shape(1) : B.shape(0), N = transB ? B.shape(0) : B.shape(1);
        require(K == K2, "Gemm: inner dimensions mismatch");
        require(Y.size() == M * N, "Gemm: Y shape mismatch");
        const float *C = nullptr;
        int c_ndim = -1;
        int64_t d0 = 0, d1 = 0;
        if (in.size() > 2) {
            const ITensor &Ct = in[2].get();
            require(Ct.dtype() == DataType::FLOAT, "Gemm: C must be FLOAT");
            C = Ct.ptr<float>();
            c_ndim = static_cast<int>(Ct.ndim());
            d0 = Ct.ndim() >= 1 ? Ct.shape(0) : 0;
            d1 = Ct.ndim() >= 2 ? Ct.shape(1) : 0;
        }
        auto fn = relu ? lcml_gemm_f32_relu : lcml_gemm_f32;
        check_status(fn(A.ptr<float>(), B.ptr<float>(), C, M, N, K, static_cast<int>(transA), static_cast<int>(transB),
                        alpha, beta, c_ndim, d0, d1, Y.ptr<float>(), stream_),
                     relu ? "Gemm + Relu" : "Gemm");
    }
};

class MatMul : public StreamOperator {
public:
    MatMul() : StreamOperator("MatMul") {}
    void forward(Span in, Span out) override {
        const ITensor &A = in[0].get(), &B = in[1].get();
        ITensor &Y = out[0].get();
        require(A.dtype() == DataType::FLOAT && B.dtype() == DataType::FLOAT, "MatMul: unfused MatMul runs in FLOAT");
        require(A.ndim() >= 1 && B.ndim() >= 1, "MatMul: scalar operands");
        // numpy matmul semantics (mat_mul.cpp:51-303): a 1-D A is [1, K], a 1-D B is [K, 1]
        // (the extra dimension does not appear in Y); batch dimensions broadcast
        const int64_t M = A.ndim() >= 2 ? A.shape(A.ndim() - 2) : 1, K = A.shape(A.ndim() - 1);
        const int64_t N = B.ndim() >= 2 ? B.shape(B.ndim() - 1) : 1;
        require((B.ndim() >= 2 ? B.shape(B.ndim() - 2) : B.shape(0)) == K, "MatMul: inner dimensions mismatch");
        const size_t ba = A.ndim() > 2 ? A.ndim() - 2 : 0, bb = B.ndim() > 2 ? B.ndim() - 2 : 0;
        const size_t nb = std::max(ba, bb);
        std::vector<int64_t> da(nb, 1), db(nb, 1), dy(nb, 1);
        for (size_t i = 0; i < ba; ++i) da[nb - ba + i] = A.shape(i);
        for (size_t i = 0; i < bb; ++i) db[nb - bb + i] = B.shape(i);
        for (size_t i = 0; i < nb; ++i) {
            require(da[i] == db[i] || da[i] == 1 || db[i] == 1, "MatMul: batch dimensions do not broadcast");
            dy[i] = std::max(da[i], db[i]);
        }
        int64_t batchY = 1, batchB = 1;
        for (size_t i = 0; i < nb; ++i) {
            batchY *= dy[i];
            batchB *= db[i];
        }
        require(Y.size() == batchY * M * N, "MatMul: Y shape mismatch");
        if (batchB == 1) {  // a 2-D right operand: A's batch folds into rows, one GEMM
            int64_t batchA = 1;
            for (auto d : da) batchA *= d;
            require(batchA == batchY, "MatMul: Y shape mismatch");
            check_status(lcml_gemm_f32(A.ptr<float>(), B.ptr<float>(), nullptr, batchY * M, N, K, 0, 0, 1.0f, 0.0f, -1, 0,
                                       0, Y.ptr<float>(), stream_),
                         "MatMul");
            return;
        }
        // one GEMM per output batch, operands found through broadcast strides
        std::vector<int64_t> sa(nb, 0), sb(nb, 0);
        for (int64_t i = static_cast<int64_t>(nb) - 1, accA = M * K, accB = K * N; i >= 0; --i) {
            sa[i] = da[i] == 1 ? 0 : accA;
            sb[i] = db[i] == 1 ? 0 : accB;
            accA *= da[i];
            accB *= db[i];
        }
        for (int64_t by = 0; by < batchY; ++by) {
            int64_t oa = 0, ob = 0, r = by;
            for (int64_t i = static_cast<int64_t>(nb) - 1; i >= 0; --i) {
                const int64_t c = r % dy[i];
                r /= dy[i];
                oa += c * sa[i];
                ob += c * sb[i];
            }
            check_status(lcml_gemm_f32(A.ptr<float>() + oa, B.ptr<float>() + ob, nullptr, M, N, K, 0, 0, 1.0f, 0.0f, -1, 0,
                                       0, Y.ptr<float>() + by * M * N, stream_),
                         "MatMul");
        }
    }
};

// ------------------------------------------------------------------ elementwise
class Unary : public StreamOperator {
    int op_;

public:
    Unary(const char *name, int op) : StreamOperator(name), op_(op) {}
    bool can_operate_inplace() const override { return true; }
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get();
        ITensor &y = out[0].get();
        require(x.dtype() == DataType::FLOAT && y.dtype() == DataType::FLOAT, get_name() + ": FLOAT only on this path");
        check_status(lcml_unary_f32(op_, x.ptr<float>(), y.ptr<float>(), x.size(), stream_), get_name().c_str());
    }
};

// true when b's shape broadcasts over a's trailing dimensions (b_n divides a_n)
bool trailing_broadcast(const ITensor &a, const ITensor &b) {
    std::vector<int64_t> bs = b.shape();
    while (!bs.empty() && bs.front() == 1) bs.erase(bs.begin());
    if (static_cast<int64_t>(bs.size()) > a.ndim()) return false;
    for (size_t i = 0; i < bs.size(); ++i)
        if (bs[bs.size() - 1 - i] != a.shape(a.ndim() - 1 - i)) return false;
    return true;
}

class Binary : public StreamOperator {
    int op_;

public:
    Binary(const char *name, int op) : StreamOperator(name), op_(op) {}
    bool can_operate_inplace() const override { return true; }
    void forward(Span in, Span out) override {
        const ITensor *a = &in[0].get(), *b = &in[1].get();
        ITensor &y = out[0].get();
        const DataType t = a->dtype();
        const bool fp8 = t == DataType::FLOAT8E4M3FN || t == DataType::FLOAT8E5M2;
        require((t == DataType::FLOAT || fp8) && b->dtype() == t && y.dtype() == t,
                get_name() + ": FLOAT, FLOAT8E4M3FN or FLOAT8E5M2 operands of one type");
        if (a->size() < b->size()) {
            require(op_ == 0 || op_ == 2, get_name() + ": left-operand broadcast is supported for Add and Mul only");
            std::swap(a, b);
        }
        require(trailing_broadcast(*a, *b), get_name() + ": unsupported broadcast");
        require(y.size() == a->size(), get_name() + ": output shape mismatch");
        if (fp8)  // decode -> half op -> encode (binary.cpp:185-283)
            check_status(lcml_binary_fp8(op_, a->ptr<uint8_t>(), b->ptr<uint8_t>(), a->size(), b->size(),
                                         y.ptr<uint8_t>(), static_cast<int>(t), stream_),
                         get_name().c_str());
        else
            check_status(lcml_binary_f32(op_, a->ptr<float>(), b->ptr<float>(), a->size(), b->size(), y.ptr<float>(),
                                         stream_),
                         get_name().c_str());
    }
};

class ReduceMax : public StreamOperator {
    std::vector<int64_t> axes_;

public:
    explicit ReduceMax(std::vector<int64_t> axes) : StreamOperator("ReduceMax"), axes_(std::move(axes)) {}
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get();
        ITensor &y = out[0].get();
        std::vector<int64_t> axes = axes_;
        if (axes.empty() && in.size() > 1 && in[1].get().host_data()) {
            const std::string &h = *in[1].get().host_data();
            axes.resize(h.size() / 8);
            std::memcpy(axes.data(), h.data(), axes.size() * 8);
        }
        require(axes.size() == 1 && norm_axis(axes[0], x.ndim()) == x.ndim() - 1, "ReduceMax: only the last axis is supported");
        require(x.dtype() == DataType::FLOAT, "ReduceMax: FLOAT only on this path");
        const int64_t cols = x.shape(x.ndim() - 1);
        check_status(lcml_reduce_max_rows(x.ptr<float>(), x.size() / cols, cols, 0, y.ptr<float>(), stream_), "ReduceMax");
    }
};

class Softmax : public StreamOperator {
    int64_t axis_;

public:
    explicit Softmax(int64_t axis) : StreamOperator("Softmax"), axis_(axis) {}
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get();
        ITensor &y = out[0].get();
        require(norm_axis(axis_, x.ndim()) == x.ndim() - 1, "Softmax: only the last axis is supported");
        const DataType t = x.dtype();
        require((t == DataType::FLOAT || t == DataType::FLOAT8E4M3FN || t == DataType::FLOAT8E5M2) && y.dtype() == t,
                "Softmax: FLOAT, FLOAT8E4M3FN or FLOAT8E5M2, the same type in and out");
        const int64_t cols = x.shape(x.ndim() - 1);
        if (t == DataType::FLOAT)
            check_status(lcml_softmax_rows(x.ptr<float>(), x.size() / cols, cols, y.ptr<float>(), stream_), "Softmax");
        else  // decode -> softmax -> encode (softmax.cpp:245-280)
            check_status(lcml_softmax_rows_fp8(x.ptr<uint8_t>(), x.size() / cols, cols, y.ptr<uint8_t>(),
                                               static_cast<int>(t), stream_),
                         "Softmax");
    }
};

class MaxPool : public StreamOperator {
    std::vector<int64_t> kernel_, strides_, pads_, dilations_;

public:
    MaxPool(std::vector<int64_t> k, std::vector<int64_t> s, std::vector<int64_t> p, std::vector<int64_t> d)
        : StreamOperator("MaxPool"), kernel_(std::move(k)), strides_(std::move(s)), pads_(std::move(p)), dilations_(std::move(d)) {}
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get();
        ITensor &y = out[0].get();
        require(x.ndim() == 4 && kernel_.size() == 2, "MaxPool: 2-D NCHW only");
        for (auto d : dilations_) require(d == 1, "MaxPool: dilation must be 1");
        const int sH = strides_.size() > 0 ? static_cast<int>(strides_[0]) : 1;
        const int sW = strides_.size() > 1 ? static_cast<int>(strides_[1]) : 1;
        const int pH = pads_.size() > 0 ? static_cast<int>(pads_[0]) : 0;
        const int pW = pads_.size() > 1 ? static_cast<int>(pads_[1]) : 0;
        require(x.dtype() == DataType::FLOAT || x.dtype() == DataType::FLOAT8E4M3FN, "MaxPool: FLOAT or FLOAT8E4M3FN");
        check_status(lcml_maxpool2d(x.data(), static_cast<int>(x.dtype()), x.shape(0) * x.shape(1), x.shape(2), x.shape(3),
                                    static_cast<int>(kernel_[0]), static_cast<int>(kernel_[1]), sH, sW, pH, pW, y.shape(2),
                                    y.shape(3), y.data(), 0, x.shape(1), stream_),
                     "MaxPool");
    }
};

class GlobalAveragePool : public StreamOperator {
public:
    GlobalAveragePool() : StreamOperator("GlobalAveragePool") {}
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get();
        ITensor &y = out[0].get();
        require(x.ndim() == 4 && y.dtype() == DataType::FLOAT, "GlobalAveragePool: NCHW input, FLOAT output");
        require(x.dtype() == DataType::FLOAT || x.dtype() == DataType::BFLOAT16, "GlobalAveragePool: FLOAT or BFLOAT16 input");
        check_status(lcml_global_avgpool(x.data(), static_cast<int>(x.dtype()), nullptr, x.shape(0), x.shape(1),
                                         x.shape(2) * x.shape(3), 0, y.ptr<float>(), stream_),
                     "GlobalAveragePool");
    }
};

// Flatten / Reshape / Identity: the output shares the input's storage when the
// executor could alias it; otherwise the bytes are copied.
class ViewOp : public StreamOperator {
public:
    explicit ViewOp(const char *name) : StreamOperator(name) {}
    bool is_output_view(size_t, const Node &) const override { return true; }
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get();
        ITensor &y = out[0].get();
        require(x.nbytes() == y.nbytes(), get_name() + ": size mismatch");
        if (x.data() != y.data())
            check_status(lcml_memcpy_async(y.data(), x.data(), x.nbytes(), 3, stream_), get_name().c_str());
    }
};

class Cast : public StreamOperator {
public:
    Cast() : StreamOperator("Cast") {}
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get();
        ITensor &y = out[0].get();
        if (x.dtype() == y.dtype()) {
            if (x.data() != y.data()) check_status(lcml_memcpy_async(y.data(), x.data(), x.nbytes(), 3, stream_), "Cast");
            return;
        }
        check_status(lcml_cast(x.data(), static_cast<int>(x.dtype()), y.data(), static_cast<int>(y.dtype()), x.size(), stream_),
                     "Cast");
    }
};

// Conv (src/onnx/operators/conv.cpp:35-255). fp32 tensors run the direct
// kernel lcml_conv2d_f32 (1-D or 2-D, group, strides, begin pads,
// dilations, optional bias); DequantizeLinear-fed FP8 convs are taken by the
// fusion pass (FusedQdqConv) before they get here.
class Conv : public StreamOperator {
    std::vector<int64_t> strides_, pads_, dilations_;
    int64_t group_;

public:
    Conv(std::vector<int64_t> strides, std::vector<int64_t> pads, std::vector<int64_t> dilations, int64_t group)
        : StreamOperator("Conv"), strides_(std::move(strides)), pads_(std::move(pads)),
          dilations_(std::move(dilations)), group_(group) {}
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get(), &w = in[1].get();
        ITensor &y = out[0].get();
        require(x.dtype() == DataType::FLOAT && w.dtype() == DataType::FLOAT && y.dtype() == DataType::FLOAT,
                "Conv: fp32 tensors here; FP8 convs run fused (DequantizeLinear -> Conv -> QuantizeLinear)");
        const size_t sd = x.ndim() - 2;  // spatial dims: 1 or 2
        require((sd == 1 || sd == 2) && w.ndim() == x.ndim() && y.ndim() == x.ndim(),
                "Conv: only 1D and 2D convolution are supported");
        const ITensor *b = in.size() > 2 ? &in[2].get() : nullptr;
        require(!b || (b->dtype() == DataType::FLOAT && b->size() == w.shape(0)), "Conv: bias must be fp32 [M]");
        auto at = [](const std::vector<int64_t> &v, size_t i, int64_t dflt) { return i < v.size() ? v[i] : dflt; };
        // a 1-D conv is the 2-D one with H = kH = oH = 1
        const int64_t H = sd == 2 ? x.shape(2) : 1, W = x.shape(sd + 1);
        const int64_t kH = sd == 2 ? w.shape(2) : 1, kW = w.shape(sd + 1);
        const int64_t oH = sd == 2 ? y.shape(2) : 1, oW = y.shape(sd + 1);
        const int sH = sd == 2 ? static_cast<int>(at(strides_, 0, 1)) : 1;
        const int sW = static_cast<int>(at(strides_, sd - 1, 1));
        const int pH = sd == 2 ? static_cast<int>(at(pads_, 0, 0)) : 0;  // begin pads (conv.cpp:119-121)
        const int pW = static_cast<int>(at(pads_, sd - 1, 0));
        const int dH = sd == 2 ? static_cast<int>(at(dilations_, 0, 1)) : 1;
        const int dW = static_cast<int>(at(dilations_, sd - 1, 1));
        check_status(lcml_conv2d_f32(x.ptr<float>(), w.ptr<float>(), b ? b->ptr<float>() : nullptr, x.shape(0),
                                     x.shape(1), H, W, w.shape(0), kH, kW, oH, oW, sH, sW, pH, pW, dH, dW,
                                     static_cast<int>(group_), y.ptr<float>(), stream_),
                     "Conv");
    }
};

// ConvTranspose (src/onnx/operators/conv_transpose.cpp:37-283), fp32, 2-D:
// the gather kernel lcml_conv_transpose2d_f32; the output extent (pads and
// output_padding) is the one the graph declares for Y.
class ConvTranspose : public StreamOperator {
    std::vector<int64_t> strides_, pads_, dilations_;
    int64_t group_;

public:
    ConvTranspose(std::vector<int64_t> strides, std::vector<int64_t> pads, std::vector<int64_t> dilations,
                  int64_t group)
        : StreamOperator("ConvTranspose"), strides_(std::move(strides)), pads_(std::move(pads)),
          dilations_(std::move(dilations)), group_(group) {}
    void forward(Span in, Span out) override {
        const ITensor &x = in[0].get(), &w = in[1].get();
        ITensor &y = out[0].get();
        require(x.dtype() == DataType::FLOAT && w.dtype() == DataType::FLOAT && y.dtype() == DataType::FLOAT,
                "ConvTranspose: fp32 tensors");
        require(x.ndim() == 4 && w.ndim() == 4 && y.ndim() == 4, "ConvTranspose: only 2D is supported");
        const ITensor *b = in.size() > 2 ? &in[2].get() : nullptr;
        require(!b || (b->dtype() == DataType::FLOAT && b->size() == y.shape(1)), "ConvTranspose: bias must be fp32 [M]");
        require(w.shape(0) == x.shape(1) && w.shape(1) * group_ == y.shape(1), "ConvTranspose: W must be [C, M/group, kH, kW]");
        auto at = [](const std::vector<int64_t> &v, size_t i, int64_t dflt) { return i < v.size() ? v[i] : dflt; };
        check_status(lcml_conv_transpose2d_f32(x.ptr<float>(), w.ptr<float>(), b ? b->ptr<float>() : nullptr, x.shape(0),
                                               x.shape(1), x.shape(2), x.shape(3), y.shape(1), w.shape(2), w.shape(3),
                                               y.shape(2), y.shape(3), static_cast<int>(at(strides_, 0, 1)),
                                               static_cast<int>(at(strides_, 1, 1)), static_cast<int>(at(pads_, 0, 0)),
                                               static_cast<int>(at(pads_, 1, 0)), static_cast<int>(at(dilations_, 0, 1)),
                                               static_cast<int>(at(dilations_, 1, 1)), static_cast<int>(group_),
                                               y.ptr<float>(), stream_),
                     "ConvTranspose");
    }
};

}// namespace

// ------------------------------------------------------------------ fused QDQ GEMM
void FusedQdqGemm::forward(Span in, Span out) {
    const ITensor &A = in[0].get(), &sa = in[1].get(), &B = in[2].get(), &sb = in[3].get();
    ITensor &Y = out[0].get();
    require(A.dtype() == DataType::FLOAT8E4M3FN && B.dtype() == DataType::FLOAT8E4M3FN, "fused Gemm: operands must be e4m3");
    const int64_t K = A.shape(A.ndim() - 1);
    const int64_t M = A.size() / K;
    const int64_t N = b_kmajor ? B.shape(0) : B.shape(B.ndim() - 1);
    require((b_kmajor ? B.shape(1) : B.shape(0)) == K, "fused Gemm: inner dimensions mismatch");
    lcml_fp8_gemm_desc d{};
    d.M = M;
    d.N = N;
    d.K = K;
    d.A = A.ptr<uint8_t>();
    d.lda = K;
    d.B = B.ptr<uint8_t>();
    d.ldb = b_kmajor ? K : N;
    d.b_kmajor = b_kmajor;
    d.scale_a = sa.ptr<float>();
    d.scale_a_mode = sa.size() > 1 ? LCML_SCALE_ROW : LCML_SCALE_TENSOR;
    d.scale_b = sb.ptr<float>();
    d.scale_b_mode = sb.size() > 1 ? LCML_SCALE_COL : LCML_SCALE_TENSOR;
    d.alpha = alpha;
    d.beta = beta;
    size_t next = 4;
    if (has_c) {
        const ITensor &C = in[next++].get();
        if (C.size() == M * N && C.ndim() == 2 && C.shape(0) == M) {
            d.c_mat = C.data();
            d.c_mat_dtype = static_cast<int>(C.dtype());
            d.ldc = N;
        } else {
            require(C.dtype() == DataType::FLOAT, "fused Gemm: broadcast C must be FLOAT");
            d.c_vec = C.ptr<float>();
            d.c_vec_mode = C.size() == 1 ? LCML_SCALE_TENSOR : (C.size() == N ? LCML_SCALE_COL : LCML_SCALE_ROW);
            require(C.size() == 1 || C.size() == N || C.size() == M, "fused Gemm: C does not broadcast");
        }
    }
    if (has_y_scale) d.y_scale = in[next++].get().ptr<float>();
    d.epilogue = epilogue;
    d.Y = Y.data();
    d.y_dtype = static_cast<int>(Y.dtype());
    d.ldy = epilogue == LCML_EPI_SILU_MUL ? N / 2 : N;
    if (row_quant) {
        ITensor &q = out[1].get(), &s = out[2].get();
        check_status(lcml_fp8_gemm_rowquant(&d, q.ptr<uint8_t>(), s.ptr<float>(), static_cast<float *>(workspace), stream_),
                     "fused Gemm + row quantization");
        return;
    }
    check_status(lcml_fp8_gemm(&d, stream_), "fused Gemm");
}

void DynamicRowQuant::forward(Span in, Span out) {
    const ITensor &x = in[0].get();
    ITensor &q = out[0].get(), &s = out[1].get();
    require(x.dtype() == DataType::FLOAT && x.ndim() == 2, "dynamic row quantization: 2-D FLOAT input");
    require(q.dtype() == DataType::FLOAT8E4M3FN && s.size() == x.shape(0), "dynamic row quantization: outputs");
    check_status(lcml_fp8_quantize_rows_dynamic(x.ptr<float>(), x.shape(0), x.shape(1), x.shape(1), s.ptr<float>(),
                                                q.ptr<uint8_t>(), stream_),
                 "dynamic row quantization");
}

void FusedQdqConv::forward(Span in, Span out) {
    size_t i = 0;
    const ITensor &x = in[i++].get(), &sx = in[i++].get(), &wp = in[i++].get(), &sw = in[i++].get();
    ITensor &y = out[0].get();
    require(x.dtype() == DataType::FLOAT8E4M3FN && wp.dtype() == DataType::FLOAT8E4M3FN, "fused Conv: e4m3 operands");
    require(y.dtype() == DataType::FLOAT8E4M3FN, "fused Conv: e4m3 output");
    lcml_fp8_conv_desc d = desc;
    d.X = x.ptr<uint8_t>();
    d.scale_x = sx.ptr<float>();
    d.Wp = wp.ptr<uint8_t>();
    d.scale_w = sw.ptr<float>();
    d.scale_w_mode = sw.size() > 1 ? LCML_SCALE_AXIS : LCML_SCALE_TENSOR;
    if (has_bias) d.bias = in[i++].get().ptr<float>();
    if (has_residual) {
        const ITensor &r = in[i++].get(), &rs = in[i++].get();
        require(r.dtype() == DataType::FLOAT8E4M3FN && r.size() == y.size(), "fused Conv: residual shape");
        d.residual = r.data();
        d.residual_dtype = LCML_DTYPE_FLOAT8E4M3FN;
        d.residual_scale = rs.ptr<float>();
    }
    d.y_scale = in[i++].get().ptr<float>();
    d.Y = y.data();
    d.y_dtype = LCML_DTYPE_FLOAT8E4M3FN;
    d.workspace = workspace;
    check_status(lcml_fp8_conv(&d, stream_), "fused Conv");
}

void QdqMaxPool::forward(Span in, Span out) {
    const ITensor &x = in[0].get();
    ITensor &y = out[0].get();
    require(x.ndim() == 4 && x.dtype() == DataType::FLOAT8E4M3FN && y.dtype() == DataType::FLOAT8E4M3FN,
            "e4m3 MaxPool: 4-D e4m3 input and output");
    check_status(lcml_maxpool2d(x.data(), LCML_DTYPE_FLOAT8E4M3FN, x.shape(0) * x.shape(1), x.shape(2), x.shape(3), kH, kW,
                                sH, sW, pH, pW, y.shape(2), y.shape(3), y.data(), nhwc ? 1 : 0, x.shape(1), stream_),
                 "e4m3 MaxPool");
}

void QdqGlobalAveragePool::forward(Span in, Span out) {
    const ITensor &x = in[0].get(), &sx = in[1].get();
    ITensor &y = out[0].get();
    require(x.ndim() == 4 && x.dtype() == DataType::FLOAT8E4M3FN && y.dtype() == DataType::FLOAT,
            "e4m3 GlobalAveragePool: 4-D e4m3 input, FLOAT output");
    check_status(lcml_global_avgpool(x.data(), LCML_DTYPE_FLOAT8E4M3FN, sx.ptr<float>(), x.shape(0), x.shape(1),
                                     x.shape(2) * x.shape(3), nhwc ? 1 : 0, y.ptr<float>(), stream_),
                 "e4m3 GlobalAveragePool");
}

// ------------------------------------------------------------------ registration
REGISTER_TO_DEFAULT_OPSET(QuantizeLinear) { return std::make_unique<QuantizeLinear>(get_int(node, "axis", 1)); };
REGISTER_TO_DEFAULT_OPSET(DequantizeLinear) { return std::make_unique<DequantizeLinear>(get_int(node, "axis", 1)); };
std::unique_ptr<Operator> make_gemm_f32_relu(const Node &node) {
    auto g = std::make_unique<Gemm>(get_float(node, "alpha", 1.0f), get_float(node, "beta", 1.0f),
                                    get_int(node, "transA", 0), get_int(node, "transB", 0));
    g->relu = true;
    return g;
}

REGISTER_TO_DEFAULT_OPSET(Gemm) {
    return std::make_unique<Gemm>(get_float(node, "alpha", 1.0f), get_float(node, "beta", 1.0f), get_int(node, "transA", 0),
                                  get_int(node, "transB", 0));
};
REGISTER_TO_DEFAULT_OPSET(MatMul) { return std::make_unique<MatMul>(); };
REGISTER_TO_DEFAULT_OPSET(Conv) {
    if (auto p = node.try_get_attr("auto_pad")) {
        const std::string s = p->get<AttributeType::STRING>();
        if (!s.empty() && s != "NOTSET") throw Error("Conv: auto_pad " + s + " is not supported (explicit pads only)");
    }
    return std::make_unique<Conv>(get_ints(node, "strides"), get_ints(node, "pads"), get_ints(node, "dilations"),
                                  get_int(node, "group", 1));
};
REGISTER_TO_DEFAULT_OPSET(ConvTranspose) {
    if (auto p = node.try_get_attr("auto_pad")) {
        const std::string s = p->get<AttributeType::STRING>();
        if (!s.empty() && s != "NOTSET")
            throw Error("ConvTranspose: auto_pad " + s + " is not supported (explicit pads only)");
    }
    return std::make_unique<ConvTranspose>(get_ints(node, "strides"), get_ints(node, "pads"),
                                           get_ints(node, "dilations"), get_int(node, "group", 1));
};
REGISTER_TO_DEFAULT_OPSET(Relu) { return std::make_unique<Unary>("Relu", 0); };
REGISTER_TO_DEFAULT_OPSET(Sigmoid) { return std::make_unique<Unary>("Sigmoid", 1); };
REGISTER_TO_DEFAULT_OPSET(Abs) { return std::make_unique<Unary>("Abs", 2); };
REGISTER_TO_DEFAULT_OPSET(Add) { return std::make_unique<Binary>("Add", 0); };
REGISTER_TO_DEFAULT_OPSET(Sub) { return std::make_unique<Binary>("Sub", 1); };
REGISTER_TO_DEFAULT_OPSET(Mul) { return std::make_unique<Binary>("Mul", 2); };
REGISTER_TO_DEFAULT_OPSET(Div) { return std::make_unique<Binary>("Div", 3); };
REGISTER_TO_DEFAULT_OPSET(ReduceMax) { return std::make_unique<ReduceMax>(get_ints(node, "axes")); };
REGISTER_TO_DEFAULT_OPSET(Softmax) { return std::make_unique<Softmax>(get_int(node, "axis", -1)); };
REGISTER_TO_DEFAULT_OPSET(MaxPool) {
    return std::make_unique<MaxPool>(get_ints(node, "kernel_shape"), get_ints(node, "strides"), get_ints(node, "pads"),
                                     get_ints(node, "dilations"));
};
REGISTER_TO_DEFAULT_OPSET(GlobalAveragePool) { return std::make_unique<GlobalAveragePool>(); };
REGISTER_TO_DEFAULT_OPSET(Flatten) { return std::make_unique<ViewOp>("Flatten"); };
REGISTER_TO_DEFAULT_OPSET(Reshape) { return std::make_unique<ViewOp>("Reshape"); };
REGISTER_TO_DEFAULT_OPSET(Identity) { return std::make_unique<ViewOp>("Identity"); };
REGISTER_TO_DEFAULT_OPSET(Cast) { return std::make_unique<Cast>(); };

// Forces the registrations above into any binary that links this library.
int operators_registered() { return static_cast<int>(OperatorSet::get_default().operator_names().size()); }

}// namespace lcml::onnx
