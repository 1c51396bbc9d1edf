// lcml_onnx.h — C++ host side of the B200 FP8 operator path.
//
// Mirrors LuisaML's ONNX API so that code written against it keeps working:
//   Model / Graph / Node / Variable / Attribute   include/onnx/onnx.h:31-421
//   OperatorSet + REGISTER_TO_DEFAULT_OPSET       include/onnx/onnx.h:338-385
//   Operator (forward, is_output_view, ...)       include/onnx/operator.h:16-54
//   ITensor / TensorTable                         include/onnx/tensor.h:24-160, tensor_table.h:22-214
//   NetworkInstance                               include/onnx/network_instance.h:37-298
// What changes: tensor storage is a device pointer (not a LuisaCompute DSL
// array), and Operator::forward enqueues CUDA work on the instance's stream
// through the C ABI of lcml_fp8.h instead of emitting shader AST. Fatal
// conditions the reference asserts on (LUISA_ASSERT) throw lcml::onnx::Error.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <span>
#include <stdexcept>
#include <string>
#include <string_view>
#include <unordered_map>
#include <variant>
#include <vector>

#include "lcml_fp8.h"

namespace lcml::onnx {

class Error : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

// ONNX TensorProto.DataType (include/onnx/onnx.h:31-60).
enum class DataType : int {
    UNDEFINED = 0, FLOAT = 1, UINT8 = 2, INT8 = 3, UINT16 = 4, INT16 = 5, INT32 = 6, INT64 = 7, STRING = 8,
    BOOL = 9, FLOAT16 = 10, DOUBLE = 11, UINT32 = 12, UINT64 = 13, COMPLEX64 = 14, COMPLEX128 = 15,
    BFLOAT16 = 16, FLOAT8E4M3FN = 17, FLOAT8E4M3FNUZ = 18, FLOAT8E5M2 = 19, FLOAT8E5M2FNUZ = 20, UINT4 = 21,
    INT4 = 22, FLOAT4E2M1 = 23, FLOAT8E8M0 = 24, UINT2 = 25, INT2 = 26, FLOAT16QUANTIZED = 27,
};

enum class AttributeType : int {
    UNDEFINED = 0, FLOAT = 1, INT = 2, STRING = 3, TENSOR = 4, GRAPH = 5, FLOATS = 6, INTS = 7, STRINGS = 8,
    TENSORS = 9, GRAPHS = 10, SPARSE_TENSOR = 11, SPARSE_TENSORS = 12, TYPE_PROTO = 13, TYPE_PROTOS = 14,
};

const char *dtype_name(DataType t);
DataType dtype_from_name(std::string_view name);  // "FLOAT", "FLOAT8E4M3FN", ...
size_t dtype_size(DataType t);                     // bytes per element (0: unsupported here; 0 for packed FP4)
// Bytes of n elements: n * dtype_size, or (n + 1) / 2 for FLOAT4E2M1 (two codes
// per byte, element 2i in the low nibble of byte i, as the reference's FP4Data).
size_t dtype_nbytes(DataType t, size_t n);

class Graph;
class OperatorSet;

class Attribute : public std::variant<float, int64_t, std::string, std::shared_ptr<Graph>, std::vector<float>,
                                      std::vector<int64_t>, std::vector<std::string>,
                                      std::vector<std::shared_ptr<Graph>>> {
    std::string name_;

public:
    using variant::variant;
    Attribute() = default;
    template <typename T>
    Attribute(std::string name, T &&value) : variant(std::forward<T>(value)), name_(std::move(name)) {}
    const std::string &get_name() const { return name_; }
    static AttributeType type_of(const Attribute &a);
    template <AttributeType T>
    const auto &get() const {
        if constexpr (T == AttributeType::FLOAT) return std::get<0>(*this);
        else if constexpr (T == AttributeType::INT) return std::get<1>(*this);
        else if constexpr (T == AttributeType::STRING) return std::get<2>(*this);
        else if constexpr (T == AttributeType::GRAPH) return std::get<3>(*this);
        else if constexpr (T == AttributeType::FLOATS) return std::get<4>(*this);
        else if constexpr (T == AttributeType::INTS) return std::get<5>(*this);
        else if constexpr (T == AttributeType::STRINGS) return std::get<6>(*this);
        else return std::get<7>(*this);
    }
};

class Variable {
    std::string name_;
    DataType dtype_ = DataType::UNDEFINED;
    std::vector<size_t> shape_;
    std::string raw_data_;
    uint64_t buffer_start_ = 0, buffer_end_ = 0;
    bool is_constant_ = false;

public:
    Variable() = default;
    Variable(std::string name, DataType dtype, std::vector<size_t> shape, std::string raw_data = {},
             uint64_t buffer_start = 0, uint64_t buffer_end = 0)
        : name_(std::move(name)), dtype_(dtype), shape_(std::move(shape)), raw_data_(std::move(raw_data)),
          buffer_start_(buffer_start), buffer_end_(buffer_end) {}
    const std::string &get_name() const { return name_; }
    DataType get_dtype() const { return dtype_; }
    const std::vector<size_t> &get_shape() const { return shape_; }
    const std::string &get_raw_data() const { return raw_data_; }
    bool is_trainable_weight() const { return buffer_end_ > buffer_start_; }
    std::pair<uint64_t, uint64_t> get_buffer_range() const { return {buffer_start_, buffer_end_}; }
    void set_is_constant(bool v) { is_constant_ = v; }
    bool is_constant() const { return is_constant_; }
    void set_shape(std::vector<size_t> s) { shape_ = std::move(s); }
    void set_dtype(DataType t) { dtype_ = t; }
};

class Node {
    std::string name_, op_type_;
    std::vector<const Variable *> inputs_, outputs_;
    std::map<std::string, Attribute, std::less<>> attributes_;

public:
    Node() = default;
    Node(std::string name, std::string op_type) : name_(std::move(name)), op_type_(std::move(op_type)) {}
    const std::string &get_name() const { return name_; }
    const std::string &get_op_type() const { return op_type_; }
    const std::vector<const Variable *> &get_inputs() const { return inputs_; }
    const std::vector<const Variable *> &get_outputs() const { return outputs_; }
    const std::map<std::string, Attribute, std::less<>> &get_attributes() const { return attributes_; }
    void add_input(const Variable &v) { inputs_.push_back(&v); }
    void add_output(const Variable &v) { outputs_.push_back(&v); }
    void set_attribute(Attribute a) { attributes_.emplace(a.get_name(), std::move(a)); }
    bool has_attribute(std::string_view n) const { return attributes_.find(n) != attributes_.end(); }
    const Attribute &get_attribute(std::string_view n) const;
    const Attribute *try_get_attr(std::string_view n) const {
        auto it = attributes_.find(n);
        return it == attributes_.end() ? nullptr : &it->second;
    }
};

class Graph {
    std::string name_;
    const Graph *parent_ = nullptr;
    std::map<std::string, std::unique_ptr<Variable>, std::less<>> variables_;  // stable addresses
    std::vector<const Variable *> inputs_, outputs_;
    std::vector<Node> nodes_;

public:
    Graph() = default;
    explicit Graph(std::string name) : name_(std::move(name)) {}
    Variable &add_variable(Variable &&v);
    const Variable &get_var(std::string_view name) const;
    Variable *find_var(std::string_view name);
    void add_input(std::string_view name) { inputs_.push_back(&get_var(name)); }
    void add_output(std::string_view name) { outputs_.push_back(&get_var(name)); }
    void add_node(Node &&n) { nodes_.push_back(std::move(n)); }
    void set_parent(const Graph *p) { parent_ = p; }
    const Graph *parent() const { return parent_; }
    const std::string &get_name() const { return name_; }
    const std::map<std::string, std::unique_ptr<Variable>, std::less<>> &get_variables() const { return variables_; }
    const std::vector<const Variable *> &get_inputs() const { return inputs_; }
    const std::vector<const Variable *> &get_outputs() const { return outputs_; }
    const std::vector<Node> &get_nodes() const { return nodes_; }
    void mark_constants();
    static Graph from_json_text(std::string_view json, const OperatorSet &opset);
};

class ITensor;
class TensorTable;
class NetworkInstance;

class Operator {
    std::string name_;

public:
    explicit Operator(std::string name) : name_(std::move(name)) {}
    virtual ~Operator() = default;
    const std::string &get_name() const { return name_; }
    virtual void forward(std::span<std::reference_wrapper<ITensor>> inputs,
                         std::span<std::reference_wrapper<ITensor>> outputs) = 0;
    virtual bool is_output_view(size_t, const Node &) const { return false; }
    virtual bool can_operate_inplace() const { return false; }
    virtual bool need_outline() const { return true; }
    virtual void set_environment(NetworkInstance &, TensorTable &) {}
    virtual void set_warp_size(uint32_t) {}
};

class OperatorSet {
public:
    using Factory = std::function<std::unique_ptr<Operator>(const Node &)>;

private:
    std::string domain_;
    int64_t version_;
    std::map<std::string, Factory, std::less<>> factories_;

public:
    OperatorSet(std::string domain, int64_t version) : domain_(std::move(domain)), version_(version) {}
    const std::string &get_domain() const { return domain_; }
    int64_t get_version() const { return version_; }
    void register_operator(std::string name, Factory f) { factories_.insert_or_assign(std::move(name), std::move(f)); }
    std::unique_ptr<Operator> create_operator(std::string_view name, const Node &node) const;
    bool has_operator(std::string_view name) const { return factories_.find(name) != factories_.end(); }
    std::vector<std::string> operator_names() const;
    static OperatorSet &get_default();

    struct RegHelper {
        std::string name;
        OperatorSet &opset;
        explicit RegHelper(std::string n, OperatorSet &s = OperatorSet::get_default()) : name(std::move(n)), opset(s) {}
        bool operator<<(Factory f) {
            opset.register_operator(std::move(name), std::move(f));
            return true;
        }
    };
};

#ifndef REGISTER_TO_DEFAULT_OPSET
#define REGISTER_TO_DEFAULT_OPSET(name)                                                             \
    [[maybe_unused]] static auto _RegOp##name = ::lcml::onnx::OperatorSet::RegHelper(#name) << []( \
                                                    [[maybe_unused]] ::lcml::onnx::Node const &node)
#endif

class Model {
    int64_t ir_version_ = 0;
    std::string producer_name_, producer_version_;
    std::shared_ptr<Graph> graph_ = std::make_shared<Graph>();
    OperatorSet *opset_ = &OperatorSet::get_default();

public:
    Model() = default;
    Model(int64_t ir, std::string pn, std::string pv)
        : ir_version_(ir), producer_name_(std::move(pn)), producer_version_(std::move(pv)) {}
    void set_graph(Graph &&g) {
        graph_ = std::make_shared<Graph>(std::move(g));
        graph_->mark_constants();
    }
    const Graph &get_graph() const { return *graph_; }
    Graph &mutable_graph() { return *graph_; }
    OperatorSet &get_opset() const { return *opset_; }
    void set_opset(OperatorSet &s) { opset_ = &s; }
    int64_t get_ir_version() const { return ir_version_; }
    const std::string &get_producer_name() const { return producer_name_; }
    const std::string &get_producer_version() const { return producer_version_; }
    static Model load_from_json(std::string_view json);
};

// ---------------------------------------------------------------------------
// Tensors: shape + dtype + device pointer. Constants loaded from the model
// also keep a host copy (used for shape/axes inputs and scalar scales).
// ---------------------------------------------------------------------------
class ITensor {
public:
    using size_type = int64_t;
    using shape_type = std::vector<int64_t>;

protected:
    shape_type shape_;
    DataType dtype_ = DataType::UNDEFINED;

public:
    ITensor() = default;
    ITensor(DataType t, shape_type s) : shape_(std::move(s)), dtype_(t) {}
    virtual ~ITensor() = default;
    const shape_type &shape() const { return shape_; }
    size_type shape(size_t d) const { return shape_.at(d); }
    shape_type strides() const;  // row-major, in elements
    size_type ndim() const { return static_cast<size_type>(shape_.size()); }
    size_type size() const;
    DataType dtype() const { return dtype_; }
    size_t nbytes() const { return dtype_nbytes(dtype_, static_cast<size_t>(size())); }
    void reshape(shape_type s);
    virtual void *data() = 0;
    virtual const void *data() const = 0;
    virtual bool is_constant() const { return false; }
    virtual bool is_view() const { return false; }
    // Host copy of the contents when the tensor is a constant from the model.
    virtual const std::string *host_data() const { return nullptr; }
    template <typename T>
    T *ptr() { return static_cast<T *>(data()); }
    template <typename T>
    const T *ptr() const { return static_cast<const T *>(data()); }
};

class DeviceTensor : public ITensor {
    void *ptr_ = nullptr;
    bool owned_ = false;
    bool constant_ = false;
    bool view_ = false;
    std::string host_;

public:
    DeviceTensor(DataType t, shape_type s, void *ptr, bool owned) : ITensor(t, std::move(s)), ptr_(ptr), owned_(owned) {}
    ~DeviceTensor() override;
    DeviceTensor(const DeviceTensor &) = delete;
    DeviceTensor &operator=(const DeviceTensor &) = delete;
    // Allocates device memory for the tensor (not on the hot path: prepare time).
    static std::unique_ptr<DeviceTensor> allocate(DataType t, shape_type s);
    // Wraps memory the caller owns (graph inputs/outputs, weight-buffer slices).
    static std::unique_ptr<DeviceTensor> borrow(DataType t, shape_type s, void *ptr);
    void *data() override { return ptr_; }
    const void *data() const override { return ptr_; }
    bool is_constant() const override { return constant_; }
    bool is_view() const override { return view_; }
    const std::string *host_data() const override { return host_.empty() ? nullptr : &host_; }
    void set_constant(std::string host_copy) {
        constant_ = true;
        host_ = std::move(host_copy);
    }
    void set_view(bool v) { view_ = v; }
};

class TensorTable {
    std::map<std::string, std::unique_ptr<ITensor>, std::less<>> owned_;
    std::map<std::string, ITensor *, std::less<>> all_;

public:
    void bind(const std::string &name, ITensor &t) { all_[name] = &t; }
    void own(const std::string &name, std::unique_ptr<ITensor> t) {
        all_[name] = t.get();
        owned_[name] = std::move(t);
    }
    ITensor &at(std::string_view name);
    bool contains(std::string_view name) const { return all_.find(name) != all_.end(); }
    void clear() {
        all_.clear();
        owned_.clear();
    }
    size_t size() const { return all_.size(); }
};

// ---------------------------------------------------------------------------
// NetworkInstance: binds external tensors, creates operators and tensors once
// (prepare), fuses QDQ node groups into single kernels, then runs the nodes in
// graph order on one CUDA stream (network_instance.cpp:584-655 runs them in
// schedule order inside one shader).
// ---------------------------------------------------------------------------
struct FusionInfo;  // per-node fusion decisions (defined in the executor)

class NetworkInstance {
public:
    NetworkInstance();
    ~NetworkInstance();
    NetworkInstance(const NetworkInstance &) = delete;
    NetworkInstance &operator=(const NetworkInstance &) = delete;

    void set_model(Model model);
    void set_input(std::string_view name, ITensor &tensor);
    void set_output(std::string_view name, ITensor &tensor);
    // Device buffer holding every initializer that has data_offsets
    // (network_instance.h:206-208 takes a LuisaCompute ByteBuffer).
    void set_weight_buffer(const void *device_ptr, size_t bytes);
    void set_stream(lcml_stream_t s) { stream_ = s; }
    lcml_stream_t stream() const { return stream_; }
    // Host-staged I/O (no reference counterpart: the reference reads and
    // writes its bound buffers itself). A bound input may name a host buffer
    // (pinned for asynchronous copies) of the same size: every forward()
    // first copies it into the bound device tensor on a second stream. That
    // copy waits only until the previous forward's last reader of the input
    // has run, so it overlaps the rest of that forward. A bound output may
    // name a host buffer that forward() fills (device -> host on the
    // instance's stream) after the last node. nullptr removes the binding.
    void set_input_host(std::string_view name, const void *host);
    void set_output_host(std::string_view name, void *host);
    // Off (default): the host-staged outputs are copied on the instance's
    // stream, so they are complete when that stream is. On: they are copied
    // on a third stream after the last node, overlapping the next forward's
    // nodes; the next forward's writer of an output waits only for that
    // copy to have read it. The host buffers are then complete after
    // wait_outputs() (the host waits for the copies enqueued so far), or on
    // a stream `s` after wait_outputs(s) (the stream waits for them).
    void enable_async_output_copy(bool e) { async_out_ = e; }
    void wait_outputs(lcml_stream_t s = nullptr);
    // Kept for source compatibility with the reference; no effect on the CUDA path.
    void set_warp_size(uint32_t w) { warp_size_ = w; }
    uint32_t warp_size() const { return warp_size_; }
    bool use_warp_optimization() const { return warp_size_ > 1; }
    void set_use_cooperative_vector(bool e) { coop_vec_ = e; }
    bool use_cooperative_vector() const { return coop_vec_; }
    void enable_logging(bool e) { logging_ = e; }
    // Disables the QDQ / activation fusion pass (every node runs its own kernel).
    void enable_fusion(bool e) {
        fusion_enabled_ = e;
        reset();
    }
    // Intermediate tensors share one device arena by lifetime (on by default,
    // the role of build_last_use_map + the pooled allocation in the reference,
    // network_instance.cpp:369-582): a tensor's bytes are reused once its last
    // reader has run. Off: every intermediate has its own allocation, so all of
    // them stay readable after forward() (for inspection and tests).
    void enable_memory_reuse(bool e) {
        reuse_memory_ = e;
        reset();
    }
    // After prepare: bytes of the intermediate arena (or of the separate
    // intermediate allocations when reuse is off), and the bytes the
    // intermediates would take without reuse.
    size_t intermediate_bytes() const { return intermediate_bytes_; }
    size_t intermediate_bytes_unplanned() const { return intermediate_unplanned_; }

    const Model &get_model() const { return model_; }
    TensorTable &tensor_table() { return table_; }

    // Prepare on first call (operators, tensors, fusion), then enqueue every node.
    void forward();
    // Drops the prepared state (e.g. after rebinding tensors of other shapes).
    void reset();

    // Introspection for tests and tooling.
    size_t num_nodes() const { return model_.get_graph().get_nodes().size(); }
    size_t num_executed_nodes() const;
    std::vector<std::string> executed_node_summary() const;
    const FusionInfo *fusion_info(size_t node_index) const;
    // True when the named tensor is stored NHWC (outputs of fused convolutions
    // and pools); its shape() stays the ONNX NCHW shape.
    bool is_nhwc(std::string_view name) const { return nhwc_.find(name) != nhwc_.end(); }

private:
    void prepare();
    void create_tensors();
    void run_fusion_pass();
    void fold_constants();
    void allocate_intermediates();

    Model model_;
    std::map<std::string, ITensor *, std::less<>> inputs_, outputs_;
    const void *weight_buffer_ = nullptr;
    size_t weight_bytes_ = 0;
    lcml_stream_t stream_ = nullptr;
    uint32_t warp_size_ = 32;
    bool coop_vec_ = false, logging_ = false, fusion_enabled_ = true, reuse_memory_ = true;
    size_t intermediate_bytes_ = 0, intermediate_unplanned_ = 0;
    bool prepared_ = false;
    TensorTable table_;
    std::vector<std::unique_ptr<Operator>> ops_;
    std::vector<std::unique_ptr<FusionInfo>> fusion_;
    std::set<std::string, std::less<>> nhwc_;
    std::map<std::string, const void *, std::less<>> host_in_;
    std::map<std::string, void *, std::less<>> host_out_;
    lcml_stream_t copy_stream_ = nullptr;
    lcml_event_t in_ready_ = nullptr, in_free_ = nullptr;
    bool in_free_recorded_ = false;
    bool async_out_ = false;
    lcml_stream_t out_stream_ = nullptr;
    lcml_event_t out_ready_ = nullptr, out_free_ = nullptr;
    bool last_out_async_ = false;  // the last forward copied its host outputs on out_stream_
};

// Throws Error with lcml_last_error() when a C-ABI call fails.
void check_status(int status, const char *what);

}// namespace lcml::onnx
