// LuisaML-JSON model loading and the IR types of lcml_onnx.h.
// Follows the reference loader's schema (src/onnx/onnx.cpp:87-242): string
// enum names for dtypes and attribute types, quoted 64-bit integers, base64
// `raw_data` or `data_offsets` [start, end) into an external weight blob,
// `value_info` shapes for intermediates, and every node's op must be
// registered (the reference asserts at onnx.cpp:228-229; this throws).
#include <cstring>
#include <set>

#include "../../include/lcml_onnx.h"
#include "json.h"

namespace lcml::onnx {

namespace {

struct DtypeRow {
    DataType t;
    const char *name;
    size_t size;
};

constexpr DtypeRow kDtypes[] = {
    {DataType::UNDEFINED, "UNDEFINED", 0}, {DataType::FLOAT, "FLOAT", 4},     {DataType::UINT8, "UINT8", 1},
    {DataType::INT8, "INT8", 1},           {DataType::UINT16, "UINT16", 2},   {DataType::INT16, "INT16", 2},
    {DataType::INT32, "INT32", 4},         {DataType::INT64, "INT64", 8},     {DataType::STRING, "STRING", 0},
    {DataType::BOOL, "BOOL", 1},           {DataType::FLOAT16, "FLOAT16", 2}, {DataType::DOUBLE, "DOUBLE", 8},
    {DataType::UINT32, "UINT32", 4},       {DataType::UINT64, "UINT64", 8},   {DataType::COMPLEX64, "COMPLEX64", 0},
    {DataType::COMPLEX128, "COMPLEX128", 0}, {DataType::BFLOAT16, "BFLOAT16", 2},
    {DataType::FLOAT8E4M3FN, "FLOAT8E4M3FN", 1}, {DataType::FLOAT8E4M3FNUZ, "FLOAT8E4M3FNUZ", 1},
    {DataType::FLOAT8E5M2, "FLOAT8E5M2", 1}, {DataType::FLOAT8E5M2FNUZ, "FLOAT8E5M2FNUZ", 1},
    {DataType::UINT4, "UINT4", 0},         {DataType::INT4, "INT4", 0},       {DataType::FLOAT4E2M1, "FLOAT4E2M1", 0},
    {DataType::FLOAT8E8M0, "FLOAT8E8M0", 1}, {DataType::UINT2, "UINT2", 0},  {DataType::INT2, "INT2", 0},
    {DataType::FLOAT16QUANTIZED, "FLOAT16QUANTIZED", 2},
};

constexpr const char *kAttrNames[] = {"UNDEFINED", "FLOAT",   "INT",           "STRING",         "TENSOR",
                                      "GRAPH",     "FLOATS",  "INTS",          "STRINGS",        "TENSORS",
                                      "GRAPHS",    "SPARSE_TENSOR", "SPARSE_TENSORS", "TYPE_PROTO", "TYPE_PROTOS"};

int b64(unsigned char c) {
    if (c >= 'A' && c <= 'Z') return c - 'A';
    if (c >= 'a' && c <= 'z') return c - 'a' + 26;
    if (c >= '0' && c <= '9') return c - '0' + 52;
    if (c == '+') return 62;
    if (c == '/') return 63;
    return -1;
}

// Base64 decode as the reference does (onnx.cpp:68-85): stop at '=', skip
// characters outside the alphabet.
std::string base64_decode(std::string_view in) {
    std::string out;
    out.reserve(in.size() * 3 / 4);
    int32_t val = 0, bits = -8;
    for (char ch : in) {
        if (ch == '=') break;
        const int v = b64(static_cast<unsigned char>(ch));
        if (v < 0) continue;
        val = (val << 6) + v;
        bits += 6;
        if (bits >= 0) {
            out.push_back(static_cast<char>((val >> bits) & 0xff));
            bits -= 8;
        }
    }
    return out;
}

std::vector<size_t> shape_from_type(const json::Value &v) {
    std::vector<size_t> shape;
    const json::Value &tt = v["type"]["tensor_type"];
    const json::Value *sh = tt.find("shape");
    if (!sh || !sh->contains("dim")) {
        shape.push_back(1);  // the reference's default for a missing shape (onnx.cpp:92-94)
        return shape;
    }
    for (const auto &d : (*sh)["dim"].items()) {
        const json::Value *dv = d.find("dim_value");
        if (!dv) throw Error("symbolic dimension (dim_param) in '" + v["name"].as_string() + "' is not supported");
        shape.push_back(static_cast<size_t>(dv->as_i64()));
    }
    return shape;
}

Variable variable_from_json(const json::Value &v) {
    return Variable(v["name"].as_string(), dtype_from_name(v["type"]["tensor_type"]["elem_type"].as_string()),
                    shape_from_type(v));
}

Variable initializer_from_json(const json::Value &v) {
    std::vector<size_t> shape;
    if (const json::Value *dims = v.find("dims")) {
        for (const auto &d : dims->items()) shape.push_back(static_cast<size_t>(d.as_i64()));
    } else {
        shape.push_back(1);
    }
    std::string raw;
    uint64_t start = 0, end = 0;
    if (const json::Value *off = v.find("data_offsets")) {
        start = (*off)[0].as_u64();
        end = (*off)[1].as_u64();
    } else if (const json::Value *rd = v.find("raw_data")) {
        raw = base64_decode(rd->as_string());
    }
    return Variable(v["name"].as_string(), dtype_from_name(v["data_type"].as_string()), std::move(shape),
                    std::move(raw), start, end);
}

AttributeType attr_type_from_name(std::string_view n) {
    for (size_t i = 0; i < sizeof(kAttrNames) / sizeof(kAttrNames[0]); ++i)
        if (n == kAttrNames[i]) return static_cast<AttributeType>(i);
    throw Error("unknown attribute type '" + std::string(n) + "'");
}

Graph graph_from_json(const json::Value &g, const OperatorSet &opset, const Graph *parent);

Attribute attribute_from_json(const json::Value &a, const Graph *parent) {
    std::string name = a["name"].as_string();
    switch (attr_type_from_name(a["type"].as_string())) {
        case AttributeType::FLOAT: return Attribute(std::move(name), static_cast<float>(a["f"].as_f64()));
        case AttributeType::INT: return Attribute(std::move(name), static_cast<int64_t>(a["i"].as_i64()));
        case AttributeType::STRING: return Attribute(std::move(name), base64_decode(a["s"].as_string()));
        case AttributeType::FLOATS: {
            std::vector<float> v;
            if (const json::Value *f = a.find("floats"))
                for (const auto &x : f->items()) v.push_back(static_cast<float>(x.as_f64()));
            return Attribute(std::move(name), std::move(v));
        }
        case AttributeType::INTS: {
            std::vector<int64_t> v;
            if (const json::Value *f = a.find("ints"))
                for (const auto &x : f->items()) v.push_back(x.as_i64());
            return Attribute(std::move(name), std::move(v));
        }
        case AttributeType::STRINGS: {
            std::vector<std::string> v;
            if (const json::Value *f = a.find("strings"))
                for (const auto &x : f->items()) v.push_back(base64_decode(x.as_string()));
            return Attribute(std::move(name), std::move(v));
        }
        case AttributeType::GRAPH:
            return Attribute(std::move(name),
                             std::make_shared<Graph>(graph_from_json(a["g"], OperatorSet::get_default(), parent)));
        case AttributeType::GRAPHS: {
            std::vector<std::shared_ptr<Graph>> v;
            for (const auto &x : a["graphs"].items())
                v.push_back(std::make_shared<Graph>(graph_from_json(x, OperatorSet::get_default(), parent)));
            return Attribute(std::move(name), std::move(v));
        }
        default: throw Error("unsupported attribute type for '" + name + "'");
    }
}

Graph graph_from_json(const json::Value &g, const OperatorSet &opset, const Graph *parent) {
    Graph graph(g.contains("name") ? g["name"].as_string() : std::string("graph"));
    graph.set_parent(parent);
    if (const json::Value *in = g.find("input"))
        for (const auto &v : in->items()) graph.add_input(graph.add_variable(variable_from_json(v)).get_name());
    if (const json::Value *out = g.find("output"))
        for (const auto &v : out->items()) graph.add_output(graph.add_variable(variable_from_json(v)).get_name());
    if (const json::Value *init = g.find("initializer"))
        for (const auto &v : init->items()) graph.add_variable(initializer_from_json(v));
    if (const json::Value *vi = g.find("value_info"))
        for (const auto &v : vi->items()) {
            Variable var = variable_from_json(v);
            if (Variable *existing = graph.find_var(var.get_name())) {
                // value_info repeating an initializer or an input: keep the first
                (void)existing;
                continue;
            }
            graph.add_variable(std::move(var));
        }
    for (const auto &n : g["node"].items()) {
        Node node(n.contains("name") ? n["name"].as_string() : std::string(), n["op_type"].as_string());
        for (const auto &i : n["input"].items()) {
            const std::string &vn = i.as_string();
            if (vn.empty()) continue;  // absent optional input
            node.add_input(graph.get_var(vn));
        }
        for (const auto &o : n["output"].items()) {
            const std::string &vn = o.as_string();
            if (!graph.find_var(vn)) throw Error("node output '" + vn + "' has no value_info/shape");
            node.add_output(graph.get_var(vn));
        }
        if (const json::Value *attrs = n.find("attribute"))
            for (const auto &a : attrs->items()) node.set_attribute(attribute_from_json(a, &graph));
        if (!opset.has_operator(node.get_op_type())) throw Error("Operator not found: " + node.get_op_type());
        graph.add_node(std::move(node));
    }
    return graph;
}

void collect_outputs(const Graph &g, std::set<std::string> &names) {
    for (const auto &n : g.get_nodes()) {
        for (const auto *o : n.get_outputs()) names.insert(o->get_name());
        for (const auto &kv : n.get_attributes()) {
            const auto t = Attribute::type_of(kv.second);
            if (t == AttributeType::GRAPH) collect_outputs(*kv.second.get<AttributeType::GRAPH>(), names);
            else if (t == AttributeType::GRAPHS)
                for (const auto &sub : kv.second.get<AttributeType::GRAPHS>()) collect_outputs(*sub, names);
        }
    }
}

}// namespace

const char *dtype_name(DataType t) {
    for (const auto &r : kDtypes)
        if (r.t == t) return r.name;
    return "UNKNOWN";
}

DataType dtype_from_name(std::string_view name) {
    for (const auto &r : kDtypes)
        if (name == r.name) return r.t;
    // the ONNX protobuf JSON writer may also emit plain integers
    if (!name.empty() && name[0] >= '0' && name[0] <= '9') {
        const int v = std::atoi(std::string(name).c_str());
        for (const auto &r : kDtypes)
            if (static_cast<int>(r.t) == v) return r.t;
    }
    throw Error("unknown element type '" + std::string(name) + "'");
}

size_t dtype_size(DataType t) {
    for (const auto &r : kDtypes)
        if (r.t == t) return r.size;
    return 0;
}

size_t dtype_nbytes(DataType t, size_t n) { return t == DataType::FLOAT4E2M1 ? (n + 1) / 2 : n * dtype_size(t); }

AttributeType Attribute::type_of(const Attribute &a) {
    switch (a.index()) {
        case 0: return AttributeType::FLOAT;
        case 1: return AttributeType::INT;
        case 2: return AttributeType::STRING;
        case 3: return AttributeType::GRAPH;
        case 4: return AttributeType::FLOATS;
        case 5: return AttributeType::INTS;
        case 6: return AttributeType::STRINGS;
        case 7: return AttributeType::GRAPHS;
        default: return AttributeType::UNDEFINED;
    }
}

const Attribute &Node::get_attribute(std::string_view n) const {
    auto it = attributes_.find(n);
    if (it == attributes_.end()) throw Error("Attribute not found: " + std::string(n));
    return it->second;
}

Variable &Graph::add_variable(Variable &&v) {
    auto it = variables_.find(v.get_name());
    if (it != variables_.end()) return *it->second;
    std::string key = v.get_name();
    auto &slot = variables_[key];
    slot = std::make_unique<Variable>(std::move(v));
    return *slot;
}

const Variable &Graph::get_var(std::string_view name) const {
    auto it = variables_.find(name);
    if (it != variables_.end()) return *it->second;
    if (parent_) return parent_->get_var(name);
    throw Error("Variable not found: " + std::string(name));
}

Variable *Graph::find_var(std::string_view name) {
    auto it = variables_.find(name);
    return it == variables_.end() ? nullptr : it->second.get();
}

void Graph::mark_constants() {
    std::set<std::string> produced;
    collect_outputs(*this, produced);
    std::set<std::string> inputs;
    for (const auto *v : inputs_) inputs.insert(v->get_name());
    // Like the reference (onnx.cpp:38-48): every variable no node produces is
    // constant -- except the graph inputs, which the caller binds.
    for (auto &kv : variables_)
        kv.second->set_is_constant(!produced.count(kv.first) && !inputs.count(kv.first));
}

Graph Graph::from_json_text(std::string_view text, const OperatorSet &opset) {
    return graph_from_json(json::Value::parse(text), opset, nullptr);
}

std::unique_ptr<Operator> OperatorSet::create_operator(std::string_view name, const Node &node) const {
    auto it = factories_.find(name);
    if (it == factories_.end()) throw Error("Operator not found: " + std::string(name));
    return it->second(node);
}

std::vector<std::string> OperatorSet::operator_names() const {
    std::vector<std::string> v;
    for (const auto &kv : factories_) v.push_back(kv.first);
    return v;
}

OperatorSet &OperatorSet::get_default() {
    static OperatorSet opset{"default", 21};
    return opset;
}

Model Model::load_from_json(std::string_view text) {
    const json::Value doc = json::Value::parse(text);
    const json::Value *ir = doc.find("ir_version");
    Model m(ir ? ir->as_i64() : 0, doc.contains("producer_name") ? doc["producer_name"].as_string() : "",
            doc.contains("producer_version") ? doc["producer_version"].as_string() : "");
    m.set_graph(graph_from_json(doc["graph"], m.get_opset(), nullptr));
    return m;
}

// ---------------------------------------------------------------------------
ITensor::shape_type ITensor::strides() const {
    shape_type s(shape_.size(), 1);
    for (int i = static_cast<int>(shape_.size()) - 2; i >= 0; --i) s[i] = s[i + 1] * shape_[i + 1];
    return s;
}

ITensor::size_type ITensor::size() const {
    size_type n = 1;
    for (auto d : shape_) n *= d;
    return n;
}

void ITensor::reshape(shape_type s) {
    size_type n = 1;
    for (auto d : s) n *= d;
    if (n != size()) throw Error("reshape changes the element count");
    shape_ = std::move(s);
}

DeviceTensor::~DeviceTensor() {
    if (owned_ && ptr_) lcml_device_free(ptr_);
}

std::unique_ptr<DeviceTensor> DeviceTensor::allocate(DataType t, shape_type s) {
    size_t n = 1;
    for (auto d : s) n *= static_cast<size_t>(d);
    const size_t bytes = dtype_nbytes(t, n);
    void *p = nullptr;
    // round up to 256 B so every tensor starts 256-byte aligned and vector
    // tails never read past the allocation
    check_status(lcml_device_alloc(((bytes + 255) / 256) * 256, &p), "lcml_device_alloc");
    return std::make_unique<DeviceTensor>(t, std::move(s), p, true);
}

std::unique_ptr<DeviceTensor> DeviceTensor::borrow(DataType t, shape_type s, void *ptr) {
    return std::make_unique<DeviceTensor>(t, std::move(s), ptr, false);
}

ITensor &TensorTable::at(std::string_view name) {
    auto it = all_.find(name);
    if (it == all_.end()) throw Error("TensorTable: key not found: " + std::string(name));
    return *it->second;
}

void check_status(int status, const char *what) {
    if (status != LCML_OK) throw Error(std::string(what) + ": " + lcml_last_error());
}

}// namespace lcml::onnx
