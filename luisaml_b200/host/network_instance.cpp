// NetworkInstance: the graph executor (network_instance.cpp in the reference).
//
// prepare (first forward):
//   0. create one Operator per node from the opset        (reference :356-365)
//   1. bind external inputs/outputs with strict dtype and shape checks (:40-86)
//   2. create constant tensors: `data_offsets` initializers become views into
//      the caller's device weight buffer (e4m3 blobs padded to 4 bytes, :215-232),
//      `raw_data` initializers are uploaded once and keep a host copy
//   3. fusion pass: DequantizeLinear -> Gemm/MatMul -> (Relu) -> (Cast | QuantizeLinear)
//      node groups become one FusedQdqGemm (scales, bias, activation and output
//      cast in the GEMM epilogue, so no dequantized operand ever reaches HBM);
//      DequantizeLinear -> Conv -> (Add residual) -> (Relu) -> QuantizeLinear
//      becomes one FusedQdqConv with an NHWC e4m3 output; QDQ MaxPool and
//      GlobalAveragePool read e4m3 directly; nodes left without readers drop out
//   4. allocate the intermediates the remaining nodes touch; view ops alias
// forward: every non-folded node runs in graph order on the instance's stream
// (the reference runs them in schedule order inside one generated shader).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <set>
#include <sstream>

#include "operators.h"

namespace lcml::onnx {

struct FusionInfo {
    bool skip = false;                      // folded into another node's kernel
    std::string note;                       // what happened to the node
    std::unique_ptr<Operator> op;           // replacement operator (fused group)
    std::vector<std::string> inputs, outputs;  // replacement I/O variable names
};

namespace {

bool is_gemm_like(const std::string &op) { return op == "Gemm" || op == "MatMul"; }

int64_t attr_int(const Node &n, const char *name, int64_t dflt) {
    if (auto p = n.try_get_attr(name)) return p->get<AttributeType::INT>();
    return dflt;
}

float attr_float(const Node &n, const char *name, float dflt) {
    if (auto p = n.try_get_attr(name)) return p->get<AttributeType::FLOAT>();
    return dflt;
}

ITensor::shape_type to_shape(const std::vector<size_t> &s) {
    ITensor::shape_type r;
    for (auto d : s) r.push_back(static_cast<int64_t>(d));
    return r;
}

}// namespace

NetworkInstance::NetworkInstance() = default;
NetworkInstance::~NetworkInstance() {
    // release operators before the tensors they may reference
    ops_.clear();
    fusion_.clear();
    table_.clear();
    if (copy_stream_) {
        lcml_stream_synchronize(copy_stream_);
        lcml_stream_destroy(copy_stream_);
    }
    if (out_stream_) {
        lcml_stream_synchronize(out_stream_);
        lcml_stream_destroy(out_stream_);
    }
    lcml_event_destroy(in_ready_);
    lcml_event_destroy(in_free_);
    lcml_event_destroy(out_ready_);
    lcml_event_destroy(out_free_);
}

void NetworkInstance::wait_outputs(lcml_stream_t s) {
    const bool async = out_stream_ && last_out_async_;
    if (s) {
        if (async) check_status(lcml_stream_wait_event(s, out_free_), "wait_outputs");
        else if (s != stream_) {  // the copies ran on the instance's stream
            lcml_event_t e = nullptr;
            check_status(lcml_event_create(&e), "event");
            check_status(lcml_event_record(e, stream_), "record");
            check_status(lcml_stream_wait_event(s, e), "wait_outputs");
            lcml_event_destroy(e);
        }
        return;
    }
    check_status(lcml_stream_synchronize(async ? out_stream_ : stream_), "wait_outputs");
}

void NetworkInstance::set_input_host(std::string_view name, const void *host) {
    if (!inputs_.count(std::string(name))) throw Error("set_input_host: input '" + std::string(name) + "' is not bound");
    if (host) host_in_[std::string(name)] = host;
    else host_in_.erase(std::string(name));
}

void NetworkInstance::set_output_host(std::string_view name, void *host) {
    if (!outputs_.count(std::string(name))) throw Error("set_output_host: output '" + std::string(name) + "' is not bound");
    if (host) host_out_[std::string(name)] = host;
    else host_out_.erase(std::string(name));
}

void NetworkInstance::set_model(Model model) {
    model_ = std::move(model);
    reset();
}

void NetworkInstance::set_input(std::string_view name, ITensor &t) {
    inputs_[std::string(name)] = &t;
    reset();
}

void NetworkInstance::set_output(std::string_view name, ITensor &t) {
    outputs_[std::string(name)] = &t;
    reset();
}

void NetworkInstance::set_weight_buffer(const void *p, size_t bytes) {
    weight_buffer_ = p;
    weight_bytes_ = bytes;
    reset();
}

void NetworkInstance::reset() {
    prepared_ = false;
    ops_.clear();
    fusion_.clear();
    table_.clear();
    nhwc_.clear();
}

const FusionInfo *NetworkInstance::fusion_info(size_t i) const { return i < fusion_.size() ? fusion_[i].get() : nullptr; }

size_t NetworkInstance::num_executed_nodes() const {
    size_t n = 0;
    for (const auto &f : fusion_)
        if (!f->skip) ++n;
    return n;
}

std::vector<std::string> NetworkInstance::executed_node_summary() const {
    std::vector<std::string> out;
    const auto &nodes = model_.get_graph().get_nodes();
    for (size_t i = 0; i < nodes.size() && i < fusion_.size(); ++i) {
        std::string s = nodes[i].get_op_type() + " " + nodes[i].get_name() + ": ";
        s += fusion_[i]->skip ? "folded" : (fusion_[i]->op ? "fused kernel" : "kernel");
        if (!fusion_[i]->note.empty()) s += " (" + fusion_[i]->note + ")";
        out.push_back(s);
    }
    return out;
}

void NetworkInstance::create_tensors() {
    const Graph &g = model_.get_graph();
    // 1. externals, strictly validated (network_instance.cpp:40-69)
    auto bind = [&](const char *role, const Variable &v, std::map<std::string, ITensor *, std::less<>> &ext) {
        auto it = ext.find(v.get_name());
        if (it == ext.end()) return;
        ITensor &t = *it->second;
        if (t.dtype() != v.get_dtype())
            throw Error(std::string(role) + " '" + v.get_name() + "' element type mismatch: expected " +
                        dtype_name(v.get_dtype()) + ", got " + dtype_name(t.dtype()));
        const auto expected = to_shape(v.get_shape());
        if (t.shape() != expected) {
            std::ostringstream os;
            os << role << " '" << v.get_name() << "' shape mismatch: expected [";
            for (auto d : expected) os << d << ",";
            os << "], got [";
            for (auto d : t.shape()) os << d << ",";
            os << "]";
            throw Error(os.str());
        }
        table_.bind(v.get_name(), t);
    };
    for (const auto *v : g.get_inputs()) bind("Input", *v, inputs_);
    for (const auto *v : g.get_outputs()) bind("Output", *v, outputs_);

    // 2. constants
    for (const auto &kv : g.get_variables()) {
        const Variable &v = *kv.second;
        if (table_.contains(v.get_name()) || !v.is_constant()) continue;
        const bool fp4 = v.get_dtype() == DataType::FLOAT4E2M1;
        size_t n = 1;
        for (auto d : v.get_shape()) n *= d;
        const size_t nbytes = dtype_nbytes(v.get_dtype(), n);
        if (v.is_trainable_weight()) {
            if (!weight_buffer_) throw Error("Weight buffer not set but required for variable: " + v.get_name());
            auto [b, e] = v.get_buffer_range();
            // blob extents as the reference checks them (network_instance.cpp:218-227):
            // FP8 padded to 4 bytes, FP4 two codes per byte
            const bool fp8 = v.get_dtype() == DataType::FLOAT8E4M3FN || v.get_dtype() == DataType::FLOAT8E5M2;
            const size_t expected = fp8 ? ((n + 3) / 4) * 4 : nbytes;
            if (e - b != expected) throw Error("Weight buffer size mismatch for variable: " + v.get_name());
            if (e > weight_bytes_) throw Error("Weight buffer too small for variable: " + v.get_name());
            auto t = DeviceTensor::borrow(v.get_dtype(), to_shape(v.get_shape()),
                                          const_cast<uint8_t *>(static_cast<const uint8_t *>(weight_buffer_) + b));
            t->set_constant({});
            table_.own(v.get_name(), std::move(t));
        } else if (!v.get_raw_data().empty()) {
            if (nbytes == 0) throw Error("unsupported element type for constant " + v.get_name());
            if (v.get_raw_data().size() < nbytes) throw Error("raw_data too short for " + v.get_name());
            std::string bytes = v.get_raw_data().substr(0, nbytes);
            // FP4 raw_data holds element 2i in the HIGH nibble of byte i (the
            // reference's loader, network_instance.cpp:242-246), device storage
            // in the low nibble (FP4Data): swap the nibbles on upload
            if (fp4)
                for (auto &c : bytes) c = static_cast<char>(((static_cast<uint8_t>(c) & 0x0f) << 4) | (static_cast<uint8_t>(c) >> 4));
            auto t = DeviceTensor::allocate(v.get_dtype(), to_shape(v.get_shape()));
            check_status(lcml_memcpy_async(t->data(), bytes.data(), nbytes, 1, stream_), "upload constant");
            t->set_constant(bytes);
            table_.own(v.get_name(), std::move(t));
        }
    }
}

void NetworkInstance::run_fusion_pass() {
    const Graph &g = model_.get_graph();
    const auto &nodes = g.get_nodes();
    std::map<std::string, int> producer;
    std::map<std::string, std::vector<int>> consumers;
    std::set<std::string> graph_outputs;
    for (const auto *v : g.get_outputs()) graph_outputs.insert(v->get_name());
    for (size_t i = 0; i < nodes.size(); ++i) {
        for (const auto *o : nodes[i].get_outputs()) producer[o->get_name()] = static_cast<int>(i);
        for (const auto *in : nodes[i].get_inputs()) consumers[in->get_name()].push_back(static_cast<int>(i));
    }
    auto sole_consumer = [&](const std::string &var) -> int {
        if (graph_outputs.count(var)) return -1;
        auto it = consumers.find(var);
        if (it == consumers.end() || it->second.size() != 1) return -1;
        return it->second[0];
    };
    auto producer_of = [&](const std::string &var) -> int {
        auto it = producer.find(var);
        return it == producer.end() ? -1 : it->second;
    };

    // a DequantizeLinear usable as a fused operand: e4m3 input, zero point absent or all zero
    auto dq_ok = [&](int d) {
        if (d < 0 || nodes[d].get_op_type() != "DequantizeLinear") return false;
        const Node &dn = nodes[d];
        if (dn.get_inputs()[0]->get_dtype() != DataType::FLOAT8E4M3FN) return false;
        if (dn.get_outputs()[0]->get_dtype() != DataType::FLOAT) return false;
        if (dn.get_inputs().size() > 2) {
            const std::string &zp = dn.get_inputs()[2]->get_raw_data();
            if (!dn.get_inputs()[2]->is_constant()) return false;
            for (char c : zp)
                if (c != 0) return false;
        }
        return true;
    };
    // per-axis scale of an operand: number of scale elements and the axis it runs along
    auto dq_scale_len = [&](int d) -> int64_t {
        size_t n = 1;
        for (auto s : nodes[d].get_inputs()[1]->get_shape()) n *= s;
        return static_cast<int64_t>(n);
    };

    auto host_floats = [&](const Variable &v) -> std::vector<float> {
        std::vector<float> out;
        if (!table_.contains(v.get_name())) return out;
        const std::string *h = table_.at(v.get_name()).host_data();
        if (!h || v.get_dtype() != DataType::FLOAT) return out;
        out.resize(h->size() / 4);
        std::memcpy(out.data(), h->data(), out.size() * 4);
        return out;
    };

    // ---- Rule: gate/up GEMM pair + Sigmoid / Mul / Mul (SiLU(gate) * up) -> one GEMM
    // over the two weights interleaved in 128-row groups, SiLU*up in the epilogue.
    for (size_t mi = 0; mi < nodes.size(); ++mi) {
        const Node &m2 = nodes[mi];
        if (m2.get_op_type() != "Mul" || m2.get_inputs().size() != 2) continue;
        for (int side = 0; side < 2; ++side) {
            const int m1 = producer_of(m2.get_inputs()[side]->get_name());
            const int gu = producer_of(m2.get_inputs()[1 - side]->get_name());
            if (m1 < 0 || gu < 0 || nodes[m1].get_op_type() != "Mul" || nodes[gu].get_op_type() != "Gemm") continue;
            // m1 = Mul(g, Sigmoid(g)) in either order
            int gg = -1, sg = -1;
            for (int k = 0; k < 2; ++k) {
                const int a = producer_of(nodes[m1].get_inputs()[k]->get_name());
                const int b = producer_of(nodes[m1].get_inputs()[1 - k]->get_name());
                if (a >= 0 && b >= 0 && nodes[a].get_op_type() == "Gemm" && nodes[b].get_op_type() == "Sigmoid" &&
                    nodes[b].get_inputs()[0] == nodes[a].get_outputs()[0]) {
                    gg = a;
                    sg = b;
                }
            }
            if (gg < 0) continue;
            const Node &G = nodes[gg], &U = nodes[gu];
            const std::string gname = G.get_outputs()[0]->get_name(), uname = U.get_outputs()[0]->get_name();
            // consumers: g -> {Sigmoid, m1}; Sigmoid -> {m1}; m1 -> {m2}; u -> {m2}
            if (graph_outputs.count(gname) || graph_outputs.count(uname) || consumers[gname].size() != 2 ||
                sole_consumer(nodes[sg].get_outputs()[0]->get_name()) != m1 ||
                sole_consumer(nodes[m1].get_outputs()[0]->get_name()) != static_cast<int>(mi) ||
                sole_consumer(uname) != static_cast<int>(mi))
                continue;
            if (G.get_inputs()[0] != U.get_inputs()[0] || G.get_inputs().size() != 2 || U.get_inputs().size() != 2)
                continue;
            if (attr_int(G, "transB", 0) != 1 || attr_int(U, "transB", 0) != 1 || attr_int(G, "transA", 0) ||
                attr_int(U, "transA", 0) || attr_float(G, "alpha", 1.0f) != 1.0f || attr_float(U, "alpha", 1.0f) != 1.0f)
                continue;
            const int da = producer_of(G.get_inputs()[0]->get_name());
            const int dg = producer_of(G.get_inputs()[1]->get_name());
            const int du = producer_of(U.get_inputs()[1]->get_name());
            if (!dq_ok(da) || !dq_ok(dg) || !dq_ok(du)) continue;
            const Variable &qa = *nodes[da].get_inputs()[0];
            const Variable &wg = *nodes[dg].get_inputs()[0], &wu = *nodes[du].get_inputs()[0];
            if (qa.get_shape().size() != 2 || wg.get_shape() != wu.get_shape() || wg.get_shape().size() != 2) continue;
            const int64_t F = static_cast<int64_t>(wg.get_shape()[0]), K = static_cast<int64_t>(wg.get_shape()[1]);
            const int64_t M = static_cast<int64_t>(qa.get_shape()[0]);
            if (F % 128 != 0 || !wg.is_constant() || !wu.is_constant() || !table_.contains(wg.get_name()) ||
                !table_.contains(wu.get_name()))
                continue;
            const int64_t la = dq_scale_len(da);
            if (la != 1 && (la != M || attr_int(nodes[da], "axis", 1) != 0)) continue;
            std::vector<float> sgv = host_floats(*nodes[dg].get_inputs()[1]), suv = host_floats(*nodes[du].get_inputs()[1]);
            auto per_row = [&](std::vector<float> v, int d) -> std::vector<float> {
                if (v.size() == 1) return std::vector<float>(static_cast<size_t>(F), v[0]);
                if (static_cast<int64_t>(v.size()) == F && attr_int(nodes[d], "axis", 1) == 0) return v;
                return {};
            };
            sgv = per_row(sgv, dg);
            suv = per_row(suv, du);
            if (sgv.empty() || suv.empty()) continue;
            // interleave [gate 128 rows; up 128 rows] per group, weights on the device, scales on the host
            auto wcat = DeviceTensor::allocate(DataType::FLOAT8E4M3FN, {2 * F, K});
            std::vector<float> scat(static_cast<size_t>(2 * F));
            const uint8_t *pg = table_.at(wg.get_name()).ptr<uint8_t>(), *pu = table_.at(wu.get_name()).ptr<uint8_t>();
            for (int64_t grp = 0; grp < F / 128; ++grp) {
                uint8_t *dst = wcat->ptr<uint8_t>() + grp * 256 * K;
                check_status(lcml_memcpy_async(dst, pg + grp * 128 * K, 128 * K, 3, stream_), "interleave gate");
                check_status(lcml_memcpy_async(dst + 128 * K, pu + grp * 128 * K, 128 * K, 3, stream_), "interleave up");
                for (int64_t r = 0; r < 128; ++r) {
                    scat[grp * 256 + r] = sgv[grp * 128 + r];
                    scat[grp * 256 + 128 + r] = suv[grp * 128 + r];
                }
            }
            wcat->set_constant({});
            auto st = DeviceTensor::allocate(DataType::FLOAT, {2 * F});
            check_status(lcml_memcpy_async(st->data(), scat.data(), scat.size() * 4, 1, stream_), "upload scales");
            check_status(lcml_stream_synchronize(stream_), "interleave");  // host scale buffer goes out of scope
            st->set_constant(std::string(reinterpret_cast<const char *>(scat.data()), scat.size() * 4));
            const std::string wname = m2.get_name() + "#gate_up_weight", sname = m2.get_name() + "#gate_up_scale";
            table_.own(wname, std::move(wcat));
            table_.own(sname, std::move(st));
            auto op = std::make_unique<FusedQdqGemm>();
            op->epilogue = LCML_EPI_SILU_MUL;
            auto &fi = *fusion_[mi];
            fi.inputs = {qa.get_name(), nodes[da].get_inputs()[1]->get_name(), wname, sname};
            fi.outputs = {m2.get_outputs()[0]->get_name()};
            fi.note = "gate/up Gemm pair + Sigmoid + Mul + Mul fused into one FP8 GEMM (SiLU*up epilogue)";
            fi.op = std::move(op);
            for (int f : {gg, gu, sg, m1}) {
                fusion_[f]->skip = true;
                fusion_[f]->note = "folded into the gate/up GEMM at " + m2.get_name();
            }
            break;
        }
    }

    // ---- Rule: Abs -> ReduceMax(last axis, keepdims 0) -> Div(448) -> QuantizeLinear(axis 0)
    // on a 2-D tensor -> one dynamic per-row quantization kernel producing q and s.
    for (size_t qi = 0; qi < nodes.size(); ++qi) {
        const Node &q = nodes[qi];
        if (q.get_op_type() != "QuantizeLinear" || q.get_inputs().size() < 2) continue;
        const Variable &x = *q.get_inputs()[0];
        if (x.get_shape().size() != 2 || x.get_dtype() != DataType::FLOAT) continue;
        if (attr_int(q, "axis", 1) != 0 || q.get_outputs()[0]->get_dtype() != DataType::FLOAT8E4M3FN) continue;
        if (q.get_inputs().size() > 2) continue;
        const int d = producer_of(q.get_inputs()[1]->get_name());
        if (d < 0 || nodes[d].get_op_type() != "Div") continue;
        const int r = producer_of(nodes[d].get_inputs()[0]->get_name());
        const std::vector<float> c = host_floats(*nodes[d].get_inputs()[1]);
        if (r < 0 || nodes[r].get_op_type() != "ReduceMax" || c.size() != 1 || c[0] != 448.0f) continue;
        const std::vector<int64_t> axes = [&] {
            if (auto p = nodes[r].try_get_attr("axes")) return p->get<AttributeType::INTS>();
            return std::vector<int64_t>{};
        }();
        if (axes.size() != 1 || (axes[0] != -1 && axes[0] != 1) || attr_int(nodes[r], "keepdims", 1) != 0) continue;
        const int a = producer_of(nodes[r].get_inputs()[0]->get_name());
        if (a < 0 || nodes[a].get_op_type() != "Abs" || nodes[a].get_inputs()[0] != &x) continue;
        if (sole_consumer(nodes[a].get_outputs()[0]->get_name()) != r ||
            sole_consumer(nodes[r].get_outputs()[0]->get_name()) != d)
            continue;
        bool late = true;  // every consumer of the scale runs after the QuantizeLinear
        for (int cidx : consumers[nodes[d].get_outputs()[0]->get_name()])
            if (cidx < static_cast<int>(qi)) late = false;
        if (!late) continue;
        auto &fi = *fusion_[qi];
        fi.op = std::make_unique<DynamicRowQuant>();
        fi.inputs = {x.get_name()};
        fi.outputs = {q.get_outputs()[0]->get_name(), nodes[d].get_outputs()[0]->get_name()};
        fi.note = "Abs + ReduceMax + Div + QuantizeLinear fused into one dynamic per-row quantization";
        for (int f : {a, r, d}) {
            fusion_[f]->skip = true;
            fusion_[f]->note = "folded into the dynamic quantization at " + q.get_name();
        }
    }

    for (size_t gi = 0; gi < nodes.size(); ++gi) {
        const Node &gn = nodes[gi];
        if (!is_gemm_like(gn.get_op_type())) continue;
        if (fusion_[gi]->skip || fusion_[gi]->op) continue;
        const bool is_gemm = gn.get_op_type() == "Gemm";
        if (is_gemm && attr_int(gn, "transA", 0) != 0) continue;
        const int da = producer_of(gn.get_inputs()[0]->get_name());
        const int db = producer_of(gn.get_inputs()[1]->get_name());
        if (!dq_ok(da) || !dq_ok(db)) continue;
        const Variable &qa = *nodes[da].get_inputs()[0];
        const Variable &qb = *nodes[db].get_inputs()[0];
        if (qb.get_shape().size() != 2 || qa.get_shape().size() < 2) continue;
        const bool transB = is_gemm && attr_int(gn, "transB", 0) != 0;
        const int64_t K = static_cast<int64_t>(qa.get_shape().back());
        const int64_t N = static_cast<int64_t>(transB ? qb.get_shape()[0] : qb.get_shape()[1]);
        int64_t M = 1;
        for (size_t i = 0; i + 1 < qa.get_shape().size(); ++i) M *= static_cast<int64_t>(qa.get_shape()[i]);
        // scale layouts: A per tensor or per row (axis 0 of a 2-D A); B per tensor or per output column
        const int64_t la = dq_scale_len(da), lb = dq_scale_len(db);
        if (la != 1) {
            if (qa.get_shape().size() != 2 || la != M || attr_int(nodes[da], "axis", 1) != 0) continue;
        }
        if (lb != 1) {
            const int64_t axis = attr_int(nodes[db], "axis", 1);
            const int64_t want = transB ? 0 : 1;
            if (lb != N || (axis != want && axis != want - 2)) continue;
        }
        (void)K;

        auto op = std::make_unique<FusedQdqGemm>();
        op->alpha = is_gemm ? attr_float(gn, "alpha", 1.0f) : 1.0f;
        op->beta = is_gemm ? attr_float(gn, "beta", 1.0f) : 1.0f;
        std::string b_name = qb.get_name();
        if (transB) {
            op->b_kmajor = 1;
        } else if (qb.is_constant() && table_.contains(qb.get_name())) {
            // [K, N] constant weight: transpose once into the K-major layout the tensor cores read
            ITensor &src = table_.at(qb.get_name());
            auto t = DeviceTensor::allocate(DataType::FLOAT8E4M3FN, {N, static_cast<int64_t>(qb.get_shape()[0])});
            check_status(lcml_fp8_transpose(src.ptr<uint8_t>(), src.shape(0), src.shape(1), t->ptr<uint8_t>(), stream_),
                         "transpose weight");
            t->set_constant({});
            b_name = qb.get_name() + "#kmajor";
            table_.own(b_name, std::move(t));
            op->b_kmajor = 1;
        } else {
            op->b_kmajor = 0;
        }
        auto &fi = *fusion_[gi];
        fi.inputs = {qa.get_name(), nodes[da].get_inputs()[1]->get_name(), b_name, nodes[db].get_inputs()[1]->get_name()};
        if (is_gemm && gn.get_inputs().size() > 2) {
            op->has_c = true;
            fi.inputs.push_back(gn.get_inputs()[2]->get_name());
        }
        // epilogue chain: (Relu) then (Cast to BFLOAT16/FLOAT | QuantizeLinear with a constant per-tensor scale)
        std::string out = gn.get_outputs()[0]->get_name();
        std::vector<int> folded;
        int c = sole_consumer(out);
        if (c >= 0 && nodes[c].get_op_type() == "Relu") {
            op->epilogue = LCML_EPI_RELU;
            folded.push_back(c);
            out = nodes[c].get_outputs()[0]->get_name();
            c = sole_consumer(out);
        }
        if (c >= 0 && nodes[c].get_op_type() == "Cast") {
            const DataType to = nodes[c].get_outputs()[0]->get_dtype();
            if (to == DataType::BFLOAT16 || to == DataType::FLOAT) {
                folded.push_back(c);
                out = nodes[c].get_outputs()[0]->get_name();
            }
        } else if (c >= 0 && nodes[c].get_op_type() == "QuantizeLinear") {
            const Node &qn = nodes[c];
            const Variable &qs = *qn.get_inputs()[1];
            size_t qsn = 1;
            for (auto s : qs.get_shape()) qsn *= s;
            bool zp_ok = qn.get_inputs().size() < 3;
            if (!zp_ok && qn.get_inputs()[2]->is_constant()) {
                zp_ok = true;
                for (char ch : qn.get_inputs()[2]->get_raw_data())
                    if (ch != 0) zp_ok = false;
            }
            if (qsn == 1 && qs.is_constant() && zp_ok && qn.get_outputs()[0]->get_dtype() == DataType::FLOAT8E4M3FN) {
                folded.push_back(c);
                op->has_y_scale = true;
                fi.inputs.push_back(qs.get_name());
                out = qn.get_outputs()[0]->get_name();
            }
        }
        fi.outputs = {out};
        std::string note = "DequantizeLinear x2";
        for (int f : folded) note += " + " + nodes[f].get_op_type();
        fi.note = note + " fused into one FP8 GEMM";
        fi.op = std::move(op);
        for (int f : folded) {
            fusion_[f]->skip = true;
            fusion_[f]->note = "folded into " + gn.get_op_type() + " " + gn.get_name();
        }
    }
    // ---- Convolutional part, in graph order (a tensor's layout is known once its
    // producer has been visited): fused QDQ Conv, e4m3 MaxPool, e4m3 GlobalAveragePool.
    // Their e4m3 outputs are stored NHWC, the implicit GEMM's row-major output.
    std::set<std::string> nhwc;
    std::vector<FusedQdqConv *> convs;
    int64_t conv_ws = 0;
    auto scalar_of = [&](const Variable &v, float &val) {
        const std::vector<float> f = host_floats(v);
        if (f.size() != 1) return false;
        val = f[0];
        return true;
    };
    // QuantizeLinear to e4m3 with a constant per-tensor scale and no zero point
    auto static_q = [&](int qi) {
        if (qi < 0 || nodes[qi].get_op_type() != "QuantizeLinear") return false;
        const Node &qn = nodes[qi];
        float s;
        if (!scalar_of(*qn.get_inputs()[1], s) || qn.get_outputs()[0]->get_dtype() != DataType::FLOAT8E4M3FN) return false;
        if (qn.get_inputs().size() > 2) {
            if (!qn.get_inputs()[2]->is_constant()) return false;
            for (char ch : qn.get_inputs()[2]->get_raw_data())
                if (ch != 0) return false;
        }
        return true;
    };
    auto ints_or = [&](const Node &n, const char *name, std::vector<int64_t> dflt) {
        if (auto p = n.try_get_attr(name)) return p->get<AttributeType::INTS>();
        return dflt;
    };
    auto auto_pad_ok = [&](const Node &n) {
        if (auto p = n.try_get_attr("auto_pad")) {
            const std::string s = p->get<AttributeType::STRING>();
            return s.empty() || s == "NOTSET";
        }
        return true;
    };
    for (size_t ci = 0; ci < nodes.size(); ++ci) {
        const Node &cn = nodes[ci];
        if (fusion_[ci]->skip || fusion_[ci]->op) continue;
        const std::string &kind = cn.get_op_type();
        if (kind == "Conv") {
            const int64_t G = attr_int(cn, "group", 1);  // grouped: conv.cpp:62-63, :122-139
            if (cn.get_inputs().size() < 2 || G < 1 || !auto_pad_ok(cn)) continue;
            const int dx = producer_of(cn.get_inputs()[0]->get_name());
            const int dw = producer_of(cn.get_inputs()[1]->get_name());
            if (!dq_ok(dx) || !dq_ok(dw) || dq_scale_len(dx) != 1) continue;
            const Variable &xq = *nodes[dx].get_inputs()[0], &wq = *nodes[dw].get_inputs()[0];
            const Variable &yv = *cn.get_outputs()[0];
            if (!wq.is_constant() || !table_.contains(wq.get_name()) || wq.get_shape().size() != 4 ||
                xq.get_shape().size() != 4 || yv.get_shape().size() != 4)
                continue;
            const int64_t M = static_cast<int64_t>(wq.get_shape()[0]), C = static_cast<int64_t>(wq.get_shape()[1]);
            const int64_t lw = dq_scale_len(dw);
            if (lw != 1 && (lw != M || attr_int(nodes[dw], "axis", 1) != 0)) continue;
            if (static_cast<int64_t>(xq.get_shape()[1]) != C * G || M % G != 0) continue;  // C: channels per group
            const auto ks = ints_or(cn, "kernel_shape", {static_cast<int64_t>(wq.get_shape()[2]), static_cast<int64_t>(wq.get_shape()[3])});
            const auto st = ints_or(cn, "strides", {1, 1});
            const auto pd = ints_or(cn, "pads", {0, 0, 0, 0});
            const auto dl = ints_or(cn, "dilations", {1, 1});
            if (ks.size() != 2 || st.size() != 2 || pd.size() != 4 || dl.size() != 2) continue;
            if (ks[0] != static_cast<int64_t>(wq.get_shape()[2]) || ks[1] != static_cast<int64_t>(wq.get_shape()[3])) continue;
            std::vector<int> folded;
            auto op = std::make_unique<FusedQdqConv>();
            auto &fi = *fusion_[ci];
            fi.inputs = {xq.get_name(), nodes[dx].get_inputs()[1]->get_name(), "", nodes[dw].get_inputs()[1]->get_name()};
            if (cn.get_inputs().size() > 2) {
                const Variable &bv = *cn.get_inputs()[2];
                if (!bv.is_constant() || bv.get_dtype() != DataType::FLOAT || !table_.contains(bv.get_name())) continue;
                op->has_bias = true;
                fi.inputs.push_back(bv.get_name());
            }
            // epilogue chain: (Add of a DequantizeLinear'd NHWC e4m3 residual) (Relu) QuantizeLinear
            std::string out = yv.get_name();
            int c = sole_consumer(out);
            int epi = LCML_EPI_NONE;
            if (c >= 0 && nodes[c].get_op_type() == "Add" && nodes[c].get_inputs().size() == 2) {
                const Node &an = nodes[c];
                const Variable *other = an.get_inputs()[0]->get_name() == out ? an.get_inputs()[1] : an.get_inputs()[0];
                const int dr = producer_of(other->get_name());
                if (dq_ok(dr) && dq_scale_len(dr) == 1 && nhwc.count(nodes[dr].get_inputs()[0]->get_name()) &&
                    nodes[dr].get_inputs()[0]->get_shape() == yv.get_shape() && an.get_outputs()[0]->get_shape() == yv.get_shape()) {
                    op->has_residual = true;
                    fi.inputs.push_back(nodes[dr].get_inputs()[0]->get_name());
                    fi.inputs.push_back(nodes[dr].get_inputs()[1]->get_name());
                    folded.push_back(c);
                    out = an.get_outputs()[0]->get_name();
                    c = sole_consumer(out);
                }
            }
            if (c >= 0 && nodes[c].get_op_type() == "Relu") {
                epi = LCML_EPI_RELU;
                folded.push_back(c);
                out = nodes[c].get_outputs()[0]->get_name();
                c = sole_consumer(out);
            }
            if (!static_q(c)) {
                fi.inputs.clear();
                continue;  // the output must be requantized to stay on the e4m3 path
            }
            folded.push_back(c);
            fi.inputs.push_back(nodes[c].get_inputs()[1]->get_name());
            out = nodes[c].get_outputs()[0]->get_name();
            lcml_fp8_conv_desc &d = op->desc;
            d.N = static_cast<int64_t>(xq.get_shape()[0]);
            d.C = C * G;
            d.H = static_cast<int64_t>(xq.get_shape()[2]);
            d.W = static_cast<int64_t>(xq.get_shape()[3]);
            d.M = M;
            d.kH = ks[0];
            d.kW = ks[1];
            d.oH = static_cast<int64_t>(yv.get_shape()[2]);
            d.oW = static_cast<int64_t>(yv.get_shape()[3]);
            d.sH = static_cast<int>(st[0]);
            d.sW = static_cast<int>(st[1]);
            d.pH = static_cast<int>(pd[0]);
            d.pW = static_cast<int>(pd[1]);
            d.dH = static_cast<int>(dl[0]);
            d.dW = static_cast<int>(dl[1]);
            d.group = static_cast<int>(G);
            d.x_nhwc = nhwc.count(xq.get_name()) ? 1 : 0;
            d.epilogue = epi;
            // the output extent of the graph must be what these pads and strides give
            if (d.oH != (d.H + pd[0] + pd[2] - d.dH * (d.kH - 1) - 1) / d.sH + 1 ||
                d.oW != (d.W + pd[1] + pd[3] - d.dW * (d.kW - 1) - 1) / d.sW + 1) {
                fi.inputs.clear();
                continue;
            }
            // weights packed once into the GEMM's K-major [M, Kp] layout
            const int64_t Kp = lcml_fp8_conv_packed_k(C, d.kH, d.kW);
            auto wp = DeviceTensor::allocate(DataType::FLOAT8E4M3FN, {M, Kp});
            check_status(lcml_fp8_conv_pack_weight(table_.at(wq.get_name()).ptr<uint8_t>(), M, C, d.kH, d.kW,
                                                   wp->ptr<uint8_t>(), stream_),
                         "pack conv weight");
            wp->set_constant({});
            const std::string wname = wq.get_name() + "#packed";
            if (!table_.contains(wname)) table_.own(wname, std::move(wp));
            fi.inputs[2] = wname;
            conv_ws = std::max<int64_t>(conv_ws, lcml_fp8_conv_workspace_size(&d));
            std::string note = "DequantizeLinear x2 + Conv";
            for (int f : folded) note += " + " + nodes[f].get_op_type();
            fi.note = note + " fused into one implicit-GEMM conv";
            fi.outputs = {out};
            convs.push_back(op.get());
            fi.op = std::move(op);
            for (int f : folded) {
                fusion_[f]->skip = true;
                fusion_[f]->note = "folded into Conv " + cn.get_name();
            }
            nhwc.insert(out);
        } else if (kind == "MaxPool") {
            const int dx = producer_of(cn.get_inputs()[0]->get_name());
            const int q = sole_consumer(cn.get_outputs()[0]->get_name());
            if (!dq_ok(dx) || dq_scale_len(dx) != 1 || !static_q(q) || !auto_pad_ok(cn)) continue;
            float s_in, s_out;
            if (!scalar_of(*nodes[dx].get_inputs()[1], s_in) || !scalar_of(*nodes[q].get_inputs()[1], s_out) ||
                s_in != s_out || !(s_in > 0.0f))
                continue;  // same positive scale: the max commutes with the encoding
            const auto ks = ints_or(cn, "kernel_shape", {});
            const auto st = ints_or(cn, "strides", {1, 1});
            const auto pd = ints_or(cn, "pads", {0, 0, 0, 0});
            const auto dl = ints_or(cn, "dilations", {1, 1});
            if (ks.size() != 2 || st.size() != 2 || pd.size() != 4 || dl != std::vector<int64_t>{1, 1} ||
                attr_int(cn, "ceil_mode", 0) != 0 || cn.get_outputs().size() != 1)
                continue;
            const Variable &xq = *nodes[dx].get_inputs()[0];
            auto op = std::make_unique<QdqMaxPool>();
            op->kH = static_cast<int>(ks[0]);
            op->kW = static_cast<int>(ks[1]);
            op->sH = static_cast<int>(st[0]);
            op->sW = static_cast<int>(st[1]);
            op->pH = static_cast<int>(pd[0]);
            op->pW = static_cast<int>(pd[1]);
            op->nhwc = nhwc.count(xq.get_name()) > 0;
            auto &fi = *fusion_[ci];
            fi.inputs = {xq.get_name()};
            fi.outputs = {nodes[q].get_outputs()[0]->get_name()};
            fi.note = "DequantizeLinear + MaxPool + QuantizeLinear (same scale) run as one e4m3 max pool";
            if (op->nhwc) nhwc.insert(fi.outputs[0]);
            fi.op = std::move(op);
            fusion_[q]->skip = true;
            fusion_[q]->note = "folded into MaxPool " + cn.get_name();
        } else if (kind == "GlobalAveragePool") {
            const int dx = producer_of(cn.get_inputs()[0]->get_name());
            if (!dq_ok(dx) || dq_scale_len(dx) != 1 || cn.get_outputs()[0]->get_dtype() != DataType::FLOAT) continue;
            const Variable &xq = *nodes[dx].get_inputs()[0];
            auto op = std::make_unique<QdqGlobalAveragePool>();
            op->nhwc = nhwc.count(xq.get_name()) > 0;
            auto &fi = *fusion_[ci];
            fi.inputs = {xq.get_name(), nodes[dx].get_inputs()[1]->get_name()};
            fi.outputs = {cn.get_outputs()[0]->get_name()};
            fi.note = "DequantizeLinear + GlobalAveragePool read the e4m3 tensor directly";
            fi.op = std::move(op);  // [N, C, 1, 1] is the same in both layouts
        }
    }
    if (!convs.empty() && conv_ws > 0) {
        auto ws = DeviceTensor::allocate(DataType::UINT8, {conv_ws});
        for (auto *c : convs) c->workspace = ws->data();
        table_.own("#conv_workspace", std::move(ws));
    }

    // ---- fp32 Gemm -> Relu (graphs without QDQ on the activations, e.g. the MLP): one kernel
    for (size_t i = 0; i < nodes.size(); ++i) {
        FusionInfo &fi = *fusion_[i];
        if (fi.skip || fi.op || nodes[i].get_op_type() != "Gemm") continue;
        const auto &outs = nodes[i].get_outputs();
        if (outs.size() != 1 || outs[0]->get_dtype() != DataType::FLOAT) continue;
        const int r = sole_consumer(outs[0]->get_name());
        if (r < 0 || nodes[r].get_op_type() != "Relu" || fusion_[r]->skip || fusion_[r]->op) continue;
        bool fp32 = true;
        for (const auto *x : nodes[i].get_inputs()) fp32 = fp32 && x->get_dtype() == DataType::FLOAT;
        if (!fp32) continue;
        fi.op = make_gemm_f32_relu(nodes[i]);
        for (const auto *x : nodes[i].get_inputs()) fi.inputs.push_back(x->get_name());
        fi.outputs = {nodes[r].get_outputs()[0]->get_name()};
        fi.note = "fp32 Gemm + Relu in one kernel";
        fusion_[r]->skip = true;
        fusion_[r]->note = "Relu folded into the preceding Gemm";
    }

    // ---- Dead nodes: a node that still runs but whose outputs nobody reads any more
    // (a DequantizeLinear whose consumers all read its e4m3 input inside a fusion) is dropped.
    auto effective_inputs = [&](size_t i) {
        std::vector<std::string> v = fusion_[i]->inputs;
        if (v.empty())
            for (const auto *x : nodes[i].get_inputs()) v.push_back(x->get_name());
        return v;
    };
    auto effective_outputs = [&](size_t i) {
        std::vector<std::string> v = fusion_[i]->outputs;
        if (v.empty())
            for (const auto *x : nodes[i].get_outputs()) v.push_back(x->get_name());
        return v;
    };
    for (bool changed = true; changed;) {
        changed = false;
        std::set<std::string> live(graph_outputs.begin(), graph_outputs.end());
        for (size_t i = 0; i < nodes.size(); ++i)
            if (!fusion_[i]->skip)
                for (const auto &n : effective_inputs(i)) live.insert(n);
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (fusion_[i]->skip) continue;
            bool used = false;
            for (const auto &n : effective_outputs(i)) used |= live.count(n) > 0;
            if (!used) {
                fusion_[i]->skip = true;
                fusion_[i]->note = "its output is only read inside fusions";
                changed = true;
            }
        }
    }

    // every reader of an NHWC tensor must be one of the layout-aware fused kernels
    nhwc_.insert(nhwc.begin(), nhwc.end());
    for (const auto &name : nhwc) {
        if (graph_outputs.count(name)) throw Error("tensor '" + name + "' is stored NHWC but is a graph output");
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (fusion_[i]->skip) continue;
            const auto ins = effective_inputs(i);
            if (std::find(ins.begin(), ins.end(), name) == ins.end()) continue;
            const Operator *o = fusion_[i]->op.get();
            const bool aware = dynamic_cast<const FusedQdqConv *>(o) || dynamic_cast<const QdqMaxPool *>(o) ||
                               dynamic_cast<const QdqGlobalAveragePool *>(o);
            if (!aware)
                throw Error("NHWC tensor '" + name + "' reaches " + nodes[i].get_op_type() + " " + nodes[i].get_name() +
                            ", which cannot read that layout");
        }
    }
}

// DequantizeLinear / QuantizeLinear whose inputs are all constants (e.g. the
// DQ of a weight feeding an fp32 Gemm) run once here; the node is then folded.
void NetworkInstance::fold_constants() {
    const Graph &g = model_.get_graph();
    const auto &nodes = g.get_nodes();
    std::set<std::string> graph_outputs;
    for (const auto *v : g.get_outputs()) graph_outputs.insert(v->get_name());
    for (size_t i = 0; i < nodes.size(); ++i) {
        if (fusion_[i]->skip) continue;
        const std::string &op = nodes[i].get_op_type();
        if (op != "DequantizeLinear" && op != "QuantizeLinear") continue;
        bool all_const = true;
        for (const auto *in : nodes[i].get_inputs())
            if (!in->is_constant() || !table_.contains(in->get_name())) all_const = false;
        const Variable &out = *nodes[i].get_outputs()[0];
        if (!all_const || graph_outputs.count(out.get_name()) || table_.contains(out.get_name())) continue;
        auto t = DeviceTensor::allocate(out.get_dtype(), to_shape(out.get_shape()));
        std::vector<std::reference_wrapper<ITensor>> ins, outs;
        for (const auto *in : nodes[i].get_inputs()) ins.emplace_back(table_.at(in->get_name()));
        outs.emplace_back(*t);
        ops_[i]->set_environment(*this, table_);
        ops_[i]->forward(ins, outs);
        t->set_constant({});
        table_.own(out.get_name(), std::move(t));
        fusion_[i]->skip = true;
        fusion_[i]->note = "constant-folded at prepare";
    }
}

void NetworkInstance::prepare() {
    const Graph &g = model_.get_graph();
    const auto &nodes = g.get_nodes();
    ops_.clear();
    fusion_.clear();
    table_.clear();
    nhwc_.clear();
    for (const auto &n : nodes) {
        ops_.push_back(model_.get_opset().create_operator(n.get_op_type(), n));
        fusion_.push_back(std::make_unique<FusionInfo>());
    }
    create_tensors();
    if (fusion_enabled_) {
        run_fusion_pass();
        fold_constants();
    }

    allocate_intermediates();
    prepared_ = true;
}

// 4. Intermediates touched by nodes that still run; view ops alias their input.
// With memory reuse, each intermediate lives from the step of the node that
// writes it to the step of its last reader (a view's readers count for the
// tensor it aliases), and the tensors are placed in one arena: largest first,
// each at the lowest 256-byte aligned offset whose range no tensor of an
// overlapping lifetime occupies (the reference colours registers with the
// same last-use information, network_instance.cpp:369-474, :476-582). Nodes
// run in order on one stream, so a dead tensor's bytes are rewritten only
// after its readers have run.
void NetworkInstance::allocate_intermediates() {
    const Graph &g = model_.get_graph();
    const auto &nodes = g.get_nodes();
    auto io_inputs = [&](size_t i) {
        std::vector<std::string> v;
        if (!fusion_[i]->inputs.empty()) return fusion_[i]->inputs;
        for (const auto *x : nodes[i].get_inputs()) v.push_back(x->get_name());
        return v;
    };
    auto io_outputs = [&](size_t i) {
        std::vector<std::string> v;
        if (!fusion_[i]->outputs.empty()) return fusion_[i]->outputs;
        for (const auto *x : nodes[i].get_outputs()) v.push_back(x->get_name());
        return v;
    };
    struct Life {
        std::string name;
        size_t bytes;
        int first, last;
        size_t offset = 0;
    };
    std::vector<Life> lives;
    std::map<std::string, size_t> life_of;   // planned tensor -> index in lives
    std::map<std::string, std::string> alias;  // view -> the tensor whose bytes it names
    std::vector<std::pair<std::string, size_t>> views;  // (view name, node index) in creation order
    auto root = [&](std::string n) {
        for (auto it = alias.find(n); it != alias.end(); it = alias.find(n)) n = it->second;
        return n;
    };
    int step = 0;
    for (size_t i = 0; i < nodes.size(); ++i, ++step) {
        if (fusion_[i]->skip) {
            --step;
            continue;
        }
        for (const auto &name : io_inputs(i)) {
            auto it = life_of.find(root(name));
            if (it != life_of.end()) lives[it->second].last = step;
            else if (!table_.contains(name) && !alias.count(name))
                throw Error("input '" + name + "' of node " + nodes[i].get_name() + " is not bound");
        }
        for (const auto &name : io_outputs(i)) {
            if (table_.contains(name) || life_of.count(name) || alias.count(name)) continue;
            const Variable &v = g.get_var(name);
            const std::string src = nodes[i].get_inputs().empty() ? std::string() : nodes[i].get_inputs()[0]->get_name();
            const bool view = ops_[i]->is_output_view(0, nodes[i]) && !src.empty() &&
                              (table_.contains(src) || life_of.count(root(src)));
            if (view) {
                alias[name] = src;
                views.emplace_back(name, i);
                continue;
            }
            life_of[name] = lives.size();
            lives.push_back({name, ((dtype_nbytes(v.get_dtype(), [&] {
                                         size_t n = 1;
                                         for (auto d : v.get_shape()) n *= d;
                                         return n;
                                     }()) + 255) / 256) * 256,
                             step, step});
        }
    }
    // a graph output the caller did not bind stays intact to the end (the
    // reference never reclaims graph outputs, network_instance.cpp:453-456)
    for (const auto *o : g.get_outputs()) {
        auto it = life_of.find(root(o->get_name()));
        if (it != life_of.end()) lives[it->second].last = step;
    }
    size_t unplanned = 0;
    for (const auto &l : lives) unplanned += l.bytes;
    intermediate_unplanned_ = unplanned;
    if (reuse_memory_ && !lives.empty()) {
        std::vector<size_t> order(lives.size());
        for (size_t k = 0; k < order.size(); ++k) order[k] = k;
        std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return lives[a].bytes > lives[b].bytes; });
        std::vector<size_t> placed;
        size_t arena = 0;
        for (size_t k : order) {
            Life &t = lives[k];
            // offsets of placed tensors alive at the same time, by start
            std::vector<std::pair<size_t, size_t>> busy;
            for (size_t p : placed)
                if (lives[p].first <= t.last && t.first <= lives[p].last)
                    busy.emplace_back(lives[p].offset, lives[p].offset + lives[p].bytes);
            std::sort(busy.begin(), busy.end());
            size_t off = 0;
            for (const auto &[b, e] : busy) {
                if (off + t.bytes <= b) break;  // fits in the gap before this range
                off = std::max(off, e);
            }
            t.offset = off;
            arena = std::max(arena, off + t.bytes);
            placed.push_back(k);
        }
        auto buf = DeviceTensor::allocate(DataType::UINT8, {static_cast<int64_t>(arena)});
        uint8_t *base = buf->ptr<uint8_t>();
        table_.own("#intermediate_arena", std::move(buf));
        for (const auto &t : lives) {
            const Variable &v = g.get_var(t.name);
            table_.own(t.name, DeviceTensor::borrow(v.get_dtype(), to_shape(v.get_shape()), base + t.offset));
        }
        intermediate_bytes_ = arena;
    } else {
        for (const auto &t : lives) {
            const Variable &v = g.get_var(t.name);
            table_.own(t.name, DeviceTensor::allocate(v.get_dtype(), to_shape(v.get_shape())));
        }
        intermediate_bytes_ = unplanned;
    }
    for (const auto &[name, i] : views) {
        const Variable &v = g.get_var(name);
        ITensor &src = table_.at(alias.at(name));
        auto t = DeviceTensor::borrow(v.get_dtype(), to_shape(v.get_shape()), src.data());
        t->set_view(true);
        if (t->nbytes() != src.nbytes()) throw Error(nodes[i].get_op_type() + ": view changes the byte size");
        table_.own(name, std::move(t));
    }
}

void NetworkInstance::forward() {
    if (!prepared_) prepare();
    const auto &nodes = model_.get_graph().get_nodes();
    std::vector<std::reference_wrapper<ITensor>> ins, outs;
    // host-staged inputs: copy on the second stream once the previous
    // forward's last reader of them has run; this forward's nodes wait for it
    size_t last_reader = nodes.size();
    if (!host_in_.empty()) {
        if (!copy_stream_) {
            check_status(lcml_stream_create(&copy_stream_), "copy stream");
            check_status(lcml_event_create(&in_ready_), "event");
            check_status(lcml_event_create(&in_free_), "event");
        }
        if (in_free_recorded_) check_status(lcml_stream_wait_event(copy_stream_, in_free_), "wait");
        for (const auto &[name, host] : host_in_) {
            ITensor &t = *inputs_.at(name);
            check_status(lcml_memcpy_async(t.data(), host, t.nbytes(), 1, copy_stream_), "input copy");
        }
        check_status(lcml_event_record(in_ready_, copy_stream_), "record");
        check_status(lcml_stream_wait_event(stream_, in_ready_), "wait");
        for (size_t i = 0; i < nodes.size(); ++i) {
            if (fusion_[i]->skip) continue;
            auto reads = [&](const std::string &n) { return host_in_.count(n) > 0; };
            bool r = false;
            if (!fusion_[i]->inputs.empty()) {
                for (const auto &n : fusion_[i]->inputs) r = r || reads(n);
            } else {
                for (const auto *x : nodes[i].get_inputs()) r = r || reads(x->get_name());
            }
            if (r) last_reader = i;
        }
    }
    // the previous forward copied its outputs on the output stream: the
    // first node that writes a bound output waits until that copy has read it
    size_t first_out_writer = nodes.size();
    if (last_out_async_) {
        auto writes = [&](const std::string &n) { return outputs_.count(n) > 0; };
        for (size_t i = 0; i < nodes.size() && first_out_writer == nodes.size(); ++i) {
            if (fusion_[i]->skip) continue;
            bool w = false;
            if (!fusion_[i]->outputs.empty()) {
                for (const auto &n : fusion_[i]->outputs) w = w || writes(n);
            } else {
                for (const auto *x : nodes[i].get_outputs()) w = w || writes(x->get_name());
            }
            if (w) first_out_writer = i;
        }
    }
    for (size_t i = 0; i < nodes.size(); ++i) {
        FusionInfo &fi = *fusion_[i];
        if (fi.skip) continue;
        if (i == first_out_writer) check_status(lcml_stream_wait_event(stream_, out_free_), "wait");
        ins.clear();
        outs.clear();
        if (!fi.inputs.empty()) {
            for (const auto &n : fi.inputs) ins.emplace_back(table_.at(n));
        } else {
            for (const auto *x : nodes[i].get_inputs()) ins.emplace_back(table_.at(x->get_name()));
        }
        if (!fi.outputs.empty()) {
            for (const auto &n : fi.outputs) outs.emplace_back(table_.at(n));
        } else {
            for (const auto *x : nodes[i].get_outputs()) outs.emplace_back(table_.at(x->get_name()));
        }
        Operator &op = fi.op ? *fi.op : *ops_[i];
        op.set_environment(*this, table_);
        if (logging_) std::fprintf(stderr, "[lcml] node %zu %s (%s)\n", i, nodes[i].get_op_type().c_str(), op.get_name().c_str());
        op.forward(ins, outs);
        if (i == last_reader) {
            check_status(lcml_event_record(in_free_, stream_), "record");
            in_free_recorded_ = true;
        }
    }
    last_out_async_ = false;
    if (host_out_.empty()) return;
    lcml_stream_t out = stream_;
    if (async_out_) {
        if (!out_stream_) {
            check_status(lcml_stream_create(&out_stream_), "output stream");
            check_status(lcml_event_create(&out_ready_), "event");
            check_status(lcml_event_create(&out_free_), "event");
        }
        check_status(lcml_event_record(out_ready_, stream_), "record");
        check_status(lcml_stream_wait_event(out_stream_, out_ready_), "wait");
        out = out_stream_;
    }
    for (const auto &[name, host] : host_out_) {
        ITensor &t = *outputs_.at(name);
        check_status(lcml_memcpy_async(host, t.data(), t.nbytes(), 2, out), "output copy");
    }
    if (async_out_) {
        check_status(lcml_event_record(out_free_, out_stream_), "record");
        last_out_async_ = true;
    }
}

}// namespace lcml::onnx
