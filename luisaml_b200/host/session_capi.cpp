// C ABI over NetworkInstance (include/lcml_session.h).
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/lcml_onnx.h"
#include "../../include/lcml_session.h"

namespace lcml::onnx {
int operators_registered();
}

using namespace lcml::onnx;

struct lcml_network {
    NetworkInstance inst;
    std::vector<std::unique_ptr<DeviceTensor>> bound;  // borrowed wrappers of caller buffers
};

namespace {
thread_local std::string t_err;

int fail(int status, const std::string &msg) {
    t_err = msg;
    return status;
}

template <typename F>
int guard(F &&f) {
    try {
        f();
        return LCML_OK;
    } catch (const std::exception &e) {
        return fail(LCML_ERR_INVALID_ARGUMENT, e.what());
    }
}

ITensor::shape_type to_shape(const int64_t *shape, int ndim) {
    ITensor::shape_type s;
    for (int i = 0; i < ndim; ++i) s.push_back(shape[i]);
    return s;
}
}// namespace

extern "C" {

const char *lcml_network_last_error(void) { return t_err.c_str(); }

int lcml_opset_size(void) { return operators_registered(); }

int lcml_network_create(const char *json, size_t len, lcml_network **out) {
    if (!json || !out) return fail(LCML_ERR_INVALID_ARGUMENT, "lcml_network_create: null argument");
    *out = nullptr;
    return guard([&] {
        auto net = std::make_unique<lcml_network>();
        net->inst.set_model(Model::load_from_json(std::string_view(json, len)));
        *out = net.release();
    });
}

void lcml_network_destroy(lcml_network *net) { delete net; }

int lcml_network_info(const lcml_network *net, int64_t *num_nodes, int64_t *num_inputs, int64_t *num_outputs) {
    if (!net) return fail(LCML_ERR_INVALID_ARGUMENT, "null network");
    const Graph &g = net->inst.get_model().get_graph();
    if (num_nodes) *num_nodes = static_cast<int64_t>(g.get_nodes().size());
    if (num_inputs) *num_inputs = static_cast<int64_t>(g.get_inputs().size());
    if (num_outputs) *num_outputs = static_cast<int64_t>(g.get_outputs().size());
    return LCML_OK;
}

int lcml_network_set_weight_buffer(lcml_network *net, const void *p, size_t bytes) {
    if (!net) return fail(LCML_ERR_INVALID_ARGUMENT, "null network");
    return guard([&] { net->inst.set_weight_buffer(p, bytes); });
}

int lcml_network_set_input(lcml_network *net, const char *name, const void *p, int dtype, const int64_t *shape, int ndim) {
    if (!net || !name || (ndim > 0 && !shape)) return fail(LCML_ERR_INVALID_ARGUMENT, "lcml_network_set_input: null argument");
    return guard([&] {
        net->bound.push_back(DeviceTensor::borrow(static_cast<DataType>(dtype), to_shape(shape, ndim), const_cast<void *>(p)));
        net->inst.set_input(name, *net->bound.back());
    });
}

int lcml_network_set_output(lcml_network *net, const char *name, void *p, int dtype, const int64_t *shape, int ndim) {
    if (!net || !name || (ndim > 0 && !shape)) return fail(LCML_ERR_INVALID_ARGUMENT, "lcml_network_set_output: null argument");
    return guard([&] {
        net->bound.push_back(DeviceTensor::borrow(static_cast<DataType>(dtype), to_shape(shape, ndim), p));
        net->inst.set_output(name, *net->bound.back());
    });
}

int lcml_network_set_input_host(lcml_network *net, const char *name, const void *host) {
    if (!net || !name) return fail(LCML_ERR_INVALID_ARGUMENT, "lcml_network_set_input_host: null argument");
    return guard([&] { net->inst.set_input_host(name, host); });
}

int lcml_network_set_output_host(lcml_network *net, const char *name, void *host) {
    if (!net || !name) return fail(LCML_ERR_INVALID_ARGUMENT, "lcml_network_set_output_host: null argument");
    return guard([&] { net->inst.set_output_host(name, host); });
}

int lcml_network_set_async_outputs(lcml_network *net, int enable) {
    if (!net) return fail(LCML_ERR_INVALID_ARGUMENT, "null network");
    net->inst.enable_async_output_copy(enable != 0);
    return LCML_OK;
}

int lcml_network_wait_outputs(lcml_network *net, lcml_stream_t stream) {
    if (!net) return fail(LCML_ERR_INVALID_ARGUMENT, "null network");
    return guard([&] { net->inst.wait_outputs(stream); });
}

int lcml_network_set_fusion(lcml_network *net, int enable) {
    if (!net) return fail(LCML_ERR_INVALID_ARGUMENT, "null network");
    net->inst.enable_fusion(enable != 0);
    return LCML_OK;
}

int lcml_network_set_memory_reuse(lcml_network *net, int enable) {
    if (!net) return fail(LCML_ERR_INVALID_ARGUMENT, "null network");
    net->inst.enable_memory_reuse(enable != 0);
    return LCML_OK;
}

int lcml_network_memory(const lcml_network *net, size_t *intermediate_bytes, size_t *unplanned_bytes) {
    if (!net || !intermediate_bytes || !unplanned_bytes) return fail(LCML_ERR_INVALID_ARGUMENT, "null argument");
    *intermediate_bytes = net->inst.intermediate_bytes();
    *unplanned_bytes = net->inst.intermediate_bytes_unplanned();
    return LCML_OK;
}

int lcml_network_set_stream(lcml_network *net, lcml_stream_t s) {
    if (!net) return fail(LCML_ERR_INVALID_ARGUMENT, "null network");
    net->inst.set_stream(s);
    return LCML_OK;
}

int lcml_network_forward(lcml_network *net) {
    if (!net) return fail(LCML_ERR_INVALID_ARGUMENT, "null network");
    return guard([&] { net->inst.forward(); });
}

int lcml_network_executed_nodes(const lcml_network *net, int64_t *executed) {
    if (!net || !executed) return fail(LCML_ERR_INVALID_ARGUMENT, "null argument");
    *executed = static_cast<int64_t>(net->inst.num_executed_nodes());
    return LCML_OK;
}

int lcml_network_tensor(const lcml_network *net, const char *name, void **device_ptr, int *dtype, int64_t *shape,
                        int max_ndim, int *ndim, int *nhwc) {
    if (!net || !name || !device_ptr || !dtype || !ndim || (max_ndim > 0 && !shape))
        return fail(LCML_ERR_INVALID_ARGUMENT, "lcml_network_tensor: null argument");
    auto &inst = const_cast<NetworkInstance &>(net->inst);
    if (!inst.tensor_table().contains(name))
        return fail(LCML_ERR_INVALID_ARGUMENT, std::string("lcml_network_tensor: no tensor '") + name +
                                                   "' (not prepared yet, or not materialized by the fused graph)");
    ITensor &t = inst.tensor_table().at(name);
    *device_ptr = t.data();
    *dtype = static_cast<int>(t.dtype());
    *ndim = static_cast<int>(t.ndim());
    for (int i = 0; i < max_ndim && i < *ndim; ++i) shape[i] = t.shape(i);
    if (nhwc) *nhwc = inst.is_nhwc(name) ? 1 : 0;
    return LCML_OK;
}

int lcml_network_summary(const lcml_network *net, char *buf, size_t len) {
    if (!net || !buf || len == 0) return fail(LCML_ERR_INVALID_ARGUMENT, "null argument");
    std::string s;
    for (const auto &l : net->inst.executed_node_summary()) s += l + "\n";
    std::strncpy(buf, s.c_str(), len - 1);
    buf[len - 1] = '\0';
    return LCML_OK;
}

}// extern "C"
