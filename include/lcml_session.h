/*
 * lcml_session.h — C ABI over the C++ NetworkInstance (include/lcml_onnx.h)
 * for hosts that bind through a foreign-function interface (Python ctypes in
 * this repository's tests and bench). Mirrors the reference's executor use
 * in tests/onnx/test_onnx_inference.cpp:150-224: load the LuisaML-JSON model
 * (Model::load_from_json, src/onnx/onnx.cpp:235), bind the weight buffer and
 * the named inputs/outputs (NetworkInstance::set_weight_buffer / set_input /
 * set_output, include/onnx/network_instance.h:185-208) and run forward()
 * (network_instance.cpp:701). Device pointers are caller-owned.
 * Every function returns 0 or an lcml_status; lcml_network_last_error()
 * has the message.
 */
#ifndef LCML_SESSION_H
#define LCML_SESSION_H

#include <stddef.h>
#include <stdint.h>

#include "lcml_fp8.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lcml_network lcml_network;

const char *lcml_network_last_error(void);
/* Parses a LuisaML-JSON model; every node's op must be registered. */
int lcml_network_create(const char *json, size_t json_len, lcml_network **out);
void lcml_network_destroy(lcml_network *net);
/* Number of nodes and of registered operator names (introspection). */
int lcml_network_info(const lcml_network *net, int64_t *num_nodes, int64_t *num_inputs, int64_t *num_outputs);
int lcml_network_set_weight_buffer(lcml_network *net, const void *device_ptr, size_t bytes);
/* Binds a caller-owned device tensor: dtype is an ONNX DataType number,
 * shape/ndim must equal the graph's declaration for that name. */
int lcml_network_set_input(lcml_network *net, const char *name, const void *device_ptr, int dtype,
                           const int64_t *shape, int ndim);
int lcml_network_set_output(lcml_network *net, const char *name, void *device_ptr, int dtype, const int64_t *shape,
                            int ndim);
/* Host-staged I/O (no reference counterpart). `host` (pinned, of the bound
 * tensor's byte size; NULL removes it) is copied into the bound input at the
 * start of every forward on a second stream, overlapping the previous
 * forward once that forward's last reader of the input has run; a bound
 * output's host buffer is filled after the last node, on the network's
 * stream. The tensor must be bound (set_input / set_output) first. */
int lcml_network_set_input_host(lcml_network *net, const char *name, const void *host);
int lcml_network_set_output_host(lcml_network *net, const char *name, void *host);
/* 1: host-staged outputs are copied on a third stream after the last node,
 * overlapping the next forward (whose writer of each output waits only for
 * that copy); the host buffers are complete after lcml_network_wait_outputs.
 * 0 (default): copied on the network's stream. */
int lcml_network_set_async_outputs(lcml_network *net, int enable);
/* stream NULL: the host waits until every output copy enqueued so far is
 * done; otherwise `stream` waits for them (enqueued, no host wait). */
int lcml_network_wait_outputs(lcml_network *net, lcml_stream_t stream);
/* 1 (default): QDQ node groups run as fused kernels; 0: one kernel per node. */
int lcml_network_set_fusion(lcml_network *net, int enable);
int lcml_network_set_stream(lcml_network *net, lcml_stream_t stream);
/* 1 (default): intermediates share one device arena by lifetime (the last-use
 * analysis and pooled allocation of network_instance.cpp:369-582), so an
 * intermediate's bytes are reused once its last reader has run; 0: one
 * allocation per intermediate, all readable after forward (inspection). */
int lcml_network_set_memory_reuse(lcml_network *net, int enable);
/* After the first forward: device bytes of the intermediates as allocated
 * (the arena, or the sum of the separate allocations), and the bytes they
 * would take with one allocation each. */
int lcml_network_memory(const lcml_network *net, size_t *intermediate_bytes, size_t *unplanned_bytes);
/* Enqueues the whole graph on the stream (prepares on the first call). */
int lcml_network_forward(lcml_network *net);
/* After forward: nodes that launched work, and a one-line-per-node summary. */
int lcml_network_executed_nodes(const lcml_network *net, int64_t *executed);
int lcml_network_summary(const lcml_network *net, char *buf, size_t len);
/* After forward: the device buffer of any tensor of the graph (inputs,
 * outputs, intermediates, constants), like NetworkInstance::get_tensor_table()
 * (include/onnx/network_instance.h:231). shape receives up to max_ndim
 * extents of the ONNX shape; *nhwc is 1 when the tensor is stored NHWC (the
 * outputs of fused convolutions and pools), else 0. With memory reuse off
 * (lcml_network_set_memory_reuse) every intermediate keeps its contents until
 * the next forward; with it on, an intermediate's bytes may hold a later
 * tensor once its last reader has run. */
int lcml_network_tensor(const lcml_network *net, const char *name, void **device_ptr, int *dtype, int64_t *shape,
                        int max_ndim, int *ndim, int *nhwc);
/* Number of operators registered in the default opset. */
int lcml_opset_size(void);

#ifdef __cplusplus
}
#endif

#endif /* LCML_SESSION_H */
