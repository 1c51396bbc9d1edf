"""NetworkInstance on the GPU: whole graphs through the C++ executor.

* the reference's fp32 MLP known-answer fixture (tests/onnx/output/, copied to
  tests/golden/simple_mlp/) must reproduce output_ref.bin within the
  reference's own tolerance (abs 1e-3, tests/onnx/test_onnx_inference.cpp:232)
  and equal the CPU oracle's K-ordered fma result bit for bit;
* the QDQ MLP benchmark graph (e4m3 weights + DequantizeLinear) must equal the
  oracle bit for bit;
* a fully quantized graph (QuantizeLinear on activations) runs as fused FP8
  GEMMs and agrees with the unfused node-by-node execution and the oracle.
"""
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, assert_close

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.array(a, copy=True)).to(dev)


def test_reference_fp32_mlp_fixture(dev):
    import torch
    from luisaml_b200.session import Network
    d = os.path.join(GOLDEN, "simple_mlp")
    net = Network(open(os.path.join(d, "simple_mlp.onnx.json")).read())
    blob = np.fromfile(os.path.join(d, "simple_mlp.safetensors"), dtype=np.uint8)
    x = np.fromfile(os.path.join(d, "input_ref.bin"), dtype=np.float32).reshape(1, 784)
    ref = np.fromfile(os.path.join(d, "output_ref.bin"), dtype=np.float32).reshape(1, 10)
    wb, xt = _t(blob, dev), _t(x, dev)
    y = torch.empty((1, 10), dtype=torch.float32, device=dev)
    net.set_weight_buffer(wb)
    net.set_input("input", xt)
    net.set_output("output", y)
    net.forward()
    got = y.cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-3, (got, ref)
    # oracle: the same graph with gemm.cpp's loop on the host
    f = lambda name, off, shape: np.frombuffer(blob[off[0]:off[1]].tobytes(), dtype=np.float32).reshape(shape)  # noqa: E731
    import json
    inits = {i["name"]: i for i in json.load(open(os.path.join(d, "simple_mlp.onnx.json")))["graph"]["initializer"]}
    W = {k: f(k, v["data_offsets"], [int(s) for s in v["dims"]]) for k, v in inits.items()}
    h = oracle.relu(oracle.gemm(x, W["net.0.weight"], W["net.0.bias"], transB=1))
    h = oracle.relu(oracle.gemm(h, W["net.2.weight"], W["net.2.bias"], transB=1))
    h = oracle.gemm(h, W["net.4.weight"], W["net.4.bias"], transB=1)
    assert np.array_equal(got, h)


@pytest.mark.parametrize("fusion", [True, False])
def test_qdq_mlp_graph(dev, fusion):
    import torch
    from luisaml_b200 import graphs
    from luisaml_b200.session import Network
    text, blob, meta = graphs.mlp(batch=32)
    net = Network(text)
    net.set_fusion(fusion)
    x = np.random.default_rng(1000).random((32, 784), dtype=np.float32)
    y = torch.empty((32, 10), dtype=torch.float32, device=dev)
    net.set_weight_buffer(_t(np.frombuffer(blob, dtype=np.uint8), dev))
    net.set_input("input", _t(x, dev))
    net.set_output("output", y)
    net.forward()
    net.forward()  # a second forward reuses the prepared state
    h = x
    for i, L in enumerate(meta["layers"]):
        w = oracle.dequantize(L["q"], L["s"][0])
        h = oracle.gemm(h, w, L["bias"], transB=1)
        if i < 2:
            h = oracle.relu(h)
    assert np.array_equal(y.cpu().numpy(), h)
    # DQ of constant weights folded at prepare; with fusion each hidden Gemm runs with its Relu
    assert net.executed_nodes() == (3 if fusion else 8)


def test_host_staged_io(dev):
    """Host-staged inputs and outputs: forwards issued back to back, each
    with its own pinned input and output, give the device-bound results; the
    input copy of one forward (on the executor's second stream) must not
    overwrite the device input before the previous forward has read it, and
    with asynchronous output copies the next forward must not overwrite the
    device output before the previous copy has read it."""
    import torch
    from luisaml_b200 import graphs
    from luisaml_b200.session import Network
    B = 2048
    text, blob, meta = graphs.mlp(batch=B)
    wb = _t(np.frombuffer(blob, dtype=np.uint8), dev)
    xs = [np.random.default_rng(2000 + i).random((B, 784), dtype=np.float32) for i in range(4)]
    ref_net = Network(text)
    ref_net.set_weight_buffer(wb)
    xd = torch.empty((B, 784), dtype=torch.float32, device=dev)
    yd = torch.empty((B, 10), dtype=torch.float32, device=dev)
    ref_net.set_input("input", xd)
    ref_net.set_output("output", yd)
    want = []
    for x in xs:
        xd.copy_(torch.from_numpy(x))
        ref_net.forward()
        want.append(yd.cpu().numpy())
    net = Network(text)
    net.set_weight_buffer(wb)
    net.set_input("input", torch.empty((B, 784), dtype=torch.float32, device=dev))
    net.set_output("output", torch.empty((B, 10), dtype=torch.float32, device=dev))
    net.set_stream(torch.cuda.current_stream(dev).cuda_stream)
    hin = [torch.from_numpy(x).pin_memory() for x in xs]
    hout = [torch.full((B, 10), np.nan).pin_memory() for _ in xs]
    for rep in range(2):
        for i in range(len(xs)):
            net.set_input_host("input", hin[i])
            net.set_output_host("output", hout[i])
            net.forward()
        torch.cuda.synchronize()
        for i in range(len(xs)):
            np.testing.assert_array_equal(hout[i].numpy(), want[i])
            hout[i].fill_(np.nan)
    with pytest.raises(Exception):
        net.set_input_host("no_such_input", hin[0])
    # asynchronous output copies (third stream): the next forward's last
    # Gemm waits only for the previous copy of the output to have read it
    net.set_async_outputs(True)
    for rep in range(2):
        for i in range(len(xs)):
            net.set_input_host("input", hin[i])
            net.set_output_host("output", hout[i])
            net.forward()
        net.wait_outputs()
        for i in range(len(xs)):
            np.testing.assert_array_equal(hout[i].numpy(), want[i])
            hout[i].fill_(np.nan)
    s = torch.cuda.Stream(dev)
    net.forward()
    net.wait_outputs(s.cuda_stream)  # the stream waits: its copy of the host output sees the finished one
    got = torch.empty((B, 10), dtype=torch.float32, device=dev)
    with torch.cuda.stream(s):
        got.copy_(hout[len(xs) - 1], non_blocking=True)
    s.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), want[len(xs) - 1])
    # back to copies on the network's stream: the first writer of the output
    # still waits for the last asynchronous copy, and wait_outputs() now waits
    # for the network's stream
    net.set_async_outputs(False)
    for i in range(len(xs)):
        net.set_input_host("input", hin[i])
        net.set_output_host("output", hout[i])
        net.forward()
    net.wait_outputs()
    for i in range(len(xs)):
        np.testing.assert_array_equal(hout[i].numpy(), want[i])


def _quantized_mlp(batch, dims, seed):
    """x -> QuantizeLinear(static s_x) -> DequantizeLinear -> Gemm(DQ W, b) -> Relu
    -> QuantizeLinear(static) -> DequantizeLinear -> Gemm -> ... (activations and weights QDQ)."""
    from luisaml_b200.export import GraphBuilder, qdq_weight, scale_from_amax
    b = GraphBuilder("qdq_mlp_full")
    b.input("x", "FLOAT", (batch, dims[0]))
    rng = np.random.default_rng(seed)
    h = "x"
    meta = []
    for li in range(len(dims) - 1):
        sx = np.float32([0.02 if li else 1.0 / 448 * 4.5])  # calibrated-style static activation scales
        b.const(f"sx{li}", sx[0:1].reshape(()))
        q = b.value(f"xq{li}", "FLOAT8E4M3FN", (batch, dims[li]))
        b.node("QuantizeLinear", [h, f"sx{li}"], [q])
        dq = b.value(f"xdq{li}", "FLOAT", (batch, dims[li]))
        b.node("DequantizeLinear", [q, f"sx{li}"], [dq])
        w = (rng.standard_normal((dims[li + 1], dims[li])) / np.sqrt(dims[li])).astype(np.float32)
        wdq, wq, ws = qdq_weight(b, f"w{li}", w, axis=0)
        bias = (rng.standard_normal(dims[li + 1]) * 0.01).astype(np.float32)
        b.const(f"b{li}", bias)
        last = li == len(dims) - 2
        out = "y" if last else b.value(f"g{li}", "FLOAT", (batch, dims[li + 1]))
        if last:
            b.output("y", "FLOAT", (batch, dims[li + 1]))
        b.node("Gemm", [dq, wdq, f"b{li}"], [out], transB=1)
        if not last:
            r = b.value(f"r{li}", "FLOAT", (batch, dims[li + 1]))
            b.node("Relu", [out], [r])
            h = r
        meta.append((sx, wq, ws, bias))
    return b.to_json(), bytes(b.blob), meta


def test_fully_quantized_graph_fuses(dev):
    import torch
    from luisaml_b200.session import Network
    batch, dims = 64, (256, 512, 384, 128)
    text, blob, meta = _quantized_mlp(batch, dims, seed=5)
    x = np.random.default_rng(6).standard_normal((batch, dims[0])).astype(np.float32)
    outs = {}
    for fusion in (True, False):
        net = Network(text)
        net.set_fusion(fusion)
        y = torch.empty((batch, dims[-1]), dtype=torch.float32, device=dev)
        net.set_weight_buffer(_t(np.frombuffer(blob, dtype=np.uint8), dev))
        net.set_input("x", _t(x, dev))
        net.set_output("y", y)
        net.forward()
        outs[fusion] = y.cpu().numpy()
        if fusion:
            s = net.summary()
            assert s.count("fused kernel") == 3 and "folded" in s, s
            # the input QuantizeLinear + 3 fused GEMMs; each Relu -> QuantizeLinear pair
            # is folded into the previous GEMM, which stores e4m3 directly
            assert net.executed_nodes() == 1 + 3
    # oracle: quantize activations, dequantize both, gemm.cpp's loop
    h = x
    for li, (sx, wq, ws, bias) in enumerate(meta):
        hq = oracle.quantize(h, sx[0])
        a = oracle.dequantize(hq, sx[0])
        w = oracle.dequantize(wq, ws, axis=0)
        h = oracle.gemm(a, w, bias, transB=1)
        if li < len(meta) - 1:
            h = oracle.relu(h)
    assert_close(outs[True], h, what="fused graph vs oracle")
    assert_close(outs[False], h, what="unfused graph vs oracle")


def _run_ffn(dev, text, blob, x, fusion):
    import torch
    from luisaml_b200.session import Network
    net = Network(text)
    net.set_fusion(fusion)
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=dev)
    net.set_weight_buffer(_t(np.frombuffer(blob, dtype=np.uint8), dev))
    net.set_input("x", _t(x, dev))
    net.set_output("y", y)
    net.forward()
    return net, y.float().cpu().numpy()


def test_ffn_graph_fused_vs_oracle(dev):
    """Llama-style FFN as ONNX nodes: the fusion pass must turn it into four
    kernels (two dynamic per-row quantizations, the gate/up GEMM with the
    SiLU*up epilogue, the down GEMM with residual and bf16 store) and match
    the oracle chain and the unfused node-by-node execution."""
    from conftest import assert_close_bf16
    from luisaml_b200 import graphs
    T, D, F = 256, 512, 1024
    text, blob, meta = graphs.ffn(T, D, F)
    x = np.random.default_rng(3000).standard_normal((T, D)).astype(np.float32)
    net, y_fused = _run_ffn(dev, text, blob, x, True)
    assert net.executed_nodes() == 4, net.summary()
    _, y_unfused = _run_ffn(dev, text, blob, x, False)
    xq, sx = oracle.quantize_dynamic_rows(x)
    g = oracle.qdq_gemm(xq, sx, meta["wg_q"], meta["wg_s"])
    u = oracle.qdq_gemm(xq, sx, meta["wu_q"], meta["wu_s"])
    h = oracle.silu_mul(g, u)
    hq, sh = oracle.quantize_dynamic_rows(h)
    ref = oracle.qdq_gemm(hq, sh, meta["wd_q"], meta["wd_s"]) + x
    assert_close_bf16(y_fused, ref, what="fused FFN vs oracle")
    assert_close_bf16(y_unfused, ref, what="unfused FFN vs oracle")


def test_ffn_config_shape_stage_by_stage(dev):
    """The configuration's FFN, 4096 tokens x d_model 4096 x ffn 11008,
    through NetworkInstance, each stage held to the oracle on the executor's
    own input (read back with lcml_network_tensor):
      * x's dynamic per-token quantization: codes and scales bit-exact (all rows);
      * the gate/up GEMM with the SiLU*up epilogue (a 22016-wide CTA-pair GEMM,
        fp32 h): sampled token rows at rtol 2e-3 / atol 1e-3 against the
        oracle's K-ordered fp32 chain on the executor's x codes;
      * h's dynamic per-token quantization: bit-exact on the executor's h (all rows);
      * the down GEMM + residual, bf16 out: sampled rows at rtol 2e-3 /
        atol 1e-3 plus the bf16 half ulp, on the executor's h codes."""
    import torch
    from conftest import assert_close_bf16
    from luisaml_b200 import graphs
    from luisaml_b200.session import Network
    T, D, F = 4096, 4096, 11008
    text, blob, meta = graphs.ffn(T, D, F)
    x = np.random.default_rng(3001).standard_normal((T, D)).astype(np.float32)
    net = Network(text)
    net.set_memory_reuse(False)  # keep every intermediate readable
    y = torch.empty((T, D), dtype=torch.bfloat16, device=dev)
    net.set_weight_buffer(_t(np.frombuffer(blob, dtype=np.uint8), dev))
    net.set_input("x", _t(x, dev))
    net.set_output("y", y)
    net.forward()
    torch.cuda.synchronize()
    assert net.executed_nodes() == 4, net.summary()
    import luisaml_b200 as lb
    assert lb.device_error() == 0
    xq, sx = net.read_tensor("x_q"), net.read_tensor("x_scale")
    xq_ref, sx_ref = oracle.quantize_dynamic_rows(x)
    assert np.array_equal(sx, sx_ref) and np.array_equal(xq, xq_ref), "x quantization differs from the oracle"
    rows = np.unique(np.concatenate([[0, 1, 127, 128, 2047, 4095], np.random.default_rng(5).integers(0, T, 10)]))
    h = net.read_tensor("h")
    g = oracle.qdq_gemm(xq[rows], sx[rows], meta["wg_q"], meta["wg_s"])
    u = oracle.qdq_gemm(xq[rows], sx[rows], meta["wu_q"], meta["wu_s"])
    assert_close(h[rows], oracle.silu_mul(g, u), what="gate/up GEMM + SiLU*up at the config shape")
    hq, sh = net.read_tensor("h_q"), net.read_tensor("h_scale")
    hq_ref, sh_ref = oracle.quantize_dynamic_rows(h)
    assert np.array_equal(sh, sh_ref) and np.array_equal(hq, hq_ref), "h quantization differs from the oracle"
    ref = oracle.qdq_gemm(hq[rows], sh[rows], meta["wd_q"], meta["wd_s"]) + x[rows]
    assert_close_bf16(y.float().cpu().numpy()[rows], ref, what="down GEMM + residual at the config shape")
    # the default lifetime-planned arena: the same output bit for bit
    net2 = Network(text)
    y2 = torch.empty((T, D), dtype=torch.bfloat16, device=dev)
    net2.set_weight_buffer(_t(np.frombuffer(blob, dtype=np.uint8), dev))
    net2.set_input("x", _t(x, dev))
    net2.set_output("y", y2)
    net2.forward()
    torch.cuda.synchronize()
    assert torch.equal(y, y2)
    arena, unplanned = net2.memory()
    assert arena < unplanned, (arena, unplanned)


def test_dynamic_row_quant_all_zero_row(dev):
    """An all-zero token row: the fused executor's dynamic quantization uses
    scale 1 (codes 0), the kernel rule for an all-zero slice; the unfused
    ONNX chain Abs -> ReduceMax -> Div(448) -> QuantizeLinear computes
    scale 0 and 0 / 0 = NaN codes (0x7f) for that row. Both are pinned."""
    import torch
    from luisaml_b200 import graphs
    from luisaml_b200.session import Network
    T, D, F = 128, 256, 256
    text, blob, meta = graphs.ffn(T, D, F)
    x = np.random.default_rng(3002).standard_normal((T, D)).astype(np.float32)
    x[5] = 0.0
    out = {}
    for fusion in (True, False):
        net = Network(text)
        net.set_fusion(fusion)
        net.set_memory_reuse(False)
        y = torch.empty((T, D), dtype=torch.bfloat16, device=dev)
        net.set_weight_buffer(_t(np.frombuffer(blob, dtype=np.uint8), dev))
        net.set_input("x", _t(x, dev))
        net.set_output("y", y)
        net.forward()
        torch.cuda.synchronize()
        out[fusion] = (net.read_tensor("x_q"), net.read_tensor("x_scale"))
    q, s = out[True]
    assert s[5] == 1.0 and (q[5] == 0).all()
    q, s = out[False]
    assert s[5] == 0.0 and (q[5] == 0x7f).all()
    np.testing.assert_array_equal(out[True][0][:5], out[False][0][:5])


def _run_graph(dev, b, inputs, outputs, fusion=True, reuse=True):
    """Runs a GraphBuilder graph: inputs {name: np array}, outputs {name: (shape, torch dtype)}."""
    import torch
    from luisaml_b200.session import Network
    net = Network(b.to_json())
    net.set_fusion(fusion)
    net.set_memory_reuse(reuse)
    if b.blob:
        net.set_weight_buffer(_t(np.frombuffer(bytes(b.blob), dtype=np.uint8), dev))
    for k, v in inputs.items():
        net.set_input(k, _t(v, dev))
    outs = {k: torch.empty(shape, dtype=dt, device=dev) for k, (shape, dt) in outputs.items()}
    for k, t in outs.items():
        net.set_output(k, t)
    net.forward()
    torch.cuda.synchronize()
    return net, {k: t.cpu().numpy() for k, t in outs.items()}


def test_fp32_conv_graph(dev):
    """An fp32 Conv node (no QDQ: conv.cpp:115-207) through NetworkInstance,
    grouped with bias and stride, then Relu: bit-exact against the oracle in
    the reference's summation order."""
    import torch
    from luisaml_b200.export import GraphBuilder
    rng = np.random.default_rng(77)
    b = GraphBuilder("conv_f32")
    b.input("x", "FLOAT", (2, 8, 12, 12))
    W = rng.standard_normal((6, 4, 3, 3)).astype(np.float32)
    bias = rng.standard_normal(6).astype(np.float32)
    b.const("w", W)
    b.const("b", bias)
    c = b.value("c", "FLOAT", (2, 6, 6, 6))
    b.node("Conv", ["x", "w", "b"], [c], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1], group=2)
    b.output("y", "FLOAT", (2, 6, 6, 6))
    b.node("Relu", [c], ["y"])
    x = rng.standard_normal((2, 8, 12, 12)).astype(np.float32)
    _, out = _run_graph(dev, b, {"x": x}, {"y": ((2, 6, 6, 6), torch.float32)})
    ref = oracle.relu(oracle.conv2d(x, W, bias, strides=(2, 2), pads=(1, 1, 1, 1), group=2, lanes=4))
    np.testing.assert_array_equal(out["y"], ref)


def test_qdq_depthwise_conv_graph(dev):
    """A QDQ depthwise conv (group = channels) fused by the executor: Q(x) ->
    DQ -> Conv(DQ(W), group=C) -> Relu -> Q -> DQ -> GlobalAveragePool, fused
    and unfused, against the oracle (codes within one step, pooled output
    within the GEMM tolerance)."""
    import torch
    from luisaml_b200.export import GraphBuilder, qdq_weight
    rng = np.random.default_rng(78)
    N, C, H = 2, 32, 10
    b = GraphBuilder("dw_qdq")
    b.input("x", "FLOAT", (N, C, H, H))
    sx = np.float32(0.01)
    b.const("sx", np.float32(sx).reshape(()))
    xq = b.value("xq", "FLOAT8E4M3FN", (N, C, H, H))
    b.node("QuantizeLinear", ["x", "sx"], [xq])
    xdq = b.value("xdq", "FLOAT", (N, C, H, H))
    b.node("DequantizeLinear", [xq, "sx"], [xdq])
    Wt = (rng.standard_normal((C, 1, 3, 3)) * 0.3).astype(np.float32)
    wdq, wq, ws = qdq_weight(b, "w", Wt, axis=0)
    bias = (rng.standard_normal(C) * 0.01).astype(np.float32)
    b.const("bias", bias)
    cv = b.value("cv", "FLOAT", (N, C, H, H))
    b.node("Conv", [xdq, wdq, "bias"], [cv], kernel_shape=[3, 3], pads=[1, 1, 1, 1], group=C)
    r = b.value("r", "FLOAT", (N, C, H, H))
    b.node("Relu", [cv], [r])
    sy = np.float32(0.004)
    b.const("sy", np.float32(sy).reshape(()))
    yq = b.value("yq", "FLOAT8E4M3FN", (N, C, H, H))
    b.node("QuantizeLinear", [r, "sy"], [yq])
    ydq = b.value("ydq", "FLOAT", (N, C, H, H))
    b.node("DequantizeLinear", [yq, "sy"], [ydq])
    b.output("y", "FLOAT", (N, C, 1, 1))
    b.node("GlobalAveragePool", [ydq], ["y"])
    x = (rng.standard_normal((N, C, H, H))).astype(np.float32)
    h = oracle.conv2d(oracle.dequantize(oracle.quantize(x, sx), sx), oracle.dequantize(wq, ws, axis=0), bias,
                      pads=(1, 1, 1, 1), group=C)
    codes = oracle.quantize(oracle.relu(h), sy)
    ref = oracle.global_avgpool(oracle.dequantize(codes, sy))
    for fusion in (True, False):
        net, out = _run_graph(dev, b, {"x": x}, {"y": ((N, C, 1, 1), torch.float32)}, fusion=fusion)
        if fusion:
            assert "implicit-GEMM conv" in net.summary() or "fused" in net.summary()
        # one e4m3 step per pooled pixel at most moves the mean by sy * 2^-3 * |y| / 100
        assert_close(out["y"], ref, rtol=2e-3, atol=1e-3, what=f"depthwise fusion={fusion}")


def test_qdq_matmul_graph(dev):
    """A MatMul node (mat_mul.cpp:51-186) with DequantizeLinear'd operands:
    x -> Q -> DQ -> MatMul(DQ(W [K, N] e4m3, per-column scales)) + Add(bias),
    fused into one FP8 GEMM (W transposed to K-major at prepare) and unfused,
    against the oracle."""
    import torch
    from luisaml_b200.export import GraphBuilder, qdq_weight
    rng = np.random.default_rng(79)
    M, K, N = 96, 256, 200
    b = GraphBuilder("matmul_qdq")
    b.input("x", "FLOAT", (M, K))
    sx = np.float32(oracle.scale_from_amax(4.5))
    b.const("sx", np.float32(sx).reshape(()))
    xq = b.value("xq", "FLOAT8E4M3FN", (M, K))
    b.node("QuantizeLinear", ["x", "sx"], [xq])
    xdq = b.value("xdq", "FLOAT", (M, K))
    b.node("DequantizeLinear", [xq, "sx"], [xdq])
    Wt = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    wdq, wq, ws = qdq_weight(b, "w", Wt, axis=1)
    b.output("y", "FLOAT", (M, N))
    b.node("MatMul", [xdq, wdq], ["y"])
    x = rng.standard_normal((M, K)).astype(np.float32)
    aq = oracle.quantize(x, sx)
    ref = oracle.qdq_gemm(aq, np.float32([sx]), wq, ws, b_kmajor=False)
    for fusion in (True, False):
        net, out = _run_graph(dev, b, {"x": x}, {"y": ((M, N), torch.float32)}, fusion=fusion)
        assert_close(out["y"], ref, what=f"QDQ MatMul fusion={fusion}")
        if fusion:
            assert net.executed_nodes() == 2, net.summary()  # input quantize + one fused GEMM


def test_matmul_nd_broadcast_graph(dev):
    """fp32 MatMul with numpy batch broadcasting (mat_mul.cpp:187-303):
    [2, 1, 5, 8] @ [3, 8, 4] -> [2, 3, 5, 4], and a 1-D right operand
    [2, 3, 5, 4] @ [4] -> [2, 3, 5], against numpy in float64."""
    import torch
    from luisaml_b200.export import GraphBuilder
    rng = np.random.default_rng(80)
    b = GraphBuilder("matmul_nd")
    b.input("a", "FLOAT", (2, 1, 5, 8))
    b.input("b", "FLOAT", (3, 8, 4))
    b.input("v", "FLOAT", (4,))
    b.output("y", "FLOAT", (2, 3, 5, 4))
    b.node("MatMul", ["a", "b"], ["y"])
    b.output("z", "FLOAT", (2, 3, 5))
    b.node("MatMul", ["y", "v"], ["z"])
    a = rng.standard_normal((2, 1, 5, 8)).astype(np.float32)
    bb = rng.standard_normal((3, 8, 4)).astype(np.float32)
    v = rng.standard_normal(4).astype(np.float32)
    _, out = _run_graph(dev, b, {"a": a, "b": bb, "v": v},
                        {"y": ((2, 3, 5, 4), torch.float32), "z": ((2, 3, 5), torch.float32)})
    want_y = np.matmul(a.astype(np.float64), bb.astype(np.float64))
    assert_close(out["y"], want_y, rtol=1e-5, atol=1e-5, what="batched matmul")
    assert_close(out["z"], np.matmul(out["y"].astype(np.float64), v), rtol=1e-5, atol=1e-5, what="matrix-vector")


def test_fp8_typed_binary_softmax_graph(dev):
    """Add and Softmax nodes on FLOAT8E4M3FN-typed tensors (no scales), the
    reference's quantized Binary / Softmax paths, through NetworkInstance."""
    import torch
    from luisaml_b200.export import GraphBuilder
    rng = np.random.default_rng(81)
    b = GraphBuilder("fp8_typed")
    b.input("p", "FLOAT8E4M3FN", (16, 40))
    b.input("q", "FLOAT8E4M3FN", (40,))
    s = b.value("s", "FLOAT8E4M3FN", (16, 40))
    b.node("Add", ["p", "q"], [s])
    b.output("y", "FLOAT8E4M3FN", (16, 40))
    b.node("Softmax", [s], ["y"], axis=-1)
    p = oracle.e4m3_encode((rng.standard_normal((16, 40)) * 2).astype(np.float32))
    q = oracle.e4m3_encode((rng.standard_normal(40)).astype(np.float32))
    _, out = _run_graph(dev, b, {"p": p, "q": q}, {"y": ((16, 40), torch.uint8)})
    sq = oracle.binary_fp8(0, p, q, 17)
    ref = oracle.e4m3_encode(oracle.softmax_rows(oracle.e4m3_decode(sq)).astype(np.float16).astype(np.float32))
    g, w = oracle.e4m3_decode(out["y"]).astype(np.float64), oracle.e4m3_decode(ref).astype(np.float64)
    assert (np.abs(g - w) <= np.maximum(np.abs(w) * 0.125, 2.0 ** -9) + 1e-12).all()
