"""QDQ graphs of the benchmark configurations, written as LuisaML-JSON + a
weight blob with luisaml_b200.export. Seeded synthetic weights (numpy PCG64,
seed = 1000 * config + tensor index); no checkpoint or dataset is involved.

Each builder returns (json_text, blob bytes, meta) where meta holds the
host-side arrays a checker needs (e4m3 weights, scales, biases).
"""
from __future__ import annotations

import numpy as np

from .export import GraphBuilder, qdq_weight, scale_from_amax


def mlp(batch=32, dims=(784, 512, 512, 10), seed_base=1000):
    """Simple MLP (scripts/simple_mlp.py shape, widened as the benchmark asks):
    Gemm(transB=1) + Relu per hidden layer, weights N(0, 1/sqrt(fan_in)) passed
    through per-tensor QuantizeLinear/DequantizeLinear (weights stored e4m3,
    DequantizeLinear in the graph), biases N(0, 0.01), fp32 activations."""
    b = GraphBuilder("simple_mlp_qdq")
    x = b.input("input", "FLOAT", (batch, dims[0]))
    meta = {"layers": []}
    h = x
    for li in range(len(dims) - 1):
        rng = np.random.default_rng(seed_base + 2 * li)
        w = (rng.standard_normal((dims[li + 1], dims[li])) / np.sqrt(dims[li])).astype(np.float32)
        bias = (np.random.default_rng(seed_base + 2 * li + 1).standard_normal(dims[li + 1]) * 0.01).astype(np.float32)
        wdq, q, s = qdq_weight(b, f"net.{2 * li}.weight", w)
        b.const(f"net.{2 * li}.bias", bias)
        last = li == len(dims) - 2
        out = "output" if last else b.value(f"linear_{li}", "FLOAT", (batch, dims[li + 1]))
        if last:
            b.output("output", "FLOAT", (batch, dims[li + 1]))
        b.node("Gemm", [h, wdq, f"net.{2 * li}.bias"], [out], transA=0, transB=1, alpha=1.0, beta=1.0)
        if not last:
            r = b.value(f"relu_{li}", "FLOAT", (batch, dims[li + 1]))
            b.node("Relu", [out], [r])
            h = r
        meta["layers"].append({"q": q, "s": s, "bias": bias})
    return b.to_json(), bytes(b.blob), meta


def _dynamic_row_qdq(b: GraphBuilder, src: str, name: str, rows: int, cols: int) -> str:
    """Per-token dynamic quantization written as plain ONNX nodes:
    Abs -> ReduceMax(axes=[-1], keepdims=0) -> Div(448) -> QuantizeLinear(axis 0)
    -> DequantizeLinear(axis 0). Returns the DequantizeLinear output."""
    a = b.value(f"{name}_abs", "FLOAT", (rows, cols))
    b.node("Abs", [src], [a])
    m = b.value(f"{name}_amax", "FLOAT", (rows,))
    b.node("ReduceMax", [a], [m], axes=[-1], keepdims=0)
    s = b.value(f"{name}_scale", "FLOAT", (rows,))
    b.node("Div", [m, "fp8_max"], [s])
    q = b.value(f"{name}_q", "FLOAT8E4M3FN", (rows, cols))
    b.node("QuantizeLinear", [src, s], [q], axis=0)
    dq = b.value(f"{name}_dq", "FLOAT", (rows, cols))
    b.node("DequantizeLinear", [q, s], [dq], axis=0)
    return dq


def ffn(tokens=4096, d_model=4096, ffn_dim=11008, seed_base=3000):
    """Llama-style FFN block: y = bf16(x + DQ(Q(h)) @ W_down^T) with
    h = SiLU(DQ(Q(x)) @ W_gate^T) * (DQ(Q(x)) @ W_up^T). Weights N(0, 0.02)
    stored e4m3 with per-output-channel scales; activations quantized per
    token (scale = row amax / 448) by explicit ONNX nodes; the residual is the
    down Gemm's C input."""
    T, D, F = tokens, d_model, ffn_dim
    b = GraphBuilder("llama_ffn_qdq")
    b.input("x", "FLOAT", (T, D))
    b.const("fp8_max", np.float32(448.0))
    xdq = _dynamic_row_qdq(b, "x", "x", T, D)
    meta = {}
    rng = lambda i: np.random.default_rng(seed_base + i)  # noqa: E731
    wg = (rng(1).standard_normal((F, D), dtype=np.float32) * np.float32(0.02))
    wu = (rng(2).standard_normal((F, D), dtype=np.float32) * np.float32(0.02))
    wd = (rng(3).standard_normal((D, F), dtype=np.float32) * np.float32(0.02))
    g_dq, meta["wg_q"], meta["wg_s"] = qdq_weight(b, "w_gate", wg, axis=0)
    u_dq, meta["wu_q"], meta["wu_s"] = qdq_weight(b, "w_up", wu, axis=0)
    d_dq, meta["wd_q"], meta["wd_s"] = qdq_weight(b, "w_down", wd, axis=0)
    del wg, wu, wd
    g = b.value("gate", "FLOAT", (T, F))
    b.node("Gemm", [xdq, g_dq], [g], transB=1)
    u = b.value("up", "FLOAT", (T, F))
    b.node("Gemm", [xdq, u_dq], [u], transB=1)
    sg = b.value("gate_sigmoid", "FLOAT", (T, F))
    b.node("Sigmoid", [g], [sg])
    silu = b.value("gate_silu", "FLOAT", (T, F))
    b.node("Mul", [g, sg], [silu])
    h = b.value("h", "FLOAT", (T, F))
    b.node("Mul", [silu, u], [h])
    hdq = _dynamic_row_qdq(b, h, "h", T, F)
    y32 = b.value("y_f32", "FLOAT", (T, D))
    b.node("Gemm", [hdq, d_dq, "x"], [y32], transB=1, alpha=1.0, beta=1.0)
    b.output("y", "BFLOAT16", (T, D))
    b.node("Cast", [y32], ["y"], to=16)
    return b.to_json(), bytes(b.blob), meta


def resnet50(batch=128, image=224, width=64, blocks=(3, 4, 6, 3), num_classes=1000, seed_base=5000,
             calib_batch=2):
    """ResNet-50 v1.5 (bottleneck blocks, stride on the 3x3) as a fully
    quantized QDQ graph, the shape of the reference's ResNet test models:
    every Conv reads DequantizeLinear'd e4m3 activations and weights
    (per-output-channel scales), adds its bias (batch norm folded in),
    optionally the residual, applies Relu and is requantized with a static
    per-tensor scale; max pool and global average pool read e4m3; the
    classifier is a QDQ Gemm. Weights are He-normal (the last conv of each
    residual branch scaled by 0.25, like a small batch-norm gamma), biases
    N(0, 0.01). Activation scales are calibrated (amax / 448) on a seeded
    synthetic batch run through the same fake-quantized network on the CPU.

    meta: "plan" (the whole network as steps the oracle replays),
    "segments" [(input name, input scale, output name, output scale, plan
    steps)] for a block-wise replay from the executor's own intermediates,
    "conv_io" (per fused conv: the e4m3 tensors it reads and writes with their
    scales, its plan step and whether Relu follows) for a conv-by-conv replay,
    "flop_per_image", "convs"."""
    import torch
    import torch.nn.functional as F

    N = batch
    b = GraphBuilder("resnet50_qdq")
    b.input("x", "FLOAT", (N, 3, image, image))
    plan, segments = [], []
    counter = [0]

    def rng():
        counter[0] += 1
        return np.random.default_rng(seed_base + counter[0])

    calib = torch.from_numpy(np.random.default_rng(seed_base).standard_normal(
        (calib_batch, 3, image, image)).astype(np.float32))

    def fq(t, s):  # fake quantization on the CPU for calibration
        return (t / s).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).to(torch.float32) * s

    def quant(src, cal, name, shape):
        """QuantizeLinear of fp32 value `src` with a scale calibrated on `cal`."""
        s = scale_from_amax(float(cal.abs().max()))
        sname = b.const(f"{name}_scale", np.float32(s))
        q = b.value(f"{name}_q", "FLOAT8E4M3FN", shape)
        b.node("QuantizeLinear", [src, sname], [q])
        plan.append(("qdq", np.float32(s)))
        return {"q": q, "s": np.float32(s), "sname": sname, "shape": shape, "cal": fq(cal, float(s))}

    def dq(act, tag):
        out = b.value(f"{act['q']}_dq_{tag}", "FLOAT", act["shape"])
        b.node("DequantizeLinear", [act["q"], act["sname"]], [out])
        return out

    flops = [0]
    convs = []
    conv_io = []  # per fused conv: input, residual, output (names + scales), its plan step, Relu

    def record(x, step, y, relu_on, res=None):
        conv_io.append({"x": x["q"], "x_scale": x["s"], "res": res["q"] if res else None,
                        "res_scale": res["s"] if res else None, "y": y["q"], "y_scale": y["s"],
                        "conv": step, "relu": relu_on})

    def conv(act, cout, k, stride, pad, name, gain=1.0):
        n, cin, h, w = act["shape"]
        wt = (rng().standard_normal((cout, cin, k, k)) * np.sqrt(2.0 / (cin * k * k)) * gain).astype(np.float32)
        bias = (rng().standard_normal(cout) * 0.01).astype(np.float32)
        wdq, wq, ws = qdq_weight(b, f"{name}.weight", wt, axis=0)
        b.const(f"{name}.bias", bias)
        oh, ow = (h + 2 * pad - k) // stride + 1, (w + 2 * pad - k) // stride + 1
        out = b.value(f"{name}_out", "FLOAT", (n, cout, oh, ow))
        b.node("Conv", [dq(act, name), wdq, f"{name}.bias"], [out], kernel_shape=[k, k], strides=[stride, stride],
               pads=[pad, pad, pad, pad], dilations=[1, 1], group=1)
        plan.append(("conv", wq, ws, bias, stride, pad))
        wdeq = torch.from_numpy(wq.view(np.uint8).copy()).view(torch.float8_e4m3fn).to(torch.float32) * \
            torch.from_numpy(ws).view(-1, 1, 1, 1)
        cal = F.conv2d(act["cal"], wdeq, torch.from_numpy(bias), stride=stride, padding=pad)
        flops[0] += 2 * cout * oh * ow * cin * k * k
        convs.append((name, (cin, h, w), (cout, oh, ow), k, stride, pad))
        return out, (n, cout, oh, ow), cal

    def relu(src, shape, name):
        out = b.value(f"{name}_relu", "FLOAT", shape)
        b.node("Relu", [src], [out])
        plan.append(("relu",))
        return out

    # stem: quantize the input, 7x7/2 conv, Relu, 3x3/2 max pool (same scale in and out)
    seg_start = len(plan)
    a = quant("x", calib, "input", (N, 3, image, image))
    x_in = a
    y, shp, cal = conv(a, width, 7, 2, 3, "stem")
    a = quant(relu(y, shp, "stem"), torch.relu(cal), "stem", shp)
    record(x_in, plan[-3], a, True)
    mp_shape = (N, width, (shp[2] + 2 - 3) // 2 + 1, (shp[3] + 2 - 3) // 2 + 1)
    mp = b.value("maxpool_out", "FLOAT", mp_shape)
    b.node("MaxPool", [dq(a, "maxpool")], [mp], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1])
    plan.append(("maxpool",))
    mq = b.value("maxpool_q", "FLOAT8E4M3FN", mp_shape)
    b.node("QuantizeLinear", [mp, a["sname"]], [mq])
    a = {"q": mq, "s": a["s"], "sname": a["sname"], "shape": mp_shape,
         "cal": F.max_pool2d(a["cal"], 3, 2, 1)}
    segments.append(("x", None, a["q"], a["s"], plan[seg_start:]))

    for si, nblocks in enumerate(blocks):
        planes = width * (2 ** si)
        for bi in range(nblocks):
            stride = 2 if (si > 0 and bi == 0) else 1
            name = f"layer{si + 1}.{bi}"
            seg_start = len(plan)
            blk_in = a
            plan.append(("block_begin",))
            res = a
            if bi == 0:  # projection shortcut (emitted first: its output is ready before the Add)
                plan.append(("downsample_begin",))
                y, shp, cal = conv(a, planes * 4, 1, stride, 0, f"{name}.downsample")
                res = quant(y, cal, f"{name}.downsample", shp)
                record(a, plan[-2], res, False)
                plan.append(("downsample_end",))
            y, shp, cal = conv(a, planes, 1, 1, 0, f"{name}.conv1")
            h1 = quant(relu(y, shp, f"{name}.conv1"), torch.relu(cal), f"{name}.conv1", shp)
            record(a, plan[-3], h1, True)
            y, shp, cal = conv(h1, planes, 3, stride, 1, f"{name}.conv2")
            h2 = quant(relu(y, shp, f"{name}.conv2"), torch.relu(cal), f"{name}.conv2", shp)
            record(h1, plan[-3], h2, True)
            y, shp, cal = conv(h2, planes * 4, 1, 1, 0, f"{name}.conv3", gain=0.25)
            s_out = b.value(f"{name}_sum", "FLOAT", shp)
            b.node("Add", [y, dq(res, f"{name}.add")], [s_out])
            plan.append(("add",))
            a = quant(relu(s_out, shp, name), torch.relu(cal + res["cal"]), f"{name}.out", shp)
            record(h2, plan[-4], a, True, res=res)
            segments.append((blk_in["q"], blk_in["s"], a["q"], a["s"], plan[seg_start:]))

    # head: global average pool on e4m3, flatten, QDQ classifier
    seg_start = len(plan)
    n, c = a["shape"][0], a["shape"][1]
    g = b.value("gap_out", "FLOAT", (n, c, 1, 1))
    b.node("GlobalAveragePool", [dq(a, "gap")], [g])
    plan.append(("gap",))
    fl = b.value("flat", "FLOAT", (n, c))
    b.node("Flatten", [g], [fl], axis=1)
    gcal = a["cal"].mean(dim=(2, 3))
    f = quant(fl, gcal, "fc_in", (n, c))
    wt = (rng().standard_normal((num_classes, c)) / np.sqrt(c)).astype(np.float32)
    bias = (rng().standard_normal(num_classes) * 0.01).astype(np.float32)
    wdq, wq, ws = qdq_weight(b, "fc.weight", wt, axis=0)
    b.const("fc.bias", bias)
    b.output("logits", "FLOAT", (n, num_classes))
    b.node("Gemm", [dq(f, "fc"), wdq, "fc.bias"], ["logits"], transB=1)
    plan.append(("fc", wq, ws, bias))
    flops[0] += 2 * c * num_classes
    segments.append((a["q"], a["s"], "logits", None, plan[seg_start:]))
    meta = {"plan": plan, "segments": segments, "conv_io": conv_io, "flop_per_image": flops[0], "convs": convs}
    return b.to_json(), bytes(b.blob), meta
