"""QDQ graphs of the benchmark configurations, written as LuisaML-JSON + a
weight blob with luisaml_b200.export. Seeded synthetic weights (numpy PCG64,
seed = 1000 * config + tensor index); no checkpoint or dataset is involved.

Each builder returns (json_text, blob bytes, meta) where meta holds the
host-side arrays a checker needs (e4m3 weights, scales, biases).
"""
from __future__ import annotations

import numpy as np

from .export import GraphBuilder, qdq_weight


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
