"""LuisaML-JSON model writer for QDQ graphs.

Produces the same file pair the reference's exporter writes
(scripts/export_onnx.py:114-203): a JSON model in the protobuf-JSON shape the
loader parses (src/onnx/onnx.cpp:87-242; string dtype/attribute enums, quoted
64-bit integers, `value_info` for every intermediate) and a raw weight blob
addressed by `data_offsets` [start, end). e4m3 initializers occupy
ceil(n/4)*4 bytes of the blob (network_instance.cpp:222-224); every tensor
starts 256-byte aligned so TMA can read weights in place. Small constants
(scales, zero points, shapes) go inline as base64 `raw_data`.

The `onnx` package is not needed: the reference's exporter depends on it and
it is not installed here.
"""
from __future__ import annotations

import base64
import json

import numpy as np

_DT = {np.dtype(np.float32): "FLOAT", np.dtype(np.uint8): "UINT8", np.dtype(np.int64): "INT64",
       np.dtype(np.int32): "INT32", np.dtype(np.float16): "FLOAT16"}


class GraphBuilder:
    def __init__(self, name: str = "graph"):
        self.name = name
        self.nodes, self.inits, self.inputs, self.outputs, self.values = [], [], [], [], []
        self.blob = bytearray()
        self._declared = set()
        self._n = 0

    # ---------------------------------------------------------------- variables
    @staticmethod
    def _value(name, dtype, shape):
        return {"name": name, "type": {"tensor_type": {"elem_type": dtype,
                                                       "shape": {"dim": [{"dim_value": str(int(d))} for d in shape]}}}}

    def input(self, name, dtype, shape):
        self.inputs.append(self._value(name, dtype, shape))
        self._declared.add(name)
        return name

    def output(self, name, dtype, shape):
        self.outputs.append(self._value(name, dtype, shape))
        self._declared.add(name)
        return name

    def value(self, name, dtype, shape):
        if name not in self._declared:
            self.values.append(self._value(name, dtype, shape))
            self._declared.add(name)
        return name

    def weight(self, name, array, dtype=None):
        """Initializer stored in the external blob (data_offsets)."""
        a = np.ascontiguousarray(array)
        dtype = dtype or _DT[a.dtype]
        pad = (-len(self.blob)) % 256
        self.blob.extend(b"\0" * pad)
        start = len(self.blob)
        raw = a.tobytes()
        if dtype == "FLOAT8E4M3FN":
            raw += b"\0" * ((-len(raw)) % 4)
        self.blob.extend(raw)
        self.inits.append({"dims": [str(int(d)) for d in a.shape], "data_type": dtype, "name": name,
                           "data_offsets": [start, len(self.blob)]})
        self.value(name, dtype, a.shape)
        return name

    def const(self, name, array, dtype=None):
        """Initializer stored inline (base64 raw_data)."""
        a = np.ascontiguousarray(array)
        dtype = dtype or _DT[a.dtype]
        entry = {"data_type": dtype, "name": name, "raw_data": base64.b64encode(a.tobytes()).decode()}
        if a.ndim:
            entry["dims"] = [str(int(d)) for d in a.shape]
        self.inits.append(entry)
        self.value(name, dtype, a.shape if a.ndim else (1,))
        return name

    # ---------------------------------------------------------------- nodes
    def node(self, op_type, inputs, outputs, name=None, **attrs):
        self._n += 1
        attr = []
        for k, v in attrs.items():
            if isinstance(v, bool) or isinstance(v, (int, np.integer)):
                attr.append({"name": k, "i": str(int(v)), "type": "INT"})
            elif isinstance(v, float):
                attr.append({"name": k, "f": float(v), "type": "FLOAT"})
            elif isinstance(v, str):
                attr.append({"name": k, "s": base64.b64encode(v.encode()).decode(), "type": "STRING"})
            elif isinstance(v, (list, tuple)) and all(isinstance(x, (int, np.integer)) for x in v):
                attr.append({"name": k, "ints": [str(int(x)) for x in v], "type": "INTS"})
            elif isinstance(v, (list, tuple)):
                attr.append({"name": k, "floats": [float(x) for x in v], "type": "FLOATS"})
            else:
                raise TypeError(f"attribute {k}: {type(v)}")
        n = {"input": list(inputs), "output": list(outputs), "name": name or f"node_{op_type.lower()}_{self._n}",
             "op_type": op_type}
        if attr:
            n["attribute"] = attr
        self.nodes.append(n)
        return outputs[0] if len(outputs) == 1 else outputs

    def to_json(self, producer="luisaml_b200") -> str:
        g = {"node": self.nodes, "name": self.name, "initializer": self.inits, "input": self.inputs,
             "output": self.outputs, "value_info": self.values}
        return json.dumps({"ir_version": "10", "producer_name": producer, "producer_version": "1", "graph": g})


# ---------------------------------------------------------------- offline quantization
def e4m3_encode(x) -> np.ndarray:
    """fp32 -> e4m3 bytes on the host, same rules as the CUDA encoder and the
    reference codec (FP8E4M3FN::from_float, include/onnx/fp_quantized.h:149-223):
    NaN -> 0x7f, +-0 -> 0x00, |x| > 448 -> +-448, round-to-nearest-even, a
    nonzero value that rounds to zero keeps its sign. Integer formulation:
    (a + 0x7ffff + lsb) >> 20 rounds the 23-bit mantissa to 3 bits with the
    carry landing in the exponent; e4m3 subnormals are rint(|x| * 512)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    sign = (u >> 24) & 0x80
    a = u & 0x7FFFFFFF
    normal = ((a + 0x7FFFF + ((a >> 20) & 1)) >> 20) - (120 << 3)
    with np.errstate(invalid="ignore", over="ignore"):
        sub = np.rint(np.where(a < 0x3C800000, np.abs(x), 0).astype(np.float32) * np.float32(512)).astype(np.uint64)
    r = np.where(a >= 0x3C800000, normal, sub)
    out = sign | r
    out = np.where(a > 0x43E00000, sign | 0x7E, out)
    out = np.where(a == 0, 0, out)
    out = np.where(a > 0x7F800000, 0x7F, out)
    return out.astype(np.uint8).reshape(x.shape)


def scale_from_amax(amax) -> np.float32:
    """amax / 448 in fp32 (1 for amax == 0): the scale every dynamic mode uses."""
    a = np.float32(amax)
    return np.float32(a / np.float32(448.0)) if a > 0 else np.float32(1.0)


def quantize(x, scale, axis=None) -> np.ndarray:
    """QuantizeLinear on the host: e4m3(x / s) with an fp32 divide."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    s = np.asarray(scale, dtype=np.float32)
    if axis is not None and s.size > 1:
        shp = [1] * x.ndim
        shp[axis] = s.size
        s = s.reshape(shp)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        return e4m3_encode((x / s).astype(np.float32))


def qdq_weight(b: GraphBuilder, name, w_fp32, axis=None):
    """Quantizes a weight offline (e4m3 initializer in the blob + fp32 scale,
    per tensor or per `axis`) and emits its DequantizeLinear. Returns
    (DQ output name, e4m3 bytes, scales)."""
    w = np.ascontiguousarray(w_fp32, dtype=np.float32)
    if axis is None:
        s = np.float32([scale_from_amax(np.abs(w).max())])
        q = quantize(w, s[0])
        b.const(name + "_scale", s[0:1].reshape(()))
    else:
        red = tuple(i for i in range(w.ndim) if i != axis)
        s = np.array([scale_from_amax(a) for a in np.abs(w).max(axis=red)], dtype=np.float32)
        q = quantize(w, s, axis=axis)
        b.const(name + "_scale", s)
    b.weight(name + "_q", q, "FLOAT8E4M3FN")
    out = b.value(name + "_dq", "FLOAT", w.shape)
    b.node("DequantizeLinear", [name + "_q", name + "_scale"], [out], **({"axis": axis} if axis is not None else {}))
    return out, q, s
