"""TEST INFRASTRUCTURE ONLY — numpy/ctypes front end of the CPU oracle.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this package, and only as the checker. The product path
(``luisaml_b200``) never imports it.

``liboracle.so`` is this directory's plain-C restatement of the reference
algorithms (see ``oracle.c`` for the file:line each function follows).
``_ref/libref_codec.so`` is the reference's own CPU codec compiled from
``include/onnx/fp_quantized.h`` where it lies in the reference tree; it only
exists where that tree does, and is used to pin the restatement.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(HERE, "liboracle.so")
_REF = os.path.join(HERE, "_ref", "libref_codec.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64 = ctypes.c_int64


def build(quiet: bool = True) -> None:
    """Compile liboracle.so (and _ref/ when $LCML_REFERENCE_TREE names a reference checkout)."""
    out = subprocess.run(["make", "-C", HERE, "all", "REF=" + os.environ.get("LCML_REFERENCE_TREE", "")],
                         capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _load():
    if not os.path.exists(_LIB):
        build()
    lib = ctypes.CDLL(_LIB)
    lib.orc_e4m3_from_float.restype = ctypes.c_uint8
    lib.orc_e4m3_from_float.argtypes = [ctypes.c_float]
    lib.orc_e4m3_to_float.restype = ctypes.c_float
    lib.orc_e4m3_to_float.argtypes = [ctypes.c_uint8]
    for fmt in ("e5m2", "e2m1"):
        enc, dec = getattr(lib, f"orc_{fmt}_from_float"), getattr(lib, f"orc_{fmt}_to_float")
        enc.restype, enc.argtypes = ctypes.c_uint8, [ctypes.c_float]
        dec.restype, dec.argtypes = ctypes.c_float, [ctypes.c_uint8]
    lib.orc_cast.restype = ctypes.c_int
    lib.orc_amax.restype = ctypes.c_float
    lib.orc_scale_from_amax.restype = ctypes.c_float
    lib.orc_scale_from_amax.argtypes = [ctypes.c_float]
    lib.orc_sigmoid1.restype = ctypes.c_float
    lib.orc_sigmoid1.argtypes = [ctypes.c_float]
    lib.orc_num_threads.restype = ctypes.c_int
    return lib


lib = _load()


def ref_lib():
    """The reference's own compiled codec, or None where the tree is absent."""
    if not os.path.exists(_REF):
        return None
    r = ctypes.CDLL(_REF)
    r.lcml_ref_e4m3_from_float.restype = ctypes.c_uint8
    r.lcml_ref_e4m3_from_float.argtypes = [ctypes.c_float]
    r.lcml_ref_e4m3_to_float.restype = ctypes.c_float
    r.lcml_ref_e4m3_to_float.argtypes = [ctypes.c_uint8]
    for fmt in ("e4m3", "e5m2", "e2m1"):
        f = getattr(r, f"lcml_ref_{fmt}_count_mismatch")
        f.restype = ctypes.c_int64
        f.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint32)]
        enc, dec = getattr(r, f"lcml_ref_{fmt}_from_float"), getattr(r, f"lcml_ref_{fmt}_to_float")
        enc.restype, enc.argtypes = ctypes.c_uint8, [ctypes.c_float]
        dec.restype, dec.argtypes = ctypes.c_float, [ctypes.c_uint8]
    r.lcml_ref_e4m3_quantize_tensor.argtypes = [_f32p, ctypes.c_float, _u8p, _i64]
    return r


def _f(a):
    return a.ctypes.data_as(_f32p)


def _u(a):
    return a.ctypes.data_as(_u8p)


def num_threads() -> int:
    return int(lib.orc_num_threads())


# --------------------------------------------------------------------------- codec
def e4m3_encode(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint8)
    lib.orc_e4m3_encode_n(_f(x), _u(y), _i64(x.size))
    return y


def e4m3_decode(q) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    y = np.empty(q.shape, dtype=np.float32)
    lib.orc_e4m3_decode_n(_u(q), _f(y), _i64(q.size))
    return y


# ONNX type numbers of the Cast restatement and their numpy storage
CAST_TYPES = {1: np.float32, 10: np.float16, 16: np.uint16, 17: np.uint8, 19: np.uint8, 23: np.uint8}


def cast(x, src: int, dst: int, n: int | None = None) -> np.ndarray:
    """Cast (cast.cpp:10-162) of n elements of storage `x` (type code `src`)
    to type `dst` (ONNX numbers; 16 = bf16 held as uint16, 23 = FP4 E2M1 packed
    two per byte, element 2i in the low nibble). Returns the raw storage."""
    x = np.ascontiguousarray(x)
    if n is None:
        n = x.size * 2 if src == 23 else x.size
    out = np.zeros((n + 1) // 2 if dst == 23 else n, dtype=CAST_TYPES[dst])
    rc = lib.orc_cast(x.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(src), out.ctypes.data_as(ctypes.c_void_p),
                      ctypes.c_int(dst), _i64(n))
    if rc != 0:
        raise ValueError(f"oracle cast {src} -> {dst} unsupported")
    return out


def binary_fp8(op: int, a, b, dtype: int) -> np.ndarray:
    """FP8-typed Add/Sub/Mul/Div (op 0..3) with b broadcast over a (binary.cpp:185-283)."""
    a = np.ascontiguousarray(a, dtype=np.uint8)
    b = np.ascontiguousarray(b, dtype=np.uint8)
    y = np.empty(a.shape, dtype=np.uint8)
    lib.orc_binary_fp8(ctypes.c_int(op), _u(a), _u(b), _i64(a.size), _i64(b.size), _u(y), ctypes.c_int(dtype))
    return y


def e5m2_encode(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return np.array([lib.orc_e5m2_from_float(float(v)) for v in x.ravel()], dtype=np.uint8).reshape(x.shape)


def e2m1_encode(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return np.array([lib.orc_e2m1_from_float(float(v)) for v in x.ravel()], dtype=np.uint8).reshape(x.shape)


# --------------------------------------------------------------------------- QDQ
def amax(x) -> np.float32:
    x = np.ascontiguousarray(x, dtype=np.float32)
    lib.orc_amax.argtypes = [_f32p, _i64]
    return np.float32(lib.orc_amax(_f(x), _i64(x.size)))


def scale_from_amax(a) -> np.float32:
    return np.float32(lib.orc_scale_from_amax(ctypes.c_float(float(a))))


def quantize(x, scale, axis: int | None = None) -> np.ndarray:
    """ONNX QuantizeLinear to float8e4m3fn (zp 0, saturate 1).

    ``scale`` is a scalar (per-tensor) or a 1-D array along ``axis``.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    s = np.ascontiguousarray(np.atleast_1d(np.asarray(scale, dtype=np.float32)))
    if s.size == 1 and axis is None:
        outer, alen, inner, per_axis = 1, 1, x.size, 0
    else:
        ax = axis % x.ndim
        outer = int(np.prod(x.shape[:ax], dtype=np.int64))
        alen = x.shape[ax]
        inner = int(np.prod(x.shape[ax + 1:], dtype=np.int64))
        per_axis = 1
        assert s.size == alen
    y = np.empty(x.shape, dtype=np.uint8)
    lib.orc_quantize_axis(_f(x), _i64(outer), _i64(alen), _i64(inner), _f(s), ctypes.c_int(per_axis), _u(y))
    return y


def quantize_dynamic_rows(x):
    """Per-row (per-token) dynamic quantization: s[r] = amax(row)/448."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = int(np.prod(x.shape[:-1], dtype=np.int64))
    cols = x.shape[-1]
    s = np.empty(rows, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint8)
    lib.orc_quantize_dynamic_rows(_f(x), _i64(rows), _i64(cols), _f(s), _u(y))
    return y, s


def dequantize(q, scale, axis: int | None = None) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    s = np.ascontiguousarray(np.atleast_1d(np.asarray(scale, dtype=np.float32)))
    if s.size == 1 and axis is None:
        outer, alen, inner, per_axis = 1, 1, q.size, 0
    else:
        ax = axis % q.ndim
        outer = int(np.prod(q.shape[:ax], dtype=np.int64))
        alen = q.shape[ax]
        inner = int(np.prod(q.shape[ax + 1:], dtype=np.int64))
        per_axis = 1
    y = np.empty(q.shape, dtype=np.float32)
    lib.orc_dequantize_axis(_u(q), _i64(outer), _i64(alen), _i64(inner), _f(s), ctypes.c_int(per_axis), _f(y))
    return y


# --------------------------------------------------------------------------- Gemm / Conv
def gemm(A, B, C=None, alpha=1.0, beta=1.0, transA=0, transB=0, rows=None, lanes=1) -> np.ndarray:
    """ONNX Gemm in fp32 with the reference's fma accumulation: K-ordered
    (lanes=1, gemm.cpp:153-157), or the four-lane order of its vector path
    for byte-buffer operands (lanes=4, gemm.cpp:123-152)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M = A.shape[1] if transA else A.shape[0]
    K = A.shape[0] if transA else A.shape[1]
    N = B.shape[0] if transB else B.shape[1]
    r0, r1 = (0, M) if rows is None else rows
    Y = np.empty((r1 - r0, N), dtype=np.float32)
    if C is None:
        cptr, cnd, d0, d1 = None, -1, 0, 0
    else:
        C = np.ascontiguousarray(C, dtype=np.float32)
        cnd = C.ndim
        d0 = C.shape[0] if C.ndim >= 1 else 0
        d1 = C.shape[1] if C.ndim >= 2 else 0
        cptr = _f(C)
    lib.orc_gemm_f32_rows_lanes(_f(A), _f(B), cptr, _i64(M), _i64(N), _i64(K), ctypes.c_int(transA),
                                ctypes.c_int(transB), ctypes.c_float(alpha), ctypes.c_float(beta),
                                ctypes.c_int(cnd), _i64(d0), _i64(d1), _f(Y), _i64(r0), _i64(r1),
                                ctypes.c_int(lanes))
    return Y


def qdq_gemm(Aq, sa, Bq, sb, b_kmajor=True, bias=None, rows=None) -> np.ndarray:
    """DequantizeLinear on both e4m3 operands, then gemm.cpp's fp32 loop.

    Aq [M,K]; Bq [N,K] when ``b_kmajor`` (Gemm transB=1) else [K,N].
    ``sa``: scalar or [M]; ``sb``: scalar or [N]. Returns fp32 [rows, N].
    """
    Aq = np.ascontiguousarray(Aq, dtype=np.uint8)
    Bq = np.ascontiguousarray(Bq, dtype=np.uint8)
    M, K = Aq.shape
    N = Bq.shape[0] if b_kmajor else Bq.shape[1]
    sa = np.ascontiguousarray(np.atleast_1d(np.asarray(sa, dtype=np.float32)))
    sb = np.ascontiguousarray(np.atleast_1d(np.asarray(sb, dtype=np.float32)))
    r0, r1 = (0, M) if rows is None else rows
    Y = np.empty((r1 - r0, N), dtype=np.float32)
    bptr = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        bptr = _f(bias)
    lib.orc_qdq_gemm_rows(_u(Aq), _f(sa), ctypes.c_int(int(sa.size > 1)), _u(Bq), _f(sb),
                          ctypes.c_int(int(sb.size > 1)), ctypes.c_int(int(bool(b_kmajor))), bptr,
                          _i64(M), _i64(N), _i64(K), _f(Y), _i64(r0), _i64(r1))
    return Y


def conv2d(X, W, bias=None, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group=1,
           images=None, lanes=1) -> np.ndarray:
    """ONNX Conv (2-D NCHW) following conv.cpp; output shape from the ONNX formula.
    lanes=1: one fma chain over (kh, kw, c); lanes=4: the reference's fp32
    order (per tap four lane sums over the channels, conv.cpp:150-191)."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    W = np.ascontiguousarray(W, dtype=np.float32)
    N, C, H, Wd = X.shape
    M, Cg, kH, kW = W.shape
    sH, sW = strides
    dH, dW = dilations
    pH, pW = pads[0], pads[1]
    pHe, pWe = (pads[2], pads[3]) if len(pads) == 4 else (pads[0], pads[1])
    oH = (H + pH + pHe - dH * (kH - 1) - 1) // sH + 1
    oW = (Wd + pW + pWe - dW * (kW - 1) - 1) // sW + 1
    n0, n1 = (0, N) if images is None else images
    Y = np.empty((n1 - n0, M, oH, oW), dtype=np.float32)
    bptr = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        bptr = _f(bias)
    ci = ctypes.c_int
    lib.orc_conv2d_f32_lanes(_f(X), _f(W), bptr, _i64(N), _i64(C), _i64(H), _i64(Wd), _i64(M), _i64(kH),
                             _i64(kW), _i64(oH), _i64(oW), ci(sH), ci(sW), ci(pH), ci(pW), ci(dH), ci(dW),
                             ci(group), _f(Y), _i64(n0), _i64(n1), ci(lanes))
    return Y


def conv_transpose2d(X, W, bias=None, strides=(1, 1), pads=(0, 0, 0, 0), dilations=(1, 1), group=1,
                     output_padding=(0, 0)) -> np.ndarray:
    """ONNX ConvTranspose (2-D NCHW, W [C, M/group, kH, kW]) following
    conv_transpose.cpp; output extent (H - 1) * s - pads + d * (k - 1) + 1 + output_padding."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    W = np.ascontiguousarray(W, dtype=np.float32)
    N, C, H, Wd = X.shape
    _, Mg, kH, kW = W.shape
    M = Mg * group
    sH, sW = strides
    dH, dW = dilations
    oH = (H - 1) * sH - pads[0] - pads[2] + dH * (kH - 1) + 1 + output_padding[0]
    oW = (Wd - 1) * sW - pads[1] - pads[3] + dW * (kW - 1) + 1 + output_padding[1]
    Y = np.empty((N, M, oH, oW), dtype=np.float32)
    bptr = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, dtype=np.float32)
        bptr = _f(bias)
    ci = ctypes.c_int
    lib.orc_conv_transpose2d_f32(_f(X), _f(W), bptr, _i64(N), _i64(C), _i64(H), _i64(Wd), _i64(M), _i64(kH),
                                 _i64(kW), _i64(oH), _i64(oW), ci(sH), ci(sW), ci(pads[0]), ci(pads[1]), ci(dH),
                                 ci(dW), ci(group), _f(Y))
    return Y


# --------------------------------------------------------------------------- memory-bound ops
def relu(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib.orc_relu(_f(x), _f(y), _i64(x.size))
    return y


def sigmoid(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib.orc_sigmoid(_f(x), _f(y), _i64(x.size))
    return y


def silu_mul(g, u):
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    y = np.empty_like(g)
    lib.orc_silu_mul(_f(g), _f(u), _f(y), _i64(g.size))
    return y


def softmax_rows(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    cols = x.shape[-1]
    lib.orc_softmax_rows(_f(x), _f(y), _i64(x.size // cols), _i64(cols))
    return y


def maxpool2d(x, kernel, strides, pads):
    x = np.ascontiguousarray(x, dtype=np.float32)
    N, C, H, W = x.shape
    kH, kW = kernel
    sH, sW = strides
    pH, pW = pads[0], pads[1]
    pHe, pWe = (pads[2], pads[3]) if len(pads) == 4 else (pH, pW)
    oH = (H + pH + pHe - kH) // sH + 1
    oW = (W + pW + pWe - kW) // sW + 1
    y = np.empty((N, C, oH, oW), dtype=np.float32)
    ci = ctypes.c_int
    lib.orc_maxpool2d(_f(x), _f(y), _i64(N * C), _i64(H), _i64(W), ci(kH), ci(kW), ci(sH), ci(sW),
                      ci(pH), ci(pW), _i64(oH), _i64(oW))
    return y


def global_avgpool(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    N, C, H, W = x.shape
    y = np.empty((N, C, 1, 1), dtype=np.float32)
    lib.orc_global_avgpool(_f(x), _f(y), _i64(N * C), _i64(H * W))
    return y


def replay_plan(plan, x):
    """Runs a QDQ convolutional network given as a list of steps (the order the
    reference's NetworkInstance executes the graph's nodes,
    src/onnx/network_instance.cpp:584-655), each through the restated operator:
      ("qdq", s)                 QuantizeLinear + DequantizeLinear, per-tensor scale
      ("conv", wq, ws, b, st, p) Conv on DequantizeLinear(wq, ws per output channel)
      ("relu",) ("maxpool",) (3x3 / 2 / pad 1) ("gap",) ("add",)
      ("fc", wq, ws, b)          Gemm(transB=1) on the dequantized weight
      ("block_begin",) / ("downsample_begin",) / ("downsample_end",)
                                 residual bookkeeping of a bottleneck block: the
                                 block input is kept, a projection branch runs
                                 from it first, and its output becomes the
                                 residual the later ("add",) uses.
    """
    h, blk_in, res = x, None, None
    for step in plan:
        kind = step[0]
        if kind == "qdq":
            h = dequantize(quantize(h, step[1]), step[1])
        elif kind == "conv":
            _, wq, ws, bias, stride, pad = step
            h = conv2d(h, dequantize(wq, ws, axis=0), bias, strides=(stride, stride), pads=(pad, pad, pad, pad))
        elif kind == "relu":
            h = relu(h)
        elif kind == "maxpool":
            h = maxpool2d(h, (3, 3), (2, 2), (1, 1, 1, 1))
        elif kind == "block_begin":
            blk_in = res = h
        elif kind == "downsample_begin":
            h = blk_in
        elif kind == "downsample_end":
            res, h = h, blk_in
        elif kind == "add":
            h = (h + res).astype(np.float32)
        elif kind == "gap":
            h = global_avgpool(h).reshape(h.shape[0], h.shape[1])
        elif kind == "fc":
            _, wq, ws, bias = step
            h = gemm(h, dequantize(wq, ws, axis=0), bias, transB=1)
        else:
            raise ValueError(f"unknown step {kind}")
    return h
