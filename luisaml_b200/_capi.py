"""ctypes binding of the C ABI in include/lcml_fp8.h (liblcml_fp8.so).

This is the binding a Python caller of the reference's operator path would
add; tests and bench.py go through it so every GPU number is measured across
the same C boundary the C++ executor uses. Loading fails loudly when the
library has not been built: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "liblcml_fp8.so")

# ONNX DataType numbers (include/onnx/onnx.h:31-60)
DTYPE_FLOAT = 1
DTYPE_FLOAT16 = 10
DTYPE_BFLOAT16 = 16
DTYPE_E4M3 = 17
PEER_SLOTS_BYTES = 512  # LCML_PEER_SLOTS_BYTES
DTYPE_E5M2 = 19
DTYPE_E2M1 = 23  # packed: two codes per byte, element 2i in the low nibble

SCALE_TENSOR = 0
SCALE_AXIS = 1
SCALE_ROW = 1
SCALE_COL = 2

# LCML_FP8_TENSOR_DYNAMIC_WORKSPACE_BYTES: scratch of lcml_fp8_quantize_tensor_dynamic
TENSOR_DYNAMIC_WORKSPACE_BYTES = 4096

EPI_NONE = 0
EPI_RELU = 1
EPI_SILU_MUL = 2

STATUS = {0: "OK", 1: "INVALID_ARGUMENT", 2: "UNSUPPORTED", 3: "CUDA", 4: "NO_DEVICE", 5: "DEVICE_TIMEOUT"}


class LcmlError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"lcml status {status} ({STATUS.get(status, '?')}): {msg}")
        self.status = status


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
        ("A", ctypes.c_void_p), ("lda", ctypes.c_int64),
        ("B", ctypes.c_void_p), ("ldb", ctypes.c_int64), ("b_kmajor", ctypes.c_int),
        ("scale_a", ctypes.c_void_p), ("scale_a_mode", ctypes.c_int),
        ("scale_b", ctypes.c_void_p), ("scale_b_mode", ctypes.c_int),
        ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
        ("c_vec", ctypes.c_void_p), ("c_vec_mode", ctypes.c_int),
        ("c_mat", ctypes.c_void_p), ("c_mat_dtype", ctypes.c_int), ("ldc", ctypes.c_int64),
        ("epilogue", ctypes.c_int),
        ("Y", ctypes.c_void_p), ("y_dtype", ctypes.c_int), ("ldy", ctypes.c_int64),
        ("y_scale", ctypes.c_void_p),
        ("row_amax", ctypes.c_void_p),
        ("y_col_offset", ctypes.c_int64),
        ("y_peers", ctypes.c_void_p),
        ("y_num_peers", ctypes.c_int),
        ("c_mat_scale", ctypes.c_void_p),
        ("variant", ctypes.c_int),
    ]


class ConvDesc(ctypes.Structure):
    _fields_ = [
        ("N", ctypes.c_int64), ("C", ctypes.c_int64), ("H", ctypes.c_int64), ("W", ctypes.c_int64),
        ("M", ctypes.c_int64), ("kH", ctypes.c_int64), ("kW", ctypes.c_int64),
        ("oH", ctypes.c_int64), ("oW", ctypes.c_int64),
        ("sH", ctypes.c_int), ("sW", ctypes.c_int), ("pH", ctypes.c_int), ("pW", ctypes.c_int),
        ("dH", ctypes.c_int), ("dW", ctypes.c_int), ("group", ctypes.c_int),
        ("X", ctypes.c_void_p), ("x_nhwc", ctypes.c_int), ("scale_x", ctypes.c_void_p),
        ("Wp", ctypes.c_void_p), ("scale_w", ctypes.c_void_p), ("scale_w_mode", ctypes.c_int),
        ("bias", ctypes.c_void_p), ("residual", ctypes.c_void_p), ("residual_dtype", ctypes.c_int),
        ("residual_scale", ctypes.c_void_p), ("epilogue", ctypes.c_int),
        ("Y", ctypes.c_void_p), ("y_dtype", ctypes.c_int), ("y_scale", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("variant", ctypes.c_int),
    ]


_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_ci = ctypes.c_int

# name -> argtypes; every function returns int status unless listed in _RESTYPES
PROTOTYPES = {
    "lcml_abi_version": [],
    "lcml_device_check": [],
    "lcml_device_error": [ctypes.POINTER(ctypes.c_int)],
    "lcml_device_alloc": [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)],
    "lcml_device_free": [_vp],
    "lcml_memcpy_async": [_vp, _vp, ctypes.c_size_t, _ci, _vp],
    "lcml_memset_async": [_vp, _ci, ctypes.c_size_t, _vp],
    "lcml_stream_synchronize": [_vp],
    "lcml_stream_create": [ctypes.POINTER(ctypes.c_void_p)],
    "lcml_stream_destroy": [_vp],
    "lcml_event_create": [ctypes.POINTER(ctypes.c_void_p)],
    "lcml_event_destroy": [_vp],
    "lcml_event_record": [_vp, _vp],
    "lcml_stream_wait_event": [_vp, _vp],
    "lcml_ipc_get_handle": [_vp, _vp],
    "lcml_ipc_open": [_vp, ctypes.POINTER(ctypes.c_void_p)],
    "lcml_ipc_close": [_vp],
    "lcml_enable_peer_access": [_ci],
    "lcml_peer_exchange_max": [_vp, _vp, _vp, _vp, _ci, _ci, ctypes.c_uint32, ctypes.c_uint32, _vp],
    "lcml_gemm_f32": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _ci, _ci, ctypes.c_float, ctypes.c_float, _ci, _c_i64,
                      _c_i64, _vp, _vp],
    "lcml_gemm_f32_relu": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _ci, _ci, ctypes.c_float, ctypes.c_float, _ci, _c_i64,
                      _c_i64, _vp, _vp],
    "lcml_fp8_quantize": [_vp, _c_i64, _c_i64, _c_i64, _vp, _ci, _vp, _vp],
    "lcml_fp8_quantize_from_amax": [_vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _vp],
    "lcml_fp8_quantize_rows_dynamic": [_vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp],
    "lcml_amax": [_vp, _c_i64, _vp, _vp],
    "lcml_fp8_quantize_tensor_dynamic": [_vp, _c_i64, _vp, _vp, _vp, _vp],
    "lcml_fp8_dequantize": [_vp, _c_i64, _c_i64, _c_i64, _vp, _ci, _vp, _ci, _vp],
    "lcml_fp8_transpose": [_vp, _c_i64, _c_i64, _vp, _vp],
    "lcml_fp8_gemm": [ctypes.POINTER(GemmDesc), _vp],
    "lcml_fp8_gemm_quantize_a": [ctypes.POINTER(GemmDesc), _vp, _c_i64, _vp, _vp, _vp, _vp],
    "lcml_fp8_gemm_simt": [ctypes.POINTER(GemmDesc), _vp],
    "lcml_fp8_gemm_rowquant": [ctypes.POINTER(GemmDesc), _vp, _vp, _vp, _vp],
    "lcml_fp8_gemm_rowquant_noalloc": [ctypes.POINTER(GemmDesc), _vp, _vp, _vp],
    "lcml_fp8_conv_workspace_size": [ctypes.POINTER(ConvDesc)],
    "lcml_fp8_conv_packed_k": [_c_i64, _c_i64, _c_i64],
    "lcml_fp8_conv_pack_weight": [_vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _vp],
    "lcml_fp8_conv": [ctypes.POINTER(ConvDesc), _vp],
    "lcml_conv2d_f32": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _ci,
                        _ci, _ci, _ci, _ci, _ci, _ci, _vp, _vp],
    "lcml_conv_transpose2d_f32": [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                  _c_i64, _ci, _ci, _ci, _ci, _ci, _ci, _ci, _vp, _vp],
    "lcml_unary_f32": [_ci, _vp, _vp, _c_i64, _vp],
    "lcml_binary_f32": [_ci, _vp, _vp, _c_i64, _c_i64, _vp, _vp],
    "lcml_reduce_max_rows": [_vp, _c_i64, _c_i64, _ci, _vp, _vp],
    "lcml_softmax_rows": [_vp, _c_i64, _c_i64, _vp, _vp],
    "lcml_binary_fp8": [_ci, _vp, _vp, _c_i64, _c_i64, _vp, _ci, _vp],
    "lcml_softmax_rows_fp8": [_vp, _c_i64, _c_i64, _vp, _ci, _vp],
    "lcml_maxpool2d": [_vp, _ci, _c_i64, _c_i64, _c_i64, _ci, _ci, _ci, _ci, _ci, _ci, _c_i64, _c_i64, _vp,
                       _ci, _c_i64, _vp],
    "lcml_global_avgpool": [_vp, _ci, _vp, _c_i64, _c_i64, _c_i64, _ci, _vp, _vp],
    "lcml_cast": [_vp, _ci, _vp, _ci, _c_i64, _vp],
}
_RESTYPES = {
    "lcml_last_error": ctypes.c_char_p,
    "lcml_launch_count": ctypes.c_uint64,
    "lcml_fp8_conv_workspace_size": ctypes.c_int64,
    "lcml_fp8_conv_packed_k": ctypes.c_int64,
}

_lib = None


def load():
    """Load liblcml_fp8.so (built in-tree by build()); raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} not built: run `python -c 'import __graft_entry__ as g; g.build()'` "
                          "or `make -C luisaml_b200`")
    lib = ctypes.CDLL(LIB_PATH)
    lib.lcml_last_error.restype = ctypes.c_char_p
    lib.lcml_last_error.argtypes = []
    lib.lcml_launch_count.restype = ctypes.c_uint64
    lib.lcml_launch_count.argtypes = []
    for name, args in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != 0:
        msg = load().lcml_last_error().decode(errors="replace")
        raise LcmlError(rc, msg)
