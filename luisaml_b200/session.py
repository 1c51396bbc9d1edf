"""ctypes binding of include/lcml_session.h: the C++ NetworkInstance driven
from Python with torch-owned device buffers (plumbing for tests and bench)."""
from __future__ import annotations

import ctypes
import os

from ._capi import LcmlError

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "liblcml_onnx.so")

_lib = None
_vp, _i64, _ci, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t


def load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} not built: run `make -C luisaml_b200`")
    lib = ctypes.CDLL(LIB_PATH)
    lib.lcml_network_last_error.restype = ctypes.c_char_p
    lib.lcml_network_create.argtypes = [ctypes.c_char_p, _sz, ctypes.POINTER(_vp)]
    lib.lcml_network_destroy.argtypes = [_vp]
    lib.lcml_network_destroy.restype = None
    lib.lcml_network_info.argtypes = [_vp, ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i64)]
    lib.lcml_network_set_weight_buffer.argtypes = [_vp, _vp, _sz]
    lib.lcml_network_set_input.argtypes = [_vp, ctypes.c_char_p, _vp, _ci, ctypes.POINTER(_i64), _ci]
    lib.lcml_network_set_output.argtypes = [_vp, ctypes.c_char_p, _vp, _ci, ctypes.POINTER(_i64), _ci]
    lib.lcml_network_set_input_host.argtypes = [_vp, ctypes.c_char_p, _vp]
    lib.lcml_network_set_output_host.argtypes = [_vp, ctypes.c_char_p, _vp]
    lib.lcml_network_set_async_outputs.argtypes = [_vp, _ci]
    lib.lcml_network_wait_outputs.argtypes = [_vp, _vp]
    lib.lcml_network_set_fusion.argtypes = [_vp, _ci]
    lib.lcml_network_set_memory_reuse.argtypes = [_vp, _ci]
    lib.lcml_network_memory.argtypes = [_vp, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]
    lib.lcml_network_set_stream.argtypes = [_vp, _vp]
    lib.lcml_network_forward.argtypes = [_vp]
    lib.lcml_network_executed_nodes.argtypes = [_vp, ctypes.POINTER(_i64)]
    lib.lcml_network_summary.argtypes = [_vp, ctypes.c_char_p, _sz]
    lib.lcml_network_tensor.argtypes = [_vp, ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.POINTER(_ci),
                                        ctypes.POINTER(_i64), _ci, ctypes.POINTER(_ci), ctypes.POINTER(_ci)]
    lib.lcml_opset_size.argtypes = []
    _lib = lib
    return lib


def _check(rc):
    if rc != 0:
        raise LcmlError(rc, load().lcml_network_last_error().decode(errors="replace"))


_TORCH_DT = {"float32": 1, "float16": 10, "bfloat16": 16, "uint8": 17}


class Network:
    """A loaded LuisaML-JSON model bound to device buffers."""

    def __init__(self, json_text: str):
        lib = load()
        data = json_text.encode()
        h = _vp()
        _check(lib.lcml_network_create(data, len(data), ctypes.byref(h)))
        self._h = h
        self._keep = []

    def close(self):
        if getattr(self, "_h", None):
            load().lcml_network_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def info(self):
        n, i, o = _i64(), _i64(), _i64()
        _check(load().lcml_network_info(self._h, ctypes.byref(n), ctypes.byref(i), ctypes.byref(o)))
        return n.value, i.value, o.value

    def set_weight_buffer(self, t):
        self._keep.append(t)
        _check(load().lcml_network_set_weight_buffer(self._h, t.data_ptr(), t.numel() * t.element_size()))

    def _bind(self, fn, name, t, dtype=None):
        self._keep.append(t)
        dt = dtype if dtype is not None else _TORCH_DT[str(t.dtype).replace("torch.", "")]
        shape = (_i64 * max(1, t.dim()))(*t.shape)
        _check(fn(self._h, name.encode(), t.data_ptr(), dt, shape, t.dim()))

    def set_input(self, name, t, dtype=None):
        self._bind(load().lcml_network_set_input, name, t, dtype)

    def set_output(self, name, t, dtype=None):
        self._bind(load().lcml_network_set_output, name, t, dtype)

    def set_input_host(self, name, t):
        """Host-staged input: the pinned host tensor `t` (the bound input's
        size) is copied in at the start of every forward, overlapping the
        previous forward once its readers of the input have run."""
        if t is not None:
            self._keep.append(t)
        _check(load().lcml_network_set_input_host(self._h, name.encode(), None if t is None else t.data_ptr()))

    def set_output_host(self, name, t):
        """Host-staged output: forward() copies the bound output into the
        pinned host tensor `t` after its last node (on the network's stream)."""
        if t is not None:
            self._keep.append(t)
        _check(load().lcml_network_set_output_host(self._h, name.encode(), None if t is None else t.data_ptr()))

    def set_async_outputs(self, enable: bool):
        """Host-staged outputs copied on a third stream, overlapping the next
        forward; they are complete after wait_outputs()."""
        _check(load().lcml_network_set_async_outputs(self._h, int(enable)))

    def wait_outputs(self, stream_handle=None):
        """No stream: the host waits for every output copy enqueued so far;
        with a stream handle: that stream waits for them."""
        _check(load().lcml_network_wait_outputs(self._h, stream_handle))

    def set_fusion(self, enable: bool):
        _check(load().lcml_network_set_fusion(self._h, int(enable)))

    def set_memory_reuse(self, enable: bool):
        """Intermediates in one lifetime-planned arena (default) or one allocation each."""
        _check(load().lcml_network_set_memory_reuse(self._h, int(enable)))

    def memory(self):
        """(intermediate bytes as allocated, bytes with one allocation each), after the first forward."""
        a, b = ctypes.c_size_t(), ctypes.c_size_t()
        _check(load().lcml_network_memory(self._h, ctypes.byref(a), ctypes.byref(b)))
        return a.value, b.value

    def set_stream(self, stream_handle: int):
        _check(load().lcml_network_set_stream(self._h, stream_handle))

    def forward(self):
        _check(load().lcml_network_forward(self._h))

    def executed_nodes(self) -> int:
        n = _i64()
        _check(load().lcml_network_executed_nodes(self._h, ctypes.byref(n)))
        return n.value

    def summary(self) -> str:
        buf = ctypes.create_string_buffer(1 << 16)
        _check(load().lcml_network_summary(self._h, buf, len(buf)))
        return buf.value.decode()

    def tensor_info(self, name: str):
        """(device pointer, ONNX dtype code, ONNX shape, stored NHWC) of any
        tensor of the prepared graph."""
        ptr, dt, nd, nh = _vp(), _ci(), _ci(), _ci()
        shape = (_i64 * 8)()
        _check(load().lcml_network_tensor(self._h, name.encode(), ctypes.byref(ptr), ctypes.byref(dt), shape, 8,
                                          ctypes.byref(nd), ctypes.byref(nh)))
        return ptr.value, dt.value, tuple(shape[i] for i in range(nd.value)), bool(nh.value)

    def read_tensor(self, name: str):
        """Host copy of a tensor after forward(), as a numpy array in storage
        order (NHWC tensors come back as N, H, W, C); fp32 as float32, bf16 as
        uint16 bit patterns, e4m3 as uint8 codes."""
        import numpy as np
        from . import check, lib as fp8_lib
        ptr, dt, shape, nhwc = self.tensor_info(name)
        npdt = {1: np.float32, 10: np.uint16, 16: np.uint16, 17: np.uint8, 19: np.uint8, 2: np.uint8, 7: np.int64,
                6: np.int32}[dt]
        if nhwc and len(shape) == 4:
            shape = (shape[0], shape[2], shape[3], shape[1])
        out = np.empty(shape, dtype=npdt)
        if out.nbytes:
            lib = fp8_lib()
            check(lib.lcml_memcpy_async(out.ctypes.data, ptr, out.nbytes, 2, None))
            check(lib.lcml_stream_synchronize(None))
        return out
