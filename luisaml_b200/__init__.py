"""luisaml_b200 — B200 (sm_100a) FP8 e4m3 operator path for LuisaML's ONNX executor.

Layers:
* ``lib/liblcml_fp8.so``  hand-written CUDA kernels behind the C ABI of
  ``include/lcml_fp8.h`` (quantize / dequantize, tcgen05 FP8 GEMM and
  implicit-GEMM conv with fused QDQ epilogues, memory-bound ops);
* ``lib/liblcml_onnx.so`` the C++ host mirror of LuisaML's operator registry,
  tensor API and NetworkInstance (``include/lcml_onnx.h``), whose operators
  call the C ABI;
* this module: torch-tensor helpers over the C ABI (device memory, streams)
  used by tests and bench.py. PyTorch is plumbing here, not the product.
"""
from __future__ import annotations

import ctypes

from . import _capi
from ._capi import (TENSOR_DYNAMIC_WORKSPACE_BYTES, DTYPE_BFLOAT16, DTYPE_E4M3, DTYPE_FLOAT, EPI_NONE, EPI_RELU, EPI_SILU_MUL, SCALE_AXIS,
                    SCALE_COL, SCALE_ROW, SCALE_TENSOR, GemmDesc, LcmlError, check)

__all__ = ["lib", "check", "LcmlError", "quantize", "quantize_from_amax", "quantize_rows_dynamic",
           "quantize_tensor_dynamic", "amax", "dequantize", "transpose_u8", "gemm", "gemm_rowquant", "launch_count",
           "device_error"]


def lib():
    return _capi.load()


def _torch():
    import torch
    return torch


def _stream():
    return ctypes.c_void_p(_torch().cuda.current_stream().cuda_stream)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("luisaml_b200 ops take CUDA tensors")


def launch_count() -> int:
    return int(lib().lcml_launch_count())


def device_error() -> int:
    code = ctypes.c_int(0)
    lib().lcml_device_error(ctypes.byref(code))
    return code.value


def _dtype_code(dt):
    torch = _torch()
    if dt == torch.float32:
        return DTYPE_FLOAT
    if dt == torch.bfloat16:
        return DTYPE_BFLOAT16
    if dt == torch.uint8:
        return DTYPE_E4M3
    raise ValueError(f"unsupported dtype {dt}")


def _axis_view(shape, axis):
    import math
    ax = axis % len(shape)
    return int(math.prod(shape[:ax])), int(shape[ax]), int(math.prod(shape[ax + 1:]))


def quantize(x, scale, axis=None, out=None):
    """QuantizeLinear (e4m3, zp 0, saturate) of fp32 ``x``; ``scale`` fp32 [1] or [x.shape[axis]]."""
    torch = _torch()
    _require_cuda(x, scale)
    assert x.dtype == torch.float32 and x.is_contiguous()
    y = out if out is not None else torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    if axis is None or scale.numel() == 1 and axis is None:
        outer, alen, inner, mode = 1, 1, x.numel(), SCALE_TENSOR
    else:
        outer, alen, inner = _axis_view(x.shape, axis)
        mode = SCALE_AXIS
    check(lib().lcml_fp8_quantize(_p(x), outer, alen, inner, _p(scale), mode, _p(y), _stream()))
    return y


def quantize_from_amax(x, amax_vec, axis, scale_out=None, out=None):
    torch = _torch()
    y = out if out is not None else torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    outer, alen, inner = _axis_view(x.shape, axis)
    check(lib().lcml_fp8_quantize_from_amax(_p(x), outer, alen, inner, _p(amax_vec), _p(scale_out), _p(y),
                                            _stream()))
    return y


def quantize_rows_dynamic(x, out=None, scale_out=None):
    """Per-row dynamic quantization of 2-D fp32 ``x``: returns (q uint8, s fp32 [rows])."""
    torch = _torch()
    _require_cuda(x)
    rows, cols = x.shape
    y = out if out is not None else torch.empty((rows, cols), dtype=torch.uint8, device=x.device)
    s = scale_out if scale_out is not None else torch.empty(rows, dtype=torch.float32, device=x.device)
    check(lib().lcml_fp8_quantize_rows_dynamic(_p(x), rows, cols, x.stride(0), _p(s), _p(y), _stream()))
    return y, s


def amax(x, out=None):
    torch = _torch()
    o = out if out is not None else torch.empty(1, dtype=torch.float32, device=x.device)
    check(lib().lcml_amax(_p(x), x.numel(), _p(o), _stream()))
    return o


def quantize_tensor_dynamic(x, workspace=None, out=None, scale_out=None):
    torch = _torch()
    ws = workspace if workspace is not None else torch.empty(TENSOR_DYNAMIC_WORKSPACE_BYTES // 4, dtype=torch.float32,
                                                             device=x.device)
    y = out if out is not None else torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    s = scale_out if scale_out is not None else torch.empty(1, dtype=torch.float32, device=x.device)
    check(lib().lcml_fp8_quantize_tensor_dynamic(_p(x), x.numel(), _p(s), _p(y), _p(ws), _stream()))
    return y, s


def dequantize(q, scale, axis=None, dtype=None):
    torch = _torch()
    dtype = dtype or torch.float32
    y = torch.empty(q.shape, dtype=dtype, device=q.device)
    if axis is None:
        outer, alen, inner, mode = 1, 1, q.numel(), SCALE_TENSOR
    else:
        outer, alen, inner = _axis_view(q.shape, axis)
        mode = SCALE_AXIS
    check(lib().lcml_fp8_dequantize(_p(q), outer, alen, inner, _p(scale), mode, _p(y), _dtype_code(dtype),
                                    _stream()))
    return y


def transpose_u8(src):
    torch = _torch()
    r, c = src.shape
    dst = torch.empty((c, r), dtype=torch.uint8, device=src.device)
    check(lib().lcml_fp8_transpose(_p(src), r, c, _p(dst), _stream()))
    return dst


def gemm(A, B, sa, sb, *, b_kmajor=True, alpha=1.0, beta=1.0, c_vec=None, c_vec_mode=None, c_mat=None,
         c_mat_scale=None, epilogue=EPI_NONE, out_dtype=None, y_scale=None, row_amax=None, out=None, simt=False,
         desc_only=False, variant=0):
    """Fused FP8 GEMM through lcml_fp8_gemm. A [M,K] e4m3 (uint8); B [N,K] (b_kmajor) or [K,N].

    sa: fp32 [1] or [M]; sb: fp32 [1] or [N]. Returns Y [M, N] (N/2 for SILU_MUL).
    variant: lcml_fp8_gemm_desc.variant (0 automatic kernel choice).
    """
    torch = _torch()
    out_dtype = out_dtype or torch.bfloat16
    M, K = A.shape
    N = B.shape[0] if b_kmajor else B.shape[1]
    n_out = N // 2 if epilogue == EPI_SILU_MUL else N
    Y = out if out is not None else torch.empty((M, n_out), dtype=out_dtype, device=A.device)
    d = GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.A, d.lda = A.data_ptr(), A.stride(0)
    d.B, d.ldb, d.b_kmajor = B.data_ptr(), B.stride(0), int(bool(b_kmajor))
    d.scale_a, d.scale_a_mode = sa.data_ptr(), SCALE_ROW if sa.numel() > 1 else SCALE_TENSOR
    d.scale_b, d.scale_b_mode = sb.data_ptr(), SCALE_COL if sb.numel() > 1 else SCALE_TENSOR
    d.alpha, d.beta = alpha, beta
    if c_vec is not None:
        d.c_vec = c_vec.data_ptr()
        if c_vec_mode is None:
            c_vec_mode = SCALE_COL if c_vec.numel() == N and N > 1 else (SCALE_ROW if c_vec.numel() == M and M > 1 else SCALE_TENSOR)
        d.c_vec_mode = c_vec_mode
    if c_mat is not None:
        d.c_mat, d.c_mat_dtype, d.ldc = c_mat.data_ptr(), _dtype_code(c_mat.dtype), c_mat.stride(0)
        if c_mat_scale is not None:  # an e4m3 (uint8) residual is decoded times this per-tensor scale
            d.c_mat_scale = c_mat_scale.data_ptr()
    d.epilogue = epilogue
    d.variant = variant
    d.Y, d.y_dtype, d.ldy = Y.data_ptr(), _dtype_code(Y.dtype), Y.stride(0)
    if y_scale is not None:
        d.y_scale = y_scale.data_ptr()
    if row_amax is not None:
        d.row_amax = row_amax.data_ptr()
    if desc_only:
        # the descriptor holds raw device pointers: keep the tensors they point into alive with it
        d._refs = (A, B, sa, sb, c_vec, c_mat, c_mat_scale, Y, y_scale, row_amax)
        return d, Y
    fn = lib().lcml_fp8_gemm_simt if simt else lib().lcml_fp8_gemm
    check(fn(ctypes.byref(d), _stream()))
    return Y


def gemm_quantize_a(A, B, sb, *, aq=None, workspace=None, **kw):
    """lcml_fp8_gemm_quantize_a: fp32 A [M, K] quantized with a dynamic
    per-tensor scale and multiplied by e4m3 B in one call (one kernel for
    M <= 4 on the GEMV path). Returns (Y, Aq or None, s). kw as for gemm()
    (variant, epilogue, out_dtype, ...)."""
    torch = _torch()
    M, K = A.shape
    s = torch.empty(1, dtype=torch.float32, device=A.device)
    fused = M <= 4 and kw.get("variant", 0) == 0
    if aq is None and not fused:
        aq = torch.empty((M, K), dtype=torch.uint8, device=A.device)
    if workspace is None and not fused:
        workspace = torch.empty(TENSOR_DYNAMIC_WORKSPACE_BYTES // 4, dtype=torch.float32, device=A.device)
    placeholder = aq if aq is not None else torch.empty((M, K), dtype=torch.uint8, device=A.device)
    d, Y = gemm(placeholder, B, s, sb, desc_only=True, **kw)
    check(lib().lcml_fp8_gemm_quantize_a(ctypes.byref(d), _p(A), A.stride(0), _p(aq) if aq is not None else None,
                                         _p(s), _p(workspace) if workspace is not None else None, _stream()))
    return Y, aq, s


def gemm_rowquant(A, B, sa, sb, *, workspace=None, **kw):
    """Fused GEMM (fp32 Y) + dynamic per-row e4m3 quantization of Y through
    lcml_fp8_gemm_rowquant. Returns (Y fp32, q uint8, s fp32 [M])."""
    torch = _torch()
    M = A.shape[0]
    d, Y = gemm(A, B, sa, sb, out_dtype=torch.float32, desc_only=True, **kw)
    q = torch.empty(Y.shape, dtype=torch.uint8, device=A.device)
    s = torch.empty(M, dtype=torch.float32, device=A.device)
    ws = workspace if workspace is not None else torch.empty(M, dtype=torch.float32, device=A.device)
    check(lib().lcml_fp8_gemm_rowquant(ctypes.byref(d), _p(q), _p(s), _p(ws), _stream()))
    return Y, q, s
