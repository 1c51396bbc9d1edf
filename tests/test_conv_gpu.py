"""FP8 convolution (lcml_fp8_conv) vs the oracle's direct conv loop
(conv.cpp:137-207 restated in oracle/oracle.c) on dequantized operands.

X is e4m3 with a per-tensor scale (NCHW for the stem, NHWC otherwise),
W is e4m3 with per-output-channel scales; outputs are NHWC.
"""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import assert_close

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.array(a, copy=True)).to(dev)


def _run_conv(dev, X, W, bias, stride, pad, nhwc_in=True, relu=False, residual=None, out="f32", y_scale=None,
              no_workspace=False, dil=1, variant=0):
    """Quantizes X (per tensor) and W (per channel) with the oracle, runs the
    GPU conv; returns (gpu NCHW fp32 result, oracle result on the dequantized
    operands, dequantization helpers)."""
    import torch
    import luisaml_b200 as lb
    N, C, H, Wd = X.shape
    M, _, kH, kW = W.shape
    sx = np.float32(oracle.scale_from_amax(oracle.amax(X)))
    xq = oracle.quantize(X, sx)
    sw = np.array([oracle.scale_from_amax(oracle.amax(W[m])) for m in range(M)], dtype=np.float32)
    wq = oracle.quantize(W, sw, axis=0)
    oH = (H + 2 * pad - dil * (kH - 1) - 1) // stride + 1
    oW = (Wd + 2 * pad - dil * (kW - 1) - 1) // stride + 1
    ref = oracle.conv2d(oracle.dequantize(xq, sx), oracle.dequantize(wq, sw, axis=0), bias, strides=(stride, stride),
                        pads=(pad, pad, pad, pad), dilations=(dil, dil))
    Kp = lb.lib().lcml_fp8_conv_packed_k(C, kH, kW)
    Wp = torch.empty((M, Kp), dtype=torch.uint8, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    wq_t = _t(wq, dev)
    lb.check(lb.lib().lcml_fp8_conv_pack_weight(ctypes.c_void_p(wq_t.data_ptr()), M, C, kH, kW,
                                                ctypes.c_void_p(Wp.data_ptr()), stream))
    xin = np.ascontiguousarray(xq.transpose(0, 2, 3, 1)) if nhwc_in else xq
    xt, sxt, swt = _t(xin, dev), _t(np.float32([sx]), dev), _t(sw, dev)
    dt = {"f32": torch.float32, "bf16": torch.bfloat16, "e4m3": torch.uint8}[out]
    Y = torch.empty((N, oH, oW, M), dtype=dt, device=dev)
    d = lb._capi.ConvDesc()
    d.N, d.C, d.H, d.W, d.M, d.kH, d.kW, d.oH, d.oW = N, C, H, Wd, M, kH, kW, oH, oW
    d.sH = d.sW = stride
    d.pH = d.pW = pad
    d.dH = d.dW = dil
    d.group = 1
    d.variant = variant
    d.X, d.x_nhwc, d.scale_x = xt.data_ptr(), int(nhwc_in), sxt.data_ptr()
    d.Wp, d.scale_w, d.scale_w_mode = Wp.data_ptr(), swt.data_ptr(), lb.SCALE_AXIS
    keep = [xt, sxt, swt, Wp]
    if bias is not None:
        bt = _t(bias, dev)
        keep.append(bt)
        d.bias = bt.data_ptr()
    res_ref = 0.0
    if residual is not None:
        rs = np.float32(oracle.scale_from_amax(oracle.amax(residual)))
        rq = oracle.quantize(residual, rs)  # NCHW
        res_ref = oracle.dequantize(rq, rs)
        rt, rst = _t(np.ascontiguousarray(rq.transpose(0, 2, 3, 1)), dev), _t(np.float32([rs]), dev)
        keep += [rt, rst]
        d.residual, d.residual_dtype, d.residual_scale = rt.data_ptr(), lb.DTYPE_E4M3, rst.data_ptr()
    d.epilogue = lb.EPI_RELU if relu else lb.EPI_NONE
    d.Y, d.y_dtype = Y.data_ptr(), {"f32": 1, "bf16": 16, "e4m3": 17}[out]
    if out == "e4m3":
        yst = _t(np.float32([y_scale]), dev)
        keep.append(yst)
        d.y_scale = yst.data_ptr()
    ws_bytes = lb.lib().lcml_fp8_conv_workspace_size(ctypes.byref(d))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    d.workspace = None if no_workspace else ws.data_ptr()
    lb.check(lb.lib().lcml_fp8_conv(ctypes.byref(d), stream))
    torch.cuda.synchronize()
    ref = ref + res_ref
    if relu:
        ref = np.maximum(ref, 0.0)
    y = Y.cpu()
    if out == "e4m3":
        got = oracle.e4m3_decode(y.numpy()).astype(np.float32)
    else:
        got = y.float().numpy()
    return got.transpose(0, 3, 1, 2), ref, ws_bytes


CASES = [
    # name, N, C, H, M, k, stride, pad, nhwc, dilation
    ("stem7x7s2_nchw", 2, 3, 64, 64, 7, 2, 3, False, 1),
    ("1x1_direct", 2, 64, 56, 256, 1, 1, 0, True, 1),
    ("3x3_pad1", 2, 64, 56, 64, 3, 1, 1, True, 1),
    ("3x3_s2", 2, 128, 56, 128, 3, 2, 1, True, 1),
    ("1x1_s2_downsample", 2, 256, 56, 512, 1, 2, 0, True, 1),
    ("3x3_7x7map", 4, 512, 7, 512, 3, 1, 1, True, 1),
    ("nchw_c8_3x3", 2, 8, 20, 32, 3, 1, 1, False, 1),       # 8-channel taps after the NHWC repack
    ("nhwc_c24_3x3_s2", 2, 24, 19, 48, 3, 2, 1, True, 1),  # C padded to 32
    ("nchw_c32_5x5", 1, 32, 17, 16, 5, 1, 2, False, 1),     # NCHW with 16-byte taps
    ("stem7x7s2_nchw_odd_hw", 2, 3, 15, 24, 7, 2, 3, False, 1),  # H*W % 4 != 0: the per-pixel repack
    ("nchw_c2_3x3", 2, 2, 16, 8, 3, 1, 1, False, 1),        # two planes into 4-channel taps
    ("nchw_c3_9x9", 1, 3, 20, 16, 9, 1, 4, False, 1),       # Kp = 336 > 256: the looped row im2col
    ("nhwc_c6_7x7_s2", 1, 6, 18, 16, 7, 2, 3, True, 1),     # NHWC repack to 8 channels, Kp = 392
    ("3x3_c16_ragged", 3, 16, 13, 24, 3, 1, 1, True, 1),    # K = 144: a partial last K-block, N = 24
    ("5x5_s2_p2", 2, 48, 23, 96, 5, 2, 2, True, 1),          # taps straddling K-blocks (48-channel taps)
    # implicit GEMM (TMA im2col) edge cases
    ("3x3_c192_ragged_tiles", 3, 192, 13, 96, 3, 1, 1, True, 1),  # 64-byte K-blocks; tiles straddle images
    ("7x7_s2_p3_c64", 2, 64, 30, 64, 7, 2, 3, True, 1),           # wide padding, odd output extent
    ("3x3_dil2_c128", 2, 128, 17, 128, 3, 1, 2, True, 2),         # dilated taps
    ("2x2_s2_nopad_c64", 1, 64, 15, 32, 2, 2, 0, True, 1),        # input rows/cols no tap reads
    ("3x3_s3_c128", 2, 128, 20, 64, 3, 3, 0, True, 1),            # traversal stride 3
    ("5x5_s1_p2_c64", 2, 64, 20, 64, 5, 1, 2, True, 1),           # two-pixel borders
    ("3x3_s1_c128_ragged", 3, 128, 11, 96, 3, 1, 1, True, 1),     # 128-byte rows; tiles straddle images
    ("3x3_s1_c64_w1", 2, 64, 1, 64, 3, 1, 1, True, 1),            # 1 x 1 images: every off-centre tap is an edge
]


def _implicit(C, k, stride, pad, nhwc):
    return nhwc and C % 64 == 0 and not (k == 1 and stride == 1 and pad == 0)


@pytest.mark.parametrize("name,N,C,H,M,k,stride,pad,nhwc,dil", CASES)
def test_conv_shapes(dev, name, N, C, H, M, k, stride, pad, nhwc, dil):
    """Every lowering vs the oracle: direct 1x1, materialized im2col (conv
    variant bit 0) and, for NHWC inputs with C % 64 == 0, the implicit GEMM
    (TMA im2col loads; the default there, with or without a workspace), whose
    result must equal the materialized one bit for bit when both run the
    single-CTA GEMM (GEMM variant 1 in bits 8-10). With automatic GEMM
    selection a small materialized conv may run split-K (another summation
    order): checked against the oracle."""
    rng = np.random.default_rng(sum(name.encode()))
    X = rng.standard_normal((N, C, H, H)).astype(np.float32)
    W = (rng.standard_normal((M, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    bias = (rng.standard_normal(M) * 0.01).astype(np.float32)
    got_auto, ref, _ = _run_conv(dev, X, W, bias, stride, pad, nhwc_in=nhwc, dil=dil, variant=1)
    assert_close(got_auto, ref, what=name + " (automatic GEMM selection)")
    single_cta = 1 << 8
    got, ref, ws = _run_conv(dev, X, W, bias, stride, pad, nhwc_in=nhwc, dil=dil, variant=1 | single_cta)
    assert (ws == 0) == (name == "1x1_direct")
    assert_close(got, ref, what=name)
    got_a, _, ws_a = _run_conv(dev, X, W, bias, stride, pad, nhwc_in=nhwc, dil=dil, variant=single_cta)
    implicit = _implicit(C, k, stride, pad, nhwc)
    assert (ws_a == 0) == (implicit or name == "1x1_direct")
    np.testing.assert_array_equal(got_a, got)
    if implicit:
        got_n, _, _ = _run_conv(dev, X, W, bias, stride, pad, nhwc_in=nhwc, no_workspace=True, dil=dil,
                                variant=single_cta)
        np.testing.assert_array_equal(got_n, got)


def test_conv_residual_relu_e4m3_out(dev):
    rng = np.random.default_rng(5)
    X = rng.standard_normal((2, 64, 28, 28)).astype(np.float32)
    W = (rng.standard_normal((256, 64, 1, 1)) * 0.1).astype(np.float32)
    R = rng.standard_normal((2, 256, 28, 28)).astype(np.float32)
    got32, ref, _ = _run_conv(dev, X, W, None, 1, 0, relu=True, residual=R)
    assert_close(got32, ref, what="residual + relu")
    ys = np.float32(oracle.scale_from_amax(np.abs(ref).max()))
    got8, _, _ = _run_conv(dev, X, W, None, 1, 0, relu=True, residual=R, out="e4m3", y_scale=ys)
    want = oracle.dequantize(oracle.quantize(ref, ys), ys)
    step = np.maximum(np.abs(want) * 0.125, ys * 2.0 ** -9)
    assert (np.abs(got8 * ys - want) <= step + 1e-7).all()


FP32_CASES = [
    # name, N, C, H, W, M, kH, kW, stride, pad, dil, group, bias
    ("3x3_pad1", 2, 8, 11, 9, 6, 3, 3, 1, 1, 1, 1, True),
    ("5x5_s2_dil", 1, 7, 17, 15, 5, 5, 3, 2, 2, 2, 1, False),   # C % 4 = 3: the lane tail
    ("grouped", 2, 12, 10, 10, 8, 3, 3, 1, 1, 1, 4, True),      # 3 channels per group: tail only
    ("grouped_wide", 1, 32, 9, 9, 16, 3, 3, 1, 0, 1, 2, True),  # 16 channels per group: four lanes
    ("depthwise", 2, 16, 13, 13, 16, 3, 3, 2, 1, 1, 16, True),
    ("1d", 3, 9, 1, 40, 7, 1, 5, 2, 2, 1, 1, True),              # a 1-D conv as H = 1
]


@pytest.mark.parametrize("name,N,C,H,W,M,kH,kW,stride,pad,dil,group,bias", FP32_CASES)
def test_conv2d_f32_matches_reference_order(dev, name, N, C, H, W, M, kH, kW, stride, pad, dil, group, bias):
    """The fp32 Conv (conv.cpp:115-207) bit for bit against the oracle in the
    reference's summation order (per tap, four lane sums over the group's
    channels), and within 1e-5 of the single fma chain."""
    import torch
    import luisaml_b200 as lb
    rng = np.random.default_rng(len(name) * 7 + C)
    X = rng.standard_normal((N, C, H, W)).astype(np.float32)
    Wt = rng.standard_normal((M, C // group, kH, kW)).astype(np.float32)
    b = rng.standard_normal(M).astype(np.float32) if bias else None
    sh = (stride, stride) if H > 1 else (1, stride)
    pd = (pad, pad, pad, pad) if H > 1 else (0, pad, 0, pad)
    dl = (dil, dil) if H > 1 else (1, dil)
    ref4 = oracle.conv2d(X, Wt, b, strides=sh, pads=pd, dilations=dl, group=group, lanes=4)
    ref1 = oracle.conv2d(X, Wt, b, strides=sh, pads=pd, dilations=dl, group=group)
    oH, oW = ref4.shape[2], ref4.shape[3]
    Y = torch.empty((N, M, oH, oW), dtype=torch.float32, device=dev)
    xt, wt = _t(X, dev), _t(Wt, dev)
    bt = _t(b, dev) if bias else None
    lb.check(lb.lib().lcml_conv2d_f32(ctypes.c_void_p(xt.data_ptr()), ctypes.c_void_p(wt.data_ptr()),
                                      ctypes.c_void_p(bt.data_ptr()) if bias else None, N, C, H, W, M, kH, kW, oH, oW,
                                      sh[0], sh[1], pd[0], pd[1], dl[0], dl[1], group, ctypes.c_void_p(Y.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    got = Y.cpu().numpy()
    np.testing.assert_array_equal(got, ref4)
    assert_close(got, ref1, rtol=1e-5, atol=1e-5, what=name)


@pytest.mark.parametrize("nhwc", [True, False])
@pytest.mark.parametrize("group,C,M", [(2, 32, 48), (64, 64, 64), (4, 24, 8)])
def test_grouped_fp8_conv(dev, nhwc, group, C, M):
    """Grouped and depthwise QDQ convs (group > 1) through lcml_fp8_conv: the
    direct kernel vs the oracle's grouped conv on the dequantized operands,
    with bias, e4m3 residual and Relu, fp32 and e4m3 outputs."""
    import torch
    import luisaml_b200 as lb
    rng = np.random.default_rng(group * 100 + C)
    N, H, k = 2, 14, 3
    X = rng.standard_normal((N, C, H, H)).astype(np.float32)
    Wt = (rng.standard_normal((M, C // group, k, k)) * 0.2).astype(np.float32)
    bias = (rng.standard_normal(M) * 0.01).astype(np.float32)
    R = rng.standard_normal((N, M, H, H)).astype(np.float32)
    sx = np.float32(oracle.scale_from_amax(oracle.amax(X)))
    xq = oracle.quantize(X, sx)
    sw = np.array([oracle.scale_from_amax(oracle.amax(Wt[m])) for m in range(M)], dtype=np.float32)
    wq = oracle.quantize(Wt, sw, axis=0)
    rs = np.float32(oracle.scale_from_amax(oracle.amax(R)))
    rq = oracle.quantize(R, rs)
    ref = oracle.conv2d(oracle.dequantize(xq, sx), oracle.dequantize(wq, sw, axis=0), bias, pads=(1, 1, 1, 1),
                        group=group)
    ref = np.maximum(ref + oracle.dequantize(rq, rs), 0.0)
    Kp = lb.lib().lcml_fp8_conv_packed_k(C // group, k, k)
    Wp = torch.empty((M, Kp), dtype=torch.uint8, device=dev)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    wqt = _t(wq, dev)
    lb.check(lb.lib().lcml_fp8_conv_pack_weight(ctypes.c_void_p(wqt.data_ptr()), M, C // group, k, k,
                                                ctypes.c_void_p(Wp.data_ptr()), st))
    xt = _t(np.ascontiguousarray(xq.transpose(0, 2, 3, 1)) if nhwc else xq, dev)
    sxt, swt, bt = _t(np.float32([sx]), dev), _t(sw, dev), _t(bias, dev)
    rt, rst = _t(np.ascontiguousarray(rq.transpose(0, 2, 3, 1)), dev), _t(np.float32([rs]), dev)
    ys = np.float32(oracle.scale_from_amax(np.abs(ref).max()))
    yst = _t(np.float32([ys]), dev)
    outs = {}
    for out, dt, code in (("f32", torch.float32, 1), ("e4m3", torch.uint8, 17)):
        Y = torch.empty((N, H, H, M), dtype=dt, device=dev)
        d = lb._capi.ConvDesc()
        d.N, d.C, d.H, d.W, d.M, d.kH, d.kW, d.oH, d.oW = N, C, H, H, M, k, k, H, H
        d.sH = d.sW = 1
        d.pH = d.pW = 1
        d.dH = d.dW = 1
        d.group = group
        d.X, d.x_nhwc, d.scale_x = xt.data_ptr(), int(nhwc), sxt.data_ptr()
        d.Wp, d.scale_w, d.scale_w_mode = Wp.data_ptr(), swt.data_ptr(), lb.SCALE_AXIS
        d.bias = bt.data_ptr()
        d.residual, d.residual_dtype, d.residual_scale = rt.data_ptr(), lb.DTYPE_E4M3, rst.data_ptr()
        d.epilogue = lb.EPI_RELU
        d.Y, d.y_dtype, d.y_scale = Y.data_ptr(), code, yst.data_ptr()
        assert lb.lib().lcml_fp8_conv_workspace_size(ctypes.byref(d)) == 0
        lb.check(lb.lib().lcml_fp8_conv(ctypes.byref(d), st))
        torch.cuda.synchronize()
        outs[out] = Y.cpu().numpy()
    got = outs["f32"].transpose(0, 3, 1, 2)
    assert_close(got, ref, what=f"grouped conv g={group}")
    # e4m3 output: the epilogue rule on the kernel's own fp32 value
    r = np.float32(1.0) / ys
    want = oracle.quantize((outs["f32"] * r).astype(np.float32), np.float32(1.0))
    np.testing.assert_array_equal(outs["e4m3"], want)


@pytest.mark.parametrize("stride,pad,dil,group,opad", [(2, 1, 1, 1, 1), (1, 0, 1, 2, 0), (3, 2, 2, 1, 2),
                                                       (2, 0, 1, 5, 0)])
def test_conv_transpose2d_f32(dev, stride, pad, dil, group, opad):
    """fp32 ConvTranspose (conv_transpose.cpp) bit for bit against the
    oracle's restatement of the reference's gather loop and lane order."""
    import torch
    import luisaml_b200 as lb
    rng = np.random.default_rng(stride * 31 + group)
    N, C, H, Wd, Mg, k = 2, 10, 7, 6, 3, 3
    X = rng.standard_normal((N, C, H, Wd)).astype(np.float32)
    Wt = rng.standard_normal((C, Mg, k, k)).astype(np.float32)
    b = rng.standard_normal(Mg * group).astype(np.float32)
    ref = oracle.conv_transpose2d(X, Wt, b, strides=(stride, stride), pads=(pad, pad, pad, pad),
                                  dilations=(dil, dil), group=group, output_padding=(opad, opad))
    M, oH, oW = ref.shape[1], ref.shape[2], ref.shape[3]
    Y = torch.empty((N, M, oH, oW), dtype=torch.float32, device=dev)
    xt, wt, bt = _t(X, dev), _t(Wt, dev), _t(b, dev)
    lb.check(lb.lib().lcml_conv_transpose2d_f32(ctypes.c_void_p(xt.data_ptr()), ctypes.c_void_p(wt.data_ptr()),
                                                ctypes.c_void_p(bt.data_ptr()), N, C, H, Wd, M, k, k, oH, oW, stride,
                                                stride, pad, pad, dil, dil, group, ctypes.c_void_p(Y.data_ptr()),
                                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    np.testing.assert_array_equal(Y.cpu().numpy(), ref)
