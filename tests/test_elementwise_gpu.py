"""Memory-bound operators around the GEMMs vs the CPU oracle (through the C ABI)."""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import assert_close

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _s():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("op", [0, 1, 2])
@pytest.mark.parametrize("n", [1, 7, 1 << 16, (1 << 20) + 3])
def test_unary(dev, op, n):
    import torch
    import luisaml_b200 as lb
    x = (np.random.default_rng(n + op).standard_normal(n) * 5).astype(np.float32)
    xt = _t(x, dev)
    y = torch.empty_like(xt)
    lb.check(lb.lib().lcml_unary_f32(op, _p(xt), _p(y), n, _s()))
    got = y.cpu().numpy()
    if op == 0:
        assert np.array_equal(got, oracle.relu(x))
    elif op == 1:
        assert_close(got, oracle.sigmoid(x), rtol=1e-6, atol=1e-7, what="sigmoid")
    else:
        assert np.array_equal(got, np.abs(x))


@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("shape,bshape", [((64, 48), (48,)), ((1000,), (1,)), ((7, 13), (7, 13)), ((5, 6, 8), (8,))])
def test_binary_broadcast(dev, op, shape, bshape):
    import torch
    import luisaml_b200 as lb
    rng = np.random.default_rng(op)
    a = rng.standard_normal(shape).astype(np.float32)
    b = (rng.standard_normal(bshape) + 3.0).astype(np.float32)
    at, bt = _t(a, dev), _t(b, dev)
    y = torch.empty_like(at)
    lb.check(lb.lib().lcml_binary_f32(op, _p(at), _p(bt), a.size, b.size, _p(y), _s()))
    ref = [a + b, a - b, a * b, a / b][op].astype(np.float32)
    assert np.array_equal(y.cpu().numpy(), ref)


def test_reduce_max_and_softmax(dev):
    import torch
    import luisaml_b200 as lb
    x = np.random.default_rng(1).standard_normal((37, 1000)).astype(np.float32) * 4
    xt = _t(x, dev)
    m = torch.empty(37, dtype=torch.float32, device=dev)
    lb.check(lb.lib().lcml_reduce_max_rows(_p(xt), 37, 1000, 1, _p(m), _s()))
    assert np.array_equal(m.cpu().numpy(), np.abs(x).max(axis=1))
    y = torch.empty_like(xt)
    lb.check(lb.lib().lcml_softmax_rows(_p(xt), 37, 1000, _p(y), _s()))
    assert_close(y.cpu().numpy(), oracle.softmax_rows(x), rtol=1e-5, atol=1e-7, what="softmax")


@pytest.mark.parametrize("nhwc", [0, 1])
def test_maxpool_resnet_stem(dev, nhwc):
    import torch
    import luisaml_b200 as lb
    x = np.random.default_rng(2).standard_normal((2, 8, 112, 112)).astype(np.float32)
    ref = oracle.maxpool2d(x, (3, 3), (2, 2), (1, 1, 1, 1))
    xin = np.ascontiguousarray(x.transpose(0, 2, 3, 1)) if nhwc else x
    xt = _t(xin, dev)
    y = torch.empty(ref.size, dtype=torch.float32, device=dev)
    lb.check(lb.lib().lcml_maxpool2d(_p(xt), 1, 16, 112, 112, 3, 3, 2, 2, 1, 1, 56, 56, _p(y), nhwc, 8, _s()))
    got = y.cpu().numpy().reshape((2, 56, 56, 8) if nhwc else ref.shape)
    if nhwc:
        got = got.transpose(0, 3, 1, 2)
    assert np.array_equal(got, ref)


def test_maxpool_e4m3_and_gap(dev):
    import torch
    import luisaml_b200 as lb
    x = np.random.default_rng(3).standard_normal((2, 4, 14, 14)).astype(np.float32)
    q = oracle.quantize(x, np.float32(0.02))
    xd = oracle.dequantize(q, np.float32(0.02))
    ref_pool = oracle.maxpool2d(xd, (3, 3), (2, 2), (1, 1, 1, 1))
    qt = _t(q, dev)
    y = torch.empty(ref_pool.size, dtype=torch.uint8, device=dev)
    lb.check(lb.lib().lcml_maxpool2d(_p(qt), 17, 8, 14, 14, 3, 3, 2, 2, 1, 1, 7, 7, _p(y), 0, 4, _s()))
    got = oracle.dequantize(y.cpu().numpy(), np.float32(0.02)).reshape(ref_pool.shape)
    assert np.array_equal(got, ref_pool)
    sc = _t(np.float32([0.02]), dev)
    g = torch.empty(8, dtype=torch.float32, device=dev)
    lb.check(lb.lib().lcml_global_avgpool(_p(qt), 17, _p(sc), 2, 4, 196, 0, _p(g), _s()))
    assert_close(g.cpu().numpy(), oracle.global_avgpool(xd).reshape(-1), rtol=1e-5, atol=1e-6, what="gap e4m3")
    xt = _t(x, dev)
    lb.check(lb.lib().lcml_global_avgpool(_p(xt), 1, None, 2, 4, 196, 0, _p(g), _s()))
    assert_close(g.cpu().numpy(), oracle.global_avgpool(x).reshape(-1), rtol=1e-5, atol=1e-6, what="gap f32")


def test_cast_roundtrip(dev):
    import torch
    import luisaml_b200 as lb
    x = np.random.default_rng(4).standard_normal(1003).astype(np.float32)
    xt = _t(x, dev)
    b = torch.empty(1003, dtype=torch.bfloat16, device=dev)
    lb.check(lb.lib().lcml_cast(_p(xt), 1, _p(b), 16, 1003, _s()))
    assert torch.equal(b, xt.bfloat16())
    f = torch.empty_like(xt)
    lb.check(lb.lib().lcml_cast(_p(b), 16, _p(f), 1, 1003, _s()))
    assert torch.equal(f, b.float())


@pytest.mark.parametrize("C,HW", [(8, 49), (64, 5), (6, 49), (12, 17), (8, 100)])
@pytest.mark.parametrize("dtype", [1, 16, 17])
def test_gap_nhwc(dev, dtype, C, HW):
    """NHWC GlobalAveragePool (the ResNet head's layout) vs the oracle's
    per-channel sequential sum: C % 4 == 0 takes the four-channel vector
    kernel (e4m3 with HW <= 64: all pixels loaded up front; otherwise 8
    pixels per unrolled step plus a tail), the others one channel per
    thread. fp32 and bf16 inputs sum in the oracle's order: bit-exact;
    e4m3 sums the codes' values before the scale (rtol 1e-5 / atol 1e-6, as
    the NCHW test)."""
    import torch
    import luisaml_b200 as lb
    N = 3
    rng = np.random.default_rng(C * 100 + HW)
    x = rng.standard_normal((N, HW, C)).astype(np.float32)
    if dtype == 1:
        xt, xd, sc = _t(x, dev), x, None
    elif dtype == 16:
        xt = _t(x, dev).bfloat16()
        xd, sc = xt.float().cpu().numpy(), None
    else:
        s = np.float32(0.02)
        q = oracle.quantize(x, s)
        xt, xd, sc = _t(q, dev), oracle.dequantize(q, s), _t(np.float32([s]), dev)
    want = oracle.global_avgpool(np.ascontiguousarray(xd.transpose(0, 2, 1)).reshape(N, C, HW, 1)).reshape(N, C)
    g = torch.empty(N * C, dtype=torch.float32, device=dev)
    lb.check(lb.lib().lcml_global_avgpool(_p(xt), dtype, _p(sc) if sc is not None else None, N, C, HW, 1, _p(g),
                                          _s()))
    got = g.cpu().numpy().reshape(N, C)
    if dtype == 17:
        assert_close(got, want, rtol=1e-5, atol=1e-6, what="gap nhwc e4m3")
    else:
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("layout,C,k,s,p", [("nhwc", 64, 3, 2, 1), ("nhwc", 8, 3, 2, 1), ("nchw", 64, 3, 2, 1),
                                             ("nhwc", 32, 2, 2, 0), ("nhwc", 16, 3, 1, 1)])
def test_maxpool_e4m3_qdq_semantics(dev, layout, C, k, s, p):
    """e4m3 MaxPool equals DequantizeLinear -> MaxPool -> QuantizeLinear at the
    same scale: -0 comes out as 0x00, NaN taps are ignored and an all-NaN
    window gives the saturated -inf code 0xfe. NHWC with C % 16 == 0 takes the
    16-byte vector kernel (3x3 windows unrolled at compile time, others read
    at run time), the others the scalar one."""
    import torch
    import luisaml_b200 as lb
    rng = np.random.default_rng(C)
    N, H, W = 2, 23, 30
    q = rng.integers(0, 256, size=(N, C, H, W), dtype=np.uint8)
    q[rng.random(q.shape) < 0.05] = 0x80
    q[:, :, 4:7, 4:7] = 0x7f   # the window centred at (5, 5) is all NaN
    q[:, :, 10, :] = 0xff
    oH, oW = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    want = oracle.quantize(oracle.maxpool2d(oracle.e4m3_decode(q).astype(np.float32), (k, k), (s, s), (p, p, p, p)),
                           np.float32(1.0))
    nhwc = layout == "nhwc"
    qin = np.ascontiguousarray(q.transpose(0, 2, 3, 1)) if nhwc else q
    y = torch.empty(N * C * oH * oW, dtype=torch.uint8, device=dev)
    lb.check(lb.lib().lcml_maxpool2d(_p(_t(qin, dev)), 17, N * C, H, W, k, k, s, s, p, p, oH, oW, _p(y), int(nhwc), C,
                                     _s()))
    got = y.cpu().numpy().reshape((N, oH, oW, C) if nhwc else (N, C, oH, oW))
    if nhwc:
        got = got.transpose(0, 3, 1, 2)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("dtype", [17, 19])
@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_binary_fp8_typed(dev, dtype, op):
    """Add/Sub/Mul/Div on FP8-typed tensors (binary.cpp:185-283): every pair
    of codes (256 x 256, decode -> half op -> encode) bit-exact against the
    oracle, and a row broadcast."""
    import ctypes
    import torch
    import luisaml_b200 as lb
    codes = np.arange(256, dtype=np.uint8)
    a = np.repeat(codes, 256)
    b = np.tile(codes, 256)
    want = oracle.binary_fp8(op, a, b, dtype)
    at, bt = _t(a, dev), _t(b, dev)
    y = torch.empty(a.size, dtype=torch.uint8, device=dev)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lb.check(lb.lib().lcml_binary_fp8(op, ctypes.c_void_p(at.data_ptr()), ctypes.c_void_p(bt.data_ptr()), a.size,
                                      b.size, ctypes.c_void_p(y.data_ptr()), dtype, st))
    np.testing.assert_array_equal(y.cpu().numpy(), want)
    row = np.arange(0, 256, 3, dtype=np.uint8)  # broadcast of one row over 256 rows
    a2 = np.random.default_rng(op).integers(0, 256, size=(256, row.size), dtype=np.uint8)
    want2 = oracle.binary_fp8(op, a2, row, dtype)
    a2t, rt = _t(a2, dev), _t(row, dev)
    y2 = torch.empty(a2.shape, dtype=torch.uint8, device=dev)
    lb.check(lb.lib().lcml_binary_fp8(op, ctypes.c_void_p(a2t.data_ptr()), ctypes.c_void_p(rt.data_ptr()), a2.size,
                                      row.size, ctypes.c_void_p(y2.data_ptr()), dtype, st))
    np.testing.assert_array_equal(y2.cpu().numpy(), want2)


@pytest.mark.parametrize("dtype", [17, 19])
def test_softmax_fp8_typed(dev, dtype):
    """Softmax of an FP8-typed tensor (softmax.cpp:245-280): decode, softmax,
    encode of the half-rounded result; codes equal to the oracle's fp32
    softmax of the decoded values except flips to the neighbouring code
    (exp differs in its last bits between implementations)."""
    import ctypes
    import torch
    import luisaml_b200 as lb
    rng = np.random.default_rng(dtype)
    x = (rng.standard_normal((64, 200)) * 3).astype(np.float32)
    if dtype == 17:
        xq, dec, enc = oracle.e4m3_encode(x), oracle.e4m3_decode, oracle.e4m3_encode
    else:
        xq = oracle.e5m2_encode(x)
        dec = lambda q: oracle.cast(q, 19, 1).reshape(q.shape)  # noqa: E731
        enc = oracle.e5m2_encode
    ref = oracle.softmax_rows(dec(xq)).astype(np.float16).astype(np.float32)
    want = enc(ref)
    xt = _t(xq, dev)
    y = torch.empty(xq.shape, dtype=torch.uint8, device=dev)
    lb.check(lb.lib().lcml_softmax_rows_fp8(ctypes.c_void_p(xt.data_ptr()), 64, 200, ctypes.c_void_p(y.data_ptr()),
                                            dtype, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    got = y.cpu().numpy()
    g, w = dec(got).astype(np.float64), dec(want).astype(np.float64)
    step = np.maximum(np.abs(w) * (0.125 if dtype == 17 else 0.25), 2.0 ** (-9 if dtype == 17 else -16))
    assert (np.abs(g - w) <= step + 1e-12).all()
    assert (got == want).mean() > 0.99
