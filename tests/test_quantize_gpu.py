"""QuantizeLinear / DequantizeLinear kernels vs the reference codec, bit-exact.

Every check goes through the C ABI (lcml_fp8_quantize & co.). Expected bytes
come from the golden vectors (the reference's own codec) or the CPU oracle,
which test_oracle_golden.py pins to those vectors.
"""
import numpy as np
import pytest

import oracle
from conftest import golden

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _one(dev, v=1.0):
    import torch
    return torch.tensor([v], dtype=torch.float32, device=dev)


@pytest.mark.parametrize("fixture", ["e4m3_encode_structured.npz", "e4m3_encode_random.npz"])
def test_encoder_matches_reference_bytes(dev, fixture):
    import luisaml_b200 as lb
    g = golden(fixture)
    q = lb.quantize(_t(g["x"], dev), _one(dev)).cpu().numpy()  # x / 1 is exact
    bad = np.nonzero(q != g["q"])[0]
    assert bad.size == 0, f"{bad.size} mismatches; first x={g['x'][bad[0]]!r} got {q[bad[0]]:#x} want {g['q'][bad[0]]:#x}"


def test_quantize_tensor_golden(dev):
    import luisaml_b200 as lb
    g = golden("e4m3_quantize_tensor.npz")
    q = lb.quantize(_t(g["x"], dev), _one(dev, float(g["scale"]))).cpu().numpy()
    assert np.array_equal(q, g["q"])


@pytest.mark.parametrize("scale", [1.0, 0.0123, 6.1e-3, 4.0])
def test_encoder_exhaustive_all_fp32_patterns(dev, scale):
    """Every one of the 2^32 fp32 bit patterns, GPU kernel vs CPU oracle; with
    scale 1 this checks the encoder itself, with the other scales the
    multiply-by-reciprocal fast path (RN(1/s) inexact) over every input, and
    with scale 4 quotients of tiny inputs that round to (signed) zero."""
    import torch
    import luisaml_b200 as lb
    one = _one(dev, scale)
    chunk = 1 << 28
    for c in range(1 << 4):
        bits = torch.arange(c * chunk, (c + 1) * chunk, dtype=torch.int64, device=dev)
        x = bits.to(torch.int32).view(torch.float32)  # wraps to the full uint32 range
        q = lb.quantize(x.contiguous(), one).cpu().numpy()
        xc = x.cpu().numpy()
        ref = oracle.quantize(xc, np.float32(scale))
        bad = np.nonzero(q != ref)[0]
        assert bad.size == 0, f"chunk {c}: {bad.size} mismatches, first bits {xc[bad[0]:bad[0]+1].view(np.uint32)}"


@pytest.mark.parametrize("shape,axis", [((64, 48), 0), ((64, 48), 1), ((5, 32, 7), 1), ((3, 16, 16), 2),
                                        ((4, 7, 33), 1), ((1000,), 0), ((13, 17), 1)])
def test_per_axis(dev, shape, axis):
    import luisaml_b200 as lb
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(shape) * 10).astype(np.float32)
    s = (rng.random(shape[axis]) * 0.05 + 0.001).astype(np.float32)
    q = lb.quantize(_t(x, dev), _t(s, dev), axis=axis).cpu().numpy()
    assert np.array_equal(q, oracle.quantize(x, s, axis=axis))


@pytest.mark.parametrize("n", [0, 1, 15, 16, 17, 4099, 1 << 20])
def test_per_tensor_ragged_sizes(dev, n):
    import luisaml_b200 as lb
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32) * 3
    s = np.float32(0.0123)
    q = lb.quantize(_t(x, dev), _one(dev, float(s))).cpu().numpy()
    assert np.array_equal(q, oracle.quantize(x, s))


def test_unaligned_input(dev):
    import luisaml_b200 as lb
    rng = np.random.default_rng(5)
    x = rng.standard_normal(1001).astype(np.float32)
    xt = _t(x, dev)[1:]  # 4-byte offset: scalar path
    q = lb.quantize(xt, _one(dev, 0.01)).cpu().numpy()
    assert np.array_equal(q, oracle.quantize(x[1:], np.float32(0.01)))


@pytest.mark.parametrize("rows,cols", [(1, 4096), (7, 4096), (64, 11008), (3, 12), (5, 13), (2, 20000), (16, 1)])
def test_dynamic_rows(dev, rows, cols):
    import luisaml_b200 as lb
    rng = np.random.default_rng(rows * 7 + cols)
    x = (rng.standard_normal((rows, cols)) * rng.random((rows, 1)) * 50).astype(np.float32)
    if rows > 2:
        x[1] = 0.0
        x[2, 0] = np.nan
    q, s = lb.quantize_rows_dynamic(_t(x, dev))
    qr, sr = oracle.quantize_dynamic_rows(x)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), sr.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), qr)


def test_dynamic_tensor_and_amax(dev):
    import luisaml_b200 as lb
    rng = np.random.default_rng(21)
    x = (rng.standard_normal(3 * 1000 + 5) * 7).astype(np.float32)
    x[10] = np.nan
    a = lb.amax(_t(x, dev)).cpu().numpy()[0]
    assert a == oracle.amax(x)
    q, s = lb.quantize_tensor_dynamic(_t(x, dev))
    sr = oracle.scale_from_amax(oracle.amax(x))
    assert s.cpu().numpy()[0] == sr
    assert np.array_equal(q.cpu().numpy(), oracle.quantize(x, sr))


def test_quantize_from_amax(dev):
    import torch
    import luisaml_b200 as lb
    rng = np.random.default_rng(8)
    x = rng.standard_normal((40, 96)).astype(np.float32)
    am = np.abs(x).max(axis=1).astype(np.float32)
    am[3] = 0.0
    so = torch.empty(40, dtype=torch.float32, device=dev)
    q = lb.quantize_from_amax(_t(x, dev), _t(am, dev), axis=0, scale_out=so).cpu().numpy()
    sr = np.array([oracle.scale_from_amax(a) for a in am], dtype=np.float32)
    assert np.array_equal(so.cpu().numpy(), sr)
    assert np.array_equal(q, oracle.quantize(x, sr, axis=0))


@pytest.mark.parametrize("axis", [None, 0, 1])
def test_dequantize(dev, axis):
    import torch
    import luisaml_b200 as lb
    q = np.arange(256 * 6, dtype=np.uint32).astype(np.uint8).reshape(48, 32)
    s = np.float32([0.37]) if axis is None else (np.arange(q.shape[axis], dtype=np.float32) * 0.01 + 0.02)
    y = lb.dequantize(_t(q, dev), _t(s, dev), axis=axis).cpu().numpy()
    ref = oracle.dequantize(q, s if axis is not None else s[0], axis=axis)
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    m = ~np.isnan(ref)
    assert np.array_equal(y[m].view(np.uint32), ref[m].view(np.uint32))
    yb = lb.dequantize(_t(q, dev), _t(s, dev), axis=axis, dtype=torch.bfloat16).float().cpu().numpy()
    assert np.array_equal(yb[m], torch.from_numpy(ref[m]).bfloat16().float().numpy())


def test_transpose(dev):
    import luisaml_b200 as lb
    rng = np.random.default_rng(2)
    a = rng.integers(0, 256, size=(130, 77), dtype=np.uint8)
    t = lb.transpose_u8(_t(a, dev)).cpu().numpy()
    assert np.array_equal(t, a.T)


def test_invalid_arguments_are_reported(dev):
    import ctypes
    import luisaml_b200 as lb
    rc = lb.lib().lcml_fp8_quantize(None, 1, 1, 16, None, 0, None, None)
    assert rc == 1 and b"null" in lb.lib().lcml_last_error()
    rc = lb.lib().lcml_fp8_quantize(None, 1, 1, 16, None, 7, None, None)
    assert rc == 1
    assert lb.device_error() == 0
    del ctypes


@pytest.mark.parametrize("scale", [0.0123, 1.0 / 3.0, 0.7071068, 3.3e-5, 1.7e-39, 2.5e38, 1e-30])
def test_fast_reciprocal_path_is_exact(dev, scale):
    """The vector kernel multiplies by RN(1/s) and re-does near-tie elements
    with an IEEE divide; the bytes must equal e4m3(x / s) exactly, including
    for scales whose reciprocal is not usable (subnormal / huge)."""
    import luisaml_b200 as lb
    rng = np.random.default_rng(int(scale * 1e6) % 1000 + 1)
    n = 1 << 24
    x = (rng.standard_normal(n) * rng.choice([1e-3, 1.0, 30.0, 1e4], size=n)).astype(np.float32)
    s = np.float32(scale)
    # plant exact ties: x = (midpoint between e4m3 neighbours) * s rounded either way
    mids = ((oracle.e4m3_decode(np.arange(1, 126, dtype=np.uint8)).astype(np.float64) +
             oracle.e4m3_decode(np.arange(2, 127, dtype=np.uint8)).astype(np.float64)) / 2)
    t = (mids * float(s)).astype(np.float32)
    x[:t.size] = t
    x[t.size:2 * t.size] = np.nextafter(t, np.float32(np.inf))
    x[2 * t.size:3 * t.size] = np.nextafter(t, np.float32(0))
    q = lb.quantize(_t(x, dev), _one(dev, float(s))).cpu().numpy()
    ref = oracle.quantize(x, s)
    bad = np.nonzero(q != ref)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x={x[bad[0]]!r} got {q[bad[0]]:#x} want {ref[bad[0]]:#x}"
