"""Pins the CPU oracle (oracle/oracle.c) against the reference's own codec.

The golden vectors in tests/golden/ were produced by the reference's compiled
CPU codec (FP8E4M3FN::from_float / to_float, include/onnx/fp_quantized.h:149-249).
Where the reference tree is present (oracle/_ref built), the restatement is
also compared with it on all 2^32 fp32 bit patterns.
"""
import concurrent.futures as cf
import ctypes

import numpy as np
import pytest

import oracle
from conftest import golden


def test_decode_all_256_codes():
    g = golden("e4m3_decode.npz")
    got = oracle.e4m3_decode(g["codes"])
    ref = g["values"]
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))  # -0.0 included
    assert nan.sum() == 2 and nan[0x7f] and nan[0xff]


@pytest.mark.parametrize("fixture", ["e4m3_encode_structured.npz", "e4m3_encode_random.npz"])
def test_encode_matches_reference_bytes(fixture):
    g = golden(fixture)
    got = oracle.e4m3_encode(g["x"])
    bad = np.nonzero(got != g["q"])[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x={g['x'][bad[0]]!r}"


def test_encode_edge_semantics():
    # the reference's documented quirks (fp_quantized.h:151-171, :213-216)
    e = oracle.e4m3_encode
    assert e(np.float32([-0.0]))[0] == 0x00
    assert e(np.float32([np.nan]))[0] == 0x7f
    assert e(np.float32([-np.nan]))[0] == 0x7f
    assert e(np.float32([np.inf]))[0] == 0x7e and e(np.float32([-np.inf]))[0] == 0xfe
    assert e(np.float32([464.0]))[0] == 0x7e and e(np.float32([1e9]))[0] == 0x7e
    assert e(np.float32([-2.0 ** -10]))[0] == 0x80  # rounds to zero, keeps the sign
    assert e(np.float32([2.0 ** -9]))[0] == 0x01


def test_quantize_tensor_fixture():
    g = golden("e4m3_quantize_tensor.npz")
    got = oracle.quantize(g["x"], g["scale"])
    assert np.array_equal(got, g["q"])
    # the fixture's scale is amax / 448 in fp32
    assert np.float32(np.max(np.abs(g["x"])) / np.float32(448.0)) == g["scale"]


def test_dynamic_rows_matches_per_row_quantize():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((33, 70)).astype(np.float32)
    x[3] = 0.0
    q, s = oracle.quantize_dynamic_rows(x)
    assert s[3] == 1.0
    for r in range(x.shape[0]):
        assert s[r] == oracle.scale_from_amax(np.max(np.abs(x[r])))
        assert np.array_equal(q[r], oracle.quantize(x[r], s[r]))


def test_gemm_matches_float64_reference():
    rng = np.random.default_rng(3)
    A = rng.standard_normal((17, 40)).astype(np.float32)
    B = rng.standard_normal((29, 40)).astype(np.float32)
    C = rng.standard_normal(29).astype(np.float32)
    Y = oracle.gemm(A, B, C, alpha=0.5, beta=2.0, transB=1)
    ref = 0.5 * (A.astype(np.float64) @ B.T.astype(np.float64)) + 2.0 * C
    np.testing.assert_allclose(Y, ref, rtol=1e-5, atol=1e-5)


def test_conv_matches_direct_float64():
    rng = np.random.default_rng(4)
    X = rng.standard_normal((2, 4, 9, 7)).astype(np.float32)
    W = rng.standard_normal((6, 2, 3, 3)).astype(np.float32)
    b = rng.standard_normal(6).astype(np.float32)
    Y = oracle.conv2d(X, W, b, strides=(2, 1), pads=(1, 1, 1, 1), group=2)
    N, C, H, Wd = X.shape
    ref = np.zeros(Y.shape)
    Xp = np.pad(X.astype(np.float64), ((0, 0), (0, 0), (1, 1), (1, 1)))
    for n in range(N):
        for m in range(6):
            g = m // 3
            for oh in range(Y.shape[2]):
                for ow in range(Y.shape[3]):
                    patch = Xp[n, g * 2:(g + 1) * 2, oh * 2:oh * 2 + 3, ow:ow + 3]
                    ref[n, m, oh, ow] = (patch * W[m]).sum() + b[m]
    np.testing.assert_allclose(Y, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m1"])
def test_exhaustive_against_reference_codec(fmt):
    """All 2^32 fp32 bit patterns: restatement == reference codec (needs oracle/_ref)."""
    r = oracle.ref_lib()
    if r is None:
        pytest.skip("oracle/_ref not built (reference tree absent): golden vectors pin the oracle instead")
    cand = ctypes.cast(getattr(oracle.lib, f"orc_{fmt}_from_float"), ctypes.c_void_p).value
    count = getattr(r, f"lcml_ref_{fmt}_count_mismatch")
    parts = 64
    span = (1 << 32) // parts

    def run(i):
        fb = ctypes.c_uint32(0)
        bad = count(cand, i * span, (i + 1) * span, ctypes.byref(fb))
        return bad, fb.value

    with cf.ThreadPoolExecutor(8) as ex:
        res = list(ex.map(run, range(parts)))
    bad = sum(b for b, _ in res)
    assert bad == 0, f"{bad} mismatches, first at bits {[hex(f) for b, f in res if b][:3]}"


@pytest.mark.parametrize("fmt", ["e5m2", "e2m1"])
def test_minifloat_codecs_match_reference_fixture(fmt):
    """FP8 E5M2 / FP4 E2M1 (fp_quantized.h:259-378, :20-115): the decode
    table and the encodes of the reference's own codec (golden fixture)."""
    g = golden(f"{fmt}_codec.npz")
    dec = getattr(oracle.lib, f"orc_{fmt}_to_float")
    got = np.array([dec(int(c)) for c in g["codes"]], dtype=np.float32)
    ref = g["values"]
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    enc = oracle.e5m2_encode if fmt == "e5m2" else oracle.e2m1_encode
    q = enc(g["x"])
    bad = np.nonzero(q != g["q"])[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x={g['x'][bad[0]]!r}"


def test_minifloat_edge_semantics():
    e5, e2 = oracle.e5m2_encode, oracle.e2m1_encode
    assert e5(np.float32([57344.0]))[0] == 0x7b and e5(np.float32([57345.0]))[0] == 0x7c  # no saturation
    assert e5(np.float32([-np.inf]))[0] == 0xfc and e5(np.float32([np.nan]))[0] == 0x7f
    assert e5(np.float32([-1e-30]))[0] == 0x80 and e5(np.float32([2.0 ** -17]))[0] == 0x00  # tie -> even (0)
    assert e2(np.float32([7.0]))[0] == 0x7 and e2(np.float32([-np.inf]))[0] == 0xf  # saturates
    assert e2(np.float32([5.0]))[0] == 0x6 and e2(np.float32([0.25]))[0] == 0x0  # ties to even
    assert e2(np.float32([-1e-30]))[0] == 0x8 and e2(np.float32([np.nan]))[0] == 0x0


def _half_then(x):
    """fp32 values rounded to half (numpy's IEEE round-to-nearest-even), as fp32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def test_cast_restatement():
    """Cast (cast.cpp:44-72): to FP8 / FP4 through half, from FP8 / FP4
    exact; checked against numpy's half rounding and the codecs directly."""
    rng = np.random.default_rng(11)
    x = np.concatenate([rng.standard_normal(4000).astype(np.float32) * 10,
                        golden("e4m3_encode_structured.npz")["x"]]).astype(np.float32)
    xh = _half_then(x)
    assert np.array_equal(oracle.cast(x, 1, 17), oracle.e4m3_encode(xh))
    assert np.array_equal(oracle.cast(x, 1, 19), oracle.e5m2_encode(xh))
    packed = oracle.cast(x, 1, 23)
    codes = np.stack([packed & 0xf, packed >> 4], axis=1).ravel()[:x.size]
    assert np.array_equal(codes, oracle.e2m1_encode(xh))
    # the double rounding is visible: fp32 -> e4m3 directly differs for some values
    assert (oracle.cast(x, 1, 17) != oracle.e4m3_encode(x)).any()
    # fp32 -> half / bf16 round to nearest even; FP8 -> fp32 exact
    h = oracle.cast(x, 1, 10)
    nan = np.isnan(x)
    assert np.array_equal(np.isnan(h), nan)  # NaN payloads are not specified
    with np.errstate(over="ignore"):  # values past 65504 become inf, as the cast does
        assert np.array_equal(h[~nan].view(np.uint16), x[~nan].astype(np.float16).view(np.uint16))
    codes8 = np.arange(256, dtype=np.uint8)
    assert np.array_equal(oracle.cast(codes8, 17, 1), oracle.e4m3_decode(codes8), equal_nan=True)
    # FP4 odd length: the last byte's high nibble stays zero
    assert oracle.cast(np.float32([1.0, 2.0, 3.0]), 1, 23).tolist() == [0x2 | (0x4 << 4), 0x5]


def test_mlp_fixture_both_reference_summation_orders():
    """The reference's fp32 MLP fixture (tests/onnx/output/) through the
    oracle with both of the reference Gemm's summation orders: the scalar
    K-ordered fma chain (gemm.cpp:153-157) and the four-lane order of its
    vector path for byte-buffer operands (gemm.cpp:123-152). Both reproduce
    output_ref.bin within the reference test's tolerance (abs 1e-3,
    test_onnx_inference.cpp:232); they differ from each other only in fp32
    rounding."""
    import json
    import os
    from conftest import GOLDEN
    d = os.path.join(GOLDEN, "simple_mlp")
    blob = np.fromfile(os.path.join(d, "simple_mlp.safetensors"), dtype=np.uint8)
    x = np.fromfile(os.path.join(d, "input_ref.bin"), dtype=np.float32).reshape(1, 784)
    ref = np.fromfile(os.path.join(d, "output_ref.bin"), dtype=np.float32).reshape(1, 10)
    inits = {i["name"]: i for i in json.load(open(os.path.join(d, "simple_mlp.onnx.json")))["graph"]["initializer"]}
    W = {k: np.frombuffer(blob[v["data_offsets"][0]:v["data_offsets"][1]].tobytes(), dtype=np.float32).reshape(
        [int(s) for s in v["dims"]]) for k, v in inits.items()}
    outs = []
    for lanes in (1, 4):
        h = oracle.relu(oracle.gemm(x, W["net.0.weight"], W["net.0.bias"], transB=1, lanes=lanes))
        h = oracle.relu(oracle.gemm(h, W["net.2.weight"], W["net.2.bias"], transB=1, lanes=lanes))
        h = oracle.gemm(h, W["net.4.weight"], W["net.4.bias"], transB=1, lanes=lanes)
        assert np.abs(h - ref).max() <= 1e-3
        outs.append(h)
    np.testing.assert_allclose(outs[0], outs[1], rtol=1e-5, atol=1e-6)
    # and the four-lane order is a different order: it is not the scalar chain everywhere
    rng = np.random.default_rng(0)
    A, B = rng.standard_normal((16, 301)).astype(np.float32), rng.standard_normal((16, 301)).astype(np.float32)
    assert not np.array_equal(oracle.gemm(A, B, transB=1, lanes=1), oracle.gemm(A, B, transB=1, lanes=4))


def test_conv_transpose_matches_scatter_definition():
    """The gather restatement of ConvTranspose (conv_transpose.cpp) equals
    the scatter definition y[oh = ih*s - p + kh*d] += x * w in float64."""
    rng = np.random.default_rng(21)
    X = rng.standard_normal((2, 6, 5, 4)).astype(np.float32)
    W = rng.standard_normal((6, 2, 3, 2)).astype(np.float32)  # [C, M/group, kH, kW], group 3 -> M = 6
    b = rng.standard_normal(6).astype(np.float32)
    s, p, d, op = (2, 3), (1, 0, 1, 0), (1, 2), (1, 0)
    Y = oracle.conv_transpose2d(X, W, b, strides=s, pads=p, dilations=d, group=3, output_padding=op)
    N, C, H, Wd = X.shape
    oH, oW = Y.shape[2], Y.shape[3]
    ref = np.zeros((N, 6, oH, oW))
    for n in range(N):
        for c in range(C):
            g = c // 2
            for mg in range(2):
                for ih in range(H):
                    for iw in range(Wd):
                        for kh in range(3):
                            for kw in range(2):
                                oh, ow = ih * s[0] - p[0] + kh * d[0], iw * s[1] - p[1] + kw * d[1]
                                if 0 <= oh < oH and 0 <= ow < oW:
                                    ref[n, g * 2 + mg, oh, ow] += float(X[n, c, ih, iw]) * float(W[c, mg, kh, kw])
    ref += b.reshape(1, 6, 1, 1)
    np.testing.assert_allclose(Y, ref, rtol=1e-5, atol=1e-5)


def test_conv_lane_order_matches_float64():
    rng = np.random.default_rng(22)
    X = rng.standard_normal((1, 10, 7, 7)).astype(np.float32)
    W = rng.standard_normal((3, 10, 3, 3)).astype(np.float32)
    Y = oracle.conv2d(X, W, pads=(1, 1, 1, 1), lanes=4)
    ref = oracle.conv2d(X.astype(np.float32), W, pads=(1, 1, 1, 1))
    np.testing.assert_allclose(Y, ref, rtol=1e-5, atol=1e-5)
    assert not np.array_equal(Y, ref)  # a different summation order
