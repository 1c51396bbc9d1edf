"""Cast (src/onnx/operators/cast.cpp:10-162) on the GPU vs the oracle's
restatement, bit for bit, between fp32, fp16, bf16, FP8 E4M3FN, FP8 E5M2 and
packed FP4 E2M1.

To FP8 / FP4 the reference rounds the value to half first (cast.cpp:63-67),
so every half bit pattern (all 65536) through each encoder covers the whole
input domain of those casts; fp32 and bf16 sources add the double rounding.
From FP8 / FP4 every code is cast to every other type. Odd lengths and
misaligned pointers take the kernel's scalar paths and the FP4 tail.
"""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

F32, F16, BF16, E4M3, E5M2, E2M1 = 1, 10, 16, 17, 19, 23
ALL = [F32, F16, BF16, E4M3, E5M2, E2M1]
STORAGE = {F32: np.float32, F16: np.uint16, BF16: np.uint16, E4M3: np.uint8, E5M2: np.uint8, E2M1: np.uint8}


def _nbytes(t, n):
    return (n + 1) // 2 if t == E2M1 else n * np.dtype(STORAGE[t]).itemsize


def _esize(t):
    """Bytes of one element's storage unit (a packed FP4 byte for E2M1)."""
    return 1 if t == E2M1 else np.dtype(STORAGE[t]).itemsize


def _gpu_cast(dev, x_bytes, src, dst, n, offset=0):
    """Runs lcml_cast on n elements of the raw storage x_bytes; x and y start
    `offset` elements (bytes for packed FP4) into their device buffers, which
    keeps each pointer aligned to its element but breaks the kernel's vector
    alignment for offset > 0."""
    import torch
    import luisaml_b200 as lb
    xo, yo = offset * _esize(src), offset * _esize(dst)
    xin = torch.zeros(len(x_bytes) + xo + 64, dtype=torch.uint8, device=dev)
    xin[xo:xo + len(x_bytes)] = torch.from_numpy(np.frombuffer(x_bytes, dtype=np.uint8).copy()).to(dev)
    nb = _nbytes(dst, n)
    yout = torch.full((nb + yo + 64,), 0xA5, dtype=torch.uint8, device=dev)
    lb.check(lb.lib().lcml_cast(ctypes.c_void_p(xin.data_ptr() + xo), src, ctypes.c_void_p(yout.data_ptr() + yo),
                                dst, n, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    out = yout.cpu().numpy()
    assert (out[:yo] == 0xA5).all() and (out[yo + nb:] == 0xA5).all(), "cast wrote outside its output"
    return out[yo:yo + nb].tobytes()


def _values(t, raw, n):
    """Decoded float64 values of raw storage of type t (for NaN-aware compares)."""
    with np.errstate(invalid="ignore"):  # signalling-NaN bit patterns widen to quiet NaNs
        return oracle.cast(np.frombuffer(raw, dtype=np.uint8), t, F32, n).astype(np.float64)


def _assert_same(got, want, dst, n, what):
    if dst in (F32, F16, BF16):  # NaN payloads are not specified: compare NaN-ness, then bits
        gv, wv = _values(dst, got, n), _values(dst, want, n)
        nan = np.isnan(wv)
        assert np.array_equal(np.isnan(gv), nan), f"{what}: NaN positions differ"
        gb = np.frombuffer(got, dtype=STORAGE[dst]).view(np.uint32 if dst == F32 else np.uint16)
        wb = np.frombuffer(want, dtype=STORAGE[dst]).view(np.uint32 if dst == F32 else np.uint16)
        bad = np.nonzero((gb != wb) & ~nan)[0]
    else:
        g, w = np.frombuffer(got, dtype=np.uint8), np.frombuffer(want, dtype=np.uint8)
        bad = np.nonzero(g != w)[0]
    assert bad.size == 0, f"{what}: {bad.size} mismatches, first at element/byte {bad[0]}"


def _sources():
    rng = np.random.default_rng(2)
    half_all = np.arange(65536, dtype=np.uint16)
    f32 = np.concatenate([half_all.view(np.float16).astype(np.float32),
                          rng.integers(0, 2 ** 32, size=1 << 20, dtype=np.uint64).astype(np.uint32).view(np.float32),
                          (rng.standard_normal(1 << 16) * 30).astype(np.float32)])
    return {
        F16: half_all.tobytes(),
        BF16: half_all.tobytes(),  # every bf16 bit pattern
        F32: f32.tobytes(),
        E4M3: np.arange(256, dtype=np.uint8).tobytes(),
        E5M2: np.arange(256, dtype=np.uint8).tobytes(),
        E2M1: np.arange(256, dtype=np.uint8).tobytes(),  # all 16 codes in both nibbles
    }


@pytest.mark.parametrize("src", ALL)
def test_cast_all_pairs_bit_exact(dev, src):
    raw = _sources()[src]
    n = len(raw) * 2 if src == E2M1 else len(raw) // np.dtype(STORAGE[src]).itemsize
    for dst in ALL:
        if dst == src:
            continue
        want = oracle.cast(np.frombuffer(raw, dtype=np.uint8), src, dst, n).tobytes()
        got = _gpu_cast(dev, raw, src, dst, n)
        _assert_same(got, want, dst, n, f"cast {src} -> {dst}")


@pytest.mark.parametrize("n", [1, 7, 9, 1001])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_cast_ragged_and_misaligned(dev, n, offset):
    rng = np.random.default_rng(n + offset)
    x = (rng.standard_normal(n) * 100).astype(np.float32)
    x[::5] = np.float32(1e-6)
    for src, dst in [(F32, E4M3), (F32, E2M1), (F32, E5M2), (F32, F16), (BF16, E2M1)]:
        raw = x.tobytes() if src == F32 else oracle.cast(x, F32, BF16).tobytes()
        want = oracle.cast(np.frombuffer(raw, dtype=np.uint8), src, dst, n).tobytes()
        got = _gpu_cast(dev, raw, src, dst, n, offset)
        _assert_same(got, want, dst, n, f"cast {src} -> {dst} n={n} offset={offset}")
    # and back from packed FP4 with an odd count
    raw = oracle.cast(x, F32, E2M1)
    want = oracle.cast(raw, E2M1, F32, n).tobytes()
    _assert_same(_gpu_cast(dev, raw.tobytes(), E2M1, F32, n, offset), want, F32, n, "fp4 -> fp32")


def test_cast_rejects_unsupported(dev):
    """Unsupported types, a same-type "cast" and pointers not aligned to their
    element are refused on the host (nothing is launched)."""
    import torch
    import luisaml_b200 as lb
    lib = lb.lib()
    assert lib.lcml_cast(None, F32, None, 6, 4, None) == 2  # INT32 destination
    assert lib.lcml_cast(None, F32, None, F32, 4, None) == 1  # same type: a copy, not a cast
    buf = torch.zeros(256, dtype=torch.uint8, device=dev)
    p = buf.data_ptr()
    before = lb.launch_count()
    assert lib.lcml_cast(ctypes.c_void_p(p + 1), F32, ctypes.c_void_p(p + 128), E4M3, 8, None) == 1
    assert lib.lcml_cast(ctypes.c_void_p(p), E4M3, ctypes.c_void_p(p + 129), BF16, 8, None) == 1
    assert lb.launch_count() == before


def test_cast_graph_through_executor(dev):
    """Cast nodes in a graph (the reference's own way to express FP8
    conversion): x fp32 -> Cast(FLOAT8E4M3FN) -> Cast(FLOAT) and
    x -> Cast(FLOAT8E5M2) -> Cast(FLOAT16), through NetworkInstance."""
    import torch
    from luisaml_b200.export import GraphBuilder
    from luisaml_b200.session import Network
    b = GraphBuilder("cast_chain")
    b.input("x", "FLOAT", (64, 33))
    q8 = b.value("q8", "FLOAT8E4M3FN", (64, 33))
    b.node("Cast", ["x"], [q8], to=17)
    b.output("y8", "FLOAT", (64, 33))
    b.node("Cast", [q8], ["y8"], to=1)
    q5 = b.value("q5", "FLOAT8E5M2", (64, 33))
    b.node("Cast", ["x"], [q5], to=19)
    b.output("y5", "FLOAT16", (64, 33))
    b.node("Cast", [q5], ["y5"], to=10)
    net = Network(b.to_json())
    x = (np.random.default_rng(9).standard_normal((64, 33)) * 50).astype(np.float32)
    y8 = torch.empty((64, 33), dtype=torch.float32, device=dev)
    y5 = torch.empty((64, 33), dtype=torch.float16, device=dev)
    net.set_input("x", torch.from_numpy(x).to(dev))
    net.set_output("y8", y8)
    net.set_output("y5", y5)
    net.forward()
    torch.cuda.synchronize()
    want8 = oracle.cast(oracle.cast(x, F32, E4M3), E4M3, F32, x.size).reshape(x.shape)
    want5 = oracle.cast(oracle.cast(x, F32, E5M2), E5M2, F16, x.size).reshape(x.shape)
    np.testing.assert_array_equal(y8.cpu().numpy(), want8)
    np.testing.assert_array_equal(y5.cpu().numpy().view(np.uint16), want5.view(np.uint16))
