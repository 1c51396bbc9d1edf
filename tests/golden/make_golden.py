"""Regenerates the golden fixtures in this directory from the reference itself.

Run where a reference checkout exists:
    LCML_REFERENCE_TREE=<LuisaML checkout> python tests/golden/make_golden.py

* e4m3_*.npz      outputs of the reference's own CPU codec
                  (include/onnx/fp_quantized.h:149-249, compiled into
                  oracle/_ref/libref_codec.so by oracle/Makefile)
* simple_mlp/     the reference's fp32 MLP known-answer fixture, copied
                  verbatim from tests/onnx/output/ (model JSON, raw weight blob,
                  input_ref.bin, output_ref.bin — tests/onnx/generate_onnx.py)

The fixtures are committed; nothing on the GPU box reads the reference tree.
"""
from __future__ import annotations

import os
import shutil
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

REF_TREE = os.environ.get("LCML_REFERENCE_TREE", "")


def ref_encode(r, x: np.ndarray) -> np.ndarray:
    return np.array([r.lcml_ref_e4m3_from_float(float(v)) for v in x.astype(np.float32)], dtype=np.uint8)


def structured_inputs() -> np.ndarray:
    """Every positive e4m3 value, the midpoints between neighbours and one
    fp32 ulp either side of each midpoint, both signs, plus the saturation
    region, zeros, infinities, NaNs and fp32 subnormals."""
    vals = np.array([oracle.lib.orc_e4m3_to_float(c) for c in range(0x00, 0x7f)], dtype=np.float32)
    xs = [vals]
    mids = ((vals[:-1].astype(np.float64) + vals[1:].astype(np.float64)) / 2).astype(np.float32)
    xs += [mids, np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(0))]
    # below the smallest subnormal (2^-9): half of it is the round-to-zero tie
    tiny = np.float32(2.0 ** -10)
    xs.append(np.array([tiny, np.nextafter(tiny, np.float32(1)), np.nextafter(tiny, np.float32(0)),
                        np.float32(2.0 ** -11), np.float32(1e-30), np.float32(1e-45)], dtype=np.float32))
    sat = np.array([448.0, 449.0, 463.99997, 464.0, 464.00003, 479.0, 480.0, 481.0, 512.0, 1e4, 1e9,
                    3.4028235e38], dtype=np.float32)
    xs.append(sat)
    pos = np.concatenate(xs)
    special = np.array([0.0, -0.0, np.inf, -np.inf], dtype=np.float32)
    nans = np.array([0x7fc00000, 0xffc00000, 0x7f800001, 0xff800001, 0x7fffffff], dtype=np.uint32).view(np.float32)
    return np.concatenate([pos, -pos, special, nans]).astype(np.float32)


def minifloat_structured_inputs(decode, codes, sat) -> np.ndarray:
    """Every positive value of a minifloat format (decode over `codes`), the
    midpoints between neighbours and one fp32 ulp either side of each, the
    round-to-zero tie below the smallest subnormal, the region past the
    largest finite value (`sat`), both signs, zeros, infinities and NaNs."""
    vals = np.array([decode(c) for c in codes], dtype=np.float32)
    mids = ((vals[:-1].astype(np.float64) + vals[1:].astype(np.float64)) / 2).astype(np.float32)
    tiny = np.float32(vals[1] / 2)
    xs = [vals, mids, np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(0)),
          np.array([tiny, np.nextafter(tiny, np.float32(1)), np.nextafter(tiny, np.float32(0)), tiny / 2,
                    np.float32(1e-30), np.float32(1e-45)], dtype=np.float32),
          np.array(sat, dtype=np.float32)]
    pos = np.concatenate(xs)
    special = np.array([0.0, -0.0, np.inf, -np.inf], dtype=np.float32)
    nans = np.array([0x7fc00000, 0xffc00000, 0x7f800001], dtype=np.uint32).view(np.float32)
    return np.concatenate([pos, -pos, special, nans]).astype(np.float32)


def random_inputs(n: int = 65536, seed: int = 1234) -> np.ndarray:
    rng = np.random.default_rng(seed)
    bits = rng.integers(0, 2 ** 32, size=n // 2, dtype=np.uint64).astype(np.uint32).view(np.float32)
    normal = rng.standard_normal(n // 2).astype(np.float32)
    scale = np.array([1.0, 100.0, 0.01, 1e-3], dtype=np.float32)[rng.integers(0, 4, size=n // 2)]
    return np.concatenate([bits, normal * scale]).astype(np.float32)


def main() -> None:
    if not REF_TREE or not os.path.isdir(REF_TREE):
        raise SystemExit("set LCML_REFERENCE_TREE to the root of a LuisaML checkout")
    r = oracle.ref_lib()
    if r is None:
        raise SystemExit("oracle/_ref/libref_codec.so missing: run `make -C oracle` with the reference tree present")

    dec = np.array([r.lcml_ref_e4m3_to_float(c) for c in range(256)], dtype=np.float32)
    np.savez(os.path.join(HERE, "e4m3_decode.npz"), codes=np.arange(256, dtype=np.uint8), values=dec)

    xs = structured_inputs()
    np.savez(os.path.join(HERE, "e4m3_encode_structured.npz"), x=xs, q=ref_encode(r, xs))

    xr = random_inputs()
    np.savez(os.path.join(HERE, "e4m3_encode_random.npz"), x=xr, q=ref_encode(r, xr))

    # QuantizeLinear per-tensor: q = from_float(x / s), s = amax / 448 (fp32)
    rng = np.random.default_rng(2024)
    x = rng.standard_normal((128, 256)).astype(np.float32)
    amax = np.float32(np.max(np.abs(x)))
    s = np.float32(amax / np.float32(448.0))
    q = np.empty(x.size, dtype=np.uint8)
    r.lcml_ref_e4m3_quantize_tensor(x.ctypes.data_as(oracle._f32p), float(s),
                                    q.ctypes.data_as(oracle._u8p), x.size)
    np.savez(os.path.join(HERE, "e4m3_quantize_tensor.npz"), x=x, scale=np.float32(s), q=q.reshape(x.shape))

    # FP8 E5M2 and FP4 E2M1 (fp_quantized.h:259-378, :20-115): decode tables and encodes
    for fmt, ncodes, top, sat in (("e5m2", 256, 0x7c, [57344.0, 57345.0, 59392.0, 61439.0, 61440.0, 65504.0, 1e9]),
                                  ("e2m1", 16, 0x8, [6.0, 6.5, 7.0, 7.5, 8.0, 100.0, 3.4028235e38])):
        enc = getattr(r, f"lcml_ref_{fmt}_from_float")
        dec = getattr(r, f"lcml_ref_{fmt}_to_float")
        table = np.array([dec(c) for c in range(ncodes)], dtype=np.float32)
        xs = np.concatenate([minifloat_structured_inputs(dec, range(0, top), sat), random_inputs(16384, 99)])
        q = np.array([enc(float(v)) for v in xs], dtype=np.uint8)
        np.savez(os.path.join(HERE, f"{fmt}_codec.npz"), codes=np.arange(ncodes, dtype=np.uint8), values=table,
                 x=xs, q=q)

    # the reference's fp32 MLP known-answer fixture
    src = os.path.join(REF_TREE, "tests", "onnx", "output")
    dst = os.path.join(HERE, "simple_mlp")
    os.makedirs(dst, exist_ok=True)
    for name in ("simple_mlp.onnx.json", "simple_mlp.safetensors", "input_ref.bin", "output_ref.bin"):
        shutil.copyfile(os.path.join(src, name), os.path.join(dst, name))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
