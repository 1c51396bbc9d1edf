"""Shared pytest configuration.

`-m gpu` tests need a B200 and the in-tree libraries; everything else runs on
CPU. GPU tests go through the C ABI (luisaml_b200 -> liblcml_fp8.so) and check
against the CPU oracle (oracle/) or the golden fixtures (tests/golden/).
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# The parity bar for GEMM / conv outputs (rtol 2e-3, atol 1e-3 of the
# fp32-accumulated oracle); e4m3 bytes and scales are compared bit-exactly.
RTOL = 2e-3
ATOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) and the built libraries")


@pytest.fixture(scope="session")
def dev():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    import luisaml_b200 as lb
    lb.check(lb.lib().lcml_device_check())
    return torch.device("cuda:0")


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def bf16_half_ulp(x):
    """Half the bf16 spacing at |x| (8 significant bits): the largest error of
    a correct round-to-nearest cast of x to bf16."""
    a = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return np.ldexp(1.0, (e - 8).astype(np.int64))


def assert_close_bf16(got, ref, rtol=RTOL, atol=ATOL, what=""):
    """bf16 output vs fp32 oracle: the fp32 accumulation must be within
    rtol/atol and the final cast to bf16 may add its half ulp."""
    assert_close(got, ref, rtol=rtol, atol=atol, what=what, extra=bf16_half_ulp(ref))


def assert_close(got, ref, rtol=RTOL, atol=ATOL, what="", extra=0.0):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    nan_got, nan_ref = np.isnan(got), np.isnan(ref)
    if (nan_got != nan_ref).any():
        i = np.unravel_index(np.argmax(nan_got != nan_ref), got.shape)
        raise AssertionError(f"{what}: NaN mismatch ({int((nan_got != nan_ref).sum())} elements); first at {i}: "
                             f"got {got[i]} ref {ref[i]}")
    err = np.where(nan_ref, 0.0, np.abs(got - ref))
    bound = atol + rtol * np.abs(np.where(nan_ref, 0.0, ref)) + extra
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} / {bad.size} elements out of tolerance "
                             f"(rtol {rtol}, atol {atol}); worst at {i}: got {got[i]} ref {ref[i]}")
