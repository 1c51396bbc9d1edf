"""The no-allocation GEMM + per-row quantization entry point.

lcml_fp8_gemm_rowquant_noalloc serves callers that cannot allocate device
memory (a host that owns all device memory through its own buffers, or a
server that reserved the whole HBM and must not call cudaMalloc). Its row-max
scratch is a static device array inside the library instead of a caller
workspace. These tests call it through the C ABI and compare it with the
workspace entry point lcml_fp8_gemm_rowquant on the same inputs, on two calls
in a row (the second with much smaller values, so row maxima left over from
the first call would show up in its scales), check that the second call
leaves the device's free memory unchanged, and check the row limit. The
shapes cover the tensor-core GEMM (320 rows, SiLU*up) and the CUDA-core GEMV
that decode-sized batches (1 and 4 rows) take.

The file name sorts last so that a `-x` run reaches every other test first.
"""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import assert_close

pytestmark = pytest.mark.gpu

MAX_ROWS = 65536


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _operands(seed, amp, M, F, K, silu):
    rng = np.random.default_rng(seed)
    Aq, sa = oracle.quantize_dynamic_rows((rng.standard_normal((M, K)) * amp).astype(np.float32))
    W = (rng.standard_normal(((2 if silu else 1) * F, K)) * 0.05).astype(np.float32)
    sw = np.array([oracle.scale_from_amax(oracle.amax(r)) for r in W], dtype=np.float32)
    return Aq, sa, oracle.quantize(W, sw, axis=0), sw


@pytest.mark.parametrize("M,F,K,silu", [(320, 384, 256, True), (4, 1000, 512, False), (1, 4096, 4096, False)])
def test_noalloc_matches_workspace_entry_point_twice(dev, M, F, K, silu):
    import torch
    import luisaml_b200 as lb
    lib = lb.lib()
    epi = lb.EPI_SILU_MUL if silu else lb.EPI_NONE
    for call, (seed, amp) in enumerate(((71, 1.0), (72, 1e-3))):
        Aq, sa, Wq, sw = [_t(a, dev) for a in _operands(seed + M, amp, M, F, K, silu)]
        # existing entry point, caller-provided workspace
        Y_ref, q_ref, s_ref = lb.gemm_rowquant(Aq, Wq, sa, sw, epilogue=epi)
        # no-allocation entry point through the C ABI
        d, Y = lb.gemm(Aq, Wq, sa, sw, epilogue=epi, out_dtype=torch.float32, desc_only=True)
        q = torch.empty(Y.shape, dtype=torch.uint8, device=dev)
        s = torch.empty(Y.shape[0], dtype=torch.float32, device=dev)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        lb.check(lib.lcml_fp8_gemm_rowquant_noalloc(ctypes.byref(d), ctypes.c_void_p(q.data_ptr()),
                                                    ctypes.c_void_p(s.data_ptr()), stream))
        torch.cuda.synchronize()
        if call == 1:  # the first call may load the module on this device; the second must not allocate
            assert torch.cuda.mem_get_info(dev)[0] == free_before, "the no-allocation call changed free memory"
        assert_close(Y.cpu().numpy(), Y_ref.cpu().numpy(), what=f"fp32 output, amp {amp}")
        assert np.array_equal(s.cpu().numpy(), s_ref.cpu().numpy()), f"row scales differ, amp {amp}"
        assert np.array_equal(q.cpu().numpy(), q_ref.cpu().numpy()), f"e4m3 bytes differ, amp {amp}"
        # and the quantization is the oracle's for that fp32 output
        qr, sr = oracle.quantize_dynamic_rows(Y.cpu().numpy())
        assert np.array_equal(s.cpu().numpy(), sr) and np.array_equal(q.cpu().numpy(), qr)
    assert lb.device_error() == 0


def test_noalloc_rejects_rows_beyond_its_scratch(dev):
    import luisaml_b200 as lb
    d = lb.GemmDesc()
    d.M, d.N, d.K = MAX_ROWS + 1, 256, 128
    rc = lb.lib().lcml_fp8_gemm_rowquant_noalloc(ctypes.byref(d), None, None, None)
    assert rc == 1
    assert b"65536" in lb.lib().lcml_last_error()
