"""FP8 GEMM (tcgen05 kernel and SIMT kernel) vs the CPU oracle.

The oracle dequantizes both e4m3 operands (DequantizeLinear) and runs
gemm.cpp's fp32 K-ordered fma loop; outputs must agree within rtol 2e-3 /
atol 1e-3 (fp32 and bf16 outputs). e4m3 outputs must decode to within one
e4m3 rounding step of the oracle's fp32 value.
"""
import numpy as np
import pytest

import oracle
from conftest import assert_close, assert_close_bf16

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def make_operands(M, N, K, seed, per_row=False, per_col=False, b_std=1.0):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (rng.standard_normal((N, K)) * b_std).astype(np.float32)  # [N, K] = Gemm transB=1
    if per_row:
        Aq, sa = oracle.quantize_dynamic_rows(A)
    else:
        sa = np.float32([oracle.scale_from_amax(oracle.amax(A))])
        Aq = oracle.quantize(A, sa[0])
    if per_col:
        sb = np.array([oracle.scale_from_amax(oracle.amax(B[n])) for n in range(N)], dtype=np.float32)
        Bq = oracle.quantize(B, sb, axis=0)
    else:
        sb = np.float32([oracle.scale_from_amax(oracle.amax(B))])
        Bq = oracle.quantize(B, sb[0])
    return Aq, sa, Bq, sb


SHAPES = [
    (128, 256, 128),     # exactly one tile
    (200, 300, 160),     # ragged M, N, K (BN=128 kernel, TMA zero fill)
    (256, 2048, 512),    # BN=256 kernel, several k-blocks
    (32, 512, 784),      # MLP layer 1 (K = 784, not a multiple of 128)
    (1, 4096, 4096),     # skinny decode
    (16, 4096, 4096),
    (128, 4096, 4096),   # skinny sweep point
    (1000, 1000, 1000),  # K % 128 != 0, N < 2048
    (1024, 2048, 1024),
]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_gemm_shapes(dev, M, N, K, out):
    import torch
    import luisaml_b200 as lb
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=M * 31 + N * 7 + K)
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb, b_kmajor=True)
    a, b, s1, s2 = _t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev)
    y32 = lb.gemm(a, b, s1, s2, out_dtype=torch.float32)
    assert_close(y32.cpu().numpy(), ref, what=f"gemm {M}x{N}x{K} f32")
    if out == "bf16":
        Y = lb.gemm(a, b, s1, s2, out_dtype=torch.bfloat16)
        # the bf16 store is the correctly rounded fp32 epilogue value ...
        assert torch.equal(Y, y32.bfloat16())
        # ... so it is within tolerance of the oracle up to the cast's half ulp
        assert_close_bf16(Y.float().cpu().numpy(), ref, what=f"gemm {M}x{N}x{K} bf16")
    assert lb.device_error() == 0


@pytest.mark.parametrize("per_row,per_col", [(True, False), (False, True), (True, True)])
def test_gemm_scale_modes(dev, per_row, per_col):
    import torch
    import luisaml_b200 as lb
    M, N, K = 300, 512, 256
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=5, per_row=per_row, per_col=per_col, b_std=0.02)
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb)
    Y = lb.gemm(_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev), out_dtype=torch.float32)
    assert_close(Y.cpu().numpy(), ref, what="scale modes")


def test_gemm_bias_relu_alpha_beta(dev):
    import torch
    import luisaml_b200 as lb
    M, N, K = 96, 640, 384
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=9)
    bias = np.random.default_rng(1).standard_normal(N).astype(np.float32)
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb)
    ref = np.maximum(0.5 * ref + 2.0 * bias, 0.0)
    Y = lb.gemm(_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev), alpha=0.5, beta=2.0, c_vec=_t(bias, dev),
                epilogue=lb.EPI_RELU, out_dtype=torch.float32)
    assert_close(Y.cpu().numpy(), ref, what="bias+relu")


def test_gemm_residual_and_row_amax(dev):
    import torch
    import luisaml_b200 as lb
    M, N, K = 256, 512, 256
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=13)
    res = np.random.default_rng(2).standard_normal((M, N)).astype(np.float32)
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb) + res
    amax = torch.zeros(M, dtype=torch.float32, device=dev)
    Y = lb.gemm(_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev), c_mat=_t(res, dev), out_dtype=torch.float32,
                row_amax=amax)
    y = Y.cpu().numpy()
    assert_close(y, ref, what="residual")
    assert np.array_equal(amax.cpu().numpy(), np.abs(y).max(axis=1))


def test_gemm_silu_mul(dev):
    import torch
    import luisaml_b200 as lb
    M, F, K = 200, 384, 256  # F = ffn width; B holds 2F rows (gate/up interleaved by 128)
    rng = np.random.default_rng(17)
    Aq, sa = oracle.quantize_dynamic_rows(rng.standard_normal((M, K)).astype(np.float32))
    Wg = (rng.standard_normal((F, K)) * 0.05).astype(np.float32)
    Wu = (rng.standard_normal((F, K)) * 0.05).astype(np.float32)
    sg = np.array([oracle.scale_from_amax(oracle.amax(r)) for r in Wg], dtype=np.float32)
    su = np.array([oracle.scale_from_amax(oracle.amax(r)) for r in Wu], dtype=np.float32)
    Gq, Uq = oracle.quantize(Wg, sg, axis=0), oracle.quantize(Wu, su, axis=0)
    g = oracle.qdq_gemm(Aq, sa, Gq, sg)
    u = oracle.qdq_gemm(Aq, sa, Uq, su)
    ref = oracle.silu_mul(g, u)
    # interleave [gate 128 rows; up 128 rows] per group
    Bq = np.concatenate([np.concatenate([Gq[i:i + 128], Uq[i:i + 128]]) for i in range(0, F, 128)])
    sb = np.concatenate([np.concatenate([sg[i:i + 128], su[i:i + 128]]) for i in range(0, F, 128)])
    amax = torch.zeros(M, dtype=torch.float32, device=dev)
    for simt in (False, True):
        amax.zero_()
        Y = lb.gemm(_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev), epilogue=lb.EPI_SILU_MUL,
                    out_dtype=torch.float32, row_amax=amax, simt=simt)
        y = Y.cpu().numpy()
        assert y.shape == (M, F)
        assert_close(y, ref, what=f"silu_mul simt={simt}")
        assert np.array_equal(amax.cpu().numpy(), np.abs(y).max(axis=1))


def test_gemm_e4m3_output(dev):
    import torch
    import luisaml_b200 as lb
    M, N, K = 128, 512, 512
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=23)
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb)
    ys = np.float32([oracle.scale_from_amax(np.abs(ref).max())])
    Y = lb.gemm(_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev), out_dtype=torch.uint8, y_scale=_t(ys, dev))
    got = oracle.e4m3_decode(Y.cpu().numpy())
    want = oracle.e4m3_decode(oracle.quantize(ref, ys[0]))
    # one e4m3 step is at most 2^-3 relative (normal) or 2^-9 absolute (subnormal) of x / s
    step = np.maximum(np.abs(want) * 0.125, 2.0 ** -9)
    assert (np.abs(got - want) <= step + 1e-12).all()
    assert (got == want).mean() > 0.99


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (2, 1001, 4096), (3, 1000, 2048), (4, 520, 3072),
                                   (48, 640, 2048), (200, 1000, 2048)])
def test_splitk_epilogues(dev, M, N, K):
    """Skinny GEMMs run split-K in a CTA cluster (partials reduced through
    distributed shared memory): per-row / per-column scales, bias, a residual
    (fp32 and e4m3), Relu, the row |max| and every output type against the
    oracle, and against the single-CTA kernel (forced by variant 1). M > 128
    (two row tiles, the last one partial) takes split-K only when variant 3
    forces it; automatic selection gives it single-CTA tiles. M <= 4 runs the
    CUDA-core GEMV under automatic selection (variant 0) and split-K under
    variant 3, so both are checked with the same epilogues."""
    import torch
    import luisaml_b200 as lb
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=M + N + K, per_row=True, per_col=True, b_std=0.05)
    rng = np.random.default_rng(K)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    ref = np.maximum(oracle.qdq_gemm(Aq, sa, Bq, sb) + bias + res, 0.0)
    args = (_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev))
    kw = dict(c_vec=_t(bias, dev), c_mat=_t(res, dev), epilogue=lb.EPI_RELU)
    results = {}
    for mode in (0, 1, 3):
        amax = torch.zeros(M, dtype=torch.float32, device=dev)
        y = lb.gemm(*args, out_dtype=torch.float32, row_amax=amax, variant=mode, **kw).cpu().numpy()
        assert_close(y, ref, what=f"split-K {M}x{N}x{K} variant {mode}")
        assert np.array_equal(amax.cpu().numpy(), np.abs(y).max(axis=1))
        yb = lb.gemm(*args, out_dtype=torch.bfloat16, variant=mode, **kw)
        assert torch.equal(yb.cpu(), torch.from_numpy(y).bfloat16())
        results[mode] = y
    assert_close(results[0], results[1], rtol=1e-5, atol=1e-4, what="automatic vs single CTA")
    assert_close(results[3], results[1], rtol=1e-5, atol=1e-4, what="split-K vs single CTA")
    # e4m3 residual and e4m3 output (the epilogue quantization rule on the split-K sum)
    rs = np.float32(oracle.scale_from_amax(oracle.amax(res)))
    rq = oracle.quantize(res, rs)
    ys = np.float32(oracle.scale_from_amax(np.abs(ref).max()))
    y32 = lb.gemm(*args, c_vec=_t(bias, dev), c_mat=_t(rq, dev), epilogue=lb.EPI_RELU, out_dtype=torch.float32,
                  c_mat_scale=_t(np.float32([rs]), dev)).cpu().numpy()
    want32 = np.maximum(oracle.qdq_gemm(Aq, sa, Bq, sb) + bias + oracle.dequantize(rq, rs), 0.0)
    assert_close(y32, want32, what="split-K e4m3 residual")
    y8 = lb.gemm(*args, c_vec=_t(bias, dev), c_mat=_t(rq, dev), epilogue=lb.EPI_RELU, out_dtype=torch.uint8,
                 c_mat_scale=_t(np.float32([rs]), dev), y_scale=_t(np.float32([ys]), dev)).cpu().numpy()
    np.testing.assert_array_equal(y8, epilogue_quantize(y32, ys))
    assert lb.device_error() == 0


@pytest.mark.parametrize("res", [True, False])
@pytest.mark.parametrize("M,N,K,relu", [(300, 256, 64, True), (1000, 128, 192, True), (200, 64, 576, False),
                                         (777, 2048, 128, True)])
def test_fast_epilogue_kernels(dev, M, N, K, relu, res):
    """The fast-epilogue kernels (e4m3 out, column-factor table, per-tensor A
    scale, bias along N, optional e4m3 residual) against the generic epilogue
    on the same GEMM (selected by asking for the row |max|, which the fast
    kernels do not compute): e4m3 bytes identical, and equal to the epilogue
    rule applied to the oracle-checked fp32 result. Ragged M leaves the last
    tile's rows past M reading a clamped residual row; N = 64 / 128 / 256 /
    2048 covers the BN = 64, 128 and 256 kernels."""
    import torch
    import luisaml_b200 as lb
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=M + K, per_col=True)
    rng = np.random.default_rng(N)
    bias = rng.standard_normal(N).astype(np.float32)
    r32 = rng.standard_normal((M, N)).astype(np.float32)
    rs = np.float32(oracle.scale_from_amax(oracle.amax(r32)))
    rq = oracle.quantize(r32, rs)
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb) + bias + (oracle.dequantize(rq, rs) if res else 0.0)
    if relu:
        ref = np.maximum(ref, 0.0)
    ys = np.float32(oracle.scale_from_amax(np.abs(ref).max()))
    kw = dict(c_vec=_t(bias, dev), epilogue=lb.EPI_RELU if relu else lb.EPI_NONE)
    if res:
        kw.update(c_mat=_t(rq, dev), c_mat_scale=_t(np.float32([rs]), dev))
    args = (_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev))
    y32 = lb.gemm(*args, out_dtype=torch.float32, **kw).cpu().numpy()
    assert_close(y32, ref, what=f"fast-epilogue shape {M}x{N}x{K} fp32")
    fast = lb.gemm(*args, out_dtype=torch.uint8, y_scale=_t(np.float32([ys]), dev), **kw).cpu().numpy()
    amax = torch.zeros(M, dtype=torch.float32, device=dev)
    generic = lb.gemm(*args, out_dtype=torch.uint8, y_scale=_t(np.float32([ys]), dev), row_amax=amax,
                      **kw).cpu().numpy()
    np.testing.assert_array_equal(fast, generic)
    np.testing.assert_array_equal(fast, epilogue_quantize(y32, ys))
    assert lb.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(200, 300, 160), (64, 1024, 128)])
def test_simt_and_tensor_core_paths_agree(dev, M, N, K):
    import torch
    import luisaml_b200 as lb
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=3)
    a, b, s1, s2 = _t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev)
    y_tc = lb.gemm(a, b, s1, s2, out_dtype=torch.float32).cpu().numpy()
    y_simt = lb.gemm(a, b, s1, s2, out_dtype=torch.float32, simt=True).cpu().numpy()
    assert_close(y_tc, y_simt, rtol=1e-5, atol=1e-4, what="tc vs simt")


def test_mn_major_b_uses_matmul_layout(dev):
    import torch
    import luisaml_b200 as lb
    M, N, K = 100, 200, 96
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=29)
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb)
    Bkn = np.ascontiguousarray(Bq.T)  # MatMul's [K, N]
    Y = lb.gemm(_t(Aq, dev), _t(Bkn, dev), _t(sa, dev), _t(sb, dev), b_kmajor=False, out_dtype=torch.float32)
    assert_close(Y.cpu().numpy(), ref, what="[K,N] B")


def test_large_8192_sampled_rows(dev):
    """The bench configuration (M=N=K=8192): sampled rows against the oracle,
    plus a size-independent check: row sums equal A_row . (sum of B rows)."""
    import torch
    import luisaml_b200 as lb
    M = N = K = 8192
    g = torch.Generator(device=dev).manual_seed(0)
    A = torch.randn(M, K, device=dev, generator=g)
    B = torch.randn(N, K, device=dev, generator=g)
    sa = lb.amax(A)
    sa = torch.where(sa > 0, sa / 448.0, torch.ones_like(sa))
    sb = lb.amax(B)
    sb = torch.where(sb > 0, sb / 448.0, torch.ones_like(sb))
    Aq, Bq = lb.quantize(A, sa), lb.quantize(B, sb)
    Y = lb.gemm(Aq, Bq, sa, sb, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert lb.device_error() == 0
    Aqh, Bqh = Aq.cpu().numpy(), Bq.cpu().numpy()
    sah, sbh = sa.cpu().numpy(), sb.cpu().numpy()
    for r0 in (0, 4093, 8160):
        ref = oracle.qdq_gemm(Aqh, sah, Bqh, sbh, rows=(r0, r0 + 32))
        assert_close(Y[r0:r0 + 32].cpu().numpy(), ref, what=f"8192^3 rows {r0}..")
    # linearity: Y @ 1 == A . (B^T @ 1), in float64 from the dequantized operands
    Ad = oracle.e4m3_decode(Aqh).astype(np.float64) * float(sah[0])
    Bd = oracle.e4m3_decode(Bqh).astype(np.float64) * float(sbh[0])
    want = Ad @ Bd.sum(axis=0)
    got = Y.double().sum(dim=1).cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-2)



@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("M,N,K,per_row,per_col", [
    (256, 256, 128, False, False),    # one pair tile
    (300, 520, 200, True, True),      # ragged everything
    (1024, 1536, 640, False, True),
    (2048, 2048, 1024, True, False),
])
def test_kernel_variants(dev, mode, M, N, K, per_row, per_col):
    """Single-CTA (variant 1) and CTA-pair (variant 2) tensor-core kernels vs the oracle."""
    import torch
    import luisaml_b200 as lb
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=M + N + K + mode, per_row=per_row, per_col=per_col)
    bias = np.random.default_rng(M).standard_normal(N).astype(np.float32)
    ref = np.maximum(oracle.qdq_gemm(Aq, sa, Bq, sb) + bias, 0.0)
    Y = lb.gemm(_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev), c_vec=_t(bias, dev), epilogue=lb.EPI_RELU,
                out_dtype=torch.float32, variant=mode)
    assert_close(Y.cpu().numpy(), ref, what=f"variant {mode} {M}x{N}x{K}")
    assert lb.device_error() == 0


@pytest.mark.parametrize("out", ["f32", "e4m3"])
def test_pair_schedule_split_last_wave(dev, out):
    """CTA-pair kernel whose schedule ends in split tiles: with P pairs and
    P + r tiles (r <= P / 2) the last r tiles run as two 256 x 128 items each.
    M and N are ragged, so the split items include partial rows and an
    item past the last column. fp32 output and the row |max| against the
    oracle (with an fp32 residual), e4m3 output bit-identical to the
    single-CTA kernel's (same epilogue rule, fp32 sums within the tolerance)."""
    import torch
    import luisaml_b200 as lb
    pairs = torch.cuda.get_device_properties(dev).multi_processor_count // 2
    num_n = 8
    num_m = (pairs + 5 + num_n - 1) // num_n  # tiles = num_m * num_n: a few more than one wave
    M, N, K = 256 * num_m - 40, 256 * num_n - 200, 384
    tiles = num_m * num_n
    assert 0 < tiles % pairs <= pairs // 2, (tiles, pairs)
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=71, per_row=True, per_col=True)
    bias = np.random.default_rng(5).standard_normal(N).astype(np.float32)
    res = np.random.default_rng(6).standard_normal((M, N)).astype(np.float32)
    args = (_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev))
    if out == "f32":
        ref = np.maximum(oracle.qdq_gemm(Aq, sa, Bq, sb) + bias + res, 0.0)
        amax = torch.zeros(M, dtype=torch.float32, device=dev)
        Y = lb.gemm(*args, c_vec=_t(bias, dev), c_mat=_t(res, dev), epilogue=lb.EPI_RELU,
                    out_dtype=torch.float32, row_amax=amax, variant=2)
        y = Y.cpu().numpy()
        assert_close(y, ref, what="pair schedule with split tiles")
        assert np.array_equal(amax.cpu().numpy(), np.abs(y).max(axis=1))
    else:
        ys = _t(np.float32([0.05]), dev)
        got = [lb.gemm(*args, c_vec=_t(bias, dev), epilogue=lb.EPI_RELU, out_dtype=torch.uint8, y_scale=ys,
                       variant=m).cpu().numpy() for m in (2, 1)]
        assert np.mean(got[0] != got[1]) <= 1e-4
        diff = np.abs(oracle.e4m3_decode(got[0]) - oracle.e4m3_decode(got[1]))
        step = np.maximum(np.abs(oracle.e4m3_decode(got[1])), 2.0 ** -6) / 8.0
        assert (diff <= step + 1e-12).all()
    assert lb.device_error() == 0


@pytest.mark.parametrize("mode", [1, 2])
def test_kernel_variants_silu(dev, mode):
    import torch
    import luisaml_b200 as lb
    M, F, K = 512, 512, 384
    rng = np.random.default_rng(41)
    Aq, sa = oracle.quantize_dynamic_rows(rng.standard_normal((M, K)).astype(np.float32))
    W = (rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32)
    sw = np.array([oracle.scale_from_amax(oracle.amax(r)) for r in W], dtype=np.float32)
    Wq = oracle.quantize(W, sw, axis=0)  # rows already in the interleaved [gate 128; up 128] order
    full = oracle.qdq_gemm(Aq, sa, Wq, sw)
    g = np.concatenate([full[:, i:i + 128] for i in range(0, 2 * F, 256)], axis=1)
    u = np.concatenate([full[:, i + 128:i + 256] for i in range(0, 2 * F, 256)], axis=1)
    ref = oracle.silu_mul(g, u)
    Y = lb.gemm(_t(Aq, dev), _t(Wq, dev), _t(sa, dev), _t(sw, dev), epilogue=lb.EPI_SILU_MUL,
                out_dtype=torch.float32, variant=mode)
    assert_close(Y.cpu().numpy(), ref, what=f"silu variant {mode}")


@pytest.mark.parametrize("epilogue", ["silu", "none"])
def test_gemm_rowquant(dev, epilogue):
    """Gemm -> (SiLU*up) -> per-row dynamic QuantizeLinear, as the FFN uses it:
    the fp32 output matches the oracle within tolerance and the e4m3 bytes and
    scales are bit-exact given that fp32 output."""
    import torch
    import luisaml_b200 as lb
    M, F, K = 300, 384, 256
    rng = np.random.default_rng(57)
    Aq, sa = oracle.quantize_dynamic_rows(rng.standard_normal((M, K)).astype(np.float32))
    W = (rng.standard_normal((2 * F, K)) * 0.05).astype(np.float32)
    sw = np.array([oracle.scale_from_amax(oracle.amax(r)) for r in W], dtype=np.float32)
    Wq = oracle.quantize(W, sw, axis=0)
    full = oracle.qdq_gemm(Aq, sa, Wq, sw)
    if epilogue == "silu":
        g = np.concatenate([full[:, i:i + 128] for i in range(0, 2 * F, 256)], axis=1)
        u = np.concatenate([full[:, i + 128:i + 256] for i in range(0, 2 * F, 256)], axis=1)
        ref = oracle.silu_mul(g, u)
        epi = lb.EPI_SILU_MUL
    else:
        ref, epi = full, lb.EPI_NONE
    ws = torch.full((M,), 123.0, dtype=torch.float32, device=dev)  # stale contents must not matter
    Y, q, s = lb.gemm_rowquant(_t(Aq, dev), _t(Wq, dev), _t(sa, dev), _t(sw, dev), epilogue=epi, workspace=ws)
    y = Y.cpu().numpy()
    assert_close(y, ref, what=f"rowquant {epilogue} fp32")
    qr, sr = oracle.quantize_dynamic_rows(y)
    assert np.array_equal(s.cpu().numpy(), sr)
    assert np.array_equal(q.cpu().numpy(), qr)


@pytest.mark.parametrize("out", ["bf16", "f32", "e4m3"])
@pytest.mark.parametrize("mode", [1, 2])
def test_gemm_column_shard_and_peer_copies(dev, out, mode):
    """The epilogue's column-offset + extra-destination stores (the fused
    all-gather path, staged through shared memory) on one GPU: a second
    buffer on the same device stands in for a peer's output."""
    import ctypes
    import torch
    import luisaml_b200 as lb
    M, N, K, Ntot, off = 300, 512, 256, 1024, 256
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=61, per_row=True, per_col=True, b_std=0.05)
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb)
    dt = {"bf16": torch.bfloat16, "f32": torch.float32, "e4m3": torch.uint8}[out]
    Y = torch.zeros((M, Ntot), dtype=dt, device=dev)
    Y2 = torch.zeros((M, Ntot), dtype=dt, device=dev)
    ys = _t(np.float32([oracle.scale_from_amax(np.abs(ref).max())]), dev)
    d, _ = lb.gemm(_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev), out_dtype=dt, desc_only=True,
                   y_scale=ys if out == "e4m3" else None, variant=mode)
    peers = torch.tensor([Y2.data_ptr()], dtype=torch.int64, device=dev)
    d.Y, d.ldy, d.y_col_offset, d.y_peers, d.y_num_peers = Y.data_ptr(), Ntot, off, peers.data_ptr(), 1
    lb.check(lb.lib().lcml_fp8_gemm(ctypes.byref(d), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert torch.equal(Y, Y2)
    assert torch.count_nonzero(Y[:, :off].float()) == 0 and torch.count_nonzero(Y[:, off + N:].float()) == 0
    got = Y[:, off:off + N]
    if out == "e4m3":
        g = oracle.e4m3_decode(got.cpu().numpy())
        w = oracle.e4m3_decode(oracle.quantize(ref, ys.cpu().numpy()[0]))
        assert (np.abs(g - w) <= np.maximum(np.abs(w) * 0.125, 2.0 ** -9) + 1e-12).all()
    elif out == "bf16":
        assert_close_bf16(got.float().cpu().numpy(), ref, what="bf16 shard")
    else:
        assert_close(got.cpu().numpy(), ref, what="f32 shard")


def epilogue_quantize(y, s):
    """The fused epilogues' output quantization: the reference codec applied
    to RN(y * RN(1 / s)) (fp32 multiply; +-0 -> 0x00, NaN -> 0x7f, |q| > 448
    saturates, as the codec does)."""
    r = np.float32(1.0) / np.float32(s)
    return oracle.quantize((np.asarray(y, dtype=np.float32) * r).astype(np.float32), np.float32(1.0))


def test_epilogue_quantize_rule(dev):
    """The epilogue rule on hand-picked values through a 1 x K x N GEMM whose
    output equals chosen fp32 values: zeros of both signs, NaN, values past
    448 * s, subnormal e4m3 results and ties."""
    import torch
    import luisaml_b200 as lb
    vals = np.float32([0.0, -0.0, 1e-30, -1e-30, 3.0, -3.0, 500.0, -1e9, 2.0 ** -9, -2.0 ** -10, 0.5625, 17.0,
                       np.nan, 448.0, 464.0, -480.0])
    N = 64
    v = np.resize(vals, N).astype(np.float32)
    for s in (np.float32(1.0), np.float32(0.0123)):
        # Y = A * B^T + bias with A = 0 (e4m3 zeros): Y = bias exactly
        A = torch.zeros((128, 64), dtype=torch.uint8, device=dev)
        B = torch.zeros((N, 64), dtype=torch.uint8, device=dev)
        one = torch.ones(1, device=dev)
        ys = _t(np.float32([s]), dev)
        Y = lb.gemm(A, B, one, one, c_vec=_t(v, dev), out_dtype=torch.uint8, y_scale=ys)
        got = Y.cpu().numpy()
        np.testing.assert_array_equal(got, np.broadcast_to(epilogue_quantize(v, s), got.shape))


@pytest.mark.parametrize("out", ["f32", "bf16", "e4m3"])
@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("M,N,K", [(300, 528, 200), (97, 64, 64), (1000, 96, 576)])
def test_store_paths(dev, out, mode, M, N, K):
    """The TMA-store epilogue (default) and plain per-row stores (variant bit 4)
    write bit-identical outputs, including ragged edges in M and N and an
    output placed at a column offset inside a wider matrix whose other columns
    must stay untouched; the fp32 result also matches the oracle and the e4m3
    bytes follow the epilogue quantization rule exactly (the codec applied to
    RN(y * RN(1 / s)) of the fp32 result y), which differs from QuantizeLinear
    of y only for values next to an e4m3 rounding boundary."""
    import torch
    import luisaml_b200 as lb
    Aq, sa, Bq, sb = make_operands(M, N, K, seed=M * 7 + N + K, per_row=True, per_col=True)
    bias = np.random.default_rng(N).standard_normal(N).astype(np.float32)
    ref = np.maximum(oracle.qdq_gemm(Aq, sa, Bq, sb) + bias, 0.0)
    dt = {"f32": torch.float32, "bf16": torch.bfloat16, "e4m3": torch.uint8}[out]
    ys = _t(np.float32([oracle.scale_from_amax(np.abs(ref).max())]), dev)
    args = (_t(Aq, dev), _t(Bq, dev), _t(sa, dev), _t(sb, dev))
    results = []
    for m in (mode, mode | 4):
        wide = torch.zeros((M, N + 48), dtype=dt, device=dev)
        wide.view(torch.uint8).fill_(0x55)
        lb.gemm(*args, c_vec=_t(bias, dev), epilogue=lb.EPI_RELU, out=wide[:, 16:16 + N],
                y_scale=ys if out == "e4m3" else None, variant=m)
        torch.cuda.synchronize()
        assert lb.device_error() == 0
        results.append(wide.view(torch.uint8).cpu().numpy())
    np.testing.assert_array_equal(results[0], results[1])
    es = {"f32": 4, "bf16": 2, "e4m3": 1}[out]
    assert (results[0][:, :16 * es] == 0x55).all() and (results[0][:, (16 + N) * es:] == 0x55).all()
    if out == "f32":
        got = results[0].view(np.float32)[:, 16:16 + N]
        assert_close(got, ref, what=f"store paths {M}x{N}x{K}")
    elif out == "e4m3":
        y32 = lb.gemm(*args, c_vec=_t(bias, dev), epilogue=lb.EPI_RELU, out_dtype=torch.float32,
                      variant=mode).cpu().numpy()
        s = np.float32(ys.cpu()[0])
        want = epilogue_quantize(y32, s)
        np.testing.assert_array_equal(results[0][:, 16:16 + N], want)
        assert np.mean(want != oracle.quantize(y32, s)) <= 1e-3


@pytest.mark.parametrize("M,pad", [(1, 0), (2, 64), (3, 0), (4, 4), (5, 0), (64, 0)])
def test_gemm_quantize_a(dev, M, pad):
    """lcml_fp8_gemm_quantize_a: dynamic per-tensor QuantizeLinear of an fp32
    A fused with the GEMM (one GEMV kernel for M <= 4, the quantize kernels
    and the GEMM otherwise). The scale and the codes are bit-exact against
    the oracle's amax / 448 and QuantizeLinear (a NaN in A is ignored by the
    amax and becomes code 0x7f), Y is bit-identical to lcml_fp8_gemm on those
    codes and within rtol 2e-3 / atol 1e-3 of the oracle's QDQ GEMM. pad > 0
    gives A a row stride of K + pad elements (fused path only)."""
    import torch
    import luisaml_b200 as lb
    N, K = 1000, 2048
    rng = np.random.default_rng(300 + M)
    A = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    A[0, 7] = np.nan
    Abig = np.zeros((M, K + pad), np.float32)
    Abig[:, :K] = A
    At = _t(Abig, dev)[:, :K]
    B = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    Bq, sb = oracle.quantize_dynamic_rows(B)
    Bt, sbt = _t(Bq, dev), _t(sb, dev)
    aq = torch.empty((M, K), dtype=torch.uint8, device=dev)
    Y, aq_out, s = lb.gemm_quantize_a(At, Bt, sbt, aq=aq, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert lb.device_error() == 0
    s_ref = oracle.scale_from_amax(np.nanmax(np.abs(A)))
    assert np.float32(s.item()) == s_ref
    codes = aq.cpu().numpy()
    np.testing.assert_array_equal(codes, oracle.quantize(A, s_ref))
    assert codes[0, 7] == 0x7f
    Y2 = lb.gemm(aq, Bt, s, sbt, out_dtype=torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(Y.cpu().numpy(), Y2.cpu().numpy())
    rows = np.arange(1, M)  # row 0 holds the NaN code: every output of it is NaN
    if rows.size:
        ref = oracle.qdq_gemm(codes[rows], np.float32([s_ref]), Bq, sb)
        assert_close(Y.cpu().numpy()[rows], ref, what=f"fused quantize-A GEMM M={M}")
    assert np.isnan(Y.cpu().numpy()[0]).all()
    if M <= 4:  # codes are optional on the fused path; an all-zero A gets scale 1
        Y3, none, s3 = lb.gemm_quantize_a(torch.zeros((M, K), device=dev), Bt, sbt, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert none is None and s3.item() == 1.0 and not Y3.cpu().numpy().any()
