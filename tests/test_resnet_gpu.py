"""ResNet-50-shaped QDQ conv networks through the executor (LuisaML-JSON ->
NetworkInstance): every DequantizeLinear -> Conv -> (Add) -> Relu ->
QuantizeLinear group must run as one fused FP8 conv, the max pool and the
global average pool on the e4m3 bytes, and the results must agree with the
oracle replaying the same graph (quantize/dequantize, conv.cpp's loop, max
pool, mean, gemm.cpp's loop).

Every activation is requantized to e4m3 with a static scale, so an fp32
summation-order difference that lands on an e4m3 rounding boundary moves
one code by one step, and in a deep network such flips compound from layer
to layer. The full ResNet-50 is therefore checked conv by conv: each fused
conv is replayed by the oracle from the executor's own e4m3 input (read back
through lcml_network_tensor), and its output codes must match except for
rare flips to the neighbouring code. Every other stage is held to the
oracle on the executor's own input: the max pool and the head quantization
bit for bit, the pooled values to fp32 summation order, the logits at the
GEMM tolerance (rtol 2e-3 / atol 1e-3).
"""
import numpy as np
import pytest

import oracle
from conftest import assert_close

pytestmark = pytest.mark.gpu


def _run(dev, text, blob, x, ncls, reuse=False):
    """Runs the graph; with reuse=False every intermediate keeps its own
    allocation, so the conv-by-conv checks can read them back."""
    import torch
    from luisaml_b200.session import Network
    net = Network(text)
    net.set_memory_reuse(reuse)
    y = torch.empty((x.shape[0], ncls), dtype=torch.float32, device=dev)
    net.set_weight_buffer(torch.from_numpy(np.frombuffer(blob, dtype=np.uint8).copy()).to(dev))
    net.set_input("x", torch.from_numpy(x).to(dev))
    net.set_output("logits", y)
    net.forward()
    torch.cuda.synchronize()
    return net, y.cpu().numpy()


def _codes_nchw(net, name):
    q = net.read_tensor(name)
    _, _, _, nhwc = net.tensor_info(name)
    return np.ascontiguousarray(q.transpose(0, 3, 1, 2)) if nhwc else q


def _structure(net, meta):
    s = net.summary()
    nconv = sum(1 for st in meta["plan"] if st[0] == "conv")
    assert s.count("implicit-GEMM conv") == nconv, s
    # input QuantizeLinear + convs + max pool + global average pool + Flatten (a view)
    # + head QuantizeLinear + head GEMM
    assert net.executed_nodes() == nconv + 6, s


def test_small_resnet_end_to_end(dev):
    """1 bottleneck block per stage, width 16, 64x64 images: shallow enough
    that the whole forward matches the oracle end to end."""
    from luisaml_b200 import graphs
    text, blob, meta = graphs.resnet50(batch=2, image=64, width=16, blocks=(1, 1, 1, 1), num_classes=10)
    x = np.random.default_rng(4001).standard_normal((2, 3, 64, 64)).astype(np.float32)
    net, got = _run(dev, text, blob, x, 10)
    _structure(net, meta)
    ref = oracle.replay_plan(meta["plan"], x)
    assert_close(got, ref, what="small resnet logits")


def _one_step_apart(got_codes, want_codes):
    """Whether every differing pair of codes is one e4m3 step apart (the
    spacing of the larger magnitude: 2^(e-3) for normals, 2^-9 below 2^-6)."""
    g = oracle.e4m3_decode(got_codes).astype(np.float64)
    w = oracle.e4m3_decode(want_codes).astype(np.float64)
    m = np.maximum(np.abs(g), np.abs(w))
    spacing = np.where(m >= 2.0 ** -6, 2.0 ** (np.floor(np.log2(np.maximum(m, 2.0 ** -6))) - 3), 2.0 ** -9)
    return bool((np.abs(g - w) <= spacing * (1 + 1e-9)).all())


def _image_codes(net, name, imgs):
    """e4m3 codes of the given images of an activation, NCHW, copied straight
    from the device tensor (NHWC tensors hold each image contiguously)."""
    import luisaml_b200 as lb
    ptr, _, shape, nhwc = net.tensor_info(name)
    n = shape[0]
    per = int(np.prod(shape[1:]))
    out = np.empty((len(imgs), per), dtype=np.uint8)
    for i, im in enumerate(imgs):
        assert 0 <= im < n
        lb.check(lb.lib().lcml_memcpy_async(out[i].ctypes.data, ptr + im * per, per, 2, None))
    lb.check(lb.lib().lcml_stream_synchronize(None))
    if nhwc and len(shape) == 4:
        return np.ascontiguousarray(out.reshape(len(imgs), shape[2], shape[3], shape[1]).transpose(0, 3, 1, 2))
    return out.reshape((len(imgs),) + tuple(shape[1:]))


def _check_convs(net, meta, imgs):
    """Every fused conv replayed by the oracle from the executor's own e4m3
    input (and residual) codes of `imgs`: output codes equal except for rare
    flips to the neighbouring code. Returns the worst flip rate."""
    worst = 0.0
    for c in meta["conv_io"]:
        _, wq, ws, bias, stride, pad = c["conv"]
        h = oracle.conv2d(oracle.dequantize(_image_codes(net, c["x"], imgs), c["x_scale"]),
                          oracle.dequantize(wq, ws, axis=0), bias, strides=(stride, stride), pads=(pad, pad, pad, pad))
        if c["res"] is not None:
            h = (h + oracle.dequantize(_image_codes(net, c["res"], imgs), c["res_scale"])).astype(np.float32)
        if c["relu"]:
            h = oracle.relu(h)
        want = oracle.quantize(h, c["y_scale"])
        gotc = _image_codes(net, c["y"], imgs)
        diff = gotc != want
        frac = float(diff.mean())
        worst = max(worst, frac)
        assert frac <= 1e-4, (c["y"], frac)
        assert _one_step_apart(gotc[diff], want[diff]), c["y"]
    return worst


def _check_pool(net, meta, imgs):
    """The e4m3 max pool works on codes: exact."""
    stem, pool = meta["conv_io"][0]["y"], meta["segments"][0][2]
    s = meta["conv_io"][0]["y_scale"]
    want = oracle.quantize(oracle.maxpool2d(oracle.dequantize(_image_codes(net, stem, imgs), s), (3, 3), (2, 2),
                                            (1, 1, 1, 1)), s)
    np.testing.assert_array_equal(_image_codes(net, pool, imgs), want)


def _check_head(net, meta, got):
    """The head stage by stage, each stage fed the executor's own input:
    GlobalAveragePool of the last block's codes (fp32 mean: summation order
    only), the head QuantizeLinear of the executor's pooled values (bit-exact
    e4m3 codes), and the QDQ classifier Gemm on the executor's head codes at
    rtol 2e-3 / atol 1e-3 on every logit."""
    src, s_in, _, _, steps = meta["segments"][-1]
    n = got.shape[0]
    last = _image_codes(net, src, list(range(n)))
    gap_ref = oracle.global_avgpool(oracle.dequantize(last, s_in)).reshape(n, -1)
    gap = net.read_tensor("gap_out").reshape(n, -1)
    assert_close(gap, gap_ref, rtol=1e-5, atol=1e-6, what="global average pool")
    s_fc = [st for st in meta["plan"] if st[0] == "qdq"][-1][1]
    fc_q = net.read_tensor("fc_in_q")
    np.testing.assert_array_equal(fc_q, oracle.quantize(gap, s_fc))
    _, wq, ws, bias = steps[-1]
    ref = oracle.qdq_gemm(fc_q, np.float32([s_fc]), wq, ws, bias=bias)
    assert_close(got, ref, what="classifier logits")


def test_resnet50_conv_by_conv_vs_oracle(dev):
    """Full ResNet-50 v1.5 at 224x224 (batch 2). Every one of the 53 fused
    convs is replayed by the oracle from the executor's own e4m3 input (and
    residual) codes: its output codes must match except for rare flips to the
    neighbouring code. The e4m3 max pool must match exactly, the head stage
    by stage (pool, bit-exact head quantization, logits at rtol 2e-3 /
    atol 1e-3)."""
    from luisaml_b200 import graphs
    text, blob, meta = graphs.resnet50(batch=2, image=224)
    x = np.random.default_rng(4002).standard_normal((2, 3, 224, 224)).astype(np.float32)
    net, got = _run(dev, text, blob, x, 1000)
    _structure(net, meta)
    assert np.isfinite(got).all()
    assert len(meta["conv_io"]) == 53
    worst = _check_convs(net, meta, [0, 1])
    print(f"53 convs: worst flip rate {worst:.5%}")
    _check_pool(net, meta, [0, 1])
    _check_head(net, meta, got)
    # the lifetime-planned arena (the default) gives the same logits bit for bit
    net2, got2 = _run(dev, text, blob, x, 1000, reuse=True)
    np.testing.assert_array_equal(got2, got)
    arena, unplanned = net2.memory()
    assert arena < unplanned / 3, (arena, unplanned)


def test_resnet50_batch128_sampled_images(dev):
    """The configuration's batch of 128 (224x224): the conv-by-conv and pool
    checks on three sampled images (first, middle, last: the implicit-GEMM
    tiles of the full batch straddle images), the head on all 128."""
    from luisaml_b200 import graphs
    text, blob, meta = graphs.resnet50(batch=128, image=224)
    x = np.random.default_rng(4003).standard_normal((128, 3, 224, 224)).astype(np.float32)
    net, got = _run(dev, text, blob, x, 1000)
    _structure(net, meta)
    assert np.isfinite(got).all()
    imgs = [0, 77, 127]
    worst = _check_convs(net, meta, imgs)
    print(f"batch 128, images {imgs}: worst conv flip rate {worst:.5%}")
    _check_pool(net, meta, imgs)
    _check_head(net, meta, got)
    del net
    net2, got2 = _run(dev, text, blob, x, 1000, reuse=True)
    np.testing.assert_array_equal(got2, got)
    arena, unplanned = net2.memory()
    print(f"batch 128 intermediates: {arena / 2**20:.0f} MiB in the arena vs {unplanned / 2**20:.0f} MiB unplanned")
    assert arena < unplanned / 3, (arena, unplanned)
