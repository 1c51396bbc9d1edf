"""Tensor-parallel FP8 GEMM with the all-gather fused into the epilogue, on
two GPUs (skipped when fewer are visible): every rank must end up with the
whole row-major output, equal to the oracle on the full problem."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, K, N, q):
    import ctypes
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    import luisaml_b200 as lb
    from luisaml_b200 import tp
    try:
        A = torch.randn((M, K), generator=torch.Generator(device=dev).manual_seed(11), device=dev)
        start, stop = tp.shard_columns(N, world, rank)
        Bt = tp.column_block_weights(torch, K, start, stop, dev, 21, 0.05)
        Bq, sb = lb.quantize_rows_dynamic(Bt)
        Aq, sa = lb.quantize_rows_dynamic(A)
        out = tp.PeerOutputs(torch, dist, M * N * 4, dev)
        d, _ = lb.gemm(Aq, Bq, sa, sb, out_dtype=torch.float32, desc_only=True)
        d.Y, d.ldy, d.y_col_offset = out.local, N, start
        d.y_peers, d.y_num_peers = out.peer_array.data_ptr(), world - 1
        lb.check(lb.lib().lcml_fp8_gemm(ctypes.byref(d), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()
        dist.barrier()
        full = out.to_host((M, N), torch.float32).numpy()
        shards = [None] * world
        dist.all_gather_object(shards, (start, Bq.cpu().numpy(), sb.cpu().numpy()))
        if rank == 0:
            q.put((full, Aq.cpu().numpy(), sa.cpu().numpy(), shards))
        else:
            q.put(("rank1", full))
        dist.barrier()
        out.close()
    finally:
        dist.destroy_process_group()


def test_fused_allgather_two_gpus():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import oracle
    from conftest import assert_close
    M, K, N = 512, 256, 1536
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, M, K, N, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    r0 = next(r for r in res if not isinstance(r[0], str))
    r1 = next(r for r in res if isinstance(r[0], str))
    full, aq, sa, shards = r0
    bq = np.concatenate([s[1] for s in shards])
    sb = np.concatenate([s[2] for s in shards])
    ref = oracle.qdq_gemm(aq, sa, bq, sb)
    assert_close(full, ref, what="rank 0 gathered output")
    assert np.array_equal(full, r1[1]), "ranks hold different outputs"


def test_tp_config_shape_one_gpu(dev):
    """The configuration's TP GEMM problem on one GPU, 16384 x 8192 x 28672:
    A ~N(0,1) per-token dynamically quantized, B ~N(0,0.02) per-column e4m3,
    bf16 out (the CTA-pair kernel). Per-token codes and scales bit-exact on
    sampled rows, per-column codes and scales on sampled columns, and sampled
    full rows of Y (all 28672 columns, full K) at rtol 2e-3 / atol 1e-3 plus
    the bf16 half ulp."""
    import torch
    import luisaml_b200 as lb
    import oracle
    from conftest import assert_close_bf16
    from luisaml_b200 import tp
    M, K, N = 16384, 8192, 28672
    A = torch.randn((M, K), generator=torch.Generator(device=dev).manual_seed(5000), device=dev)
    Bt = tp.column_block_weights(torch, K, 0, N, dev, 5100, 0.02)
    Bq, sb = lb.quantize_rows_dynamic(Bt)  # per-column scales of B = per-row of B^T
    Aq, sa = lb.quantize_rows_dynamic(A)
    Y = lb.gemm(Aq, Bq, sa, sb, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert lb.device_error() == 0
    rng = np.random.default_rng(8)
    rows = np.unique(np.concatenate([[0, 255, 256, M - 1], rng.integers(0, M, 4)]))
    cols = np.unique(np.concatenate([[0, 127, 128, N - 1], rng.integers(0, N, 8)]))
    ri = torch.from_numpy(rows).to(dev)
    ci = torch.from_numpy(cols).to(dev)
    aq_ref, sa_ref = oracle.quantize_dynamic_rows(A[ri].cpu().numpy())
    assert np.array_equal(Aq[ri].cpu().numpy(), aq_ref) and np.array_equal(sa[ri].cpu().numpy(), sa_ref)
    bq_ref, sb_ref = oracle.quantize_dynamic_rows(Bt[ci].cpu().numpy())
    assert np.array_equal(Bq[ci].cpu().numpy(), bq_ref) and np.array_equal(sb[ci].cpu().numpy(), sb_ref)
    del Bt, A
    ref = oracle.qdq_gemm(aq_ref, sa_ref, Bq.cpu().numpy(), sb.cpu().numpy())
    assert_close_bf16(Y[ri].float().cpu().numpy(), ref, what="TP GEMM at the config shape (sampled rows)")


def test_same_process_two_devices():
    """One process drives the CTA-pair GEMM and an implicit-GEMM conv on
    device 0 and then on device 1: the kernels' shared-memory limits are set
    per device, so the second device's launches must work and give the same
    results (skipped with fewer than 2 GPUs)."""
    import ctypes
    import torch
    import luisaml_b200 as lb
    import oracle
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from conftest import assert_close
    from test_conv_gpu import _run_conv
    rng = np.random.default_rng(12)
    M, N, K = 512, 512, 1024
    Aq, sa = oracle.quantize_dynamic_rows(rng.standard_normal((M, K)).astype(np.float32))
    Bq, sb = oracle.quantize_dynamic_rows((rng.standard_normal((N, K)) * 0.05).astype(np.float32))
    ref = oracle.qdq_gemm(Aq, sa, Bq, sb)
    X = rng.standard_normal((2, 64, 14, 14)).astype(np.float32)
    W = (rng.standard_normal((64, 64, 3, 3)) * 0.05).astype(np.float32)
    results = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
            Y = lb.gemm(t(Aq), t(Bq), t(sa), t(sb), out_dtype=torch.float32, variant=2)  # CTA pair
            torch.cuda.synchronize(dev)
            assert_close(Y.cpu().numpy(), ref, what=f"CTA-pair GEMM on device {d}")
            got, cref, ws = _run_conv(dev, X, W, None, 1, 1)
            assert ws == 0  # the implicit GEMM (TMA im2col), no workspace
            assert_close(got, cref, what=f"implicit-GEMM conv on device {d}")
            results.append((Y.cpu().numpy(), got))
    np.testing.assert_array_equal(results[0][0], results[1][0])
    np.testing.assert_array_equal(results[0][1], results[1][1])


def _row_split_worker(rank, world, port, q, shape=(1024, 768, 1024)):
    import datetime
    import sys
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      WORLD_SIZE=str(world), RANK=str(rank))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    import luisaml_b200 as lb
    try:
        wl = bench.GemmWorkload(*shape, "row_split_test")
        wl.setup(dev, 77)
        stream = torch.cuda.current_stream(dev)
        for _ in range(2):  # the second step overwrites the first's output with the same values
            wl.step(stream)
        torch.cuda.synchronize()
        assert lb.device_error() == 0
        full = wl.peers.to_host((wl.M, wl.N), torch.bfloat16).view(torch.int16).numpy()
        rows = [None] * world
        dist.all_gather_object(rows, wl.A.cpu().numpy())
        q.put((rank, full, np.concatenate(rows), wl.Bq.cpu().numpy(), float(wl.sb.item()), float(wl.sa.item())))
        dist.barrier()
        wl.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape", [(1024, 768, 1024), (5120, 2048, 2048)])
def test_row_split_gemm_two_gpus(shape):
    """The headline GEMM step under torchrun (bench.GemmWorkload, M split over
    2 ranks): the amax exchange gives each rank the whole tensor's scale,
    and the GEMM epilogue's peer stores leave the full Y on every rank. Both
    ranks' Y must be equal bit for bit and equal to one GPU running the same
    problem unsplit (per-tensor dynamic quantize of all of A, then the GEMM).
    The second shape runs each rank's 2560 rows on the CTA-pair kernel with
    split tiles at the end of its schedule (80 tiles of 256 x 256 on 74
    pairs) and the peer stores in the pair epilogue."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import luisaml_b200 as lb
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_row_split_worker, args=(r, 2, port, q, shape)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    (_, y0, A, Bq, sb, sa0), (_, y1, _, _, _, sa1) = res
    np.testing.assert_array_equal(y0, y1)
    dev = torch.device("cuda", 0)
    At = torch.from_numpy(A).to(dev)
    Aq, sa = lb.quantize_tensor_dynamic(At)
    assert sa.item() == sa0 == sa1
    Y = lb.gemm(Aq, torch.from_numpy(Bq).to(dev), sa, torch.tensor([sb], device=dev), out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(Y.view(torch.int16).cpu().numpy(), y0)


def test_peer_exchange_one_gpu(dev):
    """lcml_peer_exchange_max on one GPU: with world = 1 it returns the rank's
    own value; with world = 2 and a stand-in peer array in local memory that
    no rank writes back into, rank 0's wait for slot 1 runs out after the
    20 ms limit: the kernel returns, records device error 5, leaves *out as it
    was, and has written its own word into the stand-in peer's slot 0."""
    import ctypes
    import torch
    import luisaml_b200 as lb
    lib = lb.lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    nslot = lb._capi.PEER_SLOTS_BYTES // 8
    slots = torch.zeros(nslot, dtype=torch.int64, device=dev)
    val = torch.tensor([3.25], device=dev)
    out = torch.full((1,), -7.0, device=dev)
    lb.check(lib.lcml_peer_exchange_max(p(val), p(out), p(slots), None, 0, 1, 1, 1_000_000, st))
    torch.cuda.synchronize()
    assert out.item() == 3.25 and lb.device_error() == 0
    peer = torch.zeros(nslot, dtype=torch.int64, device=dev)
    peer_ptrs = torch.tensor([peer.data_ptr()], dtype=torch.int64, device=dev)
    slots.zero_()
    out.fill_(-7.0)
    lb.check(lib.lcml_peer_exchange_max(p(val), p(out), p(slots), p(peer_ptrs), 0, 2, 1, 20_000, st))
    torch.cuda.synchronize()
    assert lb.device_error() == 5
    assert out.item() == -7.0
    word = int(peer[32 + 0].item()) & 0xFFFFFFFFFFFFFFFF  # epoch 1 -> bank 1 (slots 32..63), slot of rank 0
    assert word >> 32 == 1 and np.uint32(word & 0xFFFFFFFF).view(np.float32) == np.float32(3.25)
    with pytest.raises(lb._capi.LcmlError):
        lb.check(lib.lcml_peer_exchange_max(p(val), p(out), p(slots), None, 0, 1, 0, 1000, st))  # epoch 0


def _exchange_worker(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    import luisaml_b200 as lb
    from luisaml_b200 import tp
    try:
        x = tp.PeerExchange(torch, dist, dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        got = []
        out = torch.zeros(1, device=dev)
        for i in range(6):  # successive epochs use alternate banks; the max moves between the ranks
            v = torch.tensor([float(10 * i + (rank if i % 2 else world - 1 - rank))], device=dev)
            x.max(v.data_ptr(), out.data_ptr(), stream)
            x.barrier(stream)
            torch.cuda.synchronize()
            got.append(out.item())
        q.put((rank, got, lb.device_error()))
        dist.barrier()
        x.close()
    finally:
        dist.destroy_process_group()


def test_peer_exchange_two_gpus():
    """Max of one float and barriers over NVLink between two ranks, six
    exchanges (both slot banks, each rank holding the max in turn)."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    want = [float(10 * i + 1) for i in range(6)]
    for rank, got, err in res:
        assert err == 0, (rank, err)
        assert got == want, (rank, got)
