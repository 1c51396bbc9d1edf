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
