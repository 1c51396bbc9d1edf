"""Host-side logic of the tensor-parallel GEMM on world_size-2 gloo ranks
(CPU): column shards tile [0, N) exactly, the block-seeded weight generator
reproduces the same B under any sharding, and the handle exchange the peer
mapping relies on (all_gather_object) delivers every rank's bytes."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from luisaml_b200 import tp
        N, K = 1280, 64
        start, stop = tp.shard_columns(N, world, rank)
        shard = tp.column_block_weights(torch, K, start, stop, "cpu", 77, 0.02)
        parts = [None] * world
        dist.all_gather_object(parts, (start, stop, shard))
        handles = [None] * world
        dist.all_gather_object(handles, bytes([rank]) * 64)
        if rank == 0:
            full = tp.column_block_weights(torch, K, 0, N, "cpu", 77, 0.02)
            ok_tiling = [p[:2] for p in parts] == [(0, 768), (768, 1280)]
            ok_data = torch.equal(torch.cat([p[2] for p in parts]), full)
            ok_handles = handles == [bytes([r]) * 64 for r in range(world)]
            result_q.put((ok_tiling, ok_data, ok_handles))
    finally:
        dist.destroy_process_group()


def test_tp_sharding_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == (True, True, True)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_columns_cover_exactly(world):
    from luisaml_b200 import tp
    N = 28672
    spans = [tp.shard_columns(N, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == N
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert all(s % 256 == 0 for s, _ in spans)
