"""Tensor-parallel FP8 GEMM (N-column split) with the all-gather fused into
the GEMM epilogue.

Each rank holds all of A (quantized per token locally) and a column shard of
B; its GEMM stores every output tile both into its own full-size output and,
over NVLink, into the same place of every other rank's output (peer buffers
mapped with CUDA IPC). After one barrier every rank holds the whole
[M, N] row-major result: the all-gather happens while the GEMM runs, with no
separate collective and no re-layout pass.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _capi
from ._capi import check

BLOCK = 256  # column-block granularity of shards and of the seeded weight generator


def shard_columns(n: int, world: int, rank: int):
    """[start, stop) columns of rank's shard; shards are whole 256-column blocks."""
    blocks = (n + BLOCK - 1) // BLOCK
    per = (blocks + world - 1) // world
    start = min(rank * per * BLOCK, n)
    stop = min((rank + 1) * per * BLOCK, n)
    return start, stop


def column_block_weights(torch, k: int, start: int, stop: int, device, base_seed: int, std: float):
    """B[:, start:stop]^T as fp32 [stop - start, k], generated block by block
    (seed = base_seed + block index) so any sharding reproduces the same B."""
    rows = []
    for c0 in range(start, stop, BLOCK):
        c1 = min(c0 + BLOCK, stop)
        g = torch.Generator(device=device).manual_seed(base_seed + c0 // BLOCK)
        blk = torch.randn((BLOCK, k), generator=g, device=device) * std
        rows.append(blk[: c1 - c0])
    return torch.cat(rows) if rows else torch.empty((0, k), device=device)


class PeerOutputs:
    """A full-size output buffer on every rank, each mapped into every other
    rank's address space (CUDA IPC), plus the device array of peer pointers
    the GEMM epilogue writes through."""

    def __init__(self, torch, dist, nbytes: int, device):
        lib = _capi.load()
        self.lib, self.torch = lib, torch
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        self.nbytes = nbytes
        p = ctypes.c_void_p()
        check(lib.lcml_device_alloc(nbytes, ctypes.byref(p)))
        self.local = p.value
        handle = (ctypes.c_uint8 * 64)()
        check(lib.lcml_ipc_get_handle(ctypes.c_void_p(self.local), handle))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle))
        self.peers = []
        for r in range(self.world):
            if r == self.rank:
                continue
            q = ctypes.c_void_p()
            h = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
            check(lib.lcml_ipc_open(h, ctypes.byref(q)))
            self.peers.append(q.value)
        self.peer_array = torch.tensor(self.peers or [0], dtype=torch.int64, device=device)

    def close(self):
        for q in self.peers:
            self.lib.lcml_ipc_close(ctypes.c_void_p(q))
        self.peers = []
        if self.local:
            self.lib.lcml_device_free(ctypes.c_void_p(self.local))
            self.local = None

    def to_host(self, shape, dtype):
        """Copies the local full output to a host numpy array (synchronous)."""
        torch = self.torch
        out = torch.empty(shape, dtype=dtype)
        torch.cuda.synchronize()
        check(self.lib.lcml_memcpy_async(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(self.local),
                                         out.numel() * out.element_size(), 2, None))
        check(self.lib.lcml_stream_synchronize(None))
        return out


class PeerExchange:
    """The step's two small exchanges over NVLink (lcml_peer_exchange_max):
    the max of one device float across the ranks, and a barrier. Each rank's
    slot array (LCML_PEER_SLOTS_BYTES) is mapped into every other rank and
    zeroed before any rank may write into it; every rank then runs the same
    sequence of exchanges, which numbers them (epochs 1, 2, ...)."""

    def __init__(self, torch, dist, device, timeout_us: int = 2_000_000):
        lib = _capi.load()
        self.lib = lib
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        self.timeout_us = timeout_us
        self.buf = PeerOutputs(torch, dist, _capi.PEER_SLOTS_BYTES, device)
        check(lib.lcml_memset_async(ctypes.c_void_p(self.buf.local), 0, _capi.PEER_SLOTS_BYTES, None))
        check(lib.lcml_stream_synchronize(None))
        dist.barrier()  # every rank's slots are zero before any rank writes into them
        self.epoch = 0

    def _run(self, value, out, stream):
        self.epoch += 1
        check(self.lib.lcml_peer_exchange_max(
            ctypes.c_void_p(value), ctypes.c_void_p(out), ctypes.c_void_p(self.buf.local),
            ctypes.c_void_p(self.buf.peer_array.data_ptr()), self.rank, self.world, self.epoch, self.timeout_us,
            ctypes.c_void_p(stream)))

    def max(self, value_ptr: int, out_ptr: int, stream: int):
        """*out = max over the ranks of *value (device floats), enqueued on `stream`."""
        self._run(value_ptr, out_ptr, stream)

    def barrier(self, stream: int):
        """Returns (on the device) once every rank has reached this point of its stream."""
        self._run(None, None, stream)

    def close(self):
        self.buf.close()
