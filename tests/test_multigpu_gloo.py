"""Host-side multi-GPU logic on CPU: world_size-2 gloo ranks shard the
output rows (rns8_b200.shard.row_slab), compute their slab with the CPU
oracle standing in for the device, gather, and agree with the unsharded
result; max-over-ranks timing is reduced the way bench.py does it."""

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from rns8_b200.shard import grid_shape, output_tile, row_slab


def test_row_slab_partitions_rows():
    for m in (0, 1, 7, 8192, 8193):
        for world in (1, 2, 3, 4, 8):
            spans = [row_slab(r, world, m) for r in range(world)]
            assert sum(rows for _, rows in spans) == m
            pos = 0
            for row0, rows in spans:
                assert row0 == pos
                pos += rows
            assert max(r for _, r in spans) - min(r for _, r in spans) <= 1
    with pytest.raises(ValueError):
        row_slab(2, 2, 10)


def test_output_tile_partitions_the_output():
    assert [grid_shape(w) for w in (1, 2, 3, 4, 6, 8)] == [(1, 1), (2, 1), (3, 1), (2, 2), (3, 2), (4, 2)]
    for m, n in ((8192, 8192), (4700, 4080), (7, 3), (1, 1)):
        for world in (1, 2, 3, 4, 8):
            cover = np.zeros((m, n), np.int32)
            for r in range(world):
                row0, rows, col0, cols = output_tile(r, world, m, n)
                cover[row0:row0 + rows, col0:col0 + cols] += 1
            assert (cover == 1).all()
    with pytest.raises(ValueError):
        output_tile(4, 4, 10, 10)


def _grid_worker(rank, world, port, m, n, k, q):
    from oracle import bridge

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(43)
    A = rng.integers(-(2**20), 2**20, (m, k), dtype=np.int64, endpoint=True)
    B = rng.integers(-(2**20), 2**20, (k, n), dtype=np.int64, endpoint=True)
    row0, rows, col0, cols = output_tile(rank, world, m, n)
    # Each rank touches only its row slab of A and column slab of B.
    st, C, _ = bridge.gemm_bounded_oneshot(np.ascontiguousarray(A[row0:row0 + rows]),
                                           np.ascontiguousarray(B[:, col0:col0 + cols]), k * 2**40)
    assert st == 0
    parts = [None] * world
    dist.all_gather_object(parts, (row0, col0, C))
    if rank == 0:
        full = np.zeros((m, n), np.int64)
        for r0, c0, c in parts:
            full[r0:r0 + c.shape[0], c0:c0 + c.shape[1]] = c
        st, want, _ = bridge.gemm_bounded_oneshot(A, B, k * 2**40)
        q.put(bool(np.array_equal(full, want)))
    dist.destroy_process_group()


def test_output_tile_gemm_four_gloo_ranks():
    """2 x 2 output blocks on four gloo ranks, each from its own A row slab and
    B column slab, gathered into the unsharded product."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_grid_worker, args=(r, 4, port, 67, 45, 33, q)) for r in range(4)]
    for p in procs:
        p.start()
    ok = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert ok


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, k, q):
    import torch

    from oracle import bridge

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(42)
    A = rng.integers(-(2**20), 2**20, (m, k), dtype=np.int64, endpoint=True)
    B = rng.integers(-(2**20), 2**20, (k, n), dtype=np.int64, endpoint=True)
    row0, rows = row_slab(rank, world, m)
    st, C, _ = bridge.gemm_bounded_oneshot(np.ascontiguousarray(A[row0:row0 + rows]), B, k * 2**40)
    assert st == 0
    parts = [None] * world
    dist.all_gather_object(parts, (row0, C))
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        full = np.zeros((m, n), np.int64)
        for r0, c in parts:
            full[r0:r0 + c.shape[0]] = c
        st, want, _ = bridge.gemm_bounded_oneshot(A, B, k * 2**40)
        q.put((bool(np.array_equal(full, want)), float(t.item())))
    dist.destroy_process_group()


def test_row_slab_gemm_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 37, 24, 40, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    ok, tmax = q.get(timeout=10)
    assert ok and tmax == 2.0


# ---- plane sharding: ownership, slabs and the IPC handle exchange ------------------
from rns8_b200.shard import PlaneExchange, plane_slabs, planes_of_rank, slab_of_rank


def test_plane_ownership_and_slabs():
    for prefix in (1, 9, 18, 20):
        for world in (1, 2, 3, 8):
            owned = sorted(p for r in range(world) for p in planes_of_rank(r, world, prefix))
            assert owned == list(range(prefix))  # every plane exactly once
    for m in (1, 127, 128, 1000, 4096, 8193):
        for world in (1, 2, 4, 8):
            slab_rows, count = plane_slabs(m, world)
            assert slab_rows % 128 == 0 and 1 <= count <= world
            spans = [slab_of_rank(r, m, world) for r in range(world)]
            assert sum(rows for _, rows in spans) == m
            assert all(rows > 0 for _, rows in spans[:count]) and all(rows == 0 for _, rows in spans[count:])


class _ShmIpc:
    """Stand-in for CUDA IPC on CPU: a buffer is POSIX shared memory, its
    handle the 64-byte padded name, an opened peer buffer a mapping of it."""

    HANDLE_BYTES = 64

    def __init__(self):
        self.live = {}

    def alloc(self, nbytes):
        from multiprocessing import shared_memory

        shm = shared_memory.SharedMemory(create=True, size=nbytes)
        self.live[id(shm)] = shm
        return id(shm), shm.name.encode().ljust(self.HANDLE_BYTES, b"\0")

    def open(self, handle):
        from multiprocessing import shared_memory

        shm = shared_memory.SharedMemory(name=handle.rstrip(b"\0").decode())
        self.live[id(shm)] = shm
        return id(shm)

    def view(self, ptr):
        return np.ndarray((self.live[ptr].size,), np.int8, buffer=self.live[ptr].buf)

    def close(self, ptr):
        self.live.pop(ptr).close()

    def free(self, ptr):
        shm = self.live.pop(ptr)
        shm.close()
        shm.unlink()


def _plane_worker(rank, world, port, m, n, k, prefix, q):
    from oracle import bridge

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(7)
    A = rng.integers(-(2**62), 2**62, (m, k), dtype=np.int64)
    B = rng.integers(-(2**62), 2**62, (k, n), dtype=np.int64)
    ipc = _ShmIpc()
    ex = PlaneExchange(ipc, rank, world, m, n, prefix, buffers=2)
    mine = planes_of_rank(rank, world, prefix)
    # This rank's planes of all of C (the oracle stands in for pack + GEMM) ...
    c_all = bridge.gemm_rns(bridge.pack(A, prefix), bridge.pack(B, prefix), prefix)
    # ... stored row by row into the slab owners' buffers, as the fused epilogue does.
    table = ex.slab_table(1)
    for s, ptr in enumerate(table):
        row0, rows = slab_of_rank(s, m, world)
        dst = ipc.view(ptr)[: prefix * rows * n].reshape(prefix, rows, n)
        for p in mine:
            dst[p] = c_all[p, row0:row0 + rows]
    dist.barrier()
    ok = True
    if ex.rows:
        got = ipc.view(ex.receive_buffer(1))[: prefix * ex.rows * n].reshape(prefix, ex.rows, n)
        st, limbs = bridge.export_limbs(np.ascontiguousarray(got), prefix, 3, True)
        st_all, want = bridge.export_limbs(c_all, prefix, 3, True)
        ok = st == 0 and st_all == 0 and np.array_equal(limbs, want[ex.row0:ex.row0 + ex.rows])
    dist.barrier()  # nobody unlinks a buffer a peer still maps
    ex.close()
    oks = [None] * world
    dist.all_gather_object(oks, ok)
    if rank == 0:
        q.put(all(oks))
    dist.destroy_process_group()


def test_plane_exchange_two_gloo_ranks():
    """Two ranks, 20 planes split 10/10, 200 output rows in 128-row slabs:
    every rank receives all planes of its slab and reconstructs it."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_plane_worker, args=(r, 2, port, 200, 24, 16, 20, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    assert q.get(timeout=10)
