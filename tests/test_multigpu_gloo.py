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

from rns8_b200.shard import row_slab


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
