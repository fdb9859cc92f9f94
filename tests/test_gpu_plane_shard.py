"""Plane sharding on the GPU: the pack of selected planes, and the plane GEMM
whose epilogue scatters output row slabs into per-slab buffers (the fused
exchange) or copies them there (the copy form). On one GPU the ranks are
emulated: every virtual rank computes its planes into all slabs' buffers,
which are this GPU's memory; the result must equal, byte for byte, the
unsharded plane GEMM and the oracle. With two or more GPUs the same runs
across processes over NVLink (CUDA IPC peer buffers, an NCCL barrier)."""

from __future__ import annotations

import ctypes as C
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

FUSED, COPY = 0, 1


@pytest.fixture(scope="module")
def lib():
    import rns8_b200

    return rns8_b200.lib()


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def u32s(values):
    return (C.c_uint32 * len(values))(*values)


def pack_full(lib, src, signed, prefix):
    rows, cols = src.shape
    out = torch.empty((prefix, rows, cols), dtype=torch.int8, device="cuda")
    fn = lib.rns8_cuda_pack_i64_device if signed else lib.rns8_cuda_pack_u64_device
    assert fn(0, src.data_ptr(), rows, cols, src.stride(0), prefix, out.data_ptr(), stream()) == 0
    return out


def pack_subset(lib, src, signed, planes):
    rows, cols = src.shape
    out = torch.empty((len(planes), rows, cols), dtype=torch.int8, device="cuda")
    fn = lib.rns8_cuda_pack_i64_planes_device if signed else lib.rns8_cuda_pack_u64_planes_device
    assert fn(0, src.data_ptr(), rows, cols, src.stride(0), u32s(planes), len(planes), out.data_ptr(), stream()) == 0
    return out


@pytest.mark.parametrize("signed", [True, False])
@pytest.mark.parametrize("rows,cols,ld", [(96, 64, 64), (33, 20, 24), (5, 7, 7)])
@pytest.mark.parametrize("planes", [[1, 9, 17], [0], [19, 3, 5, 7, 2, 11, 13, 0, 1, 4, 6, 8]])
def test_pack_selected_planes(lib, signed, rows, cols, ld, planes):
    g = torch.Generator(device="cuda").manual_seed(rows * cols + len(planes))
    src = torch.randint(-(2**63), 2**63 - 1, (rows, ld), dtype=torch.int64, device="cuda", generator=g)
    src[0, : min(cols, 6)] = torch.tensor([-1, 0, 1, -(2**63), 2**63 - 1, -128], dtype=torch.int64)[: min(cols, 6)]
    view = src[:, :cols]
    full = pack_full(lib, view, signed, 20)
    sub = pack_subset(lib, view, signed, planes)
    torch.cuda.synchronize()
    for j, p in enumerate(planes):
        assert torch.equal(sub[j], full[p]), (j, p)


def run_virtual_ranks(lib, ra_full, rb_full, m, n, k, prefix, world, exchange):
    """Every virtual rank multiplies its planes and scatters them into the
    slab buffers; returns the slab buffers and the fused flags seen."""
    from rns8_b200.shard import plane_slabs, planes_of_rank, slab_of_rank

    slab_rows, count = plane_slabs(m, world)
    slabs = [torch.full((prefix, slab_of_rank(s, m, world)[1], n), 77, dtype=torch.int8, device="cuda")
             for s in range(count)]
    table = (C.c_void_p * count)(*[t.data_ptr() for t in slabs])
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    fused_seen = []
    for r in range(world):
        mine = planes_of_rank(r, world, prefix)
        if not mine:
            continue
        a = ra_full[mine].contiguous()
        b = rb_full[mine].contiguous()
        sb = lib.rns8_cuda_gemm_rns_slabs_scratch_bytes(0, m, n, k, len(mine), exchange)
        scratch = torch.empty(max(sb, 1), dtype=torch.uint8, device="cuda")
        fused = C.c_uint32(9)
        st = lib.rns8_cuda_gemm_rns_slabs_device(0, a.data_ptr(), b.data_ptr(), m, n, k, u32s(mine), len(mine), table,
                                                 count, slab_rows, exchange, scratch.data_ptr(), sb,
                                                 status.data_ptr(), C.byref(fused), stream())
        assert st == 0
        fused_seen.append(fused.value)
        torch.cuda.synchronize()
    assert int(status[0].item()) == 0
    return slabs, fused_seen


@pytest.mark.parametrize("m,n,k,world,fusable", [
    (1000, 256, 320, 2, True),   # ragged last slab, tensor cores, no split-K
    (1000, 256, 320, 8, True),   # 8 slabs of 128 rows, 2-3 planes per rank
    (512, 128, 2048, 3, False),  # few tiles: split-K, so the copy form runs
    (200, 40, 48, 2, False),     # N not a multiple of 16: SIMT GEMM, copy form
])
@pytest.mark.parametrize("exchange", [FUSED, COPY])
def test_slab_scatter_equals_unsharded_gemm(lib, oracle, m, n, k, world, fusable, exchange):
    from rns8_b200.shard import slab_of_rank

    prefix = 20
    g = torch.Generator(device="cuda").manual_seed(m + n + k + world)
    A = torch.randint(-(2**63), 2**63 - 1, (m, k), dtype=torch.int64, device="cuda", generator=g)
    B = torch.randint(-(2**63), 2**63 - 1, (k, n), dtype=torch.int64, device="cuda", generator=g)
    ra, rb = pack_full(lib, A, True, prefix), pack_full(lib, B, True, prefix)
    rc = torch.empty((prefix, m, n), dtype=torch.int8, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    sb = lib.rns8_cuda_gemm_rns_scratch_bytes(0, m, n, k, prefix)
    scratch = torch.empty(max(sb, 1), dtype=torch.uint8, device="cuda")
    assert lib.rns8_cuda_gemm_rns_device(0, ra.data_ptr(), rb.data_ptr(), rc.data_ptr(), m, n, k, prefix, 0,
                                         scratch.data_ptr(), sb, status.data_ptr(), stream()) == 0
    slabs, fused = run_virtual_ranks(lib, ra, rb, m, n, k, prefix, world, exchange)
    assert all(f == (1 if (fusable and exchange == FUSED) else 0) for f in fused), fused
    for s, buf in enumerate(slabs):
        row0, rows = slab_of_rank(s, m, world)
        assert torch.equal(buf, rc[:, row0:row0 + rows]), s
    if m * n <= 256 * 256:  # the oracle on the small cases
        want = oracle.gemm_rns(oracle.pack(A.cpu().numpy(), prefix), oracle.pack(B.cpu().numpy(), prefix), prefix)
        np.testing.assert_array_equal(torch.cat(slabs, dim=1).cpu().numpy(), want)


def test_slab_scatter_rejects_bad_layouts(lib):
    a = torch.zeros((1, 256, 64), dtype=torch.int8, device="cuda")
    b = torch.zeros((1, 64, 128), dtype=torch.int8, device="cuda")
    d = torch.zeros((21, 256, 128), dtype=torch.int8, device="cuda")  # room for any plane slot of either slab
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    one = (C.c_void_p * 1)(d.data_ptr())
    two = (C.c_void_p * 2)(d.data_ptr(), d.data_ptr())
    call = lambda table, count, rows, planes=(3,): lib.rns8_cuda_gemm_rns_slabs_device(
        0, a.data_ptr(), b.data_ptr(), 256, 128, 64, u32s(list(planes)), len(planes), table, count, rows, FUSED,
        None, 0, status.data_ptr(), None, stream())
    INVALID = 1
    assert call(one, 1, 128) == INVALID       # one slab of 128 rows cannot hold 256
    assert call(two, 2, 256) == INVALID       # the second slab would be empty
    assert call(two, 2, 128, (20,)) == INVALID  # plane index beyond the ladder
    assert call(two, 2, 128) == 0  # both slabs in one buffer: rows 0-127 of plane slot 3, written twice
    torch.cuda.synchronize()


# ---- two or more GPUs: real peers ---------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _peer_worker(rank, world, port, m, n, k, q):
    import torch.distributed as dist

    import rns8_b200
    from rns8_b200.shard import LibraryIpc, PlaneExchange, planes_of_rank

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    lib = rns8_b200.lib()
    prefix = 20
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.randint(-(2**63), 2**63 - 1, (m, k), dtype=torch.int64, device="cuda", generator=g)
    B = torch.randint(-(2**63), 2**63 - 1, (k, n), dtype=torch.int64, device="cuda", generator=g)
    ex = PlaneExchange(LibraryIpc(lib, rank), rank, world, m, n, prefix, buffers=1)
    mine = planes_of_rank(rank, world, prefix)
    idx = (C.c_uint32 * len(mine))(*mine)
    ra = torch.empty((len(mine), m, k), dtype=torch.int8, device="cuda")
    rb = torch.empty((len(mine), k, n), dtype=torch.int8, device="cuda")
    assert lib.rns8_cuda_pack_i64_planes_device(rank, A.data_ptr(), m, k, k, idx, len(mine), ra.data_ptr(), sp) == 0
    assert lib.rns8_cuda_pack_i64_planes_device(rank, B.data_ptr(), k, n, n, idx, len(mine), rb.data_ptr(), sp) == 0
    table = (C.c_void_p * ex.slab_count)(*ex.slab_table(0))
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    fused = C.c_uint32(9)
    dist.barrier()
    assert lib.rns8_cuda_gemm_rns_slabs_device(rank, ra.data_ptr(), rb.data_ptr(), m, n, k, idx, len(mine), table,
                                               ex.slab_count, ex.slab_rows, FUSED, None, 0, status.data_ptr(),
                                               C.byref(fused), sp) == 0
    flag = torch.ones(1, device="cuda")
    dist.all_reduce(flag)  # every rank's scatter has completed
    ok = True
    if ex.rows:
        out = torch.empty((ex.rows, n, 3), dtype=torch.int64, device="cuda")
        assert lib.rns8_cuda_export_limbs_device(rank, ex.receive_buffer(0), ex.rows, n, prefix, 1, 3,
                                                 out.data_ptr(), n, status.data_ptr(), sp) == 0
        # The unsharded path on this GPU for the same rows.
        fa = torch.empty((prefix, ex.rows, k), dtype=torch.int8, device="cuda")
        fb = torch.empty((prefix, k, n), dtype=torch.int8, device="cuda")
        fc = torch.empty((prefix, ex.rows, n), dtype=torch.int8, device="cuda")
        Aslab = A[ex.row0:ex.row0 + ex.rows].contiguous()
        assert lib.rns8_cuda_pack_i64_device(rank, Aslab.data_ptr(), ex.rows, k, k, prefix, fa.data_ptr(), sp) == 0
        assert lib.rns8_cuda_pack_i64_device(rank, B.data_ptr(), k, n, n, prefix, fb.data_ptr(), sp) == 0
        sb = lib.rns8_cuda_gemm_rns_scratch_bytes(rank, ex.rows, n, k, prefix)
        scratch = torch.empty(max(sb, 1), dtype=torch.uint8, device="cuda")
        assert lib.rns8_cuda_gemm_rns_device(rank, fa.data_ptr(), fb.data_ptr(), fc.data_ptr(), ex.rows, n, k, prefix,
                                             0, scratch.data_ptr(), sb, status.data_ptr(), sp) == 0
        want = torch.empty_like(out)
        assert lib.rns8_cuda_export_limbs_device(rank, fc.data_ptr(), ex.rows, n, prefix, 1, 3, want.data_ptr(), n,
                                                 status.data_ptr(), sp) == 0
        torch.cuda.synchronize()
        ok = bool(torch.equal(out, want)) and int(status[0].item()) == 0 and fused.value == 1
    dist.barrier()
    ex.close()
    oks = [None] * world
    dist.all_gather_object(oks, ok)
    if rank == 0:
        q.put(all(oks))
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_plane_exchange_across_gpus():
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, 1000, 256, 320, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    assert q.get(timeout=10)
