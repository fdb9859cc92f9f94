"""The 2-D output partition of the strong-scaling split (rns8_b200.shard.output_tile)
on one GPU: every rank's block is computed as that rank computes it — pack its
row slab of A (compact) and its column slab of B (read in place with ld = n),
plane GEMM, export into a block-sized output — and all blocks together must
equal, bit for bit, the unsharded pipeline, which is checked against the
oracle on sampled rows. Ranks are emulated one after another on cuda:0; the
split has no exchange, so nothing else differs across GPUs."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    import rns8_b200

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return rns8_b200.lib()


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def product(lib, A, B, row0, rows, col0, cols, P, bound):
    """The block [row0, row0+rows) x [col0, col0+cols) of A x B through the device seam."""
    k, n = B.shape
    ra = torch.empty((P, rows, k), dtype=torch.int8, device="cuda")
    rb = torch.empty((P, k, cols), dtype=torch.int8, device="cuda")
    rc = torch.empty((P, rows, cols), dtype=torch.int8, device="cuda")
    out = torch.full((rows, cols), 0x5A5A, dtype=torch.int64, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    s = stream()
    assert lib.rns8_cuda_pack_i64_device(0, A.data_ptr() + row0 * k * 8, rows, k, k, P, ra.data_ptr(), s) == 0
    assert lib.rns8_cuda_pack_i64_device(0, B.data_ptr() + col0 * 8, k, cols, n, P, rb.data_ptr(), s) == 0
    sb = lib.rns8_cuda_gemm_rns_scratch_bytes(0, rows, cols, k, P)
    scratch = torch.empty(max(sb, 1), dtype=torch.uint8, device="cuda")
    assert lib.rns8_cuda_gemm_rns_device(0, ra.data_ptr(), rb.data_ptr(), rc.data_ptr(), rows, cols, k, P, 0,
                                         scratch.data_ptr(), sb, status.data_ptr(), s) == 0
    assert lib.rns8_cuda_export_i64_device(0, rc.data_ptr(), rows, cols, P, bound, out.data_ptr(), cols,
                                           status.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert int(status[0].item()) == 0
    return out


@pytest.mark.parametrize("m,n,k,world", [(2048, 2048, 1024, 4), (2048, 4096, 512, 8), (1000, 1040, 304, 4),
                                         (700, 520, 96, 6),
                                         (1024, 8192, 256, 8)])  # 4096-wide B slabs: the streamed pack, strided
def test_output_blocks_equal_unsharded(lib, oracle, m, n, k, world):
    from rns8_b200.shard import output_tile

    P, bound = 9, 2**61
    rng = oracle.Rng(m + n + k + world)
    hA = rng.i64(-(2**24), 2**24, (m, k))
    hB = rng.i64(-(2**24), 2**24, (k, n))
    A, B = torch.from_numpy(hA).cuda(), torch.from_numpy(hB).cuda()
    whole = product(lib, A, B, 0, m, 0, n, P, bound)
    rows = np.linspace(0, m - 1, 8).astype(np.int64)
    planes = oracle.gemm_rns(oracle.pack(np.ascontiguousarray(hA[rows]), P), oracle.pack(hB, P), P)
    st, want = oracle.export_i64(planes, P, bound)
    assert st == 0
    np.testing.assert_array_equal(whole.cpu().numpy()[rows], want)
    for r in range(world):
        row0, nr, col0, nc = output_tile(r, world, m, n)
        block = product(lib, A, B, row0, nr, col0, nc, P, bound)
        assert torch.equal(block, whole[row0:row0 + nr, col0:col0 + nc]), f"rank {r}"


@pytest.mark.parametrize("rows,cols,ld,signed", [(64, 4096, 8192, True), (33, 8192, 12288, False), (3, 4096, 4098, True)])
def test_strided_pack_matches_oracle(lib, oracle, rows, cols, ld, signed):
    """Sources whose rows are whole 4096-element tiles take the streamed pack
    even when rows are ld apart; the planes must equal the oracle's."""
    P = 20
    rng = oracle.Rng(rows + cols + ld)
    full = rng.i64(-(2**63), 2**63 - 1, (rows, ld)) if signed else rng.u64(0, 2**64 - 1, (rows, ld))
    src = torch.from_numpy(full.view(np.int64)).cuda()
    out = torch.empty((P, rows, cols), dtype=torch.int8, device="cuda")
    fn = lib.rns8_cuda_pack_i64_device if signed else lib.rns8_cuda_pack_u64_device
    assert fn(0, src.data_ptr(), rows, cols, ld, P, out.data_ptr(), stream()) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.pack(np.ascontiguousarray(full[:, :cols]), P))


def test_block_sharded_oneshot_gathers_the_product(oracle):
    """rns8_b200.shard.gemm_i64_block_sharded for every rank of 4 and 6 (on
    one GPU, one after another) assembles the unsharded one-shot's result."""
    import rns8_b200 as r8
    from rns8_b200.shard import gemm_i64_block_sharded

    m, n, k = 300, 520, 96
    rng = oracle.Rng(77)
    A = rng.i64(-(2**20), 2**20, (m, k))
    B = rng.i64(-(2**20), 2**20, (k, n))
    desc = r8.gemm_desc(r8.Semantics.BOUNDED_I64, r8.BoundKind.GLOBAL_MAX_ABS, m, n, k, bound=k * 2**40)
    with r8.Context(0) as ctx:
        want = r8.gemm_i64_oneshot(ctx, desc, A, B)
        for world in (4, 6):
            full = np.full((m, n), 7, np.int64)
            for r in range(world):
                row0, col0, blk = gemm_i64_block_sharded(ctx, desc, A, B, r, world)
                full[row0:row0 + blk.shape[0], col0:col0 + blk.shape[1]] = blk
            np.testing.assert_array_equal(full, want)
