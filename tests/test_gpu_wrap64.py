"""WRAP_U64_MOD_2_64 on the GPU against the oracle's restatement of
src/backend_wrap64/wrap64_reference.cpp: the byte-plane seam kernels, the
tensor-core byte-pair GEMM (and its SIMT fallback), and the public API as the
reference's differential test drives it
(tests/differential/test_hip_direct_wrap64_public_cases.inc)."""

from __future__ import annotations

import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

OK, INVALID = 0, 1
TC, SIMT = 1, 2
KATS = json.loads((Path(__file__).resolve().parent / "golden" / "reference_kats.json").read_text())


@pytest.fixture(scope="module")
def lib():
    import rns8_b200

    return rns8_b200.lib()


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def dev_u64(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int64)).cuda()


def host_u64(t) -> np.ndarray:
    return t.cpu().numpy().view(np.uint64)


def limbs_of(lib, A: np.ndarray):
    rows, cols = A.shape
    d = dev_u64(A)
    planes = torch.empty((8, rows, cols), dtype=torch.uint8, device="cuda")
    assert lib.rns8_cuda_pack_wrap_u64_device(0, d.data_ptr(), rows, cols, cols, planes.data_ptr(), stream()) == OK
    return planes


def wrap_gemm(lib, A: np.ndarray, B: np.ndarray, path: int):
    m, k = A.shape
    n = B.shape[1]
    la, lb = limbs_of(lib, A), limbs_of(lib, B)
    c = torch.full((m, n), -1, dtype=torch.int64, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    st = lib.rns8_cuda_gemm_wrap_u64_device(0, la.data_ptr(), lb.data_ptr(), c.data_ptr(), m, n, k, path,
                                            status.data_ptr(), stream())
    torch.cuda.synchronize()
    return st, host_u64(c), int(status[0].item())


@pytest.mark.parametrize("rows,cols,ld", [(64, 96, 96), (33, 20, 24), (5, 7, 9), (1, 3, 3)])
def test_pack_export_round_trip(lib, rows, cols, ld):
    rng = np.random.default_rng(rows * cols)
    src = rng.integers(0, 2**64 - 1, (rows, ld), dtype=np.uint64, endpoint=True)
    d_src = dev_u64(src)
    planes = torch.empty((8, rows, cols), dtype=torch.uint8, device="cuda")
    assert lib.rns8_cuda_pack_wrap_u64_device(0, d_src.data_ptr(), rows, cols, ld, planes.data_ptr(), stream()) == OK
    torch.cuda.synchronize()
    got_planes = planes.cpu().numpy()
    for l in range(8):  # limb-major byte planes
        np.testing.assert_array_equal(got_planes[l], ((src[:, :cols] >> np.uint64(8 * l)) & np.uint64(0xFF)).astype(np.uint8))
    out = torch.full((rows, ld + 2), 7, dtype=torch.int64, device="cuda")
    assert lib.rns8_cuda_export_wrap_u64_device(0, planes.data_ptr(), rows, cols, out.data_ptr(), ld + 2,
                                                stream()) == OK
    torch.cuda.synchronize()
    got = host_u64(out)
    np.testing.assert_array_equal(got[:, :cols], src[:, :cols])
    assert (got[:, cols:] == 7).all()


@pytest.mark.parametrize("m,n,k", [
    (128, 256, 64),
    (200, 272, 48),     # ragged M and N tiles
    (64, 32, 16),
    (130, 512, 1040),   # split K to fill the SMs
])
def test_tensor_core_gemm_matches_oracle(lib, oracle, m, n, k):
    rng = np.random.default_rng(m + n + k)
    A = rng.integers(0, 2**64 - 1, (m, k), dtype=np.uint64, endpoint=True)
    B = rng.integers(0, 2**64 - 1, (k, n), dtype=np.uint64, endpoint=True)
    A[0, :] = 2**64 - 1
    B[:, -1] = 0x8080808080808080
    st, got, word = wrap_gemm(lib, A, B, TC)
    assert st == OK and word == 0
    np.testing.assert_array_equal(got, oracle.wrap64_gemm(A, B))


@pytest.mark.parametrize("k", [16384, 40000])
def test_tensor_core_gemm_worst_case_bytes(lib, oracle, k):
    """Every byte 0xFF: each diagonal sum is as large as it can be, so S_d for
    d >= 4 overflows 32 bits and relies on wrapping, and K = 40000 needs three
    16384-product units per tile. (2^64 - 1)^2 = 1 mod 2^64, so every cell is K."""
    m, n = 128, 128
    A = np.full((m, k), 2**64 - 1, np.uint64)
    B = np.full((k, n), 2**64 - 1, np.uint64)
    st, got, word = wrap_gemm(lib, A, B, TC)
    assert st == OK and word == 0
    assert (got == np.uint64(k)).all()
    # Random bytes at the same K against the oracle.
    rng = np.random.default_rng(k)
    A = rng.integers(0, 2**64 - 1, (m, k), dtype=np.uint64, endpoint=True)
    B = rng.integers(0, 2**64 - 1, (k, n), dtype=np.uint64, endpoint=True)
    st, got, word = wrap_gemm(lib, A, B, TC)
    assert st == OK and word == 0
    np.testing.assert_array_equal(got, oracle.wrap64_gemm(A, B))


@pytest.mark.parametrize("m,n,k", [(7, 3, 5), (33, 17, 100), (64, 64, 64)])
def test_simt_gemm_matches_oracle(lib, oracle, m, n, k):
    rng = np.random.default_rng(m * n * k)
    A = rng.integers(0, 2**64 - 1, (m, k), dtype=np.uint64, endpoint=True)
    B = rng.integers(0, 2**64 - 1, (k, n), dtype=np.uint64, endpoint=True)
    st, got, _ = wrap_gemm(lib, A, B, SIMT)
    assert st == OK
    np.testing.assert_array_equal(got, oracle.wrap64_gemm(A, B))
    if k % 16 or n % 16:
        st, _, _ = wrap_gemm(lib, A, B, TC)
        assert st == INVALID  # the tensor-core path needs K and N multiples of 16


# ---- public API --------------------------------------------------------------------
@pytest.fixture(scope="module")
def ctx():
    import rns8_b200 as r8

    c = r8.Context(0)
    yield c
    c.close()


def wrap_desc(r8, m, n, k):
    return r8.gemm_desc(r8.Semantics.WRAP_U64_MOD_2_64, r8.BoundKind.NONE, m, n, k)


def test_public_persistent_path_matches_reference_kat(ctx):
    """test_hip_direct_wrap64_public_cases.inc:6-200: padded leading
    dimensions, byte-limb storage, same-source pack elision, RNS calls refused
    on wrap handles, padding untouched, and the one-shot call."""
    import rns8_b200 as r8

    kat = KATS["wrap64_public_2x3x5"]
    m, n, k, lda, ldb, ldc = kat["m"], kat["n"], kat["k"], kat["lda"], kat["ldb"], 5
    A = np.array([int(v) for v in kat["A"]], np.uint64).reshape(m, lda)
    B = np.array([int(v) for v in kat["B"]], np.uint64).reshape(k, ldb)
    want = np.array([[int(v) for v in row] for row in kat["expected"]], np.uint64)
    plan = r8.Plan(ctx, wrap_desc(r8, m, n, k))
    assert plan.prefix == 0
    info = plan.backend_info()
    assert info.selected_kernel.decode().startswith("sm100a_simt_wrap64")  # K = 5: not a TMA shape
    a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
    ws = r8.Workspace(ctx, plan)
    for mat, rows, cols in ((a, m, k), (b, k, n), (c, m, n)):
        si = mat.storage_info()
        assert si.uses_byte_limb_storage == 1 and si.uses_residue_storage == 0
        assert si.device_byte_limb_bytes == rows * cols * 8 and si.device_residue_bytes == 0
        assert si.device_byte_limbs_current == 0
    a.pack_u64(A[:, :k], source_version=7)
    b.pack_u64(B[:, :n], source_version=11)
    assert a.storage_info().device_byte_limbs_current == 1
    changed = A.copy()
    changed[0, 0] = 123456789
    a.pack_u64(changed[:, :k], source_version=7)  # same source version: the pack is skipped
    with pytest.raises(r8.Error) as err:
        r8.export_wrap_u64(ctx, plan, c)
    assert err.value.status == r8.Status.INVALID_ARGUMENT  # C not current yet
    r8.gemm_wrap_u64(ctx, plan, a, b, c, ws)
    out = np.full((m, ldc), 0x1111111111111111, np.uint64)
    r8.export_wrap_u64(ctx, plan, c, out=out[:, :n])
    np.testing.assert_array_equal(out[:, :n], want)
    assert (out[:, n:] == 0x1111111111111111).all()
    with pytest.raises(r8.Error) as err:
        r8.gemm_rns(ctx, plan, a, b, c, ws)
    assert err.value.status == r8.Status.INVALID_ARGUMENT
    with pytest.raises(r8.Error) as err:
        r8.export_u64(ctx, plan, c)
    assert err.value.status == r8.Status.INVALID_ARGUMENT
    with pytest.raises(r8.Error) as err:
        a.pack_i64(A[:, :k].view(np.int64))
    assert err.value.status == r8.Status.INVALID_ARGUMENT
    one = np.full((m, ldc), 0xABABABABABABABAB, np.uint64)
    r8.gemm_wrap_u64_oneshot(ctx, wrap_desc(r8, m, n, k), A[:, :k], B[:, :n], out=one[:, :n])
    np.testing.assert_array_equal(one[:, :n], want)
    assert (one[:, n:] == 0xABABABABABABABAB).all()
    for h in (a, b, c, ws, plan):
        h.close()


@pytest.mark.parametrize("m,n,k", [(256, 512, 128), (96, 48, 33)])
def test_public_chain_and_oneshot_match_oracle(ctx, oracle, m, n, k):
    """C = A x B, then D = C x E with C's byte planes as the next A, through the
    persistent API; and the one-shot call on the same inputs."""
    import rns8_b200 as r8

    rng = np.random.default_rng(m + k)
    A = rng.integers(0, 2**64 - 1, (m, k), dtype=np.uint64, endpoint=True)
    B = rng.integers(0, 2**64 - 1, (k, n), dtype=np.uint64, endpoint=True)
    E = rng.integers(0, 2**64 - 1, (n, 64), dtype=np.uint64, endpoint=True)
    p1, p2 = r8.Plan(ctx, wrap_desc(r8, m, n, k)), r8.Plan(ctx, wrap_desc(r8, m, 64, n))
    a, b, c = (r8.Matrix.for_plan(ctx, p1, role) for role in "abc")
    e, d = r8.Matrix.for_plan(ctx, p2, "b"), r8.Matrix.for_plan(ctx, p2, "c")
    w1, w2 = r8.Workspace(ctx, p1), r8.Workspace(ctx, p2)
    a.pack_u64(A)
    b.pack_u64(B)
    e.pack_u64(E)
    r8.gemm_wrap_u64(ctx, p1, a, b, c, w1)
    r8.gemm_wrap_u64(ctx, p2, c, e, d, w2)
    want_c = oracle.wrap64_gemm(A, B)
    np.testing.assert_array_equal(r8.export_wrap_u64(ctx, p1, c), want_c)
    np.testing.assert_array_equal(r8.export_wrap_u64(ctx, p2, d), oracle.wrap64_gemm(want_c, E))
    np.testing.assert_array_equal(r8.gemm_wrap_u64_oneshot(ctx, wrap_desc(r8, m, n, k), A, B), want_c)
    for h in (a, b, c, e, d, w1, w2, p1, p2):
        h.close()


def test_public_resident_path_padded_tile_tail(ctx):
    """test_wrap64_residency_reject_cases.inc:1-128: 17 x 19 x 33 with padded
    lda 41, ldb 29, ldc 23 (matrices declare those logical leading
    dimensions), full-width values with all-ones, zero, 0x80-byte and
    alternating-byte patterns; two rounds of new sources through pack / GEMM
    / export of the same resident matrices and the one-shot call, both equal
    to sum a*b mod 2^64, C's padding untouched, source versions stamped."""
    import rns8_b200 as r8

    m, n, k, lda, ldb, ldc = 17, 19, 33, 41, 29, 23
    U = 2**64 - 1
    plan = r8.Plan(ctx, wrap_desc(r8, m, n, k))
    S, BK = r8.Semantics.WRAP_U64_MOD_2_64, r8.BoundKind.NONE
    a = r8.Matrix(ctx, m, k, S, BK, logical_ld=lda)
    b = r8.Matrix(ctx, k, n, S, BK, logical_ld=ldb)
    c = r8.Matrix(ctx, m, n, S, BK, logical_ld=ldc)
    ws = r8.Workspace(ctx, plan)
    for salt, (va, vb) in ((0x1234, (301, 302)), (0x5678, (401, 402))):
        rng = np.random.default_rng(salt)
        A = np.full((m, lda), 0xAAAAAAAAAAAAAAAA ^ salt, np.uint64)
        B = np.full((k, ldb), 0xBBBBBBBBBBBBBBBB ^ (salt << 1), np.uint64)
        A[:, :k] = rng.integers(0, U, (m, k), dtype=np.uint64, endpoint=True)
        B[:, :n] = rng.integers(0, U, (k, n), dtype=np.uint64, endpoint=True)
        special_a = {0: U, 1: 0, 2: 0x8080808080808080, 3: 0x7F807F807F807F80}
        special_b = {0: U - 1, 1: 1, 2: 0xFEFDFCFBFAF9F8F7, 3: 0x0102030405060708}
        for r in range(m):
            for q in range(k):
                if (r + q) % 13 in special_a:
                    A[r, q] = special_a[(r + q) % 13]
        for q in range(k):
            for col in range(n):
                if (q * 3 + col) % 17 in special_b:
                    B[q, col] = special_b[(q * 3 + col) % 17]
        a.pack_u64(A[:, :k], source_version=va)
        b.pack_u64(B[:, :n], source_version=vb)
        assert a.storage_info().source_version == va and b.storage_info().source_version == vb
        r8.gemm_wrap_u64(ctx, plan, a, b, c, ws)
        sentinel = 0xCDCDCDCDCDCDCDCD
        out = np.full((m, ldc), sentinel, np.uint64)
        r8.export_wrap_u64(ctx, plan, c, out=out[:, :n])
        one = np.full((m, ldc), sentinel, np.uint64)
        r8.gemm_wrap_u64_oneshot(ctx, wrap_desc(r8, m, n, k), A[:, :k], B[:, :n], out=one[:, :n])
        Ai = [[int(x) for x in row] for row in A[:, :k]]
        Bi = [[int(x) for x in row] for row in B[:, :n]]
        want = np.array([[sum(Ai[r][q] * Bi[q][col] for q in range(k)) % 2**64 for col in range(n)]
                         for r in range(m)], np.uint64)
        np.testing.assert_array_equal(out[:, :n], want)
        np.testing.assert_array_equal(one, out)
        assert (out[:, n:] == sentinel).all()
    for h in (a, b, c, ws, plan):
        h.close()


def test_wrap64_rejects_crt_metadata_and_rns_apis(ctx):
    """test_wrap64_residency_reject_cases.inc (CRT metadata and RNS APIs),
    on this backend's one context kind: bounded one-shots refuse a wrap64
    descriptor; zero leading dimensions, bounded-looking, prefixed, flagged,
    mis-tiled and tile-bounded wrap64 descriptors are INVALID_ARGUMENT (also
    when an unavailable backend is requested); a valid one requesting an
    unavailable backend is UNSUPPORTED_BACKEND; AUTO runs (2^64-1 x 2 mod
    2^64); bounded-looking wrap64 matrix descriptors are refused; the RNS and
    exact-wide calls refuse wrap64 handles, and the wrap64 calls refuse a
    bounded plan's workspace and a bounded matrix."""
    import ctypes as C

    import rns8_b200 as r8

    lib, S, BK, B, abi = r8.lib(), r8.Semantics, r8.BoundKind, r8.Backend, r8.abi
    INVALID, UNSUPPORTED = 1, 4
    U = 2**64 - 1
    A = np.array([[U]], np.uint64)
    Bm = np.array([[2]], np.uint64)
    Cm = np.zeros((1, 1), np.uint64)
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    h = ctx.handle
    desc = wrap_desc(r8, 1, 1, 1)
    assert lib.rns8_gemm_u64_oneshot(h, C.byref(desc), p(A), 1, p(Bm), 1, p(Cm), 1) == INVALID
    sA, sB, sC = np.array([[-1]], np.int64), np.array([[2]], np.int64), np.zeros((1, 1), np.int64)
    assert lib.rns8_gemm_i64_oneshot(h, C.byref(desc), p(sA), 1, p(sB), 1, p(sC), 1) == INVALID
    for lda, ldb, ldc in ((0, 1, 1), (1, 0, 1), (1, 1, 0)):
        Cm[0, 0] = 0x123456789ABCDEF0
        assert lib.rns8_gemm_wrap_u64_oneshot(h, C.byref(desc), p(A), lda, p(Bm), ldb, p(Cm), ldc) == INVALID
        assert Cm[0, 0] == 0x123456789ABCDEF0

    def plan_status(d):
        plan = C.c_void_p()
        st = lib.rns8_create_plan(h, C.byref(d), C.byref(plan))
        if plan.value:
            lib.rns8_destroy_plan(plan)
        assert st != 0 or plan.value
        return st, bool(plan.value)

    def invalid(d):
        assert lib.rns8_gemm_wrap_u64_oneshot(h, C.byref(d), p(A), 1, p(Bm), 1, p(Cm), 1) == INVALID
        assert plan_status(d) == (INVALID, False)

    def variant(**kw):
        d = wrap_desc(r8, 1, 1, 1)
        for key, val in kw.items():
            setattr(d, key, val)
        return d

    invalid(variant(bound_kind=int(BK.GLOBAL_MAX_UNSIGNED), bound=U))
    invalid(variant(bound_kind=int(BK.GLOBAL_MAX_UNSIGNED), bound=U, requested_backend=int(B.HIPBLASLT)))
    fut = variant(requested_backend=int(B.HIPBLASLT))
    assert lib.rns8_gemm_wrap_u64_oneshot(h, C.byref(fut), p(A), 1, p(Bm), 1, p(Cm), 1) == UNSUPPORTED
    assert plan_status(fut) == (UNSUPPORTED, False)
    auto = variant(requested_backend=int(B.AUTO))
    assert lib.rns8_gemm_wrap_u64_oneshot(h, C.byref(auto), p(A), 1, p(Bm), 1, p(Cm), 1) == 0
    assert int(Cm[0, 0]) == U - 1
    invalid(variant(max_prefix=9))
    invalid(variant(bound=1))
    invalid(variant(flags=1))
    invalid(variant(tile_m=32))
    invalid(variant(tile_n=96))
    tb = (C.c_uint64 * 1)(1)
    invalid(variant(tile_bounds=C.cast(tb, C.POINTER(C.c_uint64)), tile_bounds_count=1))
    invalid(variant(tile_bounds_count=1))
    invalid(variant(bound_kind=int(BK.PER_TILE_MAX_UNSIGNED), tile_m=64, tile_n=64,
                    tile_bounds=C.cast(tb, C.POINTER(C.c_uint64)), tile_bounds_count=1))
    bounded = r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 1, 1, 1, bound=2,
                           requested_backend=B.WRAP64_BYTE_LIMB)
    assert lib.rns8_gemm_wrap_u64_oneshot(h, C.byref(bounded), p(A), 1, p(Bm), 1, p(Cm), 1) == INVALID
    assert plan_status(bounded) == (UNSUPPORTED, False)

    def matrix_status(**kw):
        md = abi.MatrixDesc(rows=1, cols=1, logical_ld=1, semantics=int(S.WRAP_U64_MOD_2_64),
                            logical_layout=int(abi.Layout.ROW_MAJOR), bound_kind=int(BK.NONE))
        for key, val in kw.items():
            setattr(md, key, val)
        m = C.c_void_p()
        st = lib.rns8_create_matrix(h, C.byref(md), C.byref(m))
        if m.value:
            lib.rns8_destroy_matrix(m)
        return st, bool(m.value)

    assert matrix_status()[0] == 0
    assert matrix_status(bound_kind=int(BK.GLOBAL_MAX_UNSIGNED)) == (INVALID, False)
    assert matrix_status(max_prefix=9) == (INVALID, False)
    assert matrix_status(flags=1) == (INVALID, False)
    assert matrix_status(logical_ld=-1) == (INVALID, False)
    assert matrix_status(tile_m=32) == (INVALID, False)

    plan = r8.Plan(ctx, desc)
    ws = r8.Workspace(ctx, plan)
    a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
    assert lib.rns8_pack_i64(h, a.handle, p(sA), 1, 0) == INVALID
    a.pack_u64(A)
    b.pack_u64(Bm)
    assert lib.rns8_gemm_rns(h, plan.handle, a.handle, b.handle, c.handle, ws.handle) == INVALID
    r8.gemm_wrap_u64(ctx, plan, a, b, c, ws)
    limbs = np.zeros(1, np.uint64)
    assert lib.rns8_export_i64(h, plan.handle, c.handle, p(sC), 1) == INVALID
    assert lib.rns8_export_u64(h, plan.handle, c.handle, p(Cm), 1) == INVALID
    assert lib.rns8_export_exact_wide_signed_limbs(h, plan.handle, c.handle, p(limbs), 1, 1) == INVALID
    assert lib.rns8_export_exact_wide_unsigned_limbs(h, plan.handle, c.handle, p(limbs), 1, 1) == INVALID
    # Bounded handles on the wrap64 calls.
    bplan = r8.Plan(ctx, r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 1, 1, 1, bound=2))
    bws = r8.Workspace(ctx, bplan)
    bmat = r8.Matrix(ctx, 1, 1, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 9)
    bmat.pack_u64(Bm)
    assert lib.rns8_gemm_wrap_u64(h, plan.handle, a.handle, b.handle, c.handle, bws.handle) == INVALID
    assert lib.rns8_export_wrap_u64(h, plan.handle, bmat.handle, p(Cm), 1) == INVALID
    for obj in (bmat, bws, bplan, a, b, c, ws, plan):
        obj.close()
