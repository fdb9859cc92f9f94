"""The reference's currentness cases (tests/unit/test_semantics_currentness_cases.inc):
a per-tile bounded GEMM refuses a workspace made for a same-shape plan with
other tile bounds or other tile sizes, and matrices whose tile sizes are not
the plan's (gemm and export alike); a bounded export refuses output matrices
with too few planes or the wrong bound kind; and matrix creation whose owned
storage would overflow is RANGE_ERROR with no handle. The case that edits a
plan's private schedule fields (lines 97-149) has no public-ABI form and is
not mirrored."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

OK, INVALID, RANGE = 0, 1, 5
I64_MAX = 2**63 - 1


@pytest.fixture(scope="module")
def r8():
    import rns8_b200

    rns8_b200.lib()
    return rns8_b200


def per_tile_desc(r8, bounds, tile):
    S, BK = r8.Semantics, r8.BoundKind
    d = r8.gemm_desc(S.BOUNDED_U64, BK.PER_TILE_MAX_UNSIGNED, 65, 65, 1, tile_m=tile, tile_n=tile)
    r8.api.set_tile_bounds(d, bounds)
    return d


def test_stale_schedule_workspaces_and_matrix_tiles(r8):
    """test_semantics_currentness_cases.inc:1-95."""
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    m = n = 65
    A = np.zeros((m, 1), np.uint64)
    B = np.full((1, n), 7, np.uint64)
    A[-1, 0] = 1000000
    B[0, -1] = 1000
    with r8.Context(0) as ctx:
        plan_a = r8.Plan(ctx, per_tile_desc(r8, [0, 0, 7000000, 1000000000], 64))
        plan_b = r8.Plan(ctx, per_tile_desc(r8, [0, 0, 7000000, 999999999], 64))
        plan_t = r8.Plan(ctx, per_tile_desc(r8, [1000000000], 128))
        entries = plan_a.tile_schedule()
        assert entries and entries[0].range_bit_length == 0
        ws_a, ws_b, ws_t = (r8.Workspace(ctx, p) for p in (plan_a, plan_b, plan_t))

        def mat(rows, cols, tile):
            return r8.Matrix(ctx, rows, cols, S.BOUNDED_U64, BK.PER_TILE_MAX_UNSIGNED, 9, tile, tile)

        a, b, c = mat(m, 1, 64), mat(1, n, 64), mat(m, n, 64)
        a.pack_u64(A)
        b.pack_u64(B)
        gemm = lambda x, y, z, w: lib.rns8_gemm_rns(ctx.handle, plan_a.handle, x.handle, y.handle, z.handle,
                                                     w.handle)
        assert gemm(a, b, c, ws_a) == OK
        assert gemm(a, b, c, ws_b) == INVALID
        assert gemm(a, b, c, ws_t) == INVALID
        wrong_a, wrong_c = mat(m, 1, 128), mat(m, n, 128)
        wrong_a.pack_u64(A)
        assert gemm(wrong_a, b, c, ws_a) == INVALID
        assert gemm(a, b, wrong_c, ws_a) == INVALID
        out = np.zeros((m, n), np.uint64)
        assert lib.rns8_export_u64(ctx.handle, plan_a.handle, wrong_c.handle,
                                   out.ctypes.data_as(C.POINTER(C.c_uint64)), n) == INVALID
        assert not out.any()
        # The accepted call computed the product.
        np.testing.assert_array_equal(r8.export_u64(ctx, plan_a, c), A @ B)
        for h in (wrong_c, wrong_a, c, b, a, ws_t, ws_b, ws_a, plan_t, plan_b, plan_a):
            h.close()


def test_export_rejects_outputs_outside_the_plan_contract(r8):
    """test_semantics_currentness_cases.inc:151-182."""
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    with r8.Context(0) as ctx:
        plan = r8.Plan(ctx, r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 2, 2, 1, bound=100000))
        dst = np.full(4, 5, np.uint64)
        ptr = dst.ctypes.data_as(C.POINTER(C.c_uint64))
        vals = np.array([[1, 2], [3, 4]], np.uint64)
        c = r8.Matrix(ctx, 2, 2, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 0)
        # A fresh matrix is not device-current: this backend's export refuses
        # it, as the reference's device-resident backends do.
        assert lib.rns8_export_u64(ctx.handle, plan.handle, c.handle, ptr, 2) == INVALID
        c.pack_u64(vals)
        assert lib.rns8_export_u64(ctx.handle, plan.handle, c.handle, ptr, 2) == OK
        assert dst.tolist() == [1, 2, 3, 4]
        dst[:] = 5
        # Device-current matrices outside the plan's contract.
        wrong_prefix = r8.Matrix(ctx, 2, 2, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 1)
        wrong_prefix.pack_u64(vals)
        assert lib.rns8_export_u64(ctx.handle, plan.handle, wrong_prefix.handle, ptr, 2) == INVALID
        wrong_kind = r8.Matrix(ctx, 2, 2, S.BOUNDED_U64, BK.PER_TILE_MAX_UNSIGNED, 0)
        wrong_kind.pack_u64(vals)
        assert lib.rns8_export_u64(ctx.handle, plan.handle, wrong_kind.handle, ptr, 2) == INVALID
        assert (dst == 5).all()
        for h in (wrong_kind, wrong_prefix, c, plan):
            h.close()


def test_matrix_creation_storage_overflow(r8):
    """test_semantics_currentness_cases.inc:184-214."""
    S, BK, abi = r8.Semantics, r8.BoundKind, r8.abi
    lib = r8.lib()
    with r8.Context(0) as ctx:
        for sem, bk, mp in ((S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 9), (S.WRAP_U64_MOD_2_64, BK.NONE, 0)):
            md = abi.MatrixDesc(rows=I64_MAX // 2, cols=8, logical_ld=8, semantics=int(sem),
                                logical_layout=int(abi.Layout.ROW_MAJOR), bound_kind=int(bk), max_prefix=mp)
            h = C.c_void_p()
            assert lib.rns8_create_matrix(ctx.handle, C.byref(md), C.byref(h)) == RANGE
            assert not h.value
