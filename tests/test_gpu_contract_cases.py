"""The reference's persistent-GEMM contract cases
(tests/unit/test_semantics_workspace_cases.inc:27-146): a workspace from a
different plan is WORKSPACE_TOO_SMALL, matrices of the wrong shape, prefix or
bound kind are INVALID_ARGUMENT, and the output's source version is derived
from its inputs' (stable while they are, new when one is repacked, untouched
by a refused call). Inputs are packed first: this is a device backend, where
GEMM operands must be device-current."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

OK, INVALID, TOO_SMALL = 0, 1, 7


@pytest.fixture(scope="module")
def r8():
    import rns8_b200

    rns8_b200.lib()
    return rns8_b200


def setup(r8, ctx, bound):
    S, BK = r8.Semantics, r8.BoundKind
    desc = r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 2, 2, 2, bound=bound)
    plan = r8.Plan(ctx, desc)
    ws = r8.Workspace(ctx, plan)
    small = r8.Plan(ctx, r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 2, 2, 1, bound=bound))
    wrong_ws = r8.Workspace(ctx, small)
    a, b, c = (r8.Matrix(ctx, 2, 2, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 0) for _ in range(3))
    return plan, ws, small, wrong_ws, a, b, c


def test_incompatible_matrix_and_workspace_contracts(r8):
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    with r8.Context(0) as ctx:
        plan, ws, small, wrong_ws, a, b, c = setup(r8, ctx, 100000)
        a.pack_u64(np.array([[1, 2], [3, 4]], np.uint64))
        b.pack_u64(np.array([[5, 6], [7, 8]], np.uint64))
        gemm = lambda x, y, z, w: lib.rns8_gemm_rns(ctx.handle, plan.handle, x.handle, y.handle, z.handle, w.handle)
        assert gemm(a, b, c, ws) == OK
        assert gemm(a, b, c, wrong_ws) == TOO_SMALL
        wrong_b = r8.Matrix(ctx, 3, 2, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 0)
        wrong_b.pack_u64(np.ones((3, 2), np.uint64))
        assert gemm(a, wrong_b, c, ws) == INVALID
        wrong_c = r8.Matrix(ctx, 2, 2, S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 1)  # one plane
        assert gemm(a, b, wrong_c, ws) == INVALID
        wrong_a = r8.Matrix(ctx, 2, 2, S.BOUNDED_U64, BK.PER_TILE_MAX_UNSIGNED, 0)
        assert gemm(wrong_a, b, c, ws) == INVALID
        np.testing.assert_array_equal(r8.export_u64(ctx, plan, c), [[19, 22], [43, 50]])
        for h in (wrong_a, wrong_c, wrong_b, a, b, c, wrong_ws, ws, small, plan):
            h.close()


def test_output_source_version_stamping(r8):
    with r8.Context(0) as ctx:
        plan, ws, small, wrong_ws, a, b, c = setup(r8, ctx, 1000)
        a.pack_u64(np.array([[1, 2], [3, 4]], np.uint64), source_version=17)
        b.pack_u64(np.array([[5, 6], [7, 8]], np.uint64), source_version=23)
        r8.gemm_rns(ctx, plan, a, b, c, ws)
        v1 = c.storage_info().source_version
        assert v1 not in (0, 17, 23)
        r8.gemm_rns(ctx, plan, a, b, c, ws)
        assert c.storage_info().source_version == v1
        b.pack_u64(np.array([[8, 7], [6, 5]], np.uint64), source_version=24)
        r8.gemm_rns(ctx, plan, a, b, c, ws)
        v2 = c.storage_info().source_version
        assert v2 not in (0, v1)
        with pytest.raises(r8.Error) as err:
            r8.gemm_rns(ctx, plan, a, b, c, wrong_ws)
        assert err.value.status == r8.Status.WORKSPACE_TOO_SMALL
        assert c.storage_info().source_version == v2
        np.testing.assert_array_equal(r8.export_u64(ctx, plan, c), [[20, 17], [48, 41]])
        for h in (a, b, c, wrong_ws, ws, small, plan):
            h.close()
