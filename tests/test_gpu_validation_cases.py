"""The reference's public-API validation cases
(tests/unit/test_api_validation_cases.inc:1-120): invalid leading dimensions
and overflowing dimensions are refused before any access or allocation, and
outputs keep their bytes."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

INVALID, RANGE = 1, 5
I64_MAX = 2**63 - 1
HUGE = I64_MAX // 2 + 1


@pytest.fixture(scope="module")
def r8():
    import rns8_b200

    rns8_b200.lib()
    return rns8_b200


@pytest.fixture(scope="module")
def ctx(r8):
    c = r8.Context(0)
    yield c
    c.close()


def p(a):
    return a.ctypes.data


def test_oneshots_reject_invalid_leading_dimensions(r8, ctx):
    lib, S, BK = r8.lib(), r8.Semantics, r8.BoundKind
    a64 = np.array([1, 2, 3, 4], np.int64)
    b64 = np.array([5, 6, 7, 8], np.int64)
    c64 = np.full(4, -1, np.int64)
    u64a, u64b = a64.view(np.uint64), b64.view(np.uint64)
    cu64 = np.full(4, 99, np.uint64)
    a8, b8 = np.array([1, 2, 3, 4], np.uint8), np.array([5, 6, 7, 8], np.uint8)
    c8 = np.full(4, 77, np.uint8)
    d_i64 = r8.gemm_desc(S.BOUNDED_I64, BK.GLOBAL_MAX_ABS, 2, 2, 2, bound=1000)
    d_u64 = r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 2, 2, 2, bound=1000)
    d_ring = r8.gemm_desc(S.FINITE_RING_U8, BK.NONE, 2, 2, 2, finite_modulus=251)
    d_field = r8.gemm_desc(S.FINITE_FIELD_U8, BK.NONE, 2, 2, 2, finite_modulus=251)
    d_wrap = r8.gemm_desc(S.WRAP_U64_MOD_2_64, BK.NONE, 2, 2, 2)
    h = ctx.handle
    for lda, ldb, ldc in ((1, 2, 2), (2, 1, 2), (2, 2, 1)):
        assert lib.rns8_gemm_i64_oneshot(h, C.byref(d_i64), p(a64), lda, p(b64), ldb, p(c64), ldc) == INVALID
        assert lib.rns8_gemm_u64_oneshot(h, C.byref(d_u64), p(u64a), lda, p(u64b), ldb, p(cu64), ldc) == INVALID
        assert lib.rns8_gemm_finite_ring_u8_oneshot(h, C.byref(d_ring), 251, p(a8), lda, p(b8), ldb, p(c8),
                                                    ldc) == INVALID
        assert lib.rns8_gemm_wrap_u64_oneshot(h, C.byref(d_wrap), p(u64a), lda, p(u64b), ldb, p(cu64), ldc) == INVALID
    assert lib.rns8_gemm_finite_field_u8_oneshot(h, C.byref(d_field), 251, p(a8), 1, p(b8), 2, p(c8), 2) == INVALID
    assert (c64 == -1).all() and (cu64 == 99).all() and (c8 == 77).all()


def test_overflowing_dimensions_rejected(r8, ctx):
    lib, S, BK, abi = r8.lib(), r8.Semantics, r8.BoundKind, r8.abi
    a64 = np.array([1, 2, 3, 4], np.int64)
    b64 = np.array([5, 6, 7, 8], np.int64)
    c64 = np.full(4, -7, np.int64)
    d = r8.gemm_desc(S.BOUNDED_I64, BK.GLOBAL_MAX_ABS, HUGE, HUGE, 2, bound=1000)
    assert lib.rns8_gemm_i64_oneshot(ctx.handle, C.byref(d), p(a64), 2, p(b64), HUGE, p(c64), HUGE) == INVALID
    assert (c64 == -7).all()
    # per-tile plan whose tile count overflows
    d = r8.gemm_desc(S.BOUNDED_I64, BK.PER_TILE_MAX_ABS, I64_MAX, I64_MAX, 1, tile_m=64, tile_n=64)
    tb = (C.c_uint64 * 1)(1)
    d.tile_bounds = C.cast(tb, C.POINTER(C.c_uint64))
    d.tile_bounds_count = 2**64 - 1
    plan = C.c_void_p()
    assert lib.rns8_create_plan(ctx.handle, C.byref(d), C.byref(plan)) == RANGE and not plan.value

    def create(rows, cols, sem, bk, ld=None, max_prefix=0):
        md = abi.MatrixDesc(rows=rows, cols=cols, logical_ld=cols if ld is None else ld, semantics=int(sem),
                            logical_layout=int(abi.Layout.ROW_MAJOR), bound_kind=int(bk), max_prefix=max_prefix)
        m = C.c_void_p()
        st = lib.rns8_create_matrix(ctx.handle, C.byref(md), C.byref(m))
        assert not m.value or st == 0
        if m.value:
            lib.rns8_destroy_matrix(m)
        return st

    assert create(HUGE, 3, S.BOUNDED_I64, BK.GLOBAL_MAX_ABS) == RANGE
    assert create(I64_MAX, I64_MAX, S.FINITE_RING_U8, BK.NONE) == RANGE
    assert create(HUGE, 3, S.WRAP_U64_MOD_2_64, BK.NONE) == RANGE
    assert create(2, 3, S.BOUNDED_I64, BK.GLOBAL_MAX_ABS, ld=2) == INVALID
    assert create(2, 3, S.FINITE_RING_U8, BK.NONE, ld=2) == INVALID
    assert create(2, 3, S.WRAP_U64_MOD_2_64, BK.NONE, ld=2) == INVALID
