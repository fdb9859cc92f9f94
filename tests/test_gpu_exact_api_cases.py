"""The reference's exact-wide public-API cases
(tests/unit/test_api_exact_wide_cases.inc:1-470) through this library:
limb-layout validation, descriptor validation, handles of the wrong contract
or prefix, null handles, and the fixed-width stride and range contracts of
the limb exports on 1 x 1 x 1 products. Every refused call leaves its output
untouched."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

OK, INVALID, RANGE = 0, 1, 5
MAXP = 20


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


def exact_desc(r8, sem, m, n, k):
    return r8.gemm_desc(sem, r8.BoundKind.NONE, m, n, k, max_prefix=MAXP)


def make_matrix(r8, ctx, rows, cols, sem, bound_kind=None, max_prefix=MAXP):
    abi = r8.abi
    bk = r8.BoundKind.NONE if bound_kind is None else bound_kind
    md = abi.MatrixDesc(rows=rows, cols=cols, logical_ld=cols, semantics=int(sem),
                        logical_layout=int(abi.Layout.ROW_MAJOR), bound_kind=int(bk), max_prefix=max_prefix)
    h = C.c_void_p()
    st = r8.lib().rns8_create_matrix(ctx.handle, C.byref(md), C.byref(h))
    return st, h


def make_plan(r8, ctx, d):
    h = C.c_void_p()
    st = r8.lib().rns8_create_plan(ctx.handle, C.byref(d), C.byref(h))
    return st, h


def export_fn(r8, signed):
    lib = r8.lib()
    return lib.rns8_export_exact_wide_signed_limbs if signed else lib.rns8_export_exact_wide_unsigned_limbs


@pytest.mark.parametrize("signed", [True, False])
def test_limb_layout_rejected(r8, ctx, signed):
    sem = r8.Semantics.EXACT_WIDE_SIGNED if signed else r8.Semantics.EXACT_WIDE_UNSIGNED
    m, n, k = 1, 2, 1
    sentinel = 0x5E5E5E5E5E5E5E5E
    limbs = np.full(128, sentinel, np.uint64)
    st, plan = make_plan(r8, ctx, exact_desc(r8, sem, m, n, k))
    assert st == OK
    st, c = make_matrix(r8, ctx, m, n, sem)
    assert st == OK
    fn = export_fn(r8, signed)
    p = limbs.ctypes.data
    assert fn(ctx.handle, plan, c, p, n, 0) == INVALID
    assert fn(ctx.handle, plan, c, p, n, 33) == INVALID
    assert fn(ctx.handle, plan, c, p, n - 1, 2) == INVALID
    assert fn(ctx.handle, plan, c, p, (2**63 - 1) // 32 + 1, 32) == INVALID
    assert fn(ctx.handle, plan, c, None, n, 2) == INVALID
    # null handles
    assert fn(None, plan, c, p, n, 2) == INVALID
    assert fn(ctx.handle, None, c, p, n, 2) == INVALID
    assert fn(ctx.handle, plan, None, p, n, 2) == INVALID
    assert (limbs == np.uint64(sentinel)).all()
    r8.lib().rns8_destroy_matrix(c)
    r8.lib().rns8_destroy_plan(plan)


@pytest.mark.parametrize("signed", [True, False])
def test_exact_descriptors_require_bound_none(r8, ctx, signed):
    S, BK = r8.Semantics, r8.BoundKind
    sem = S.EXACT_WIDE_SIGNED if signed else S.EXACT_WIDE_UNSIGNED
    stale = BK.GLOBAL_MAX_ABS if signed else BK.GLOBAL_MAX_UNSIGNED
    d = exact_desc(r8, sem, 1, 1, 1)
    d.bound = 1
    assert r8.api.plan_probe(d)[0] == INVALID
    d = exact_desc(r8, sem, 1, 1, 1)
    d.bound_kind = int(stale)
    assert r8.api.plan_probe(d)[0] == INVALID
    d = exact_desc(r8, sem, 1, 1, 1)
    tb = (C.c_uint64 * 1)(1)
    d.tile_bounds = C.cast(tb, C.POINTER(C.c_uint64))
    d.tile_bounds_count = 1
    assert r8.api.plan_probe(d)[0] == INVALID
    st, h = make_matrix(r8, ctx, 1, 1, sem, bound_kind=stale)
    assert st == INVALID and not h.value


@pytest.mark.parametrize("signed", [True, False])
def test_wrong_prefix_and_wrong_contract_handles_rejected(r8, ctx, signed):
    S = r8.Semantics
    sem = S.EXACT_WIDE_SIGNED if signed else S.EXACT_WIDE_UNSIGNED
    limbs = np.array([0x8A8A8A8A8A8A8A8A, 0x8B8B8B8B8B8B8B8B], np.uint64)
    st, plan = make_plan(r8, ctx, exact_desc(r8, sem, 1, 1, 1))
    assert st == OK
    fn = export_fn(r8, signed)
    lib = r8.lib()
    st, c9 = make_matrix(r8, ctx, 1, 1, sem, max_prefix=9)  # stale prefix
    assert st == OK
    assert fn(ctx.handle, plan, c9, limbs.ctypes.data, 1, 2) == INVALID
    bounded_export = lib.rns8_export_i64 if signed else lib.rns8_export_u64
    assert bounded_export(ctx.handle, plan, c9, limbs.ctypes.data, 1) == INVALID
    st, cb = make_matrix(r8, ctx, 1, 1, S.BOUNDED_I64 if signed else S.BOUNDED_U64,
                         bound_kind=r8.BoundKind.GLOBAL_MAX_ABS if signed else r8.BoundKind.GLOBAL_MAX_UNSIGNED,
                         max_prefix=9)
    assert st == OK
    assert fn(ctx.handle, plan, cb, limbs.ctypes.data, 1, 2) == INVALID
    st, cw = make_matrix(r8, ctx, 1, 1, S.WRAP_U64_MOD_2_64, max_prefix=0)
    assert st == OK
    assert fn(ctx.handle, plan, cw, limbs.ctypes.data, 1, 2) == INVALID
    # bounded and wrap exports, and the other signedness, on an exact handle
    st, ce = make_matrix(r8, ctx, 1, 1, sem)
    assert lib.rns8_export_i64(ctx.handle, plan, ce, limbs.ctypes.data, 1) == INVALID
    assert lib.rns8_export_u64(ctx.handle, plan, ce, limbs.ctypes.data, 1) == INVALID
    assert lib.rns8_export_wrap_u64(ctx.handle, plan, ce, limbs.ctypes.data, 1) == INVALID
    assert export_fn(r8, not signed)(ctx.handle, plan, ce, limbs.ctypes.data, 1, 2) == INVALID
    assert limbs.tolist() == [0x8A8A8A8A8A8A8A8A, 0x8B8B8B8B8B8B8B8B]
    for h in (c9, cb, cw, ce):
        lib.rns8_destroy_matrix(h)
    lib.rns8_destroy_plan(plan)


def one_by_one(r8, ctx, signed, a, b):
    S = r8.Semantics
    sem = S.EXACT_WIDE_SIGNED if signed else S.EXACT_WIDE_UNSIGNED
    plan = r8.Plan(ctx, exact_desc(r8, sem, 1, 1, 1))
    mats = [r8.Matrix(ctx, 1, 1, sem, r8.BoundKind.NONE, MAXP) for _ in range(3)]
    ws = r8.Workspace(ctx, plan)
    dt = np.int64 if signed else np.uint64
    (mats[0].pack_i64 if signed else mats[0].pack_u64)(np.array([[a]], dt), source_version=1)
    (mats[1].pack_i64 if signed else mats[1].pack_u64)(np.array([[b]], dt), source_version=1)
    r8.gemm_rns(ctx, plan, mats[0], mats[1], mats[2], ws)
    return plan, mats, ws


def test_fixed_width_exports_stride_and_range(r8, ctx):
    """:252-445 — -1 x 1 in one padded limb and in 32 limbs; INT64_MIN x 1 in
    one and two limbs; INT64_MAX x 2 refused in one limb; u64 max^2 and
    u64 max x 2 with padded two-limb rows."""
    lib = r8.lib()
    fs, fu = export_fn(r8, True), export_fn(r8, False)
    plan, mats, ws = one_by_one(r8, ctx, True, -1, 1)
    padded = np.array([0, 0x4545454545454545], np.uint64)
    assert fs(ctx.handle, plan.handle, mats[2].handle, padded.ctypes.data, 2, 1) == OK
    assert padded.tolist() == [2**64 - 1, 0x4545454545454545]
    wide = np.zeros(32, np.uint64)
    assert fs(ctx.handle, plan.handle, mats[2].handle, wide.ctypes.data, 1, 32) == OK
    assert (wide == np.uint64(2**64 - 1)).all()

    plan, mats, ws = one_by_one(r8, ctx, True, -(2**63), 1)
    one = np.zeros(1, np.uint64)
    assert fs(ctx.handle, plan.handle, mats[2].handle, one.ctypes.data, 1, 1) == OK and one[0] == 2**63
    two = np.zeros(2, np.uint64)
    assert fs(ctx.handle, plan.handle, mats[2].handle, two.ctypes.data, 1, 2) == OK
    assert two.tolist() == [2**63, 2**64 - 1]

    plan, mats, ws = one_by_one(r8, ctx, True, 2**63 - 1, 2)
    small = np.array([0x3434343434343434], np.uint64)
    assert fs(ctx.handle, plan.handle, mats[2].handle, small.ctypes.data, 1, 1) == RANGE
    assert small[0] == 0x3434343434343434
    assert fs(ctx.handle, plan.handle, mats[2].handle, two.ctypes.data, 1, 2) == OK
    assert two.tolist() == [0xFFFFFFFFFFFFFFFE, 0]

    plan, mats, ws = one_by_one(r8, ctx, False, 2**64 - 1, 2**64 - 1)
    small = np.array([0x6969696969696969], np.uint64)
    assert fu(ctx.handle, plan.handle, mats[2].handle, small.ctypes.data, 1, 1) == RANGE
    assert small[0] == 0x6969696969696969
    assert fu(ctx.handle, plan.handle, mats[2].handle, two.ctypes.data, 1, 2) == OK
    assert two.tolist() == [1, 0xFFFFFFFFFFFFFFFE]

    plan, mats, ws = one_by_one(r8, ctx, False, 2**64 - 1, 2)
    one = np.array([0x5656565656565656], np.uint64)
    assert fu(ctx.handle, plan.handle, mats[2].handle, one.ctypes.data, 1, 1) == RANGE
    assert one[0] == 0x5656565656565656
    padded = np.array([0, 0, 0x6767676767676767, 0x7878787878787878], np.uint64)
    assert fu(ctx.handle, plan.handle, mats[2].handle, padded.ctypes.data, 2, 2) == OK
    assert padded.tolist() == [0xFFFFFFFFFFFFFFFE, 1, 0x6767676767676767, 0x7878787878787878]
    del lib
