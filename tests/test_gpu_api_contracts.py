"""Public-API contracts on the GPU, after the reference's differential
scenarios (tests/differential/test_hip_direct_bounded_residency_cases.inc,
…_exact_wide_residue_cases.inc, …_grouped_descriptor_cases.inc,
…_finite_persistent_cases.inc): operands that are not device-current are
refused, resident matrices are reused across same-shape calls, grouped tasks
may not share outputs, the widest limb export honours a padded leading
dimension, and finite one-shots keep the 65536-product K blocks."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


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


def bounded_plan(r8, ctx, m, n, k, bound):
    desc = r8.gemm_desc(r8.Semantics.BOUNDED_I64, r8.BoundKind.GLOBAL_MAX_ABS, m, n, k, bound=bound)
    return r8.Plan(ctx, desc)


def test_operands_must_be_device_current(r8, ctx):
    """test_hip_direct_bounded_residency_cases.inc:1-178: a GEMM whose input
    was never packed, and an export of a C no GEMM has written, are refused
    without touching anything; once packed, the same handles work."""
    m, n, k = 64, 48, 32
    rng = np.random.default_rng(1)
    A = rng.integers(-1000, 1000, (m, k), dtype=np.int64, endpoint=True)
    B = rng.integers(-1000, 1000, (k, n), dtype=np.int64, endpoint=True)
    plan = bounded_plan(r8, ctx, m, n, k, k * 10**6)
    a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
    ws = r8.Workspace(ctx, plan)
    b.pack_i64(B)
    with pytest.raises(r8.Error) as err:
        r8.gemm_rns(ctx, plan, a, b, c, ws)  # A never packed
    assert err.value.status == r8.Status.INVALID_ARGUMENT
    out = np.full((m, n), 5, np.int64)
    with pytest.raises(r8.Error) as err:
        r8.export_i64(ctx, plan, c, out=out)  # C never written
    assert err.value.status == r8.Status.INVALID_ARGUMENT
    assert (out == 5).all()
    assert c.storage_info().device_residues_current == 0
    a.pack_i64(A)
    r8.gemm_rns(ctx, plan, a, b, c, ws)
    np.testing.assert_array_equal(r8.export_i64(ctx, plan, c), A @ B)
    for h in (a, b, c, ws, plan):
        h.close()


def test_resident_matrices_reused_across_same_shape_calls(r8, ctx):
    """The same A/B/C handles serve several products: new source data is
    packed over the resident residues, storage is not reallocated, and every
    export reflects the latest inputs."""
    m, n, k = 256, 256, 128
    rng = np.random.default_rng(2)
    plan = bounded_plan(r8, ctx, m, n, k, k * 2**40)
    a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
    ws = r8.Workspace(ctx, plan)
    bytes0 = [h.storage_info().device_residue_bytes for h in (a, b, c)]
    for version in range(1, 4):
        A = rng.integers(-(2**20), 2**20, (m, k), dtype=np.int64, endpoint=True)
        B = rng.integers(-(2**20), 2**20, (k, n), dtype=np.int64, endpoint=True)
        a.pack_i64(A, source_version=10 + version)
        b.pack_i64(B, source_version=20 + version)
        r8.gemm_rns(ctx, plan, a, b, c, ws)
        np.testing.assert_array_equal(r8.export_i64(ctx, plan, c), A @ B)
        assert [h.storage_info().device_residue_bytes for h in (a, b, c)] == bytes0
    for h in (a, b, c, ws, plan):
        h.close()


def test_grouped_tasks_may_not_share_outputs(r8, ctx):
    """test_hip_direct_grouped_descriptor_cases.inc:1-187: outputs are written
    concurrently, so a grouped call whose tasks share an output, or whose
    output is another task's input, is refused before any launch."""
    m = n = k = 64
    plan = bounded_plan(r8, ctx, m, n, k, k * 2**20)
    mats = [r8.Matrix.for_plan(ctx, plan, role) for role in "abcabc"]
    a1, b1, c1, a2, b2, c2 = mats
    w1, w2 = r8.Workspace(ctx, plan), r8.Workspace(ctx, plan)
    rng = np.random.default_rng(3)
    for mat in (a1, b1, a2, b2):
        mat.pack_i64(rng.integers(-1000, 1000, (m, k), dtype=np.int64, endpoint=True))
    for tasks in ([(a1, b1, c1, w1), (a2, b2, c1, w2)],   # shared output
                  [(a1, b1, c1, w1), (c1, b2, c2, w2)]):  # output feeds the other task
        with pytest.raises(r8.Error) as err:
            r8.gemm_rns_grouped(ctx, plan, tasks)
        assert err.value.status == r8.Status.INVALID_ARGUMENT
        assert c1.storage_info().device_residues_current == 0 and c2.storage_info().device_residues_current == 0
    r8.gemm_rns_grouped(ctx, plan, [(a1, b1, c1, w1), (a2, b2, c2, w2)])
    assert c1.storage_info().device_residues_current == 1 and c2.storage_info().device_residues_current == 1
    for h in mats + [w1, w2, plan]:
        h.close()


@pytest.mark.parametrize("signed", [True, False])
def test_widest_limb_export_with_padded_rows(r8, ctx, oracle, signed):
    """test_hip_direct_exact_wide_residue_cases.inc:355-420: 32 limbs per
    element into a destination whose rows are padded; the padding keeps its
    bytes and every element matches the oracle's limbs."""
    m, n, k, limbs, pad = 5, 7, 9, 32, 3
    rng = np.random.default_rng(4 + signed)
    sem = r8.Semantics.EXACT_WIDE_SIGNED if signed else r8.Semantics.EXACT_WIDE_UNSIGNED
    dtype = np.int64 if signed else np.uint64
    lo, hi = (-(2**63), 2**63 - 1) if signed else (0, 2**64 - 1)
    A = rng.integers(lo, hi, (m, k), dtype=dtype, endpoint=True)
    B = rng.integers(lo, hi, (k, n), dtype=dtype, endpoint=True)
    plan = r8.Plan(ctx, r8.gemm_desc(sem, r8.BoundKind.NONE, m, n, k))
    a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
    ws = r8.Workspace(ctx, plan)
    (a.pack_i64 if signed else a.pack_u64)(A)
    (b.pack_i64 if signed else b.pack_u64)(B)
    r8.gemm_rns(ctx, plan, a, b, c, ws)
    ld = n + pad
    out = np.full((m, ld, limbs), 0xA5A5A5A5A5A5A5A5, np.uint64)
    fn = r8.lib().rns8_export_exact_wide_signed_limbs if signed else r8.lib().rns8_export_exact_wide_unsigned_limbs
    assert fn(ctx.handle, plan.handle, c.handle, out.ctypes.data, ld, limbs) == 0
    P = plan.prefix
    planes = oracle.gemm_rns(oracle.pack(A, P), oracle.pack(B, P), P)
    st, want = oracle.export_limbs(planes, P, limbs, signed)
    assert st == 0
    np.testing.assert_array_equal(out[:, :n], want)
    assert (out[:, n:] == np.uint64(0xA5A5A5A5A5A5A5A5)).all()
    exact = np.array(oracle.exact_product(A, B), dtype=object)
    top = (out[:, :n, -1] >> np.uint64(63)).astype(bool)
    if signed:
        assert (top == (exact < 0)).all()  # sign-extended to the top limb
    else:
        assert not top.any()
    for h in (a, b, c, ws, plan):
        h.close()


@pytest.mark.parametrize("modulus,field", [(256, False), (251, True), (255, False)])
@pytest.mark.parametrize("k", [65537, 131073])
def test_finite_oneshot_k_blocks(r8, ctx, oracle, modulus, field, k):
    """test_hip_direct_finite_persistent_cases.inc:237-261: one-shot finite
    GEMMs longer than one 65536-product block, with the largest residues."""
    m, n = 3, 17
    A = np.full((m, k), 255, np.uint8)
    B = np.full((k, n), 255, np.uint8)
    A[1, ::2] = 128
    B[::3, 2] = 1
    sem = r8.Semantics.FINITE_FIELD_U8 if field else r8.Semantics.FINITE_RING_U8
    desc = r8.gemm_desc(sem, r8.BoundKind.NONE, m, n, k, finite_modulus=modulus)
    got = r8.gemm_finite_u8_oneshot(ctx, desc, modulus, A, B, field)
    st, want = oracle.gemm_finite_u8_oneshot(A, B, modulus, field)
    assert st == 0
    np.testing.assert_array_equal(got, want)
    exact = (A.astype(object).dot(B.astype(object))) % modulus
    np.testing.assert_array_equal(got.astype(object), exact)
