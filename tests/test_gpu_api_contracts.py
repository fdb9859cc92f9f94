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


class _PackingInfo(C.Structure):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("backend", C.c_int32),
                ("semantics", C.c_int32), ("uses_resident_matrix_inputs", C.c_uint32),
                ("uses_transient_pack_workspace", C.c_uint32), ("uses_matrix_engine_pack_layout", C.c_uint32),
                ("reusable_prepack_cache_available", C.c_uint32), ("production_prepack_cache_available", C.c_uint32),
                ("flags", C.c_uint32), ("input_domain", C.c_int32), ("output_domain", C.c_int32),
                ("output_host_current", C.c_uint32), ("output_device_current", C.c_uint32),
                ("next_op_flags", C.c_uint32), ("reserved0", C.c_uint32), ("a_pack_workspace_bytes", C.c_uint64),
                ("b_pack_workspace_bytes", C.c_uint64), ("accumulator_workspace_bytes", C.c_uint64),
                ("library_workspace_bytes", C.c_uint64), ("total_transient_workspace_bytes", C.c_uint64),
                ("input_domain_name", C.c_char * 64), ("output_domain_name", C.c_char * 64),
                ("next_op_hint", C.c_char * 160), ("a_layout_version", C.c_char * 96),
                ("b_layout_version", C.c_char * 96), ("output_layout_version", C.c_char * 96),
                ("prepack_cache_scope", C.c_char * 96), ("detail", C.c_char * 256)]


def test_plan_packing_info_contract_names(r8, ctx):
    """tests/unit/test_api_plan_packing_cases.inc:1-110 on a device-resident
    backend: bounded plans read and produce residue-current planes
    (rns_centered_residue_planes_v1, next op: final export or RNS GEMM
    "without logical export"), wrap64 plans byte limbs (wrap64_byte_limb_v1,
    final export only), finite plans finite_u8_centered_residue_v1; output is
    device-current; a short struct and a null plan are INVALID_ARGUMENT."""
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    RNS, FINITE, WRAP = 1, 3, 4
    FINAL, RNS_GEMM = 1, 2

    def info_of(plan, size=C.sizeof(_PackingInfo)):
        info = _PackingInfo(struct_size=size, abi_version=1)
        return lib.rns8_get_plan_packing_info(plan.handle if plan else None, C.byref(info)), info

    cases = [
        (r8.gemm_desc(S.BOUNDED_I64, BK.GLOBAL_MAX_ABS, 2, 3, 4, bound=16), RNS, FINAL | RNS_GEMM,
         b"rns_residue_current", b"rns_centered_residue_planes_v1"),
        (r8.gemm_desc(S.WRAP_U64_MOD_2_64, BK.NONE, 2, 2, 2), WRAP, FINAL, b"wrap64_byte_limb_current",
         b"wrap64_byte_limb_v1"),
        (r8.gemm_desc(S.FINITE_FIELD_U8, BK.NONE, 2, 2, 2, finite_modulus=251), FINITE, FINAL, b"finite_u8_current",
         b"finite_u8_centered_residue_v1"),
    ]
    for desc, domain, next_op, domain_name, layout in cases:
        plan = r8.Plan(ctx, desc)
        st, info = info_of(plan)
        assert st == 0
        assert (info.semantics, info.uses_resident_matrix_inputs, info.uses_transient_pack_workspace,
                info.uses_matrix_engine_pack_layout, info.reusable_prepack_cache_available) == (
                    desc.semantics, 1, 0, 0, 0)
        assert (info.input_domain, info.output_domain) == (domain, domain)
        assert (info.output_host_current, info.output_device_current) == (0, 1)
        assert info.next_op_flags == next_op
        assert info.input_domain_name == domain_name and info.output_domain_name == domain_name
        assert info.a_layout_version == layout and info.b_layout_version == layout
        assert info.output_layout_version == layout
        assert info.prepack_cache_scope == b"device_resident_no_prepack_cache"
        if domain == RNS:
            assert b"without logical export" in info.next_op_hint
        assert info_of(plan, C.sizeof(_PackingInfo) - 1)[0] == 1
        plan.close()
    assert info_of(None)[0] == 1
