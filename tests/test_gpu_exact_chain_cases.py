"""The reference's exact-wide chain cases (tests/unit/test_exact_wide_chain_cases.inc)
through this library's public C ABI: a product's residues (and its range
record) feed the next product; an overflowing link is a RANGE_ERROR that
changes nothing; the proof counts K and ignores host padding; an output may
not alias an input; and a matrix whose higher planes were never written
(computed under a smaller prefix) cannot serve a larger-prefix plan until it
is repacked. Matrices hold 20 planes (RNS8_MAX_SUPPORTED_PREFIX), as the
reference's fixture creates them."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

OK, INVALID, RANGE = 0, 1, 5


@pytest.fixture(scope="module")
def r8():
    import rns8_b200

    rns8_b200.lib()
    return rns8_b200


class Chain:
    """Plan (fixed prefix), workspace and four m x k / k x n / m x n / m x n matrices."""

    def __init__(self, r8, ctx, signed, m=1, n=1, k=1, prefix=20):
        S, BK = r8.Semantics, r8.BoundKind
        self.r8, self.ctx, self.signed = r8, ctx, signed
        self.sem = S.EXACT_WIDE_SIGNED if signed else S.EXACT_WIDE_UNSIGNED
        d = r8.gemm_desc(self.sem, BK.NONE, m, n, k, max_prefix=prefix, flags=r8.PLAN_FORCE_FIXED_PREFIX)
        self.plan = r8.Plan(ctx, d)
        self.ws = r8.Workspace(ctx, self.plan)
        self.mats = [r8.Matrix(ctx, r, c, self.sem, BK.NONE, 20) for r, c in ((m, k), (k, n), (m, n), (m, n))]

    def pack(self, i, values, version):
        arr = np.asarray(values, np.int64 if self.signed else np.uint64)
        (self.mats[i].pack_i64 if self.signed else self.mats[i].pack_u64)(arr, source_version=version)

    def multiply(self, a, b, c, plan=None, ws=None):
        plan, ws = plan or self.plan, ws or self.ws
        return self.r8.lib().rns8_gemm_rns(self.ctx.handle, plan.handle, self.mats[a].handle, self.mats[b].handle,
                                           self.mats[c].handle, ws.handle)

    def export(self, i, limbs, plan=None):
        return self.r8.export_exact_wide_limbs(self.ctx, plan or self.plan, self.mats[i], limbs, signed=self.signed)

    def close(self):
        for h in (*self.mats, self.ws, self.plan):
            h.close()


def value_of(limbs, signed):
    v = sum(int(x) << (64 * i) for i, x in enumerate(limbs))
    bits = 64 * len(limbs)
    return v - (1 << bits) if signed and v >> (bits - 1) else v


@pytest.mark.parametrize("signed", [True, False])
def test_repeated_products(r8, signed):
    """:35-62 — x7 (or x(-7)) forty times through alternating outputs; every
    link is admitted and exports exactly in three limbs."""
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, signed)
        seven = -7 if signed else 7
        f.pack(0, [[seven]], 1)
        f.pack(1, [[seven]], 1)
        expected, inp, out = seven, 0, 2
        for step in range(40):
            assert f.multiply(inp, 1, out) == OK, step
            expected *= seven
            assert value_of(f.export(out, 3)[0, 0], signed) == expected, step
            inp, out = out, inp
        f.close()


@pytest.mark.parametrize("signed", [True, False])
def test_overflowing_link_rejected_before_changing_anything(r8, signed):
    """:64-92 — (INT64_MIN)^2 (or (2^64-1)^2) is admitted; one more factor
    exceeds M_20 / 2 and is a RANGE_ERROR that leaves the destination
    unwritten and the source as it was; with a zero factor the link runs."""
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, signed)
        big = -(2**63) if signed else 2**64 - 1
        f.pack(0, [[big]], 11)
        f.pack(1, [[big]], 12)
        assert f.multiply(0, 1, 2) == OK
        before = f.mats[2].storage_info().source_version
        assert f.multiply(2, 1, 3) == RANGE
        assert f.mats[3].storage_info().source_version == 0
        assert f.mats[2].storage_info().source_version == before
        assert value_of(f.export(2, 3)[0, 0], signed) == big * big
        f.pack(1, [[0]], 13)
        assert f.multiply(2, 1, 3) == OK
        assert value_of(f.export(3, 3)[0, 0], signed) == 0
        f.close()


def test_range_proof_counts_k_and_ignores_host_padding(r8):
    """:94-116 — 2 x 2 operands packed from rows of 3 whose third column is
    INT64_MIN padding: C = A x B, D = C x B, D exports as {29, -30, -67, 70}
    in two limbs."""
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, True, 2, 2, 2)
        a = np.array([[2, -3, -(2**63)], [-1, 4, -(2**63)]], np.int64)
        b = np.array([[5, -6, -(2**63)], [7, -8, -(2**63)]], np.int64)
        f.mats[0].pack_i64(a[:, :2], source_version=1)
        f.mats[1].pack_i64(b[:, :2], source_version=1)
        assert f.multiply(0, 1, 2) == OK
        assert f.multiply(2, 1, 3) == OK
        out = f.export(3, 2)
        assert [value_of(out[i, j], True) for i in range(2) for j in range(2)] == [29, -30, -67, 70]
        f.close()


def test_aliases_and_unwritten_higher_planes(r8):
    """:118-152 — an output aliasing an input is INVALID_ARGUMENT; a product
    computed under prefix 18 holds only 18 valid planes, so a prefix-20 plan
    refuses it as an operand and as an export source (RANGE_ERROR, output
    untouched) until the matrix is repacked."""
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, False, prefix=18)
        f.pack(0, [[17]], 1)
        f.pack(1, [[17]], 2)
        assert f.multiply(0, 1, 0) == INVALID
        assert f.multiply(0, 1, 1) == INVALID
        assert value_of(f.export(0, 1)[0, 0], False) == 17
        assert f.multiply(0, 1, 2) == OK
        larger = r8.Plan(ctx, r8.gemm_desc(S.EXACT_WIDE_UNSIGNED, BK.NONE, 1, 1, 1, max_prefix=20,
                                           flags=r8.PLAN_FORCE_FIXED_PREFIX))
        lws = r8.Workspace(ctx, larger)
        assert f.multiply(2, 1, 3, larger, lws) == RANGE
        out = np.full(3, 777, np.uint64)
        assert lib.rns8_export_exact_wide_unsigned_limbs(ctx.handle, larger.handle, f.mats[2].handle,
                                                         out.ctypes.data_as(C.c_void_p), 1, 3) == RANGE
        assert (out == 777).all()
        f.pack(2, [[17]], 3)
        assert f.multiply(2, 1, 3, larger, lws) == OK
        assert value_of(f.export(3, 3, larger)[0, 0], False) == 17 * 17
        lws.close()
        larger.close()
        f.close()


@pytest.mark.parametrize("signed", [True, False])
def test_pack_rejects_values_outside_the_matrix_range(r8, signed):
    """:170-188 — a one-plane exact-wide matrix (M = 256) cannot hold 128
    signed (centered range [-128, 127]) or 256 unsigned: pack is a
    RANGE_ERROR and the matrix keeps source version 0."""
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    with r8.Context(0) as ctx:
        m = r8.Matrix(ctx, 1, 1, S.EXACT_WIDE_SIGNED if signed else S.EXACT_WIDE_UNSIGNED, BK.NONE, 1)
        v = np.array([[128]], np.int64) if signed else np.array([[256]], np.uint64)
        fn = lib.rns8_pack_i64 if signed else lib.rns8_pack_u64
        assert fn(ctx.handle, m.handle, v.ctypes.data_as(C.c_void_p), 1, 1) == RANGE
        assert m.storage_info().source_version == 0
        m.close()


def test_cancellation_safe_wide_chain(r8):
    """test_exact_wide_axis_cases.inc:1-27 — A of INT64_MAX and B = [[h, -h],
    [-h, h]] give C = 0 exactly, so C x A is admitted (D = 0); with B all
    positive, C = 2h^2 and C x A (4h^3 > M_20 / 2) is a RANGE_ERROR that
    leaves D as it was."""
    h = 2**63 - 1
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, True, 2, 2, 2)
        f.pack(0, [[h, h], [h, h]], 1)
        f.pack(1, [[h, -h], [-h, h]], 1)
        assert f.multiply(0, 1, 2) == OK
        assert f.multiply(2, 0, 3) == OK
        assert (f.export(3, 3) == 0).all()
        version = f.mats[3].storage_info().source_version
        f.pack(1, [[h, h], [h, h]], 2)
        assert f.multiply(0, 1, 2) == OK
        assert value_of(f.export(2, 3)[0, 0], True) == 2 * h * h
        assert f.multiply(2, 0, 3) == RANGE
        assert f.mats[3].storage_info().source_version == version
        assert (f.export(3, 3) == 0).all()
        f.close()


def test_axis_bounds_through_a_heterogeneous_unsigned_chain(r8):
    """test_exact_wide_axis_cases.inc:51-68 — diag(100, 7, 1) x I x I: both
    links admitted, D exports as A in two limbs."""
    a = [[100, 0, 0], [0, 7, 0], [0, 0, 1]]
    eye = [[1, 0, 0], [0, 1, 0], [0, 0, 1]]
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, False, 3, 3, 3)
        f.pack(0, a, 1)
        f.pack(1, eye, 1)
        assert f.multiply(0, 1, 2) == OK
        assert f.multiply(2, 1, 3) == OK
        out = f.export(3, 2)
        assert out[:, :, 0].tolist() == a and (out[:, :, 1] == 0).all()
        f.close()


def test_rejected_repack_keeps_the_matrix(r8):
    """test_exact_wide_axis_cases.inc:90-102 — a one-plane matrix holding 7
    refuses 128 (RANGE_ERROR) and keeps its source version."""
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    with r8.Context(0) as ctx:
        m = r8.Matrix(ctx, 1, 1, S.EXACT_WIDE_SIGNED, BK.NONE, 1)
        m.pack_i64(np.array([[7]], np.int64), source_version=1)
        v = np.array([[128]], np.int64)
        assert lib.rns8_pack_i64(ctx.handle, m.handle, v.ctypes.data_as(C.c_void_p), 1, 2) == RANGE
        assert m.storage_info().source_version == 1
        m.close()


@pytest.mark.parametrize("signed", [True, False])
def test_export_refuses_other_interpretations(r8, signed):
    """test_exact_wide_rns_contract_cases.inc (signed and unsigned "rejects
    ... interpretations"): an exact-wide product exported as the other
    signedness, as bounded uint64 / int64, or as wrap64 is INVALID_ARGUMENT
    with the destination untouched."""
    lib = r8.lib()
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, signed)
        f.pack(0, [[-7 if signed else 7]], 1)
        f.pack(1, [[11]], 1)
        assert f.multiply(0, 1, 2) == OK
        dst = np.array([0xDDDDDDDDDDDDDDDD, 0xEEEEEEEEEEEEEEEE], np.uint64)
        ptr = dst.ctypes.data_as(C.c_void_p)
        h, p, c = ctx.handle, f.plan.handle, f.mats[2].handle
        other = lib.rns8_export_exact_wide_unsigned_limbs if signed else lib.rns8_export_exact_wide_signed_limbs
        assert other(h, p, c, ptr, 1, 2) == INVALID
        assert lib.rns8_export_u64(h, p, c, ptr, 1) == INVALID
        assert lib.rns8_export_i64(h, p, c, ptr, 1) == INVALID
        assert lib.rns8_export_wrap_u64(h, p, c, ptr, 1) == INVALID
        assert dst.tolist() == [0xDDDDDDDDDDDDDDDD, 0xEEEEEEEEEEEEEEEE]
        assert value_of(f.export(2, 2)[0, 0], signed) == (-77 if signed else 77)
        f.close()


def test_unsigned_high_bit_fixed_width(r8):
    """tests/differential/test_hip_direct_exact_wide_export_cases.inc:245-303:
    C = [2^127, 0] (2 x 2^63 x 2^63) exports in two limbs as [0, 2^63 | 0, 0],
    is a RANGE_ERROR in one limb (destination untouched), and in 32 limbs
    has every limb above the second zero."""
    lib = r8.lib()
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, False, 1, 2, 2)
        f.pack(0, [[2**63, 2**63]], 1)
        f.pack(1, [[2**63, 0], [2**63, 0]], 1)
        assert f.multiply(0, 1, 2) == OK
        two = f.export(2, 2)
        assert two.reshape(-1).tolist() == [0, 2**63, 0, 0]
        one = np.full(2, 0x9D9D9D9D9D9D9D9D, np.uint64)
        assert lib.rns8_export_exact_wide_unsigned_limbs(ctx.handle, f.plan.handle, f.mats[2].handle,
                                                         one.ctypes.data_as(C.c_void_p), 2, 1) == RANGE
        assert (one == 0x9D9D9D9D9D9D9D9D).all()
        wide = f.export(2, 32)
        assert wide[0, 0, :2].tolist() == [0, 2**63] and (wide[0, 0, 2:] == 0).all() and (wide[0, 1] == 0).all()
        f.close()


@pytest.mark.parametrize("signed", [True, False])
def test_every_fixed_limb_width(r8, signed):
    """tests/differential/test_hip_direct_exact_wide_residue_cases.inc:278-353:
    C = -1 (signed) exports as all-ones limbs and C = 1 (unsigned) as 1
    followed by zero limbs, at widths 1, 2, 3, 4, 8, 16 and 32."""
    with r8.Context(0) as ctx:
        f = Chain(r8, ctx, signed)
        f.pack(0, [[-1 if signed else 1]], 1)
        f.pack(1, [[1]], 1)
        assert f.multiply(0, 1, 2) == OK
        for width in (1, 2, 3, 4, 8, 16, 32):
            limbs = f.export(2, width)[0, 0].tolist()
            assert limbs == ([2**64 - 1] * width if signed else [1] + [0] * (width - 1)), width
        f.close()
