"""The reference's bounded-GEMM unit cases (tests/unit/test_bounded_gemm_basic_cases.inc,
test_bounded_gemm_per_tile_cases.inc, test_bounded_gemm_schedule_cases.inc)
and its bounded differential / qualification cases
(tests/differential/test_hip_direct_bounded_oneshot_cases.inc,
test_hip_direct_qualification_cases.inc) through this library's public C
ABI: input-range descriptors (bound = K * lhs_bound * rhs_bound), prefix
selection, per-tile contracts and schedules, signs, cancellation and
full-width boundaries, K-split edges, and range errors that leave outputs
untouched. Descriptor validation and schedules run on the host
(rns8_cuda_plan_probe, rns8_cuda_plan_tile_schedule_probe; no GPU); the
products run on the GPU."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

OK, INVALID, RANGE = 0, 1, 5


@pytest.fixture(scope="module")
def r8():
    import rns8_b200

    rns8_b200.lib()
    return rns8_b200


def desc(r8, semantics, m, n, k, bound=0, bound_kind=None, lhs=0, rhs=0, max_prefix=0, finite_modulus=0):
    S, BK = r8.Semantics, r8.BoundKind
    if bound_kind is None:
        bound_kind = BK.GLOBAL_MAX_ABS if semantics == S.BOUNDED_I64 else BK.GLOBAL_MAX_UNSIGNED
    return r8.gemm_desc(semantics, bound_kind, m, n, k, bound=bound, lhs_bound=lhs, rhs_bound=rhs,
                        max_prefix=max_prefix, finite_modulus=finite_modulus)


def test_input_range_descriptor_validation(r8):
    S, BK = r8.Semantics, r8.BoundKind
    st, sel, req, eb = r8.api.plan_probe(desc(r8, S.BOUNDED_I64, 2, 2, 3, bound_kind=BK.INPUT_RANGE_AND_K, lhs=7,
                                              rhs=11))
    assert st == OK and eb == 3 * 7 * 11 and sel == req
    assert r8.api.plan_probe(desc(r8, S.BOUNDED_U64, 1, 1, 4, bound=1, bound_kind=BK.INPUT_RANGE_AND_K, lhs=1,
                                  rhs=1))[0] == INVALID  # a stale global bound
    assert r8.api.plan_probe(desc(r8, S.BOUNDED_U64, 1, 1, 4, bound_kind=BK.INPUT_RANGE_AND_K, lhs=2**64 - 1,
                                  rhs=2))[0] == RANGE  # K * lhs * rhs overflows the u64 contract
    assert r8.api.plan_probe(desc(r8, S.BOUNDED_I64, 1, 1, 4, bound_kind=BK.INPUT_RANGE_AND_K, lhs=2**63,
                                  rhs=2))[0] == RANGE
    assert r8.api.plan_probe(desc(r8, S.BOUNDED_U64, 1, 1, 1, bound=1, lhs=1))[0] == INVALID  # stale lhs field
    assert r8.api.plan_probe(desc(r8, S.FINITE_RING_U8, 1, 1, 1, bound_kind=BK.NONE, lhs=1,
                                  finite_modulus=255))[0] == INVALID
    # bounded plan creation rejects insufficient prefix range (:350-358)
    assert r8.api.plan_probe(desc(r8, S.BOUNDED_I64, 1, 1, 1, bound=2**63 - 1, max_prefix=8))[0] == RANGE


def test_per_tile_plan_with_overflowing_tile_count(r8):
    """test_api_validation_cases.inc:59-71: a per-tile plan over INT64_MAX^2
    cells is a range error, before any tile bound is read."""
    S, BK = r8.Semantics, r8.BoundKind
    d = r8.gemm_desc(S.BOUNDED_I64, BK.PER_TILE_MAX_ABS, 2**63 - 1, 2**63 - 1, 1, tile_m=64, tile_n=64)
    tb = (C.c_uint64 * 1)(1)
    d.tile_bounds = C.cast(tb, C.POINTER(C.c_uint64))
    d.tile_bounds_count = 2**64 - 1
    assert r8.api.plan_probe(d)[0] == RANGE


@pytest.mark.gpu
def test_input_range_persistent_and_oneshot(r8):
    S, BK = r8.Semantics, r8.BoundKind
    with r8.Context(0) as ctx:
        d = desc(r8, S.BOUNDED_I64, 2, 2, 3, bound_kind=BK.INPUT_RANGE_AND_K, lhs=7, rhs=11)
        plan = r8.Plan(ctx, d)
        info = plan.schedule_info()
        assert info.bound_kind == BK.INPUT_RANGE_AND_K and info.effective_bound == 3 * 7 * 11
        assert info.lhs_bound == 7 and info.rhs_bound == 11
        assert info.bound_contract.decode() == "input_range_and_k_derived_output_bound"
        assert info.max_selected_prefix == info.min_required_prefix
        # Contract vocabulary of the info queries (api_plan_contract_names.inc:39-52, 462-530).
        bi = plan.backend_info()
        assert bi.accumulator_input_domain.decode() == "centered_i8_rns_residue_planes"
        assert bi.accumulator_signedness.decode() == "signed_i8x_signed_i8"
        assert bi.accumulator_type.decode() == "int32"
        assert bi.accumulator_modulus_policy.decode() == "selected_rns_modulus_ladder"
        assert bi.accumulator_safety_status.decode() == "safe_int32_k_block_split"
        a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
        ws = r8.Workspace(ctx, plan)
        a.pack_i64(np.array([[7, -2, 3], [-1, 4, -5]], np.int64), source_version=10)
        b.pack_i64(np.array([[2, -3], [6, 1], [-4, 5]], np.int64), source_version=11)
        r8.gemm_rns(ctx, plan, a, b, c, ws)
        assert r8.export_i64(ctx, plan, c).ravel().tolist() == [-10, -8, 42, -18]
        for h in (a, b, c, ws, plan):
            h.close()
        one = r8.gemm_i64_oneshot(ctx, desc(r8, S.BOUNDED_I64, 1, 2, 2, bound_kind=BK.INPUT_RANGE_AND_K, lhs=5, rhs=6),
                                  np.array([[5, -4]], np.int64), np.array([[6, -3], [2, 1]], np.int64))
        assert one.ravel().tolist() == [22, -19]
        one = r8.gemm_u64_oneshot(ctx, desc(r8, S.BOUNDED_U64, 2, 1, 2, bound_kind=BK.INPUT_RANGE_AND_K, lhs=9, rhs=8),
                                  np.array([[9, 1], [2, 3]], np.uint64), np.array([[8], [7]], np.uint64))
        assert one.ravel().tolist() == [79, 37]


@pytest.mark.gpu
@pytest.mark.parametrize("signed", [True, False])
def test_too_small_bound_keeps_padded_output(r8, signed):
    """:317-348 — a valid but too small global bound: RANGE_ERROR and every
    element of the padded output (ldc = 4 for n = 2) keeps its sentinel."""
    S = r8.Semantics
    with r8.Context(0) as ctx:
        if signed:
            A = np.array([[6], [-6]], np.int64)
            B = np.array([[7, -7, 999]], np.int64)[:, :2]
            sentinel, dtype, fn = -0x123456789, np.int64, r8.gemm_i64_oneshot
        else:
            A = np.array([[6], [8]], np.uint64)
            B = np.array([[7, 1, 999]], np.uint64)[:, :2]
            sentinel, dtype, fn = 0xBADC0FFEE0DDF00D, np.uint64, r8.gemm_u64_oneshot
        C = np.full((2, 4), sentinel, dtype)
        with pytest.raises(r8.Error) as err:
            fn(ctx, desc(r8, S.BOUNDED_I64 if signed else S.BOUNDED_U64, 2, 2, 1, bound=41), A, B, out=C[:, :2])
        assert err.value.status == r8.Status.RANGE_ERROR
        assert (C == dtype(sentinel)).all()


def test_per_tile_contracts_reject_missing_or_inconsistent_bounds(r8):
    """test_bounded_gemm_per_tile_cases.inc (per-tile bound contracts): no
    tile bounds, too few, a global bound beside them, and a signed tile bound
    beyond 2^63 are INVALID_ARGUMENT; a global signed bound of 2^63 + 1
    likewise (test_bounded_gemm_schedule_cases.inc, int64 min)."""
    S, BK = r8.Semantics, r8.BoundKind
    probe = lambda d: r8.api.plan_probe(d)[0]
    d = r8.gemm_desc(S.BOUNDED_U64, BK.PER_TILE_MAX_UNSIGNED, 65, 65, 1, tile_m=64, tile_n=64)
    assert probe(d) == INVALID
    r8.api.set_tile_bounds(d, [7, 1000, 7000000])
    assert probe(d) == INVALID
    r8.api.set_tile_bounds(d, [7, 1000, 7000000, 1000000000])
    d.bound = 1
    assert probe(d) == INVALID
    d.bound = 0
    assert probe(d) == OK
    s = r8.gemm_desc(S.BOUNDED_I64, BK.PER_TILE_MAX_ABS, 1, 1, 1)
    r8.api.set_tile_bounds(s, [2**64 - 1])
    assert probe(s) == INVALID
    assert probe(desc(r8, S.BOUNDED_I64, 1, 1, 1, bound=2**63 + 1)) == INVALID
    assert probe(desc(r8, S.BOUNDED_I64, 1, 1, 1, bound=2**63)) == OK


def test_per_tile_schedule_collapses_to_fixed_prefix(r8):
    """test_bounded_gemm_schedule_cases.inc (collapse case): when every tile
    needs the full nine moduli the schedule is one group at prefix 9, each
    entry keeps its own range bit length and the grid geometry of a 65 x 65
    output in 64 x 64 tiles."""
    import math

    S, BK = r8.Semantics, r8.BoundKind
    first_full = math.prod(r8.LADDER[:8]) // 2
    top = 2**63
    d = r8.gemm_desc(S.BOUNDED_I64, BK.PER_TILE_MAX_ABS, 65, 65, 7, tile_m=64, tile_n=64)
    r8.api.set_tile_bounds(d, [top, first_full, top, first_full])
    entries, info = r8.api.plan_tile_schedule_probe(d)
    assert (info.tile_m, info.tile_n, info.tile_rows, info.tile_cols, info.tile_count) == (64, 64, 2, 2, 4)
    assert (info.min_required_prefix, info.max_required_prefix) == (9, 9)
    assert (info.min_selected_prefix, info.max_selected_prefix) == (9, 9)
    assert (info.prefix_group_count, info.adaptive_prefix_active, info.adaptive_skip_active) == (1, 0, 0)
    assert info.range_bit_length == (2 * top).bit_length()
    assert len(entries) == 4
    for e in entries:
        assert (e.required_prefix, e.selected_prefix, e.group_index) == (9, 9, 0)
    assert entries[0].range_bit_length == (2 * top).bit_length()
    assert entries[1].range_bit_length == math.prod(r8.LADDER[:8]).bit_length()
    e0, e3 = entries[0], entries[3]
    assert (e0.row_offset, e0.col_offset, e0.row_extent, e0.col_extent) == (0, 0, 64, 64)
    assert (e3.tile_row, e3.tile_col, e3.row_offset, e3.col_offset, e3.row_extent, e3.col_extent) == (
        1, 1, 64, 64, 1, 1)


@pytest.mark.gpu
@pytest.mark.parametrize("dk", [-1, 0, 1])
def test_k_split_edges_keep_padding_and_cancel_exactly(r8, dk):
    """test_bounded_gemm_schedule_cases.inc (K-split edge cases): K one below,
    at and one above the 65536-product int32-safe block, with padded lda,
    ldb and ldc: alternating +-127 rows cancel exactly, and the padding
    columns of C keep their sentinels."""
    S = r8.Semantics
    k = 65536 + dk
    with r8.Context(0) as ctx:
        product = 127 * 127
        A = np.full((2, k + 1), 0x5A5A5A5A, np.int64)
        B = np.full((k, 3), -0x1234567, np.int64)
        A[0, :k] = np.where(np.arange(k) % 2 == 0, 127, -127)
        A[1, :k] = 127
        B[:, 0], B[:, 1] = 127, -127
        sentinel = -0x51F15E5
        Cm = np.full((2, 4), sentinel, np.int64)
        r8.gemm_i64_oneshot(ctx, desc(r8, S.BOUNDED_I64, 2, 2, k, bound=k * product), A[:, :k], B[:, :2],
                            out=Cm[:, :2])
        alt = 0 if k % 2 == 0 else product
        assert Cm.tolist() == [[alt, -alt, sentinel, sentinel], [k * product, -k * product, sentinel, sentinel]]

        Au = np.full((2, k + 1), 0xFEEDFACEFEEDFACE, np.uint64)
        Bu = np.full((k, 3), 0xDEADBEEFDEADBEEF, np.uint64)
        Au[0, :k], Au[1, :k] = 255, 1
        Bu[:, 0], Bu[:, 1] = 1, 255
        su = 0xC001D00DCAFEF00D
        Cu = np.full((2, 4), su, np.uint64)
        r8.gemm_u64_oneshot(ctx, desc(r8, S.BOUNDED_U64, 2, 2, k, bound=k * 255 * 255), Au[:, :k], Bu[:, :2],
                            out=Cu[:, :2])
        assert Cu.tolist() == [[k * 255, k * 255 * 255, su, su], [k, k * 255, su, su]]


def test_schedule_tile_grid_and_prefix_groups(r8):
    """test_bounded_gemm_schedule_cases.inc (tile grid case): a global bound
    of 1000 over 130 x 129 in 64 x 64 tiles is one group at prefix 2 (10
    range bits, adaptive skip below the default 9), a 3 x 3 grid whose last
    tile is 2 x 1; a schedule buffer of 8 is WORKSPACE_TOO_SMALL with the
    count still written."""
    S, BK = r8.Semantics, r8.BoundKind
    d = r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 130, 129, 7, bound=1000, tile_m=64, tile_n=64)
    entries, info = r8.api.plan_tile_schedule_probe(d)
    assert (info.tile_m, info.tile_n, info.tile_rows, info.tile_cols, info.tile_count) == (64, 64, 3, 3, 9)
    assert (info.min_required_prefix, info.max_required_prefix, info.min_selected_prefix,
            info.max_selected_prefix) == (2, 2, 2, 2)
    assert (info.prefix_group_count, info.adaptive_prefix_active, info.adaptive_skip_active) == (1, 0, 1)
    assert info.range_bit_length == 10
    e0, e8 = entries[0], entries[-1]
    assert (e0.tile_row, e0.tile_col, e0.row_offset, e0.col_offset, e0.row_extent, e0.col_extent) == (0, 0, 0, 0, 64,
                                                                                                    64)
    assert (e0.required_prefix, e0.selected_prefix, e0.group_index, e0.range_bit_length) == (2, 2, 0, 10)
    assert (e8.tile_row, e8.tile_col, e8.row_offset, e8.col_offset, e8.row_extent, e8.col_extent) == (2, 2, 128, 128,
                                                                                                    2, 1)
    small = (r8.abi.PlanTileScheduleEntry * 8)()
    for e in small:
        e.struct_size, e.abi_version = C.sizeof(e), 1
    written = C.c_uint64()
    st = r8.lib().rns8_cuda_plan_tile_schedule_probe(C.byref(d), small, 8, C.byref(written), None)
    assert st == 7 and written.value == 9  # RNS8_WORKSPACE_TOO_SMALL


def test_schedule_from_copied_per_tile_bounds(r8):
    """test_bounded_gemm_schedule_cases.inc (copied per-tile bounds): nine
    tile bounds from 1 to 2^40 give prefixes 1..6 in five groups (group
    index ordered by prefix), 41 range bits."""
    S, BK = r8.Semantics, r8.BoundKind
    bounds = [1, 1000, 1000000, 2**40, 5, 2000, 70000, 2**20, 2**32]
    d = r8.gemm_desc(S.BOUNDED_U64, BK.PER_TILE_MAX_UNSIGNED, 130, 129, 7, tile_m=64, tile_n=64)
    r8.api.set_tile_bounds(d, bounds)
    entries, info = r8.api.plan_tile_schedule_probe(d)
    assert (info.tile_rows, info.tile_cols, info.tile_count) == (3, 3, 9)
    assert (info.min_required_prefix, info.max_required_prefix, info.min_selected_prefix,
            info.max_selected_prefix) == (1, 6, 1, 6)
    assert (info.prefix_group_count, info.adaptive_prefix_active, info.adaptive_skip_active) == (5, 1, 1)
    assert info.range_bit_length == 41
    got = [(e.required_prefix, e.selected_prefix, e.group_index) for e in entries]
    assert got[0] == (1, 1, 0) and got[1] == (2, 2, 1) and got[2] == (3, 3, 2) and got[3] == (6, 6, 4)
    assert got[8] == (5, 5, 3)
    e8 = entries[8]
    assert (e8.row_offset, e8.col_offset, e8.row_extent, e8.col_extent) == (128, 128, 2, 1)


def test_zero_output_skips_need_the_opt_in(r8):
    """test_bounded_gemm_schedule_cases.inc (proven-zero opt-in): zero tile
    bounds flag ZERO_OUTPUT tiles only with ALLOW_PROVEN_ZERO_TILE_SKIPS;
    without it they run at prefix 1 with 0 range bits; the flag on a global
    plan is INVALID_ARGUMENT."""
    S, BK = r8.Semantics, r8.BoundKind
    bounds = [0, 1000, 0, 1000000]
    d = r8.gemm_desc(S.BOUNDED_U64, BK.PER_TILE_MAX_UNSIGNED, 65, 65, 1, tile_m=64, tile_n=64)
    r8.api.set_tile_bounds(d, bounds)
    entries, info = r8.api.plan_tile_schedule_probe(d)
    assert info.flags == 0
    assert (entries[0].range_bit_length, entries[0].required_prefix, entries[0].selected_prefix,
            entries[0].flags, entries[2].flags) == (0, 1, 1, 0, 0)
    d = r8.gemm_desc(S.BOUNDED_U64, BK.PER_TILE_MAX_UNSIGNED, 65, 65, 1, tile_m=64, tile_n=64, flags=2)
    r8.api.set_tile_bounds(d, bounds)
    entries, info = r8.api.plan_tile_schedule_probe(d)
    ZERO = 1  # RNS8_TILE_SCHEDULE_ZERO_OUTPUT
    assert info.flags == ZERO
    assert [e.flags for e in entries] == [ZERO, 0, ZERO, 0]
    assert entries[0].range_bit_length == 0 and entries[2].range_bit_length == 0
    g = r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 1, 1, 1, bound=1, flags=2)
    assert r8.api.plan_probe(g)[0] == INVALID


def test_default_and_fixed_prefix_selection(r8):
    """test_bounded_gemm_basic_cases.inc:127-169, 350-420: bound 1000 selects
    prefix 2 (adaptive skip) unless FORCE_FIXED_PREFIX keeps the default 9;
    INT64_MAX at max_prefix 8 is a RANGE_ERROR; 2^63 signed and 2^64 - 1
    unsigned need exactly prefix 9 (8 is a RANGE_ERROR)."""
    S, BK = r8.Semantics, r8.BoundKind
    d = desc(r8, S.BOUNDED_U64, 2, 2, 3, bound=1000)
    _, info = r8.api.plan_tile_schedule_probe(d)
    assert (info.min_required_prefix, info.max_required_prefix, info.min_selected_prefix, info.max_selected_prefix,
            info.adaptive_skip_active) == (2, 2, 2, 2, 1)
    d.flags = r8.PLAN_FORCE_FIXED_PREFIX
    _, info = r8.api.plan_tile_schedule_probe(d)
    assert (info.min_required_prefix, info.max_required_prefix, info.min_selected_prefix, info.max_selected_prefix,
            info.adaptive_skip_active) == (2, 2, 9, 9, 0)
    assert r8.api.plan_probe(desc(r8, S.BOUNDED_I64, 1, 1, 1, bound=2**63 - 1, max_prefix=8))[0] == RANGE
    for sem, bound in ((S.BOUNDED_I64, 2**63), (S.BOUNDED_U64, 2**64 - 1)):
        assert r8.api.plan_probe(desc(r8, sem, 1, 1, 1, bound=bound, max_prefix=8))[0] == RANGE
        _, info = r8.api.plan_tile_schedule_probe(desc(r8, sem, 1, 1, 1, bound=bound, max_prefix=9))
        assert (info.min_required_prefix, info.max_required_prefix, info.min_selected_prefix,
                info.max_selected_prefix) == (9, 9, 9, 9)


@pytest.mark.gpu
def test_oneshot_signs_cancellation_and_full_boundaries(r8):
    """test_bounded_gemm_basic_cases.inc:1-126: signs and cancellation
    (2x3 x 3x2 -> {-188, 51, -268, 881}; 123456789 - 123456789 -> 0 under
    bound 1); outputs at INT64_MAX, -INT64_MAX, INT64_MIN (bound 2^63) and
    UINT64_MAX; full-width values with padded lda = ldb = 3 and ldc = 4
    leaving the padding untouched."""
    S = r8.Semantics
    I64MIN, I64MAX, U = -(2**63), 2**63 - 1, 2**64 - 1
    with r8.Context(0) as ctx:
        A = np.array([[7, -3, 5], [-11, 13, 17]], np.int64)
        B = np.array([[2, -5], [19, 23], [-29, 31]], np.int64)
        assert r8.gemm_i64_oneshot(ctx, desc(r8, S.BOUNDED_I64, 2, 2, 3, bound=100000), A, B).ravel().tolist() == [
            -188, 51, -268, 881]
        out = np.array([[99]], np.int64)
        r8.gemm_i64_oneshot(ctx, desc(r8, S.BOUNDED_I64, 1, 1, 2, bound=1), np.array([[123456789, 123456789]],
                            np.int64), np.array([[1], [-1]], np.int64), out=out)
        assert out[0, 0] == 0
        for a, bound, want in ((I64MAX, I64MAX, I64MAX), (-I64MAX, I64MAX, -I64MAX), (I64MIN, 2**63, I64MIN)):
            got = r8.gemm_i64_oneshot(ctx, desc(r8, S.BOUNDED_I64, 1, 1, 1, bound=bound), np.array([[a]], np.int64),
                                      np.array([[1]], np.int64))
            assert got[0, 0] == want
        got = r8.gemm_u64_oneshot(ctx, desc(r8, S.BOUNDED_U64, 1, 1, 1, bound=U), np.array([[U]], np.uint64),
                                  np.array([[1]], np.uint64))
        assert int(got[0, 0]) == U
        # Padded full-width: signed
        s = 0x1020304050607
        A = np.full((2, 3), s, np.int64)
        B = np.full((2, 3), -s, np.int64)
        A[0, :2] = [I64MIN, 0]
        A[1, :2] = [I64MAX, -I64MAX]
        B[0, :2] = [1, 0]
        B[1, :2] = [0, 1]
        Cm = np.full((2, 4), s, np.int64)
        r8.gemm_i64_oneshot(ctx, desc(r8, S.BOUNDED_I64, 2, 2, 2, bound=2**63), A[:, :2], B[:, :2], out=Cm[:, :2])
        assert Cm.tolist() == [[I64MIN, 0, s, s], [I64MAX, -I64MAX, s, s]]
        # Padded full-width: unsigned
        su = 0xAAAAAAAAAAAAAAAA
        A = np.full((2, 3), su, np.uint64)
        B = np.full((2, 3), su, np.uint64)
        A[0, :2] = [U, U - 1]
        A[1, :2] = [0, 1]
        B[0, :2] = [1, 0]
        B[1, :2] = [0, 1]
        Cm = np.full((2, 4), su, np.uint64)
        r8.gemm_u64_oneshot(ctx, desc(r8, S.BOUNDED_U64, 2, 2, 2, bound=U), A[:, :2], B[:, :2], out=Cm[:, :2])
        assert [[int(x) for x in row] for row in Cm] == [[U, U - 1, su, su], [0, 1, su, su]]


def per_tile(r8, signed, bounds, flags=0, m=65, n=65, k=1):
    S, BK = r8.Semantics, r8.BoundKind
    d = r8.gemm_desc(S.BOUNDED_I64 if signed else S.BOUNDED_U64,
                     BK.PER_TILE_MAX_ABS if signed else BK.PER_TILE_MAX_UNSIGNED, m, n, k, flags=flags, tile_m=64,
                     tile_n=64)
    r8.api.set_tile_bounds(d, bounds)
    return d


@pytest.mark.gpu
def test_per_tile_oneshots(r8):
    """test_bounded_gemm_per_tile_cases.inc:1-153: too-small per-tile bounds
    (2 x 3 = 6 against 5, or against a 0 bound without the proven-zero flag)
    are RANGE_ERROR with the padded C untouched; with the flag, zero-bound
    tiles are written as zeros; unsigned and signed per-tile prefixes
    (bounds 7 .. 1e9) export every cell exactly."""
    m = n = 65
    with r8.Context(0) as ctx:
        for signed, bounds in ((True, [5, 10, 10, 10]), (False, [5, 10, 10, 10]), (False, [0, 10, 10, 10])):
            dt = np.int64 if signed else np.uint64
            fn = r8.gemm_i64_oneshot if signed else r8.gemm_u64_oneshot
            C = np.full((m, 67), -99 if signed else 123, dt)
            with pytest.raises(r8.Error) as err:
                fn(ctx, per_tile(r8, signed, bounds), np.full((m, 1), 2, dt), np.full((1, n), 3, dt), out=C[:, :n])
            assert err.value.status == r8.Status.RANGE_ERROR
            assert (C == (-99 if signed else 123)).all()
        A = np.array([[1 if r < 64 else 1000] for r in range(m)], np.uint64)
        B = np.array([[0 if c < 64 else 7 for c in range(n)]], np.uint64)
        C = np.full((m, n + 1), 0xDEADBEEFDEADBEEF, np.uint64)
        r8.gemm_u64_oneshot(ctx, per_tile(r8, False, [0, 7, 0, 7000], flags=2), A, B, out=C[:, :n])
        np.testing.assert_array_equal(C[:, :n], A @ B)
        assert (C[:, n] == 0xDEADBEEFDEADBEEF).all()
        A = np.array([[1 if r < 64 else 1000000] for r in range(m)], np.uint64)
        B = np.array([[7 if c < 64 else 1000 for c in range(n)]], np.uint64)
        got = r8.gemm_u64_oneshot(ctx, per_tile(r8, False, [7, 1000, 7000000, 1000000000]), A, B)
        np.testing.assert_array_equal(got, A @ B)
        A = np.array([[-2 if r < 64 else -1000000] for r in range(m)], np.int64)
        B = np.array([[3 if c < 64 else -1000 for c in range(n)]], np.int64)
        got = r8.gemm_i64_oneshot(ctx, per_tile(r8, True, [6, 2000, 3000000, 1000000000]), A, B)
        np.testing.assert_array_equal(got, A @ B)


@pytest.mark.gpu
def test_cancellation_and_full_width_stressors(r8):
    """tests/differential/test_hip_direct_bounded_oneshot_cases.inc:241-337:
    full-range int64 terms that cancel to results inside a small bound (the
    residue arithmetic is exact modulo M, so intermediate sums beyond int64
    do not matter); INT64_MIN / INT64_MAX and UINT64_MAX / UINT64_MAX - 42
    through an identity with max_prefix 20; and K = 65537 unsigned at the
    exact bound K * 255 * 2."""
    S = r8.Semantics
    I64MIN, I64MAX, U = -(2**63), 2**63 - 1, 2**64 - 1
    with r8.Context(0) as ctx:
        A = np.array([[I64MAX, I64MIN + 1, 37, -37], [1000000000, -1000000000, -12345, 12345]], np.int64)
        B = np.array([[1, 1], [1, 1], [1000000, 1000000], [1000000, -1000000]], np.int64)
        got = r8.gemm_i64_oneshot(ctx, desc(r8, S.BOUNDED_I64, 2, 2, 4, bound=30000000000), A, B)
        assert got.ravel().tolist() == [0, 74000000, 0, -24690000000]
        eye = np.array([[1, 0], [0, 1]])
        got = r8.gemm_i64_oneshot(ctx, desc(r8, S.BOUNDED_I64, 1, 2, 2, bound=2**63, max_prefix=20),
                                  np.array([[I64MIN, I64MAX]], np.int64), eye.astype(np.int64))
        assert got.ravel().tolist() == [I64MIN, I64MAX]
        got = r8.gemm_u64_oneshot(ctx, desc(r8, S.BOUNDED_U64, 1, 2, 2, bound=U, max_prefix=20),
                                  np.array([[U, U - 42]], np.uint64), eye.astype(np.uint64))
        assert [int(x) for x in got.ravel()] == [U, U - 42]
        k = 65537
        Au = np.full((1, k), 255, np.uint64)
        Bu = np.zeros((k, 2), np.uint64)
        Bu[:, 0], Bu[:, 1] = 1, 2
        got = r8.gemm_u64_oneshot(ctx, desc(r8, S.BOUNDED_U64, 1, 2, k, bound=k * 255 * 2), Au, Bu)
        assert [int(x) for x in got.ravel()] == [k * 255, k * 255 * 2]


@pytest.mark.gpu
def test_bounded_export_every_prefix_and_every_failing_cell(r8):
    """tests/differential/test_hip_direct_qualification_cases.inc:33-82: a
    1 x 65 output of 2s (bound 10) at prefixes 1, 7, 8, 9, 20, signed and
    unsigned, with no failing cell or one out-of-bound cell (-11 / 11) at
    every position: the export succeeds or is a RANGE_ERROR accordingly, and
    a failing export leaves all 68 destination elements untouched."""
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    cols = 65
    with r8.Context(0) as ctx:
        for prefix in (1, 7, 8, 9, 20):
            for signed in (False, True):
                sem = S.BOUNDED_I64 if signed else S.BOUNDED_U64
                bk = BK.GLOBAL_MAX_ABS if signed else BK.GLOBAL_MAX_UNSIGNED
                plan = r8.Plan(ctx, r8.gemm_desc(sem, bk, 1, cols, 1, bound=10, max_prefix=prefix,
                                                 flags=r8.PLAN_FORCE_FIXED_PREFIX))
                assert plan.prefix == prefix
                mat = r8.Matrix(ctx, 1, cols, sem, bk, prefix)
                dt = np.int64 if signed else np.uint64
                fn = lib.rns8_export_i64 if signed else lib.rns8_export_u64
                for bad in range(-1, cols):
                    vals = np.full((1, cols), 2, dt)
                    if bad >= 0:
                        vals[0, bad] = -11 if signed else 11
                    (mat.pack_i64 if signed else mat.pack_u64)(vals)
                    out = np.full(cols + 3, -777 if signed else 777, dt)
                    st = fn(ctx.handle, plan.handle, mat.handle, out.ctypes.data_as(C.c_void_p), cols + 3)
                    if bad < 0:
                        assert st == OK and out[:cols].tolist() == [2] * cols, prefix
                        assert (out[cols:] == (-777 if signed else 777)).all()
                    else:
                        assert st == RANGE, (prefix, signed, bad)
                        assert (out == (-777 if signed else 777)).all()
                mat.close()
                plan.close()


@pytest.mark.gpu
@pytest.mark.parametrize("k", [65535, 65536, 65537, 131073, 262145])
def test_persistent_gemm_spans_safe_k_blocks(r8, k):
    """tests/differential/test_hip_direct_qualification_cases.inc:84-126:
    (-127) x (-127) summed over K across one to five 65536-product blocks."""
    S, BK = r8.Semantics, r8.BoundKind
    with r8.Context(0) as ctx:
        plan = r8.Plan(ctx, r8.gemm_desc(S.BOUNDED_I64, BK.GLOBAL_MAX_ABS, 1, 1, k, bound=k * 127 * 127))
        ws = r8.Workspace(ctx, plan)
        a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
        a.pack_i64(np.full((1, k), -127, np.int64))
        b.pack_i64(np.full((k, 1), -127, np.int64))
        r8.gemm_rns(ctx, plan, a, b, c, ws)
        assert r8.export_i64(ctx, plan, c)[0, 0] == k * 127 * 127
        for h in (a, b, c, ws, plan):
            h.close()


@pytest.mark.gpu
def test_per_tile_k_split_centered_cancellation(r8):
    """tests/differential/test_hip_direct_per_tile_cases.inc:1-49: one tile
    bounded by 127^2 over K = 65537 alternating +-127: the tile runs at its
    required prefix (below the plan's 9), and C = [127^2, -127^2] with the
    padded column untouched."""
    k = 65537
    d = per_tile(r8, True, [127 * 127], m=1, n=2, k=k)
    entries, info = r8.api.plan_tile_schedule_probe(d)
    assert len(entries) == 1 and entries[0].selected_prefix == entries[0].required_prefix < 9
    A = np.full((1, k + 1), -0x55AA55AA, np.int64)
    B = np.full((k, 3), -0x55AA55AA, np.int64)
    A[0, :k] = np.where(np.arange(k) % 2 == 0, 127, -127)
    B[:, 0], B[:, 1] = 127, -127
    C = np.full((1, 3), -0x55AA55AA, np.int64)
    with r8.Context(0) as ctx:
        r8.gemm_i64_oneshot(ctx, d, A[:, :k], B[:, :2], out=C[:, :2])
    assert C.tolist() == [[127 * 127, -127 * 127, -0x55AA55AA]]


@pytest.mark.gpu
def test_persistent_prefix9_exact_k_block_reused(r8):
    """tests/differential/test_hip_direct_bounded_schedule_cases.inc:401-520:
    u64, K = 65536 exactly, prefix 9 forced, padded host layouts; the same
    resident matrices serve two rounds of new inputs."""
    S, BK = r8.Semantics, r8.BoundKind
    k = 65536
    with r8.Context(0) as ctx:
        plan = r8.Plan(ctx, r8.gemm_desc(S.BOUNDED_U64, BK.GLOBAL_MAX_UNSIGNED, 2, 2, k, bound=k * 12,
                                         flags=r8.PLAN_FORCE_FIXED_PREFIX))
        assert plan.prefix == 9
        info = plan.schedule_info()
        assert (info.min_selected_prefix, info.max_selected_prefix, info.adaptive_prefix_active) == (9, 9, 0)
        ws = r8.Workspace(ctx, plan)
        a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
        s = 0xD1FFD1FFD1FFD1FF
        for variant, (a0, a1, b0, b1) in enumerate(((1, 2, 3, 5), (2, 3, 1, 4))):
            A = np.full((2, k + 1), s, np.uint64)
            B = np.full((k, 3), s, np.uint64)
            A[0, :k], A[1, :k] = a0, a1
            B[:, 0], B[:, 1] = b0, b1
            a.pack_u64(A[:, :k], source_version=10 + variant)
            b.pack_u64(B[:, :2], source_version=20 + variant)
            r8.gemm_rns(ctx, plan, a, b, c, ws)
            out = np.full((2, 3), s, np.uint64)
            r8.export_u64(ctx, plan, c, out=out[:, :2])
            want = [[k * a0 * b0, k * a0 * b1], [k * a1 * b0, k * a1 * b1]]
            assert [[int(x) for x in row[:2]] for row in out] == want
            assert (out[:, 2] == s).all()
        for h in (a, b, c, ws, plan):
            h.close()


@pytest.mark.gpu
@pytest.mark.parametrize("signed", [True, False])
def test_export_range_errors_repeat_without_side_effects(r8, signed):
    """tests/differential/test_hip_direct_bounded_residency_cases.inc:179-306:
    a prefix-1 plan (bound 10) exporting [-11, 7] (or [11, 3]) is a
    RANGE_ERROR twice in a row, the destination keeps its fill, and the
    matrix stays device-current."""
    S, BK = r8.Semantics, r8.BoundKind
    lib = r8.lib()
    sem = S.BOUNDED_I64 if signed else S.BOUNDED_U64
    bk = BK.GLOBAL_MAX_ABS if signed else BK.GLOBAL_MAX_UNSIGNED
    with r8.Context(0) as ctx:
        plan = r8.Plan(ctx, r8.gemm_desc(sem, bk, 1, 2, 1, bound=10))
        assert plan.prefix == 1
        c = r8.Matrix(ctx, 1, 2, sem, bk, 0)
        if signed:
            c.pack_i64(np.array([[-11, 7]], np.int64))
            fill, out, fn = 0x1212121212121212, np.full(2, 0x1212121212121212, np.int64), lib.rns8_export_i64
        else:
            c.pack_u64(np.array([[11, 3]], np.uint64))
            fill, out, fn = 0xFEFEFEFEFEFEFEFE, np.full(2, 0xFEFEFEFEFEFEFEFE, np.uint64), lib.rns8_export_u64
        for _ in range(2):
            assert fn(ctx.handle, plan.handle, c.handle, out.ctypes.data_as(C.c_void_p), 2) == RANGE
            assert [int(x) for x in out] == [fill if not signed else 0x1212121212121212] * 2
            si = c.storage_info()
            assert (si.host_residues_current, si.device_residues_current) == (0, 1)
        c.close()
        plan.close()
