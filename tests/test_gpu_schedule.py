"""Per-tile bound plans on the GPU: the scheduled plane GEMM (adaptive prefix
per tile, proven-zero tiles) and the per-tile export, through the public API,
against the oracle's restatement of cpu_reference.cpp:221-260 and
api_export.cpp:365-414. Bounds are set tight, loose, zero (proven-zero
tiles) and too small (a caller's broken promise: the reference then exports
what the selected planes reconstruct, or RANGE_ERROR), and the results must
agree bit for bit, status included."""

from __future__ import annotations

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


def scaled_inputs(rng, m, n, k, signed, tile_m, zero_rows=()):
    """A with row blocks scaled by very different powers of two, so that tiles
    need different prefixes; rows in zero_rows are zero."""
    lo = -(2**10) if signed else 0
    dtype = np.int64 if signed else np.uint64
    A = rng.integers(lo, 2**10, (m, k), dtype=dtype, endpoint=True)
    B = rng.integers(lo, 2**10, (k, n), dtype=dtype, endpoint=True)
    for r0 in range(0, m, tile_m):
        A[r0:r0 + tile_m] *= dtype(2 ** int(rng.integers(0, 24)))
    for r in zero_rows:
        A[r] = 0
    return A, B


def tile_max(C, m, n, tile_m, tile_n):
    out = []
    for r0 in range(0, m, tile_m):
        for c0 in range(0, n, tile_n):
            out.append(int(np.abs(C[r0:r0 + tile_m, c0:c0 + tile_n].astype(object)).max()))
    return out


def oracle_run(oracle, A, B, plan_prefix_storage, sel, tile_m, tile_n, bounds, signed):
    P = plan_prefix_storage
    a, b = oracle.pack(A, P), oracle.pack(B, P)
    c = np.zeros((P, A.shape[0], B.shape[1]), np.int8)  # a fresh matrix holds zero planes
    oracle.gemm_rns_scheduled(a, b, c, tile_m, tile_n, sel)
    return oracle.export_scheduled(c, tile_m, tile_n, sel, bounds, signed)


def sel_of(entries, plan_prefix):
    if not entries:
        return None
    return [e.selected_prefix | (0x80 if e.flags & 1 else 0) for e in entries]


def run_public(r8, ctx, desc, A, B, signed):
    plan = r8.Plan(ctx, desc)
    a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
    ws = r8.Workspace(ctx, plan)
    (a.pack_i64 if signed else a.pack_u64)(A)
    (b.pack_i64 if signed else b.pack_u64)(B)
    r8.gemm_rns(ctx, plan, a, b, c, ws)
    try:
        out, st = (r8.export_i64 if signed else r8.export_u64)(ctx, plan, c), 0
    except r8.Error as e:
        out, st = None, int(e.status)
    entries, info = plan.tile_schedule(), plan.schedule_info()
    for h in (a, b, c, ws, plan):
        h.close()
    return st, out, entries, info


@pytest.mark.parametrize("m,n,k,tile_m,tile_n,variants", [
    (384, 512, 64, 128, 128, ("tight", "loose", "lying")),  # tensor cores; a kernel tile covers two schedule tiles
    (320, 448, 48, 64, 256, ("tight", "loose", "lying")),   # 64-row schedule tiles
    (200, 200, 40, 128, 64, ("tight", "loose", "lying")),   # N, K not multiples of 16: SIMT + masked copy
    (128, 128, 65552, 64, 64, ("tight", "lying")),          # K above 65536: split-K with the masked finalize
])
@pytest.mark.parametrize("signed", [True, False])
def test_scheduled_gemm_and_export_match_oracle(r8, ctx, oracle, m, n, k, tile_m, tile_n, variants, signed):
    rng = np.random.default_rng(m + n + k + signed)
    zero_rows = range(0, tile_m) if m > tile_m else ()  # the first row block of C is zero
    A, B = scaled_inputs(rng, m, n, k, signed, tile_m, zero_rows)
    C = A @ B  # |C| < 2^60: exact in 64-bit integers
    exact = tile_max(C, m, n, tile_m, tile_n)
    bk = r8.BoundKind.PER_TILE_MAX_ABS if signed else r8.BoundKind.PER_TILE_MAX_UNSIGNED
    sem = r8.Semantics.BOUNDED_I64 if signed else r8.Semantics.BOUNDED_U64
    all_bounds = {
        "tight": exact,
        "loose": [4 * b + 3 for b in exact],
        "lying": [b // 300 if i % 3 == 1 else b for i, b in enumerate(exact)],  # some tiles promise too little
    }
    for name in variants:
        bounds = all_bounds[name]
        for flags in (0, 2):  # ALLOW_PROVEN_ZERO_TILE_SKIPS: zero bounds skip their tiles
            desc = r8.gemm_desc(sem, bk, m, n, k, flags=flags, tile_m=tile_m, tile_n=tile_n)
            r8.api.set_tile_bounds(desc, bounds)
            st, out, entries, info = run_public(r8, ctx, desc, A, B, signed)
            sel = sel_of(entries, 9)
            if info.prefix_group_count == 1 and info.flags == 0 and info.min_selected_prefix == 9:
                sel = [9] * len(bounds)
            ost, want = oracle_run(oracle, A, B, info.max_selected_prefix, sel, tile_m, tile_n, bounds, signed)
            assert st == ost, (name, flags)
            if st == 0:
                np.testing.assert_array_equal(out, want)
                if name != "lying":
                    np.testing.assert_array_equal(out, C)
            if name == "tight":
                assert info.adaptive_prefix_active == 1  # the scaled row blocks need several prefixes
            # The one-shot entry point runs the same schedule.
            one = np.zeros((m, n), np.int64 if signed else np.uint64)
            fn = r8.gemm_i64_oneshot if signed else r8.gemm_u64_oneshot
            try:
                fn(ctx, desc, A, B, out=one)
                ost1 = 0
            except r8.Error as e:
                ost1 = int(e.status)
            assert ost1 == ost, (name, flags)
            if ost1 == 0:
                np.testing.assert_array_equal(one, want)


def test_zero_row_col_flags_and_grouped_scheduled(r8, ctx, oracle):
    """Zero row / column proofs flag tiles (ZERO_ROW_COL_PRODUCT) without
    changing values; a grouped call under a scheduled plan runs every task."""
    rng = np.random.default_rng(5)
    m, n, k, tm, tn = 256, 256, 64, 128, 128
    tasks_in = [scaled_inputs(rng, m, n, k, True, tm) for _ in range(3)]
    for A, B in tasks_in:
        A[7] = 0
        B[:, 9] = 0
    za = np.zeros(m, np.uint8)
    za[7] = 1
    zb = np.zeros(n, np.uint8)
    zb[9] = 1
    bounds = [max(tile_max(A @ B, m, n, tm, tn)[t] for A, B in tasks_in) for t in range(4)]
    desc = r8.gemm_desc(r8.Semantics.BOUNDED_I64, r8.BoundKind.PER_TILE_MAX_ABS, m, n, k, flags=4, tile_m=tm,
                        tile_n=tn)
    r8.api.set_tile_bounds(desc, bounds, za, zb)
    plan = r8.Plan(ctx, desc)
    info = plan.schedule_info()
    assert info.zero_a_row_count == 1 and info.zero_b_col_count == 1
    assert info.zero_row_col_product_count == 1 * n + (m - 1) * 1
    entries = plan.tile_schedule()
    assert [e.flags for e in entries] == [2, 2, 2, 0]  # row 7 lies in tile row 0, column 9 in tile column 0
    handles, tasks = [], []
    for A, B in tasks_in:
        a, b, c = (r8.Matrix.for_plan(ctx, plan, role) for role in "abc")
        ws = r8.Workspace(ctx, plan)
        a.pack_i64(A)
        b.pack_i64(B)
        tasks.append((a, b, c, ws))
        handles += [a, b, c, ws]
    r8.gemm_rns_grouped(ctx, plan, tasks)
    for (A, B), (_, _, c, _) in zip(tasks_in, tasks):
        np.testing.assert_array_equal(r8.export_i64(ctx, plan, c), A @ B)
    for h in handles + [plan]:
        h.close()


def test_resident_bounded_chain(r8, ctx):
    """C = A x B stays resident as residues and feeds D = C x E without an
    export (the persistent-residue model, api_gemm.cpp:938-961); only D is
    exported, with the second plan's bound."""
    rng = np.random.default_rng(9)
    m, k, n, n2 = 256, 64, 128, 96
    A = rng.integers(-(2**12), 2**12, (m, k), dtype=np.int64, endpoint=True)
    B = rng.integers(-(2**12), 2**12, (k, n), dtype=np.int64, endpoint=True)
    E = rng.integers(-(2**12), 2**12, (n, n2), dtype=np.int64, endpoint=True)
    D = (A @ B) @ E  # |D| < 2^49
    bound = int(np.abs(D).max())
    sem, bk = r8.Semantics.BOUNDED_I64, r8.BoundKind.GLOBAL_MAX_ABS
    p1 = r8.Plan(ctx, r8.gemm_desc(sem, bk, m, n, k, bound=2**40, max_prefix=8, flags=r8.PLAN_FORCE_FIXED_PREFIX))
    p2 = r8.Plan(ctx, r8.gemm_desc(sem, bk, m, n2, n, bound=bound, max_prefix=8, flags=r8.PLAN_FORCE_FIXED_PREFIX))
    a, b, c = (r8.Matrix.for_plan(ctx, p1, role) for role in "abc")
    e, d = r8.Matrix.for_plan(ctx, p2, "b"), r8.Matrix.for_plan(ctx, p2, "c")
    w1, w2 = r8.Workspace(ctx, p1), r8.Workspace(ctx, p2)
    a.pack_i64(A)
    b.pack_i64(B)
    e.pack_i64(E)
    r8.gemm_rns(ctx, p1, a, b, c, w1)
    r8.gemm_rns(ctx, p2, c, e, d, w2)  # C's residue planes are the next A
    np.testing.assert_array_equal(r8.export_i64(ctx, p2, d), D)
    for h in (a, b, c, e, d, w1, w2, p1, p2):
        h.close()
