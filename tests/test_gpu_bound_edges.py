"""Large bounded one-shots at the edges of the bound contract, on a shape of
592 output tiles (four full waves of the tensor-core kernel on 148 SMs) with
partial edge tiles in both dimensions, checked against exact products: float64
GEMMs where |C| < 2^53, closed forms where the values sit at the bound.

Cases: signed and unsigned random products, a padded output with odd ld,
a few rows exactly at the bound (cells in the fractional CRT's undecided band,
settled by the exact Garner path), every cell at the bound, and range errors
just past the bound (rejected by the exact path) and far past it (rejected by
the fraction), both leaving C untouched."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

M, N, K = 4700, 4080, 128  # 37 x 16 = 592 output tiles: four full waves on 148 SMs


@pytest.fixture(scope="module")
def r8():
    import rns8_b200

    rns8_b200.lib()
    return rns8_b200


@pytest.fixture(scope="module")
def ctx(r8):
    with r8.Context(0) as c:
        yield c


def desc(r8, signed, bound, m=M, n=N, k=K, prefix=0):
    S, BK = r8.Semantics, r8.BoundKind
    return r8.gemm_desc(S.BOUNDED_I64 if signed else S.BOUNDED_U64,
                        BK.GLOBAL_MAX_ABS if signed else BK.GLOBAL_MAX_UNSIGNED, m, n, k, bound=bound,
                        max_prefix=prefix, flags=r8.PLAN_FORCE_FIXED_PREFIX if prefix else 0)


def prefix_of(r8, ctx, d):
    plan = r8.Plan(ctx, d)
    P = plan.prefix
    plan.close()
    return P


@pytest.mark.parametrize("signed", [True, False])
def test_random_products_with_partial_tiles(r8, ctx, signed):
    rng = np.random.default_rng(11 if signed else 12)
    if signed:
        A = rng.integers(-(2**20), 2**20, (M, K), dtype=np.int64, endpoint=True)
        B = rng.integers(-(2**20), 2**20, (K, N), dtype=np.int64, endpoint=True)
        bound, fn, dt = 2**47, r8.gemm_i64_oneshot, np.int64
    else:
        A = rng.integers(0, 2**21, (M, K), dtype=np.uint64)
        B = rng.integers(0, 2**21, (K, N), dtype=np.uint64)
        bound, fn, dt = 2**49, r8.gemm_u64_oneshot, np.uint64
    d = desc(r8, signed, bound)
    out = fn(ctx, d, A, B)
    want = (A.astype(np.float64) @ B.astype(np.float64)).astype(dt)  # |C| < 2^53: exact
    np.testing.assert_array_equal(out, want)


def test_padded_output_odd_ld(r8, ctx):
    rng = np.random.default_rng(13)
    A = rng.integers(-(2**20), 2**20, (M, K), dtype=np.int64, endpoint=True)
    B = rng.integers(-(2**20), 2**20, (K, N), dtype=np.int64, endpoint=True)
    d = desc(r8, True, 2**47)
    sentinel = -0x5EED
    Cp = np.full((M, N + 1), sentinel, np.int64)
    r8.gemm_i64_oneshot(ctx, d, A, B, out=Cp[:, :N])
    np.testing.assert_array_equal(Cp[:, :N], (A.astype(np.float64) @ B.astype(np.float64)).astype(np.int64))
    assert (Cp[:, N] == sentinel).all()


def edge_inputs(rows_at_edge, extra=0):
    """B = 2^27 everywhere; A small except the listed rows, which are 2^27 in
    every column (their cells are exactly 2^61 = the bound), plus `extra` on
    the first such row's first element."""
    rng = np.random.default_rng(14)
    A = rng.integers(-(2**20), 2**20, (M, K), dtype=np.int64, endpoint=True)
    for r in rows_at_edge:
        A[r, :] = 2**27
    if rows_at_edge and extra:
        A[rows_at_edge[0], 0] += extra
    B = np.full((K, N), 2**27, np.int64)
    want = np.repeat((A.sum(axis=1) * 2**27)[:, None], N, axis=1)  # |A row sum| * 2^27 fits int64
    return A, B, want


def test_rows_at_the_bound(r8, ctx):
    rows = [0, 1777, M - 1]  # 3 x 4080 cells at v = bound
    A, B, want = edge_inputs(rows)
    d = desc(r8, True, 2**61, prefix=9)
    assert prefix_of(r8, ctx, d) == 9
    out = r8.gemm_i64_oneshot(ctx, d, A, B)
    assert (out[rows] == 2**61).all()
    np.testing.assert_array_equal(out, want)


def test_every_cell_at_the_bound(r8, ctx):
    A = np.full((M, K), 2**27, np.int64)
    B = np.full((K, N), -(2**27), np.int64)
    d = desc(r8, True, 2**61, prefix=9)
    out = r8.gemm_i64_oneshot(ctx, d, A, B)
    assert (out == -(2**61)).all()


@pytest.mark.parametrize("extra", [1, 2**27])
def test_range_errors_past_the_bound_leave_c_untouched(r8, ctx, extra):
    """extra = 1: one row at 2^61 + 2^27, inside the fraction's undecided band
    (the exact path rejects it); extra = 2^27: a row at 2^62, far outside (the
    fraction rejects it)."""
    A, B, _ = edge_inputs([5], extra=extra if extra == 1 else 0)
    if extra != 1:
        A[5, :] = 2**28  # row 5 cells: 2^28 * 2^27 * 128 = 2^62
    d = desc(r8, True, 2**61, prefix=9)
    C = np.full((M, N), 7, np.int64)
    with pytest.raises(r8.Error) as err:
        r8.gemm_i64_oneshot(ctx, d, A, B, out=C)
    assert err.value.status == r8.Status.RANGE_ERROR
    assert (C == 7).all()
