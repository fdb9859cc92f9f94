"""Exact-wide admission proofs on the device against the oracle's restatement
of src/core/exact_range.hpp:51-154: the 256-bit admission bound, the operand
maxima and the per-row / per-column records of the cell bounds, bit for bit;
and the decisions of a chained exact-wide GEMM through the public API."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

LADDER = [256, 255, 253, 251, 247, 239, 233, 229, 227, 223, 217, 211, 199, 197, 193, 191, 181, 179, 173, 167]


@pytest.fixture(scope="module")
def lib():
    import rns8_b200

    return rns8_b200.lib()


@pytest.fixture(scope="module")
def oracle():
    from oracle import bridge

    return bridge


def limbs(v: np.ndarray) -> int:
    return sum(int(x) << (64 * i) for i, x in enumerate(v))


def device_bound(lib, A: np.ndarray, B: np.ndarray):
    m, k = A.shape
    n = B.shape[1]
    signed = A.dtype == np.int64
    dA = torch.from_numpy(A.view(np.int64).copy()).cuda()
    dB = torch.from_numpy(B.view(np.int64).copy()).cuda()
    bound, amax, bmax = (np.zeros(4, np.uint64) for _ in range(3))
    rows = np.zeros((m, 8), np.uint64)
    cols = np.zeros((n, 8), np.uint64)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = lib.rns8_cuda_exact_gemm_bound_device(0, dA.data_ptr(), dB.data_ptr(), m, n, k, 1 if signed else 0,
                                               bound.ctypes.data, amax.ctypes.data, bmax.ctypes.data,
                                               rows.ctypes.data, cols.ctypes.data, stream)
    assert st == 0
    pair = lambda v: (limbs(v[:4]), limbs(v[4:]))
    return limbs(bound), limbs(amax), limbs(bmax), [pair(r) for r in rows], [pair(c) for c in cols]


def inputs(kind: str, m: int, n: int, k: int, seed: int):
    rng = np.random.default_rng(seed)
    if kind == "full_signed":
        A = rng.integers(-(2**63), 2**63 - 1, (m, k), dtype=np.int64, endpoint=True)
        B = rng.integers(-(2**63), 2**63 - 1, (k, n), dtype=np.int64, endpoint=True)
    elif kind == "full_unsigned":
        A = rng.integers(0, 2**64 - 1, (m, k), dtype=np.uint64, endpoint=True)
        B = rng.integers(0, 2**64 - 1, (k, n), dtype=np.uint64, endpoint=True)
    elif kind == "skewed":  # row / column scales spread over 60 bits: tightening picks different bounds per cell
        A = rng.integers(-(2**3), 2**3, (m, k), dtype=np.int64) << rng.integers(0, 60, (m, 1))
        B = rng.integers(-(2**3), 2**3, (k, n), dtype=np.int64) << rng.integers(0, 60, (1, n))
    elif kind == "offset":  # values far from zero with a small spread: the centered bound wins
        A = (2**62 + rng.integers(-1000, 1000, (m, k))).astype(np.int64)
        B = (-(2**61) + rng.integers(-7, 7, (k, n))).astype(np.int64)
        A[0, :] = 2**62  # a constant row: zero deviation
    else:  # extremes: INT64_MIN / INT64_MAX / 0
        A = rng.choice(np.array([-(2**63), 2**63 - 1, 0, -1], np.int64), (m, k))
        B = rng.choice(np.array([-(2**63), 2**63 - 1, 0, 1], np.int64), (k, n))
    return A, B


@pytest.mark.parametrize("kind", ["full_signed", "full_unsigned", "skewed", "offset", "extremes"])
@pytest.mark.parametrize("m,n,k", [
    (1, 1, 1),
    (33, 257, 5),       # ragged warp and 256-column tile
    (300, 64, 17),
    (2100, 40, 3),      # more than 64 groups of 32 rows: blocks loop over row groups
    (8, 8300, 2),       # more than one 8192-column stripe
])
def test_admission_bound_and_records_match_oracle(lib, oracle, kind, m, n, k):
    A, B = inputs(kind, m, n, k, m * 7 + n + k)
    st, want_bound = oracle.exact_gemm_admission(A, B, 20)
    assert st == 0
    want_rows, want_cols = oracle.exact_gemm_cell_stats(A, B)
    bound, amax, bmax, rows, cols = device_bound(lib, A, B)
    assert bound == want_bound
    assert amax == max(abs(int(v)) for v in A.ravel())
    assert bmax == max(abs(int(v)) for v in B.ravel())
    assert rows == want_rows
    assert cols == want_cols


def modulus_product(P: int) -> int:
    out = 1
    for m in LADDER[:P]:
        out *= m
    return out


def test_chained_exact_wide_gemm_decisions(oracle):
    """C = A x B (full-range int64), then D = C x E: the second GEMM's
    admission uses C's recorded row bounds (the reference keeps them in
    commit_exact_range) and E's native column ranges. The decision at each
    prefix must equal the one the reference's arithmetic gives."""
    import rns8_b200 as r8

    rng = np.random.default_rng(11)
    m, k1, n1, n2 = 24, 4, 16, 20
    A = rng.integers(-(2**63), 2**63 - 1, (m, k1), dtype=np.int64, endpoint=True)
    B = rng.integers(-(2**63), 2**63 - 1, (k1, n1), dtype=np.int64, endpoint=True)
    E = rng.integers(-40, 40, (n1, n2), dtype=np.int64, endpoint=True)
    # Reference arithmetic for the chain (exact_range.hpp:79-143, with C's rows
    # carrying only max and sum): bound2 = min(K*Cmax*Emax, max over cells).
    st, c_max = oracle.exact_gemm_admission(A, B, 20)
    assert st == 0
    c_rows, _ = oracle.exact_gemm_cell_stats(A, B)
    e_cols = [(max(abs(int(v)) for v in E[:, c]), sum(abs(int(v)) for v in E[:, c])) for c in range(n2)]
    e_max = max(abs(int(v)) for v in E.ravel())
    cells = max(min(n1 * ra * eb, rs * eb, ra * es) for ra, rs in c_rows for eb, es in e_cols)
    bound2 = min(n1 * c_max * e_max, cells)
    ctx = r8.Context(0)
    decided = []
    try:
        for P in (17, 18, 19, 20):
            d1 = r8.gemm_desc(r8.Semantics.EXACT_WIDE_SIGNED, r8.BoundKind.NONE, m, n1, k1, max_prefix=P,
                              flags=r8.PLAN_FORCE_FIXED_PREFIX)
            d2 = r8.gemm_desc(r8.Semantics.EXACT_WIDE_SIGNED, r8.BoundKind.NONE, m, n2, n1, max_prefix=P,
                              flags=r8.PLAN_FORCE_FIXED_PREFIX)
            p1, p2 = r8.Plan(ctx, d1), r8.Plan(ctx, d2)
            a, b, c = (r8.Matrix.for_plan(ctx, p1, r) for r in "abc")
            e, d = r8.Matrix.for_plan(ctx, p2, "b"), r8.Matrix.for_plan(ctx, p2, "c")
            w1, w2 = r8.Workspace(ctx, p1), r8.Workspace(ctx, p2)
            a.pack_i64(A)
            b.pack_i64(B)
            e.pack_i64(E)
            r8.gemm_rns(ctx, p1, a, b, c, w1)
            want_ok = 2 * bound2 < modulus_product(P)
            if want_ok:
                r8.gemm_rns(ctx, p2, c, e, d, w2)
                got = r8.export_exact_wide_limbs(ctx, p2, d, 3, signed=True)
                exact_c = np.array(oracle.exact_product(A, B), dtype=object)
                exact_d = exact_c.dot(E.astype(object))
                val = lambda v: (lambda x: x - (1 << 192) if x >> 191 else x)(sum(int(v[l]) << (64 * l) for l in range(3)))
                assert all(val(got[i, j]) == exact_d[i, j] for i in range(m) for j in range(n2))
            else:
                with pytest.raises(r8.Error) as err:
                    r8.gemm_rns(ctx, p2, c, e, d, w2)
                assert err.value.status == r8.Status.RANGE_ERROR
            decided.append(want_ok)
            for h in (a, b, c, e, d, w1, w2, p1, p2):
                h.close()
    finally:
        ctx.close()
    assert True in decided and False in decided, (bound2.bit_length(), decided)
