"""Pins the CPU oracle before anything is checked against it.

Three independent anchors:
  * golden outputs of the reference's own epilogue arithmetic
    (tests/golden/reducer_vectors.json, made by oracle/_ref);
  * known answers stated in the reference's tests (tests/golden/reference_kats.json);
  * exact Python big-int products for the reference's public-API sweeps
    (tests/unit/test_bounded_reference_sweeps.cpp:161-502).
"""

import json
import math
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
KATS = json.loads((GOLDEN / "reference_kats.json").read_text())
REDUCER = json.loads((GOLDEN / "reducer_vectors.json").read_text())
OK, INVALID, UNSUPPORTED, RANGE = 0, 1, 4, 5


def centered(v, m):
    r = v % m
    return r - m if r >= (m + 1) // 2 else r


def test_ladder_and_range_bits(oracle):
    assert [oracle.lib().oracle_modulus(i) for i in range(28)] == KATS["ladder"]["moduli"]
    for p, bits in KATS["prefix_range_bits"]["table"].items():
        assert abs(oracle.lib().oracle_prefix_range_bits(int(p)) - bits) <= 0.002
    for i in range(28):
        for j in range(i + 1, 28):
            assert math.gcd(KATS["ladder"]["moduli"][i], KATS["ladder"]["moduli"][j]) == 1


def test_modulus_products_and_prefix_boundaries(oracle):
    products = [int(p) for p in KATS["modulus_products"]["products"]]
    for prefix in range(1, 21):
        assert oracle.modulus_product(prefix) == products[prefix]
        assert oracle.required_prefix_for_range(products[prefix] - 1) == prefix
        assert oracle.required_prefix_for_range(products[prefix]) == (prefix + 1 if prefix < 20 else 0)
    assert products[9] > 2**64 > products[8]
    assert oracle.required_prefix_for_range(2**64 - 1) == 9
    assert oracle.required_prefix_for_range(2**64) == 9


def test_centered_residue_kats(oracle):
    for v, m, want in KATS["centered_residues"]["cases"]:
        assert oracle.lib().oracle_centered_residue_i64(v, m) == want
    r = oracle.lib().oracle_centered_residue_i64(-(2**63), 251)
    assert -125 <= r <= 125 and r == centered(-(2**63), 251)


def test_reducer_matches_reference_reducer(oracle):
    values = REDUCER["values"]
    for m_str, expected in REDUCER["reduce_to_centered_i32"].items():
        m = int(m_str)
        got = [oracle.lib().oracle_reduce_to_centered(v, m) for v in values]
        assert got == expected, m
        assert expected == [centered(v, m) for v in values]


def test_finite_u8_center_matches_reference(oracle):
    src = np.arange(256, dtype=np.uint8).reshape(1, 256)
    for m_str, expected in REDUCER["center_u8"].items():
        assert oracle.pack_finite_u8(src, int(m_str)).ravel().tolist() == expected


def test_residue_dot_k_splits(oracle):
    for case in REDUCER["residue_dot"][::7]:  # every 7th of 240 cases keeps the CPU suite fast
        k, m, lo = case["k"], case["modulus"], case["lo"]
        a = np.full(k, lo, np.int8)
        b = np.full(k * 3, 73, np.int8)
        idx = np.arange(k)
        b[::3] = np.where(case["alternating"] & (idx % 2 == 1), 1, lo).astype(np.int8)
        got = oracle.lib().oracle_centered_residue_dot(a.ctypes.data, b.ctypes.data, k, 3, m)
        assert got == case["expected"] == centered(case["exact_sum"], m)


def residues_for(v, prefix):
    return np.array([centered(v, m) for m in KATS["ladder"]["moduli"][:prefix]], np.int8)


def test_crt_known_answers(oracle):
    import ctypes as C

    out = C.c_int64()
    for v, p, bound, want in KATS["crt_roundtrips"]["signed"]:
        st = oracle.lib().oracle_reconstruct_signed(residues_for(v, p).ctypes.data, p, bound, C.addressof(out))
        assert (st, out.value if st == OK else None) == ((OK, v) if want == "ok" else (RANGE, None))
    uout = C.c_uint64()
    for v, p, bound, want in KATS["crt_roundtrips"]["unsigned"]:
        v = int(v)
        st = oracle.lib().oracle_reconstruct_unsigned(residues_for(v, p).ctypes.data, p, bound, C.addressof(uout))
        assert (st, uout.value if st == OK else None) == ((OK, v) if want == "ok" else (RANGE, None))
    for p in KATS["crt_canonical"]["prefixes"]:
        P = oracle.modulus_product(p)
        for v in (0, 1, P // 2, P - 1):
            limbs = np.zeros(4, np.uint64)
            oracle.lib().oracle_reconstruct_canonical(residues_for(v, p).ctypes.data, p, limbs.ctypes.data)
            assert oracle.from_limbs4(limbs) == v
    t = KATS["crt_threshold_prefix2"]
    assert oracle.modulus_product(2) == t["product"] and (t["product"] + 1) // 2 == t["threshold"]
    for v, bound, want, value in t["cases"]:
        out.value = 123
        st = oracle.lib().oracle_reconstruct_signed(residues_for(v, 2).ctypes.data, 2, bound, C.addressof(out))
        assert st == (OK if want == "ok" else RANGE)
        assert out.value == (value if want == "ok" else 123)  # failure leaves the output untouched
    ir = KATS["crt_insufficient_range"]
    st = oracle.lib().oracle_reconstruct_signed(residues_for(ir["value"], 8).ctypes.data, 8, ir["bound"],
                                                C.addressof(out))
    assert st == RANGE


def test_ring_gemm_known_answers(oracle):
    kat = KATS["ring_gemm_2x3x4"]
    A = np.array(kat["A"], np.int8).reshape(2, 4)
    B = np.array(kat["B"], np.int8).reshape(4, 3)
    for m in kat["moduli"]:
        assert oracle.ring_gemm(A, B, m).tolist() == kat["expected"][str(m)]
    kk = KATS["ring_gemm_k65537"]
    a = np.full((1, kk["k"]), kk["value"], np.int8)
    b = np.full((kk["k"], 1), kk["value"], np.int8)
    assert oracle.ring_gemm(a, b, kk["modulus"])[0, 0] == kk["expected"]


def test_example_bounded_i64(oracle):
    ex = KATS["example_bounded_i64"]
    A = np.array(ex["A"], np.int64).reshape(ex["m"], ex["k"])
    B = np.array(ex["B"], np.int64).reshape(ex["k"], ex["n"])
    st, C, _ = oracle.gemm_bounded_oneshot(A, B, ex["bound"])
    assert st == OK and C.ravel().tolist() == ex["expected"]


def check_exact(oracle, A, B, signed=True):
    exact = oracle.exact_product(A, B)
    flat = [v for row in exact for v in row]
    bound = max(abs(v) for v in flat) if signed else max(flat)
    st, C, _ = oracle.gemm_bounded_oneshot(A, B, bound)
    assert st == OK
    assert [int(x) for x in C.ravel()] == flat


def test_sweep_all_tiny_dims(oracle):
    # test_bounded_reference_sweeps.cpp:161-206 input formulas.
    for m in range(1, 9):
        for n in range(1, 9):
            for k in range(1, 9):
                A = np.array([[((r * 17 + c * 5 + m - n) % 11) - 5 for c in range(k)] for r in range(m)], np.int64)
                B = np.array([[((r * 7 - c * 13 + k + n) % 13) - 6 for c in range(n)] for r in range(k)], np.int64)
                check_exact(oracle, A, B)
                Au = np.array([[(r * 19 + c * 3 + m + 1) % 17 for c in range(k)] for r in range(m)], np.uint64)
                Bu = np.array([[(r * 5 + c * 11 + n + 2) % 19 for c in range(n)] for r in range(k)], np.uint64)
                check_exact(oracle, Au, Bu, signed=False)


def test_seeded_random_trials(oracle):
    # test_bounded_reference_sweeps.cpp:209-243 with its seed and draw order.
    rng = oracle.Rng(0x8A5CD13F00D)
    import ctypes as C

    for _ in range(32):
        m = 1 + rng.next() % 8
        n = 1 + rng.next() % 8
        k = 1 + rng.next() % 8
        lda, ldb = k + 1, n + 1
        sa = np.full((m, lda), 12345, np.int64)
        sb = np.full((k, ldb), -12345, np.int64)
        ua = np.full((m, lda), 99999, np.uint64)
        ub = np.full((k, ldb), 99999, np.uint64)
        for r in range(m):
            for c in range(k):
                sa[r, c] = rng.i64(-31, 31, 1)[0]
                ua[r, c] = rng.u64(0, 63, 1)[0]
        for r in range(k):
            for c in range(n):
                sb[r, c] = rng.i64(-31, 31, 1)[0]
                ub[r, c] = rng.u64(0, 63, 1)[0]
        check_exact(oracle, sa[:, :k], sb[:, :n])
        check_exact(oracle, ua[:, :k], ub[:, :n], signed=False)


@pytest.mark.parametrize("k", [65535, 65536, 65537])
def test_k_split_cancellation(oracle, k):
    # test_bounded_reference_sweeps.cpp:245-281
    kk = np.arange(k)
    A = np.where(kk % 2 == 0, 127, -127).astype(np.int64).reshape(1, k)
    B = np.stack([np.full(k, 127), np.full(k, -127)], axis=1).astype(np.int64)
    exact = [int((A[0].astype(object) * B[:, j].astype(object)).sum()) for j in range(2)]
    st, C, _ = oracle.gemm_bounded_oneshot(A, B, max(abs(v) for v in exact) or 1)
    assert st == OK and C.ravel().tolist() == exact
    Au = np.full((1, k), 255, np.uint64)
    Bu = np.stack([np.full(k, 1), np.full(k, 255)], axis=1).astype(np.uint64)
    exact = [255 * k, 255 * 255 * k]
    st, C, _ = oracle.gemm_bounded_oneshot(Au, Bu, max(exact))
    assert st == OK and [int(v) for v in C.ravel()] == exact


def test_padded_full_width_outputs(oracle):
    # test_bounded_reference_sweeps.cpp:283-368
    sentinel = 0xAAAAAAAAAAAAAAAA
    A = np.full((2, 3), sentinel, np.uint64)
    B = np.full((2, 3), sentinel, np.uint64)
    C = np.full((2, 3), sentinel, np.uint64)
    A[0, 0], A[0, 1], A[1, 0], A[1, 1] = 2**64 - 1, 2**64 - 2, 0, 1
    B[0, 0], B[0, 1], B[1, 0], B[1, 1] = 1, 0, 0, 1
    st, C, used = oracle.gemm_bounded_oneshot(A[:, :2], B[:, :2], 2**64 - 1, out=C[:, :2])
    assert st == OK and used == 9
    assert int(C[0, 0]) == 2**64 - 1 and int(C[0, 1]) == 2**64 - 2 and int(C[1, 0]) == 0 and int(C[1, 1]) == 1
    Cfull = C.base if C.base is not None else C
    assert int(Cfull.reshape(2, 3)[0, 2]) == sentinel and int(Cfull.reshape(2, 3)[1, 2]) == sentinel
    s = 0x123456789ABC
    A = np.full((2, 3), s, np.int64)
    B = np.full((2, 3), s, np.int64)
    Cs = np.full((2, 3), s, np.int64)
    A[0, 0], A[0, 1], A[1, 0], A[1, 1] = -(2**63), 2**63 - 1, -(2**63 - 1), 0
    B[0, 0], B[0, 1], B[1, 0], B[1, 1] = 1, 0, 0, 1
    st, out, used = oracle.gemm_bounded_oneshot(A[:, :2], B[:, :2], 2**63, out=Cs[:, :2])
    assert st == OK and used == 9
    assert Cs.tolist() == [[-(2**63), 2**63 - 1, s], [-(2**63 - 1), 0, s]]


@pytest.mark.parametrize("k", [65536, 65537])
def test_worst_case_accumulation(oracle, k):
    # test_bounded_reference_sweeps.cpp:475-513
    for a_val in (127, -128):
        A = np.full((1, k), a_val, np.int64)
        B = np.full((k, 1), 127, np.int64)
        st, C, _ = oracle.gemm_bounded_oneshot(A, B, abs(a_val * 127 * k))
        assert st == OK and int(C[0, 0]) == a_val * 127 * k
    Au = np.full((1, k), 255, np.uint64)
    Bu = np.full((k, 1), 255, np.uint64)
    st, C, _ = oracle.gemm_bounded_oneshot(Au, Bu, 255 * 255 * k)
    assert st == OK and int(C[0, 0]) == 255 * 255 * k


def test_prefix_selection(oracle):
    for sem, bound, max_prefix, force, want in KATS["prefix_selection"]["cases"]:
        st, sel, _, _ = oracle.plan_select_prefix(1 if sem == "i64" else 2, 1 if sem == "i64" else 2, 64, 64, 64,
                                                  bound=bound, max_prefix=max_prefix, flags=force)
        assert st == OK and sel == want


def test_range_error_when_bound_too_small(oracle):
    A = np.array([[1000, 1000]], np.int64)
    B = np.array([[1000], [1000]], np.int64)
    out = np.full((1, 1), 77, np.int64)
    st, out, _ = oracle.gemm_bounded_oneshot(A, B, 1_999_999, out=out)
    assert st == RANGE and int(out[0, 0]) == 77


def test_finite_oneshot_exact(oracle):
    rng = np.random.default_rng(7)
    for m, n, k, mod, field in [(5, 7, 9, 251, True), (8, 3, 70, 256, False), (4, 4, 4, 2, False)]:
        A = rng.integers(0, 256, (m, k), dtype=np.uint8)
        B = rng.integers(0, 256, (k, n), dtype=np.uint8)
        st, C = oracle.gemm_finite_u8_oneshot(A, B, mod, field)
        exact = (A.astype(object) % mod).dot(B.astype(object) % mod) % mod
        assert st == OK and C.astype(int).tolist() == exact.tolist()


def test_exact_wide_limbs_round_trip(oracle):
    rng = np.random.default_rng(3)
    A = rng.integers(-(2**63), 2**63 - 1, (3, 5), dtype=np.int64, endpoint=True)
    B = rng.integers(-(2**63), 2**63 - 1, (5, 4), dtype=np.int64, endpoint=True)
    exact = oracle.exact_product(A, B)
    P = 20
    st, bound = oracle.exact_gemm_admission(A, B, P)
    assert st == OK
    assert bound >= max(abs(v) for row in exact for v in row)  # admission bound is sound
    planes = oracle.gemm_rns(oracle.pack(A, P), oracle.pack(B, P), P)
    st, limbs = oracle.export_limbs(planes, P, 3, signed=True)
    assert st == OK
    for i in range(3):
        for j in range(4):
            v = sum(int(limbs[i, j, l]) << (64 * l) for l in range(3))
            v = v - (1 << 192) if v >> 191 else v
            assert v == exact[i][j]
    st, _ = oracle.export_limbs(planes, P, 1, signed=True)
    assert st == RANGE  # products of full-range int64 need more than 64 bits


def limb_boundary_planes(prefix: int, value: int, cells: int) -> np.ndarray:
    """Centered residue planes (prefix x 1 x cells) of one value in every cell."""
    def centered(v, m):
        r = v % m
        return r - m if r >= (m + 1) // 2 else r
    return np.array([[[centered(value, m)] * cells] for m in LADDER_ALL[:prefix]], np.int8)


LADDER_ALL = KATS["ladder"]["moduli"]


@pytest.mark.parametrize("case", KATS["exact_wide_limb_boundaries"]["cases"])
def test_exact_wide_limb_boundaries(oracle, case):
    """test_exact_wide_limb_boundary_cases.inc:1-127: centered half-open
    representative, one-limb edges, overflow and 32-limb widths."""
    prefix, signed, value, limbs, want = case
    st, got = oracle.export_limbs(limb_boundary_planes(prefix, int(value), 1), prefix, limbs, signed)
    if want == "range":
        assert st == RANGE
    else:
        assert st == OK
        assert [int(v) for v in got[0, 0]] == [int(v) for v in want]


# ---- WRAP_U64_MOD_2_64 -------------------------------------------------------------
def test_wrap64_public_kat(oracle):
    """Inputs of the reference's public wrap64 differential test (padded lda/ldb)."""
    kat = KATS["wrap64_public_2x3x5"]
    m, n, k = kat["m"], kat["n"], kat["k"]
    A = np.array([int(v) for v in kat["A"]], np.uint64).reshape(m, kat["lda"])[:, :k]
    B = np.array([int(v) for v in kat["B"]], np.uint64).reshape(k, kat["ldb"])[:, :n]
    want = np.array([[int(v) for v in row] for row in kat["expected"]], np.uint64)
    np.testing.assert_array_equal(oracle.wrap64_gemm(A, B), want)
    np.testing.assert_array_equal(oracle.wrap64_gemm(A, B, diagonals=True), want)


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 5, 33), (16, 24, 300)])
def test_wrap64_oracles_agree(oracle, m, n, k):
    """Native uint64 accumulation (wrap64_reference.cpp:254-290) and the 36-pair
    Comba-diagonal restatement (:166-190) agree, and match numpy's wrapping
    uint64 matmul, on random and extreme values."""
    rng = np.random.default_rng(m * 100 + k)
    A = rng.integers(0, 2**64 - 1, (m, k), dtype=np.uint64, endpoint=True)
    B = rng.integers(0, 2**64 - 1, (k, n), dtype=np.uint64, endpoint=True)
    A[0, :] = 2**64 - 1
    B[:, 0] = 0x8080808080808080
    want = A @ B  # numpy integer matmul wraps modulo 2^64
    np.testing.assert_array_equal(oracle.wrap64_gemm(A, B), want)
    np.testing.assert_array_equal(oracle.wrap64_gemm(A, B, diagonals=True), want)
