"""Generate the golden fixtures under tests/golden/ (run where the reference
tree is present; the outputs are committed so GPU boxes need no reference).

reducer_vectors.json
    Outputs of the reference's own Boost-free epilogue arithmetic
    (src/backend_common/finite_u8_reducer.hpp, residue_dot.hpp), compiled
    in place by oracle/Makefile into oracle/_ref/librns8_ref_reducer.so:
    reduce_to_centered_i32 for the 20 boundary int32 values of
    tests/unit/test_residues.cpp:46-67 and 2000 seeded values, for all 28
    ladder moduli; center_u8 for every byte and modulus 2..256; and
    centered_residue_dot for the K-split cases of
    tests/unit/test_residue_dot.cpp:9-31.

reference_kats.json
    Known answers stated in the reference's tests and examples, with
    file:line provenance, plus the exact values they imply (Python big ints).

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import ctypes as C
import json
import math
import random
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import bridge  # noqa: E402

LADDER = bridge.LADDER
INT32_BOUNDARY = [-(2**31), -(2**31) + 1, -536870912, -65537, -65536, -32769, -32768, -257, -256, -1, 0, 1, 127, 128,
                  255, 256, 32767, 32768, 65536, 2**31 - 1]


def reducer_vectors() -> dict:
    subprocess_ok = bridge.REF_SO.exists()
    if not subprocess_ok:
        bridge.build()
    ref = bridge.ref_lib()
    if ref is None:
        raise SystemExit("oracle/_ref was not built: the reference tree is required to regenerate fixtures")
    rnd = random.Random(20261201)
    values = INT32_BOUNDARY + [rnd.randint(-(2**31), 2**31 - 1) for _ in range(2000)]
    reduce = {str(m): [int(ref.ref_reduce_to_centered_i32(v, m)) for v in values] for m in LADDER}
    center = {str(m): [int(ref.ref_center_u8(b, m)) for b in range(256)] for m in range(2, 257)}
    dots = []
    for k in (65535, 65536, 65537, 131072, 131073, 262145):
        for p in range(20):
            m = LADDER[p]
            lo = -(m // 2)
            for alternating in (False, True):
                a = np.full(k, lo, np.int8)
                b = np.full(k * 3, 73, np.int8)
                idx = np.arange(k)
                vals = np.where(alternating & (idx % 2 == 1), 1, lo).astype(np.int8)
                b[::3] = vals
                got = int(ref.ref_centered_residue_dot(a.ctypes.data, b.ctypes.data, k, 3, m))
                exact = int(lo) * int(vals.astype(np.int64).sum())
                dots.append({"k": k, "modulus": m, "alternating": alternating, "lo": lo, "expected": got,
                             "exact_sum": exact})
    return {"source": "oracle/_ref/librns8_ref_reducer.so built from the reference's "
                      "src/backend_common/{finite_u8_reducer,residue_dot}.hpp",
            "values": values, "reduce_to_centered_i32": reduce, "center_u8": center, "residue_dot": dots}


def centered(v: int, m: int) -> int:
    r = v % m
    return r - m if r >= (m + 1) // 2 else r


def reference_kats() -> dict:
    prod = [math.prod(LADDER[:p]) for p in range(0, 21)]
    kats = {
        "ladder": {"source": "tests/unit/test_moduli.cpp:11-19", "moduli": LADDER},
        "prefix_range_bits": {
            "source": "tests/unit/test_moduli.cpp:62-75 (margin 0.002)",
            "table": {"4": 31.949, "5": 39.897, "6": 47.798, "7": 55.662, "8": 63.502, "9": 71.328, "10": 79.129,
                      "12": 94.612, "16": 125.040, "18": 140.024, "19": 147.458, "20": 154.842}},
        "modulus_products": {"source": "tests/unit/test_moduli.cpp:21-39", "products": [str(p) for p in prod]},
        "prefix9_full_width": {"source": "tests/unit/test_moduli.cpp:41-54",
                               "required_prefix_2^64-1": 9, "required_prefix_2^64": 9},
        "centered_residues": {
            "source": "tests/unit/test_residues.cpp:11-29",
            "cases": [[127, 256, 127], [128, 256, -128], [-128, 256, -128], [-129, 256, 127],
                      [127, 255, 127], [128, 255, -127], [-127, 255, -127], [-128, 255, 127],
                      [125, 251, 125], [126, 251, -125], [-125, 251, -125]]},
        "crt_roundtrips": {
            "source": "tests/unit/test_crt.cpp:22-43,92-106,108-137",
            "signed": [[-123456789, 9, 123456789, "ok"], [-(2**63), 9, 2**63, "ok"], [2**63, 9, 2**63, "range"]],
            "unsigned": [[2**64 - 1, 9, 2**64 - 1, "ok"], [2**64, 9, 2**64 - 1, "range"],
                         [str(prod[9] - 1), 9, 2**64 - 1, "range"]]},
        "crt_canonical": {"source": "tests/unit/test_crt.cpp:45-60", "prefixes": [1, 2, 4, 8, 9, 12, 20]},
        "crt_threshold_prefix2": {
            "source": "tests/unit/test_crt.cpp:62-90", "product": 65280, "threshold": 32640,
            "cases": [[32639, 32639, "ok", 32639], [32641, 32639, "ok", -32639], [32640, 32640, "range", None],
                      [65279, 1, "ok", -1]]},
        "crt_insufficient_range": {"source": "tests/unit/test_crt.cpp:139-144", "value": 2**63 - 1, "prefix": 8,
                                   "bound": 2**63 - 1, "status": "range"},
        "ring_gemm_2x3x4": {
            "source": "tests/unit/test_ring_gemm.cpp:27-43",
            "A": [1, -2, 3, -4, -5, 6, -7, 8], "B": [9, -10, 11, -12, 13, -14, 15, -16, 17, -18, 19, -20],
            "moduli": [255, 251]},
        "ring_gemm_k65537": {"source": "tests/unit/test_ring_gemm.cpp:45-54", "k": 65537, "value": 127,
                             "modulus": 256, "expected": centered(127 * 127 * 65537, 256)},
        "example_bounded_i64": {"source": "examples/bounded_i64_oneshot.cpp:14-27", "m": 2, "n": 2, "k": 3,
                                "bound": 100, "A": [2, -3, 4, -5, 6, 7], "B": [1, 8, -2, 9, 3, -4],
                                "expected": [20, -27, 4, -14]},
        "prefix_selection": {"source": "BASELINE.json configs; api_plan_schedule.inc:263-278",
                             "cases": [["i64", 2**49, 0, 0, 7], ["i64", 2**61, 0, 0, 8], ["i64", 2**61, 9, 1, 9],
                                       ["u64", 2**62, 0, 0, 8], ["i64", 2**63, 0, 0, 9], ["u64", 2**64 - 1, 0, 0, 9]]},
    }
    # wrap64 public-path inputs of the reference's differential test (padded
    # lda = 6, ldb = 4); the expected cells are sum a*b mod 2^64, the value
    # wrap64_reference.cpp:254-290 computes.
    u64max = 2**64 - 1
    wa = [0, 1, u64max, 0x8080808080808080, 0x0102030405060708, 0xAAAA,
          255, 256, u64max - 1, 0x7F7F7F7F7F7F7F7F, 17, 0xBBBB]
    wb = [3, u64max, 0x1112131415161718, 0xCCCC, 29, 0x8080808080808080, 31, 0xDDDD,
          0x0101010101010101, 0xFEFDFCFBFAF9F8F7, 37, 0xEEEE, 41, 43, 47, 0xFFFF, 53, 59, 61, 0x1234]
    m, n, k, lda, ldb = 2, 3, 5, 6, 4
    kats["wrap64_public_2x3x5"] = {
        "source": "tests/differential/test_hip_direct_wrap64_public_cases.inc:6-45",
        "m": m, "n": n, "k": k, "lda": lda, "ldb": ldb, "A": [str(v) for v in wa], "B": [str(v) for v in wb],
        "expected": [[str(sum(wa[r * lda + q] * wb[q * ldb + c] for q in range(k)) % 2**64) for c in range(n)]
                     for r in range(m)]}
    # Exact-wide fixed-width limb boundaries: (prefix, signed, value, limbs) ->
    # "range" or the little-endian limbs (two's complement when signed).
    def limbs_of(v: int, count: int) -> list[str]:
        u = v % (1 << (64 * count))
        return [str((u >> (64 * l)) & (2**64 - 1)) for l in range(count)]

    half3, half20 = prod[3] // 2, prod[20] // 2
    cases = [
        [3, True, str(half3), 1, limbs_of(-half3, 1)],           # centered half-open: M/2 -> -M/2
        [20, True, str(half20), 2, "range"],
        [20, True, str(half20), 3, limbs_of(-half20, 3)],
        [20, True, str(2**63 - 1), 1, limbs_of(2**63 - 1, 1)],
        [20, True, str(-(2**63)), 1, limbs_of(-(2**63), 1)],
        [20, True, "-1", 1, limbs_of(-1, 1)],
        [20, True, str(2**63), 1, "range"],
        [20, True, str(-(2**63) - 1), 1, "range"],
        [20, True, "-1", 32, limbs_of(-1, 32)],
        [20, False, str(2**64 - 1), 1, limbs_of(2**64 - 1, 1)],
        [20, False, str(2**64), 1, "range"],
        [20, False, str(2**64), 2, limbs_of(2**64, 2)],
        [20, False, "1", 32, limbs_of(1, 32)],
        [20, False, str(2**127), 1, "range"],
        [20, False, str(2**127), 2, limbs_of(2**127, 2)],
        [20, False, str(2**127), 32, limbs_of(2**127, 32)],
    ]
    kats["exact_wide_limb_boundaries"] = {"source": "tests/unit/test_exact_wide_limb_boundary_cases.inc:1-127",
                                          "cases": cases}
    # Expected values for the 2x3x4 ring GEMM KAT.
    A = np.array(kats["ring_gemm_2x3x4"]["A"]).reshape(2, 4)
    B = np.array(kats["ring_gemm_2x3x4"]["B"]).reshape(4, 3)
    exact = (A @ B).tolist()
    kats["ring_gemm_2x3x4"]["expected"] = {str(m): [[centered(v, m) for v in row] for row in exact]
                                           for m in kats["ring_gemm_2x3x4"]["moduli"]}
    return kats


def main() -> None:
    out = Path(__file__).resolve().parent
    (out / "reducer_vectors.json").write_text(json.dumps(reducer_vectors()))
    (out / "reference_kats.json").write_text(json.dumps(reference_kats(), indent=1))
    print("wrote", out / "reducer_vectors.json", out / "reference_kats.json")


if __name__ == "__main__":
    main()
