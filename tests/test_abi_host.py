"""Host-side checks of librns8.so that need no GPU: every symbol declared in
include/rns8/*.h is exported, the ctypes mirrors have the C compiler's
layouts, ladder queries match the oracle, and plan validation / prefix
selection agrees with the oracle's restatement of the reference
(src/core/moduli.cpp:234-387, api_plan_schedule.inc:263-278) over a fuzzed
descriptor set. No compute call is made."""

import ctypes as C
import random
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
INCLUDE = ROOT / "include"


def declared_symbols():
    names = set()
    for h in (INCLUDE / "rns8").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"RNS8_API\s+[\w\s\*]+?\b(rns8_\w+)\s*\(", text))
    return sorted(names)


def test_every_declared_symbol_is_exported(rns8):
    names = declared_symbols()
    assert len(names) >= 81
    lib = rns8.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing
    nm = subprocess.run(["nm", "-D", "--defined-only", str(rns8.abi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in nm.splitlines() if " T " in line}
    assert set(names) <= exported
    assert all(s.startswith("rns8_") for s in exported if not s.startswith("_"))  # nothing else leaks


def test_struct_layouts_match_c(tmp_path, rns8):
    structs = {"rns8_context_options": rns8.abi.ContextOptions, "rns8_device_info": rns8.abi.DeviceInfo,
               "rns8_gemm_desc": rns8.abi.GemmDesc, "rns8_matrix_desc": rns8.abi.MatrixDesc,
               "rns8_plan_schedule_info": rns8.abi.PlanScheduleInfo,
               "rns8_plan_backend_info": rns8.abi.PlanBackendInfo,
               "rns8_matrix_storage_info": rns8.abi.MatrixStorageInfo,
               "rns8_grouped_gemm_task": rns8.abi.GroupedGemmTask}
    src = tmp_path / "probe.c"
    lines = ['#include <stdio.h>', '#include "rns8/rns8.h"', "int main(void){"]
    lines += [f'printf("{n} %zu\\n", sizeof({n}));' for n in structs]
    lines.append("return 0;}")
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", f"-I{INCLUDE}", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    for line in out.splitlines():
        name, size = line.split()
        assert C.sizeof(structs[name]) == int(size), name


def test_abi_layout_matches_reference_header():
    """Every struct size, field offset, enumerator and numeric macro of the
    reference's public headers (tests/golden/abi_layout.json, generated from
    doublemover/RNS8 include/rns8 by tests/golden/make_abi_layout.py) is the
    same in include/rns8, as the C compiler lays them out."""
    import importlib.util
    import json

    spec = importlib.util.spec_from_file_location("make_abi_layout", ROOT / "tests" / "golden" / "make_abi_layout.py")
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    want = json.loads((ROOT / "tests" / "golden" / "abi_layout.json").read_text())
    names = {"structs": {s: list(f) for s, f in want["offsetof"].items()}, "enums": list(want["enums"]),
             "macros": list(want["macros"])}
    assert len(names["structs"]) == 20 and sum(len(f) for f in names["structs"].values()) == 443
    got = gen.probe(INCLUDE, names)
    for key in ("sizeof", "offsetof", "enums", "macros"):
        assert got[key] == want[key], key


def test_status_and_ladder_queries(rns8, oracle):
    lib = rns8.lib()
    assert lib.rns8_status_string(0) == b"success"
    assert lib.rns8_status_string(5) == b"range error"
    assert lib.rns8_status_string(999) == b"unknown status"
    # test_api_status_cases.inc:1-24: every ABI status has the reference's text.
    texts = [b"success", b"invalid argument", b"unsupported operating system", b"unsupported architecture",
             b"unsupported backend", b"range error", b"accumulation overflow risk", b"workspace too small",
             b"backend failure", b"verification failed", b"internal error"]
    assert [lib.rns8_status_string(s) for s in range(len(texts))] == texts
    assert lib.rns8_status_string(0x7FFF) == b"unknown status"
    assert lib.rns8_default_modulus_count() == 28
    for i in range(28):
        assert lib.rns8_default_modulus(i) == oracle.lib().oracle_modulus(i)
    assert lib.rns8_default_modulus(28) == 0
    for p in range(0, 30):
        assert lib.rns8_prefix_range_bits(p) == pytest.approx(oracle.lib().oracle_prefix_range_bits(p), abs=1e-12)
    assert lib.rns8_validate_default_moduli() == 0


def test_context_requires_the_cuda_backend(rns8):
    opts = rns8.abi.ContextOptions(requested_backend=int(rns8.Backend.CPU_REFERENCE))
    h = C.c_void_p()
    assert rns8.lib().rns8_create_context(-1, C.byref(opts), C.byref(h)) == rns8.Status.UNSUPPORTED_BACKEND
    assert not h
    bad = rns8.abi.ContextOptions(requested_backend=int(rns8.Backend.AUTO), flags=1)
    assert rns8.lib().rns8_create_context(-1, C.byref(bad), C.byref(h)) == rns8.Status.INVALID_ARGUMENT
    assert rns8.lib().rns8_create_context(-1, None, None) == rns8.Status.INVALID_ARGUMENT


def test_unsupported_surfaces_leave_outputs_untouched(rns8):
    lib = rns8.lib()
    out = C.c_void_p(1234)
    assert lib.rns8_create_result_cache(None, None, None, C.byref(out)) == rns8.Status.UNSUPPORTED_BACKEND
    assert out.value is None
    # wrap64 is implemented: null arguments are malformed, as in the reference (api_oneshot.cpp:597-599).
    assert lib.rns8_gemm_wrap_u64_oneshot(None, None, None, 0, None, 0, None, 0) == rns8.Status.INVALID_ARGUMENT
    assert lib.rns8_freivalds_verify(None, None, None, None, 0, 0, None) == rns8.Status.UNSUPPORTED_BACKEND
    assert lib.rns8_destroy_plan(None) == 0 and lib.rns8_destroy_matrix(None) == 0


def _fuzz_descs(seed=1234, count=3000):
    rnd = random.Random(seed)
    sems = [1, 2, 3, 4, 6, 7]
    bounds = [0, 1, 100, 2**20, 2**31, 2**49, 2**61, 2**62, 2**63 - 1, 2**63, 2**63 + 1, 2**64 - 1]
    for _ in range(count):
        sem = rnd.choice(sems)
        bk = rnd.choice([0, 1, 2, 5, 1, 2])
        d = dict(semantics=sem, bound_kind=bk, m=rnd.choice([1, 7, 512]), n=rnd.choice([1, 5, 256]),
                 k=rnd.choice([1, 3, 4096, 65537, 2**31, 2**40]), bound=rnd.choice(bounds),
                 max_prefix=rnd.choice([0, 0, 1, 5, 8, 9, 18, 20, 21]), flags=rnd.choice([0, 0, 1, 8]),
                 finite_modulus=0, lhs_bound=0, rhs_bound=0)
        if sem in (6, 7):
            d.update(bound_kind=0, bound=0, max_prefix=0, finite_modulus=rnd.choice([2, 97, 251, 256, 1, 0]))
        if sem in (3, 4):
            d.update(bound_kind=rnd.choice([0, 0, 1]), bound=rnd.choice([0, 0, 5]))
        if bk == 5 and sem in (1, 2):
            d.update(bound=0, lhs_bound=rnd.choice([1, 2**20, 2**31, 2**63]), rhs_bound=rnd.choice([1, 2**24, 2**33]))
        yield d


def test_plan_selection_matches_oracle(rns8, oracle):
    checked = 0
    for d in _fuzz_descs():
        desc = rns8.gemm_desc(d["semantics"], d["bound_kind"], d["m"], d["n"], d["k"], bound=d["bound"],
                              max_prefix=d["max_prefix"], flags=d["flags"], finite_modulus=d["finite_modulus"],
                              lhs_bound=d["lhs_bound"], rhs_bound=d["rhs_bound"])
        st, sel, req, eb = rns8.plan_probe(desc)
        ost, osel, oreq, oeb = oracle.plan_select_prefix(d["semantics"], d["bound_kind"], d["m"], d["n"], d["k"],
                                                         d["bound"], d["max_prefix"], d["flags"],
                                                         d["finite_modulus"], d["lhs_bound"], d["rhs_bound"])
        assert st == ost, d
        if st == 0:
            assert (sel, req, eb) == (osel, oreq, oeb), d
        checked += 1
    assert checked == 3000


def test_baseline_config_prefixes(rns8):
    # C1 -> 7, C3 -> 8 default / 9 forced, C4 -> 8, C5 -> 18 default / 20 forced.
    I64, U64, EWS = rns8.Semantics.BOUNDED_I64, rns8.Semantics.BOUNDED_U64, rns8.Semantics.EXACT_WIDE_SIGNED
    ABS, UNS, NONE = rns8.BoundKind.GLOBAL_MAX_ABS, rns8.BoundKind.GLOBAL_MAX_UNSIGNED, rns8.BoundKind.NONE
    F = rns8.PLAN_FORCE_FIXED_PREFIX
    cases = [(I64, ABS, 512, 2**49, 0, 0, 7), (I64, ABS, 8192, 2**61, 0, 0, 8), (I64, ABS, 8192, 2**61, 9, F, 9),
             (U64, UNS, 262144, 2**62, 0, 0, 8), (EWS, NONE, 4096, 0, 0, 0, 18), (EWS, NONE, 4096, 0, 20, F, 20)]
    for sem, bk, k, bound, mp, flags, want in cases:
        st, sel, _, _ = rns8.plan_probe(rns8.gemm_desc(sem, bk, 256, 256, k, bound=bound, max_prefix=mp, flags=flags))
        assert st == 0 and sel == want


def test_reference_reducer_fixture_matches_kernel_reduction(oracle):
    """The epilogue's reduction (v + 2^31, floor(2^32/m) mul-hi, one correction,
    minus 2^31 mod m, center) restated in numpy reproduces the reference reducer."""
    import json

    g = json.loads((ROOT / "tests/golden/reducer_vectors.json").read_text())
    v = np.array(g["values"], np.int64)
    u = (v + 2**31).astype(np.uint64)
    for m_str, expected in g["reduce_to_centered_i32"].items():
        m = np.uint64(int(m_str))
        magic = np.uint64((1 << 32) // int(m_str))
        q = (u * magic) >> np.uint64(32)
        r = u - q * m
        r = np.where(r >= m, r - m, r)
        off = np.uint64((1 << 31) % int(m_str))
        r = np.where(r >= off, r - off, r + m - off).astype(np.int64)
        r = np.where(r >= (int(m_str) + 1) // 2, r - int(m_str), r)
        assert r.tolist() == expected


# ---- per-tile bound schedules (host-only probe against the oracle) -----------------
def _schedule_cases():
    rng = np.random.default_rng(77)
    I64, U64 = 1, 2
    cases = []
    for trial in range(60):
        sem = I64 if trial % 2 == 0 else U64
        tile_m, tile_n = [64, 128, 256][trial % 3], [64, 128, 512][(trial // 3) % 3]
        m, n = int(rng.integers(1, 900)), int(rng.integers(1, 900))
        tiles = -(-m // tile_m) * -(-n // tile_n)
        top = 2**63 if sem == I64 else 2**64 - 1
        kind = trial % 5
        if kind == 0:
            bounds = [int(rng.integers(0, 2**20)) for _ in range(tiles)]
        elif kind == 1:
            bounds = [0 if rng.random() < 0.4 else int(rng.integers(1, top, dtype=np.uint64)) for _ in range(tiles)]
        elif kind == 2:
            bounds = [top] * tiles  # collapses: every tile needs the plan prefix
        elif kind == 3:
            bounds = [int(2 ** int(rng.integers(0, 60))) for _ in range(tiles)]
        else:
            bounds = [int(rng.integers(0, top, dtype=np.uint64)) for _ in range(tiles)]
        flags = [0, 1, 2, 3, 6, 7][trial % 6]  # FORCE_FIXED_PREFIX | ZERO_TILE_SKIPS | ZERO_ROW_COL_SKIPS
        za = (rng.random(m) < 0.05).astype(np.uint8) if flags & 4 else None
        zb = (rng.random(n) < 0.05).astype(np.uint8) if flags & 4 else None
        max_prefix = [0, 9, 12][trial % 3] if kind != 2 else 0
        cases.append((sem, m, n, tile_m, tile_n, max_prefix, flags, bounds, za, zb))
    return cases


@pytest.mark.parametrize("case", _schedule_cases())
def test_tile_schedule_matches_oracle(rns8, oracle, case):
    """configure_plan_schedule for per-tile bounds (api_plan_schedule.inc:178-261)
    and rns8_get_plan_tile_schedule (api_plan_public_api.inc:119-167)."""
    sem, m, n, tile_m, tile_n, max_prefix, flags, bounds, za, zb = case
    bk = rns8.BoundKind.PER_TILE_MAX_ABS if sem == 1 else rns8.BoundKind.PER_TILE_MAX_UNSIGNED
    desc = rns8.gemm_desc(sem, bk, m, n, 16, max_prefix=max_prefix, flags=flags, tile_m=tile_m, tile_n=tile_n)
    rns8.api.set_tile_bounds(desc, bounds, za, zb)
    ost, rows, summ = oracle.plan_tile_schedule(sem, m, n, tile_m, tile_n, max_prefix, flags, bounds, za, zb)
    try:
        entries, info = rns8.api.plan_tile_schedule_probe(desc)
        st = 0
    except rns8.Error as e:
        st = int(e.status)
    assert st == ost
    if st != 0:
        return
    assert len(entries) == len(rows)
    assert (info.min_required_prefix, info.max_required_prefix, info.min_selected_prefix,
            info.max_selected_prefix, info.prefix_group_count, info.range_bit_length, info.adaptive_prefix_active,
            info.adaptive_skip_active, info.flags) == tuple(summ[k] for k in (
                "min_required", "max_required", "min_selected", "max_selected", "group_count", "range_bits",
                "adaptive_prefix", "adaptive_skip", "flags"))
    tile_cols = -(-n // tile_n)
    for t, (e, row) in enumerate(zip(entries, rows)):
        assert (e.tile_row, e.tile_col) == (t // tile_cols, t % tile_cols)
        assert (e.row_offset, e.col_offset) == (e.tile_row * tile_m, e.tile_col * tile_n)
        assert e.row_extent == min(tile_m, m - e.row_offset) and e.col_extent == min(tile_n, n - e.col_offset)
        assert e.required_prefix == row[0] and e.range_bit_length == row[3]
        if summ["collapsed"]:
            # a cleared schedule reports every tile at the plan's selected prefix, group 0, no flags
            assert (e.selected_prefix, e.group_index, e.flags) == (summ["min_selected"], 0, 0)
        else:
            assert (e.selected_prefix, e.group_index, e.flags) == (row[1], row[2], row[4])
