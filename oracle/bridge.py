"""TEST INFRASTRUCTURE ONLY: ctypes bridge to the CPU oracle
(oracle/rns8_oracle.cpp) and to the reference's own reducer harness
(oracle/_ref). Imported by tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline leg as the checker or the timed CPU baseline; never by the
product package.
"""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "librns8_oracle.so"
REF_SO = HERE / "_ref" / "librns8_ref_reducer.so"

vp, i64, u64, u32, u16 = C.c_void_p, C.c_int64, C.c_uint64, C.c_uint32, C.c_uint16

_SIGS = {
    "oracle_modulus": (u16, [u32]),
    "oracle_modulus_product": (None, [u32, vp]),
    "oracle_required_prefix_for_range": (u32, [vp]),
    "oracle_prefix_range_bits": (C.c_double, [u32]),
    "oracle_centered_residue_i64": (C.c_int8, [i64, u16]),
    "oracle_centered_residue_u64": (C.c_int8, [u64, u16]),
    "oracle_reduce_to_centered": (C.c_int8, [i64, u16]),
    "oracle_set_parallel_threshold": (None, [u64]),
    "oracle_max_threads": (C.c_int, []),
    "oracle_set_threads": (None, [C.c_int]),
    "oracle_pack_i64": (None, [vp, i64, i64, i64, u32, vp]),
    "oracle_pack_u64": (None, [vp, i64, i64, i64, u32, vp]),
    "oracle_pack_finite_u8": (None, [vp, i64, i64, i64, u16, vp]),
    "oracle_export_finite_u8": (None, [vp, i64, i64, u16, vp, i64]),
    "oracle_ring_gemm_modulus": (None, [vp, vp, vp, i64, i64, i64, i64, i64, i64, u16]),
    "oracle_gemm_rns": (None, [vp, vp, vp, i64, i64, i64, u32]),
    "oracle_centered_residue_dot": (C.c_int8, [vp, vp, i64, i64, u16]),
    "oracle_reconstruct_signed": (C.c_int, [vp, u32, u64, vp]),
    "oracle_reconstruct_unsigned": (C.c_int, [vp, u32, u64, vp]),
    "oracle_reconstruct_canonical": (None, [vp, u32, vp]),
    "oracle_export_i64": (C.c_int, [vp, i64, i64, u32, u64, vp, i64]),
    "oracle_export_u64": (C.c_int, [vp, i64, i64, u32, u64, vp, i64]),
    "oracle_export_exact_wide_limbs": (C.c_int, [vp, i64, i64, u32, vp, i64, u32, C.c_int]),
    "oracle_plan_select_prefix": (C.c_int, [u32, u32, i64, i64, i64, u64, u32, u32, u32, u64, u64, vp, vp, vp]),
    "oracle_gemm_bounded_oneshot": (C.c_int, [C.c_int, u32, i64, i64, i64, u64, u32, u32, u64, u64, vp, i64, vp, i64,
                                              vp, i64, vp]),
    "oracle_gemm_finite_u8_oneshot": (C.c_int, [C.c_int, u16, i64, i64, i64, vp, i64, vp, i64, vp, i64]),
    "oracle_exact_gemm_admission": (C.c_int, [C.c_int, vp, i64, vp, i64, i64, i64, i64, u32, vp, vp, vp]),
    "oracle_exact_gemm_cell_stats": (C.c_int, [C.c_int, vp, i64, vp, i64, i64, i64, i64, vp, vp]),
    "oracle_wrap64_gemm": (None, [vp, i64, vp, i64, vp, i64, i64, i64, i64]),
    "oracle_plan_tile_schedule": (C.c_int, [u32, i64, i64, u32, u32, u32, u32, vp, vp, vp, vp, vp]),
    "oracle_gemm_rns_scheduled": (None, [vp, vp, vp, i64, i64, i64, u32, u32, vp]),
    "oracle_export_scheduled": (C.c_int, [vp, i64, i64, u32, u32, vp, vp, C.c_int, vp, i64]),
    "oracle_wrap64_gemm_diagonals": (None, [vp, i64, vp, i64, vp, i64, i64, i64, i64]),
    "oracle_rng_new": (C.c_int, [u64]),
    "oracle_rng_free": (None, [C.c_int]),
    "oracle_rng_next": (u64, [C.c_int]),
    "oracle_rng_fill_i64": (None, [C.c_int, i64, i64, vp, i64]),
    "oracle_rng_fill_u64": (None, [C.c_int, u64, u64, vp, i64]),
    "oracle_rng_fill_u8": (None, [C.c_int, u32, vp, i64]),
    "oracle_rng_skip_i64": (None, [C.c_int, i64, i64, i64]),
    "oracle_rng_skip_u64": (None, [C.c_int, u64, u64, i64]),
    "oracle_checksum_u64": (u64, [vp, i64, i64, i64]),
    "oracle_checksum_u64_from": (u64, [u64, vp, i64]),
}

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build()
        h = C.CDLL(str(ORACLE_SO))
        for name, (res, args) in _SIGS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
    return _lib


def ref_lib() -> C.CDLL | None:
    """The reference's own reducer (oracle/_ref), or None when it was not built."""
    if not REF_SO.exists():
        return None
    h = C.CDLL(str(REF_SO))
    h.ref_reduce_to_centered_i32.restype = C.c_int8
    h.ref_reduce_to_centered_i32.argtypes = [C.c_int32, u32]
    h.ref_reduce_to_centered_accelerator_i32.restype = C.c_int8
    h.ref_reduce_to_centered_accelerator_i32.argtypes = [C.c_int32, u32]
    h.ref_center_u8.restype = C.c_int8
    h.ref_center_u8.argtypes = [C.c_uint8, u32]
    h.ref_canonical_from_centered.restype = u32
    h.ref_canonical_from_centered.argtypes = [C.c_int8, u32]
    h.ref_centered_residue_dot.restype = C.c_int8
    h.ref_centered_residue_dot.argtypes = [vp, vp, i64, i64, u32]
    return h


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _ld(a: np.ndarray) -> int:
    return a.strides[0] // a.itemsize


LADDER = [256, 255, 253, 251, 247, 239, 233, 229, 227, 223, 217, 211, 199, 197,
          193, 191, 181, 179, 173, 167, 163, 157, 151, 149, 139, 137, 131, 127]


def to_limbs4(v: int) -> np.ndarray:
    return np.array([(v >> (64 * i)) & ((1 << 64) - 1) for i in range(4)], dtype=np.uint64)


def from_limbs4(a: np.ndarray) -> int:
    v = sum(int(a[i]) << (64 * i) for i in range(4))
    return v - (1 << 256) if v >> 255 else v


def modulus_product(prefix: int) -> int:
    out = np.zeros(4, np.uint64)
    lib().oracle_modulus_product(prefix, _p(out))
    return from_limbs4(out)


def required_prefix_for_range(r: int) -> int:
    return int(lib().oracle_required_prefix_for_range(_p(to_limbs4(r))))


def pack(src: np.ndarray, prefix: int) -> np.ndarray:
    rows, cols = src.shape
    out = np.zeros((prefix, rows, cols), np.int8)
    fn = lib().oracle_pack_i64 if src.dtype == np.int64 else lib().oracle_pack_u64
    fn(_p(src), rows, cols, _ld(src), prefix, _p(out))
    return out


def pack_finite_u8(src: np.ndarray, modulus: int) -> np.ndarray:
    rows, cols = src.shape
    out = np.zeros((rows, cols), np.int8)
    lib().oracle_pack_finite_u8(_p(src), rows, cols, _ld(src), modulus, _p(out))
    return out


def gemm_rns(a: np.ndarray, b: np.ndarray, prefix: int) -> np.ndarray:
    """a: (P, m, k) int8, b: (P, k, n) int8 -> (P, m, n) int8 (planes >= prefix)."""
    a = np.ascontiguousarray(a[:prefix])
    b = np.ascontiguousarray(b[:prefix])
    _, m, k = a.shape
    n = b.shape[2]
    c = np.zeros((prefix, m, n), np.int8)
    lib().oracle_gemm_rns(_p(a), _p(b), _p(c), m, n, k, prefix)
    return c


def ring_gemm(a: np.ndarray, b: np.ndarray, modulus: int) -> np.ndarray:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), np.int8)
    lib().oracle_ring_gemm_modulus(_p(a), _p(b), _p(c), m, n, k, k, n, n, modulus)
    return c


def export_i64(planes: np.ndarray, prefix: int, bound: int) -> tuple[int, np.ndarray]:
    planes = np.ascontiguousarray(planes[:prefix])
    _, m, n = planes.shape
    out = np.zeros((m, n), np.int64)
    st = lib().oracle_export_i64(_p(planes), m, n, prefix, bound, _p(out), n)
    return int(st), out


def export_u64(planes: np.ndarray, prefix: int, bound: int) -> tuple[int, np.ndarray]:
    planes = np.ascontiguousarray(planes[:prefix])
    _, m, n = planes.shape
    out = np.zeros((m, n), np.uint64)
    st = lib().oracle_export_u64(_p(planes), m, n, prefix, bound, _p(out), n)
    return int(st), out


def export_limbs(planes: np.ndarray, prefix: int, limbs: int, signed: bool) -> tuple[int, np.ndarray]:
    planes = np.ascontiguousarray(planes[:prefix])
    _, m, n = planes.shape
    out = np.zeros((m, n, limbs), np.uint64)
    st = lib().oracle_export_exact_wide_limbs(_p(planes), m, n, prefix, _p(out), n, limbs, 1 if signed else 0)
    return int(st), out


def plan_select_prefix(semantics, bound_kind, m, n, k, bound=0, max_prefix=0, flags=0, finite_modulus=0,
                       lhs_bound=0, rhs_bound=0) -> tuple[int, int, int, int]:
    sel, req, eb = C.c_uint32(), C.c_uint32(), C.c_uint64()
    st = lib().oracle_plan_select_prefix(int(semantics), int(bound_kind), m, n, k, bound, max_prefix, flags,
                                         finite_modulus, lhs_bound, rhs_bound, C.addressof(sel), C.addressof(req),
                                         C.addressof(eb))
    return int(st), sel.value, req.value, eb.value


def gemm_bounded_oneshot(A: np.ndarray, B: np.ndarray, bound: int, *, bound_kind=None, max_prefix=0, flags=0,
                         lhs_bound=0, rhs_bound=0, out: np.ndarray | None = None) -> tuple[int, np.ndarray, int]:
    signed = A.dtype == np.int64
    m, k = A.shape
    n = B.shape[1]
    if bound_kind is None:
        bound_kind = 1 if signed else 2
    out = np.zeros((m, n), A.dtype) if out is None else out
    used = C.c_uint32()
    st = lib().oracle_gemm_bounded_oneshot(1 if signed else 0, bound_kind, m, n, k, bound, max_prefix, flags,
                                           lhs_bound, rhs_bound, _p(A), _ld(A), _p(B), _ld(B), _p(out), _ld(out),
                                           C.addressof(used))
    return int(st), out, used.value


def gemm_finite_u8_oneshot(A: np.ndarray, B: np.ndarray, modulus: int, field: bool) -> tuple[int, np.ndarray]:
    m, k = A.shape
    n = B.shape[1]
    out = np.zeros((m, n), np.uint8)
    st = lib().oracle_gemm_finite_u8_oneshot(1 if field else 0, modulus, m, n, k, _p(A), _ld(A), _p(B), _ld(B),
                                             _p(out), n)
    return int(st), out


def exact_gemm_admission(A: np.ndarray, B: np.ndarray, prefix: int) -> tuple[int, int]:
    m, k = A.shape
    n = B.shape[1]
    bound = np.zeros(4, np.uint64)
    amax = np.zeros(4, np.uint64)
    bmax = np.zeros(4, np.uint64)
    st = lib().oracle_exact_gemm_admission(1 if A.dtype == np.int64 else 0, _p(A), _ld(A), _p(B), _ld(B), m, n, k,
                                           prefix, _p(bound), _p(amax), _p(bmax))
    return int(st), from_limbs4(bound)


def exact_gemm_cell_stats(A: np.ndarray, B: np.ndarray) -> tuple[list[tuple[int, int]], list[tuple[int, int]]]:
    """Per output row and column: (max, sum) of the exact-wide cell bounds."""
    m, k = A.shape
    n = B.shape[1]
    rows = np.zeros((m, 8), np.uint64)
    cols = np.zeros((n, 8), np.uint64)
    lib().oracle_exact_gemm_cell_stats(1 if A.dtype == np.int64 else 0, _p(A), _ld(A), _p(B), _ld(B), m, n, k,
                                       _p(rows), _p(cols))
    pair = lambda v: (from_limbs4(v[:4]), from_limbs4(v[4:]))
    return [pair(r) for r in rows], [pair(c) for c in cols]


def wrap64_gemm(A: np.ndarray, B: np.ndarray, diagonals: bool = False) -> np.ndarray:
    """C = A x B mod 2^64 over uint64 (A, B may be row-padded views)."""
    m, k = A.shape
    n = B.shape[1]
    out = np.zeros((m, n), np.uint64)
    fn = lib().oracle_wrap64_gemm_diagonals if diagonals else lib().oracle_wrap64_gemm
    fn(_p(A), _ld(A), _p(B), _ld(B), _p(out), n, m, n, k)
    return out


def plan_tile_schedule(semantics: int, m: int, n: int, tile_m: int, tile_n: int, max_prefix: int, flags: int,
                       tile_bounds, zero_a_rows=None, zero_b_cols=None):
    """(status, per-tile rows (required, selected, group, range_bits, flags), summary dict)."""
    tiles = -(-m // tile_m) * -(-n // tile_n)
    tb = np.ascontiguousarray(np.asarray(tile_bounds, np.uint64))
    za = np.ascontiguousarray(np.asarray(zero_a_rows if zero_a_rows is not None else np.zeros(m), np.uint8))
    zb = np.ascontiguousarray(np.asarray(zero_b_cols if zero_b_cols is not None else np.zeros(n), np.uint8))
    out = np.zeros((tiles, 5), np.uint32)
    summ = np.zeros(10, np.uint32)
    st = lib().oracle_plan_tile_schedule(semantics, m, n, tile_m, tile_n, max_prefix, flags, _p(tb), _p(za), _p(zb),
                                         _p(out), _p(summ))
    keys = ["min_required", "max_required", "min_selected", "max_selected", "group_count", "range_bits",
            "adaptive_prefix", "adaptive_skip", "flags", "collapsed"]
    return int(st), out, dict(zip(keys, (int(v) for v in summ)))


def gemm_rns_scheduled(a: np.ndarray, b: np.ndarray, c: np.ndarray, tile_m: int, tile_n: int, sel) -> np.ndarray:
    """C planes updated in place under a tile schedule (sel: prefix | 0x80 for proven zero)."""
    _, m, k = a.shape
    n = b.shape[2]
    s = np.ascontiguousarray(np.asarray(sel, np.uint8))
    lib().oracle_gemm_rns_scheduled(_p(a), _p(b), _p(c), m, n, k, tile_m, tile_n, _p(s))
    return c


def export_scheduled(planes: np.ndarray, tile_m: int, tile_n: int, sel, tile_bounds, signed: bool):
    _, m, n = planes.shape
    s = np.ascontiguousarray(np.asarray(sel, np.uint8))
    tb = np.ascontiguousarray(np.asarray(tile_bounds, np.uint64))
    out = np.zeros((m, n), np.int64 if signed else np.uint64)
    st = lib().oracle_export_scheduled(_p(np.ascontiguousarray(planes)), m, n, tile_m, tile_n, _p(s), _p(tb),
                                       1 if signed else 0, _p(out), n)
    return int(st), out


class Rng:
    """std::mt19937_64 + std::uniform_int_distribution (libstdc++), as the
    reference's tests and benchmark draw their inputs."""

    def __init__(self, seed: int):
        self.h = lib().oracle_rng_new(seed)

    def next(self) -> int:
        return int(lib().oracle_rng_next(self.h))

    def i64(self, lo: int, hi: int, shape) -> np.ndarray:
        out = np.empty(shape, np.int64)
        lib().oracle_rng_fill_i64(self.h, lo, hi, _p(out), out.size)
        return out

    def u64(self, lo: int, hi: int, shape) -> np.ndarray:
        out = np.empty(shape, np.uint64)
        lib().oracle_rng_fill_u64(self.h, lo, hi, _p(out), out.size)
        return out

    def u8(self, hi: int, shape) -> np.ndarray:
        """uniform_int_distribution<uint32_t>(0, hi) per byte (the reference's finite lanes)."""
        out = np.empty(shape, np.uint8)
        lib().oracle_rng_fill_u8(self.h, hi, _p(out), out.size)
        return out

    def skip_i64(self, lo: int, hi: int, count: int) -> None:
        lib().oracle_rng_skip_i64(self.h, lo, hi, count)

    def skip_u64(self, lo: int, hi: int, count: int) -> None:
        lib().oracle_rng_skip_u64(self.h, lo, hi, count)

    def __del__(self):
        try:
            lib().oracle_rng_free(self.h)
        except Exception:
            pass


def checksum(values: np.ndarray) -> int:
    v = np.ascontiguousarray(values).view(np.uint64).reshape(values.shape[0], -1)
    return int(lib().oracle_checksum_u64(_p(v), v.shape[0], v.shape[1], v.shape[1]))


# ---- independent exact-integer checker (Python big ints) -------------------
def exact_product(A: np.ndarray, B: np.ndarray) -> list[list[int]]:
    a = [[int(x) for x in row] for row in A]
    b = [[int(x) for x in row] for row in B]
    m, k, n = len(a), len(b), len(b[0])
    return [[sum(a[i][t] * b[t][j] for t in range(k)) for j in range(n)] for i in range(m)]
