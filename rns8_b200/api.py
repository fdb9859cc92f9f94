"""Pythonic wrapper over the rns8 C ABI, mirroring the reference's C++ RAII
wrapper (include/rns8/rns8.hpp: Error/check, Context, Plan, Matrix,
Workspace, grouped and one-shot helpers). Host matrices are numpy arrays in
row-major order; a padded leading dimension is taken from the row stride.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import abi
from .abi import BoundKind, Backend, Semantics, Status, lib


class Error(RuntimeError):
    def __init__(self, status: int, where: str = ""):
        self.status = Status(status)
        super().__init__(f"{where}: {abi.status_string(status)} ({self.status.name})")


def check(status: int, where: str = "rns8") -> None:
    if status != Status.SUCCESS:
        raise Error(status, where)


def _ptr(arr: np.ndarray) -> int:
    return arr.ctypes.data


def _ld(arr: np.ndarray) -> int:
    if arr.ndim != 2 or arr.strides[1] != arr.itemsize or arr.strides[0] % arr.itemsize:
        raise ValueError("expected a row-major 2-D array (padded rows allowed)")
    return arr.strides[0] // arr.itemsize


def gemm_desc(semantics, bound_kind, m, n, k, bound=0, max_prefix=0, flags=0, finite_modulus=0, lhs_bound=0,
              rhs_bound=0, tile_m=0, tile_n=0, requested_backend=Backend.AUTO) -> abi.GemmDesc:
    return abi.GemmDesc(semantics=int(semantics), bound_kind=int(bound_kind), requested_backend=int(requested_backend),
                        m=m, n=n, k=k, bound=bound, max_prefix=max_prefix, flags=flags,
                        finite_modulus=finite_modulus, lhs_bound=lhs_bound, rhs_bound=rhs_bound, tile_m=tile_m,
                        tile_n=tile_n)


def set_tile_bounds(desc: abi.GemmDesc, tile_bounds, zero_a_rows=None, zero_b_cols=None) -> abi.GemmDesc:
    """Attach per-tile bounds (and zero row/column masks) to a descriptor; the
    arrays are kept alive on the descriptor object."""
    tb = (C.c_uint64 * len(tile_bounds))(*[int(v) for v in tile_bounds])
    desc._keep = [tb]
    desc.tile_bounds = C.cast(tb, C.POINTER(C.c_uint64))
    desc.tile_bounds_count = len(tile_bounds)
    if zero_a_rows is not None:
        za = (C.c_uint8 * len(zero_a_rows))(*[int(v) for v in zero_a_rows])
        zb = (C.c_uint8 * len(zero_b_cols))(*[int(v) for v in zero_b_cols])
        desc._keep += [za, zb]
        desc.zero_a_rows = C.cast(za, C.POINTER(C.c_uint8))
        desc.zero_a_rows_count = len(zero_a_rows)
        desc.zero_b_cols = C.cast(zb, C.POINTER(C.c_uint8))
        desc.zero_b_cols_count = len(zero_b_cols)
    return desc


def _entries(fn, count_fn) -> list:
    written = C.c_uint64()
    check(count_fn(None, 0, C.byref(written)), "tile schedule count")
    arr = (abi.PlanTileScheduleEntry * max(written.value, 1))()
    for e in arr:
        e.struct_size, e.abi_version = C.sizeof(abi.PlanTileScheduleEntry), abi.ABI_VERSION
    check(fn(arr, written.value, C.byref(written)), "tile schedule")
    return list(arr)[: written.value]


def plan_tile_schedule_probe(desc: abi.GemmDesc) -> tuple[list, abi.PlanScheduleInfo]:
    """Host-only: the tile schedule and schedule info rns8_create_plan would build."""
    info = abi.PlanScheduleInfo()
    f = lib().rns8_cuda_plan_tile_schedule_probe
    entries = _entries(lambda a, c, w: f(C.byref(desc), a, c, w, C.byref(info)),
                       lambda a, c, w: f(C.byref(desc), a, c, w, None))
    return entries, info


class _Handle:
    _destroy = ""

    def __init__(self):
        self.handle = C.c_void_p()

    def close(self):
        if self.handle:
            getattr(lib(), self._destroy)(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class Context(_Handle):
    _destroy = "rns8_destroy_context"

    def __init__(self, device_id: int = -1, backend: Backend | None = None):
        super().__init__()
        opts = abi.ContextOptions(requested_backend=int(backend)) if backend is not None else None
        check(lib().rns8_create_context(device_id, C.byref(opts) if opts else None, C.byref(self.handle)),
              "rns8_create_context")

    def device_info(self) -> abi.DeviceInfo:
        info = abi.DeviceInfo()
        check(lib().rns8_get_device_info(self.handle, C.byref(info)), "rns8_get_device_info")
        return info


class Plan(_Handle):
    _destroy = "rns8_destroy_plan"

    def __init__(self, ctx: Context, desc: abi.GemmDesc):
        super().__init__()
        self.desc = desc
        check(lib().rns8_create_plan(ctx.handle, C.byref(desc), C.byref(self.handle)), "rns8_create_plan")

    def schedule_info(self) -> abi.PlanScheduleInfo:
        info = abi.PlanScheduleInfo()
        check(lib().rns8_get_plan_schedule_info(self.handle, C.byref(info)), "rns8_get_plan_schedule_info")
        return info

    def tile_schedule(self) -> list:
        f = lib().rns8_get_plan_tile_schedule
        return _entries(lambda a, c, w: f(self.handle, a, c, w), lambda a, c, w: f(self.handle, a, c, w))

    def backend_info(self) -> abi.PlanBackendInfo:
        info = abi.PlanBackendInfo()
        check(lib().rns8_get_plan_backend_info(self.handle, C.byref(info)), "rns8_get_plan_backend_info")
        return info

    @property
    def prefix(self) -> int:
        return self.schedule_info().max_selected_prefix


class Matrix(_Handle):
    _destroy = "rns8_destroy_matrix"

    def __init__(self, ctx: Context, rows: int, cols: int, semantics, bound_kind, max_prefix: int = 0,
                 tile_m: int = 0, tile_n: int = 0, logical_ld: int = 0):
        super().__init__()
        desc = abi.MatrixDesc(rows=rows, cols=cols, logical_ld=logical_ld or cols, semantics=int(semantics),
                              logical_layout=int(abi.Layout.ROW_MAJOR), bound_kind=int(bound_kind),
                              max_prefix=max_prefix, tile_m=tile_m, tile_n=tile_n)
        self.ctx = ctx
        self.rows, self.cols = rows, cols
        check(lib().rns8_create_matrix(ctx.handle, C.byref(desc), C.byref(self.handle)), "rns8_create_matrix")

    @classmethod
    def for_plan(cls, ctx: Context, plan: Plan, role: str) -> "Matrix":
        d = plan.desc
        rows, cols = {"a": (d.m, d.k), "b": (d.k, d.n), "c": (d.m, d.n)}[role]
        sem = Semantics(d.semantics)
        if sem in (Semantics.FINITE_RING_U8, Semantics.FINITE_FIELD_U8):
            return cls(ctx, rows, cols, sem, BoundKind.NONE, 0)
        bk = BoundKind(d.bound_kind)
        if bk == BoundKind.INPUT_RANGE_AND_K:
            bk = BoundKind.GLOBAL_MAX_ABS if sem == Semantics.BOUNDED_I64 else BoundKind.GLOBAL_MAX_UNSIGNED
        # Wrap64 and per-tile matrices carry the plan's tile dimensions.
        tiled = sem == Semantics.WRAP_U64_MOD_2_64 or bk in (BoundKind.PER_TILE_MAX_ABS,
                                                             BoundKind.PER_TILE_MAX_UNSIGNED)
        tm, tn = (plan.desc.tile_m, plan.desc.tile_n) if tiled else (0, 0)
        return cls(ctx, rows, cols, sem, bk, plan.prefix, tm, tn)

    def pack_i64(self, src: np.ndarray, source_version: int = 0) -> None:
        src = np.asarray(src)
        assert src.dtype == np.int64
        check(lib().rns8_pack_i64(self.ctx.handle, self.handle, _ptr(src), _ld(src), source_version), "rns8_pack_i64")

    def pack_u64(self, src: np.ndarray, source_version: int = 0) -> None:
        src = np.asarray(src)
        assert src.dtype == np.uint64
        check(lib().rns8_pack_u64(self.ctx.handle, self.handle, _ptr(src), _ld(src), source_version), "rns8_pack_u64")

    def pack_finite_u8(self, modulus: int, src: np.ndarray, source_version: int = 0) -> None:
        src = np.asarray(src)
        assert src.dtype == np.uint8
        check(lib().rns8_pack_finite_u8(self.ctx.handle, self.handle, modulus, _ptr(src), _ld(src), source_version),
              "rns8_pack_finite_u8")

    def storage_info(self) -> abi.MatrixStorageInfo:
        info = abi.MatrixStorageInfo()
        check(lib().rns8_get_matrix_storage_info(self.handle, C.byref(info)), "rns8_get_matrix_storage_info")
        return info


class Workspace(_Handle):
    _destroy = "rns8_destroy_workspace"

    def __init__(self, ctx: Context, plan: Plan):
        super().__init__()
        check(lib().rns8_create_workspace(ctx.handle, plan.handle, C.byref(self.handle)), "rns8_create_workspace")


def gemm_rns(ctx: Context, plan: Plan, a: Matrix, b: Matrix, c: Matrix, ws: Workspace) -> None:
    check(lib().rns8_gemm_rns(ctx.handle, plan.handle, a.handle, b.handle, c.handle, ws.handle), "rns8_gemm_rns")


def gemm_wrap_u64(ctx: Context, plan: Plan, a: Matrix, b: Matrix, c: Matrix, ws: Workspace) -> None:
    """C = A x B mod 2^64 on byte-limb (WRAP_U64_MOD_2_64) matrices."""
    check(lib().rns8_gemm_wrap_u64(ctx.handle, plan.handle, a.handle, b.handle, c.handle, ws.handle),
          "rns8_gemm_wrap_u64")


def gemm_finite_u8(ctx: Context, plan: Plan, modulus: int, a: Matrix, b: Matrix, c: Matrix, ws: Workspace) -> None:
    check(lib().rns8_gemm_finite_u8(ctx.handle, plan.handle, modulus, a.handle, b.handle, c.handle, ws.handle),
          "rns8_gemm_finite_u8")


def _tasks(tasks) -> tuple[C.Array, int]:
    arr = (abi.GroupedGemmTask * len(tasks))()
    for i, (a, b, c, ws) in enumerate(tasks):
        arr[i] = abi.GroupedGemmTask(a=a.handle.value, b=b.handle.value, c=c.handle.value, workspace=ws.handle.value)
    return arr, len(tasks)


def gemm_rns_grouped(ctx: Context, plan: Plan, tasks) -> None:
    arr, n = _tasks(tasks)
    check(lib().rns8_gemm_rns_grouped(ctx.handle, plan.handle, arr, n), "rns8_gemm_rns_grouped")


def gemm_finite_u8_grouped(ctx: Context, plan: Plan, modulus: int, tasks) -> None:
    arr, n = _tasks(tasks)
    check(lib().rns8_gemm_finite_u8_grouped(ctx.handle, plan.handle, modulus, arr, n), "rns8_gemm_finite_u8_grouped")


def export_i64(ctx: Context, plan: Plan, c: Matrix, out: np.ndarray | None = None) -> np.ndarray:
    out = np.zeros((plan.desc.m, plan.desc.n), np.int64) if out is None else out
    check(lib().rns8_export_i64(ctx.handle, plan.handle, c.handle, _ptr(out), _ld(out)), "rns8_export_i64")
    return out


def export_u64(ctx: Context, plan: Plan, c: Matrix, out: np.ndarray | None = None) -> np.ndarray:
    out = np.zeros((plan.desc.m, plan.desc.n), np.uint64) if out is None else out
    check(lib().rns8_export_u64(ctx.handle, plan.handle, c.handle, _ptr(out), _ld(out)), "rns8_export_u64")
    return out


def export_wrap_u64(ctx: Context, plan: Plan, c: Matrix, out: np.ndarray | None = None) -> np.ndarray:
    out = np.zeros((plan.desc.m, plan.desc.n), np.uint64) if out is None else out
    check(lib().rns8_export_wrap_u64(ctx.handle, plan.handle, c.handle, _ptr(out), _ld(out)), "rns8_export_wrap_u64")
    return out


def export_finite_u8(ctx: Context, plan: Plan, modulus: int, c: Matrix, out: np.ndarray | None = None) -> np.ndarray:
    out = np.zeros((plan.desc.m, plan.desc.n), np.uint8) if out is None else out
    check(lib().rns8_export_finite_u8(ctx.handle, plan.handle, modulus, c.handle, _ptr(out), _ld(out)),
          "rns8_export_finite_u8")
    return out


def export_exact_wide_limbs(ctx: Context, plan: Plan, c: Matrix, limb_count: int, signed: bool = True,
                            out: np.ndarray | None = None) -> np.ndarray:
    """Returns a (m, n, limb_count) uint64 array of little-endian limbs (written
    into `out` when given: C-contiguous, that shape)."""
    shape = (plan.desc.m, plan.desc.n, limb_count)
    out = np.zeros(shape, np.uint64) if out is None else out
    assert out.shape == shape and out.flags.c_contiguous
    fn = lib().rns8_export_exact_wide_signed_limbs if signed else lib().rns8_export_exact_wide_unsigned_limbs
    check(fn(ctx.handle, plan.handle, c.handle, _ptr(out), plan.desc.n, limb_count), "rns8_export_exact_wide_limbs")
    return out


def gemm_i64_oneshot(ctx: Context, desc: abi.GemmDesc, A: np.ndarray, B: np.ndarray,
                     out: np.ndarray | None = None) -> np.ndarray:
    out = np.zeros((desc.m, desc.n), np.int64) if out is None else out
    check(lib().rns8_gemm_i64_oneshot(ctx.handle, C.byref(desc), _ptr(A), _ld(A), _ptr(B), _ld(B), _ptr(out),
                                      _ld(out)), "rns8_gemm_i64_oneshot")
    return out


def gemm_u64_oneshot(ctx: Context, desc: abi.GemmDesc, A: np.ndarray, B: np.ndarray,
                     out: np.ndarray | None = None) -> np.ndarray:
    out = np.zeros((desc.m, desc.n), np.uint64) if out is None else out
    check(lib().rns8_gemm_u64_oneshot(ctx.handle, C.byref(desc), _ptr(A), _ld(A), _ptr(B), _ld(B), _ptr(out),
                                      _ld(out)), "rns8_gemm_u64_oneshot")
    return out


def gemm_wrap_u64_oneshot(ctx: Context, desc: abi.GemmDesc, A: np.ndarray, B: np.ndarray,
                          out: np.ndarray | None = None) -> np.ndarray:
    out = np.zeros((desc.m, desc.n), np.uint64) if out is None else out
    check(lib().rns8_gemm_wrap_u64_oneshot(ctx.handle, C.byref(desc), _ptr(A), _ld(A), _ptr(B), _ld(B), _ptr(out),
                                           _ld(out)), "rns8_gemm_wrap_u64_oneshot")
    return out


def gemm_finite_u8_oneshot(ctx: Context, desc: abi.GemmDesc, modulus: int, A: np.ndarray, B: np.ndarray,
                           field: bool, out: np.ndarray | None = None) -> np.ndarray:
    out = np.zeros((desc.m, desc.n), np.uint8) if out is None else out
    fn = lib().rns8_gemm_finite_field_u8_oneshot if field else lib().rns8_gemm_finite_ring_u8_oneshot
    check(fn(ctx.handle, C.byref(desc), modulus, _ptr(A), _ld(A), _ptr(B), _ld(B), _ptr(out), _ld(out)),
          "rns8_gemm_finite_u8_oneshot")
    return out


def plan_probe(desc: abi.GemmDesc) -> tuple[int, int, int, int]:
    """Host-only plan validation: (status, selected_prefix, required_prefix, effective_bound)."""
    sel, req, eb = C.c_uint32(), C.c_uint32(), C.c_uint64()
    st = lib().rns8_cuda_plan_probe(C.byref(desc), C.byref(sel), C.byref(req), C.byref(eb))
    return int(st), sel.value, req.value, eb.value
