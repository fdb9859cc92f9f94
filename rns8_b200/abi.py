"""ctypes view of the rns8 C ABI exported by librns8.so.

The structures mirror include/rns8/rns8.h field for field (the reference's
include/rns8/rns8.h:17-647); tests check every size against the C compiler's.
Loading never falls back to anything: if librns8.so is missing or does not
export an expected symbol, `lib()` raises.
"""

from __future__ import annotations

import ctypes as C
import enum
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "_build" / "librns8.so"
ABI_VERSION = 1

c_status = C.c_uint32
c_enum = C.c_uint32


class Status(enum.IntEnum):
    SUCCESS = 0
    INVALID_ARGUMENT = 1
    UNSUPPORTED_OS = 2
    UNSUPPORTED_ARCH = 3
    UNSUPPORTED_BACKEND = 4
    RANGE_ERROR = 5
    ACCUMULATION_OVERFLOW_RISK = 6
    WORKSPACE_TOO_SMALL = 7
    BACKEND_FAILURE = 8
    VERIFICATION_FAILED = 9
    INTERNAL_ERROR = 10


class Semantics(enum.IntEnum):
    BOUNDED_I64 = 1
    BOUNDED_U64 = 2
    EXACT_WIDE_SIGNED = 3
    EXACT_WIDE_UNSIGNED = 4
    WRAP_U64_MOD_2_64 = 5
    FINITE_RING_U8 = 6
    FINITE_FIELD_U8 = 7


class BoundKind(enum.IntEnum):
    NONE = 0
    GLOBAL_MAX_ABS = 1
    GLOBAL_MAX_UNSIGNED = 2
    PER_TILE_MAX_ABS = 3
    PER_TILE_MAX_UNSIGNED = 4
    INPUT_RANGE_AND_K = 5


class Layout(enum.IntEnum):
    ROW_MAJOR = 1
    COLUMN_MAJOR = 2


class Backend(enum.IntEnum):
    AUTO = 0
    CPU_REFERENCE = 1
    HIP_DIRECT = 2
    HIPBLASLT = 3
    CK = 4
    ROCWMMA = 5
    WRAP64_BYTE_LIMB = 6
    HIP_VECTOR_ALU_INT64 = 7
    AMDGPU_BUILTINS = 8
    CUDA_SM100 = 9


PLAN_FORCE_FIXED_PREFIX = 0x1
PLAN_ALLOW_PROVEN_ZERO_TILE_SKIPS = 0x2
PLAN_ALLOW_PROVEN_ZERO_ROW_COL_SKIPS = 0x4
DEFAULT_MODULUS_COUNT = 28
DEFAULT_BOUNDED_PREFIX = 9
MAX_SUPPORTED_PREFIX = 20
SAFE_INT32_K_BLOCK = 65536

GEMM_AUTO = 0
GEMM_TENSOR_CORE = 1
GEMM_SIMT = 2


class _Struct(C.Structure):
    """Base: struct_size / abi_version filled on construction."""

    def __init__(self, **kw):
        super().__init__()
        self.struct_size = C.sizeof(self)
        self.abi_version = ABI_VERSION
        for k, v in kw.items():
            setattr(self, k, v)


class ContextOptions(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("requested_backend", c_enum),
                ("flags", C.c_uint32)]


class DeviceInfo(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("backend", c_enum),
                ("device_id", C.c_int32), ("hip_available", C.c_uint32), ("hip_runtime_version", C.c_uint32),
                ("hip_driver_version", C.c_uint32), ("global_mem_bytes", C.c_uint64), ("name", C.c_char * 128),
                ("gcn_arch", C.c_char * 64), ("detail", C.c_char * 256)]


class GemmDesc(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("semantics", c_enum),
                ("bound_kind", c_enum), ("requested_backend", c_enum), ("m", C.c_int64), ("n", C.c_int64),
                ("k", C.c_int64), ("bound", C.c_uint64), ("max_prefix", C.c_uint32), ("tile_m", C.c_uint32),
                ("tile_n", C.c_uint32), ("finite_modulus", C.c_uint32), ("flags", C.c_uint32),
                ("tile_bounds", C.POINTER(C.c_uint64)), ("tile_bounds_count", C.c_uint64),
                ("lhs_bound", C.c_uint64), ("rhs_bound", C.c_uint64), ("zero_a_rows", C.POINTER(C.c_uint8)),
                ("zero_a_rows_count", C.c_uint64), ("zero_b_cols", C.POINTER(C.c_uint8)),
                ("zero_b_cols_count", C.c_uint64)]


class PlanTileScheduleEntry(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("flags", C.c_uint32),
                ("tile_row", C.c_uint64), ("tile_col", C.c_uint64), ("row_offset", C.c_int64),
                ("col_offset", C.c_int64), ("row_extent", C.c_int64), ("col_extent", C.c_int64),
                ("required_prefix", C.c_uint32), ("selected_prefix", C.c_uint32), ("group_index", C.c_uint32),
                ("range_bit_length", C.c_uint32)]


class MatrixDesc(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("rows", C.c_int64), ("cols", C.c_int64),
                ("logical_ld", C.c_int64), ("semantics", c_enum), ("logical_layout", c_enum),
                ("bound_kind", c_enum), ("tile_m", C.c_uint32), ("tile_n", C.c_uint32), ("max_prefix", C.c_uint32),
                ("flags", C.c_uint32)]


class PlanScheduleInfo(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("tile_m", C.c_uint32),
                ("tile_n", C.c_uint32), ("tile_rows", C.c_uint64), ("tile_cols", C.c_uint64),
                ("tile_count", C.c_uint64), ("min_required_prefix", C.c_uint32),
                ("max_required_prefix", C.c_uint32), ("min_selected_prefix", C.c_uint32),
                ("max_selected_prefix", C.c_uint32), ("prefix_group_count", C.c_uint32),
                ("adaptive_prefix_active", C.c_uint32), ("adaptive_skip_active", C.c_uint32),
                ("range_bit_length", C.c_uint32), ("flags", C.c_uint32), ("bound_kind", c_enum),
                ("reserved0", C.c_uint32), ("effective_bound", C.c_uint64), ("lhs_bound", C.c_uint64),
                ("rhs_bound", C.c_uint64), ("zero_a_row_count", C.c_uint64), ("zero_b_col_count", C.c_uint64),
                ("zero_row_col_product_count", C.c_uint64), ("bound_contract", C.c_char * 96)]


class PlanBackendInfo(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("backend", c_enum),
                ("is_accelerator", C.c_uint32), ("is_correctness_backend", C.c_uint32),
                ("is_matrix_engine_backend", C.c_uint32), ("compiled_kernel_available", C.c_uint32),
                ("exact_differential_validated", C.c_uint32), ("performance_validated", C.c_uint32),
                ("flags", C.c_uint32), ("workspace_required_bytes", C.c_uint64),
                ("selected_kernel", C.c_char * 128), ("accelerator_library", C.c_char * 64),
                ("accelerator_version", C.c_char * 64), ("capability_status", C.c_char * 128),
                ("epilogue_mode", C.c_char * 96), ("workspace_mode", C.c_char * 96),
                ("isa_evidence", C.c_char * 128), ("autotune_key", C.c_char * 1024),
                ("accumulator_k_block_size", C.c_uint64), ("accumulator_k_block_cap", C.c_uint64),
                ("accumulator_modulus", C.c_uint64), ("accumulator_max_lhs_abs", C.c_uint64),
                ("accumulator_max_rhs_abs", C.c_uint64), ("accumulator_max_product", C.c_uint64),
                ("accumulator_uses_int32_inner_product", C.c_uint32),
                ("accumulator_safe_for_k_block", C.c_uint32), ("accumulator_input_domain", C.c_char * 64),
                ("accumulator_signedness", C.c_char * 64), ("accumulator_type", C.c_char * 64),
                ("accumulator_modulus_policy", C.c_char * 128), ("accumulator_safety_status", C.c_char * 128)]


class MatrixStorageInfo(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("backend", c_enum),
                ("semantics", c_enum), ("logical_layout", c_enum), ("bound_kind", c_enum), ("rows", C.c_int64),
                ("cols", C.c_int64), ("logical_ld", C.c_int64), ("max_prefix", C.c_uint32),
                ("finite_modulus", C.c_uint32), ("matrix_instance_id", C.c_uint64), ("source_version", C.c_uint64),
                ("host_residues_current", C.c_uint32), ("device_residues_current", C.c_uint32),
                ("host_byte_limbs_current", C.c_uint32), ("device_byte_limbs_current", C.c_uint32),
                ("host_native_current", C.c_uint32), ("device_native_current", C.c_uint32),
                ("uses_residue_storage", C.c_uint32), ("uses_byte_limb_storage", C.c_uint32),
                ("uses_native_storage", C.c_uint32), ("hip_device_id", C.c_int32), ("flags", C.c_uint32),
                ("host_residue_bytes", C.c_uint64), ("device_residue_bytes", C.c_uint64),
                ("host_byte_limb_bytes", C.c_uint64), ("device_byte_limb_bytes", C.c_uint64),
                ("host_native_bytes", C.c_uint64), ("device_native_bytes", C.c_uint64),
                ("layout_version", C.c_char * 96), ("storage_scope", C.c_char * 96), ("detail", C.c_char * 256)]


class GroupedGemmTask(_Struct):
    _fields_ = [("struct_size", C.c_uint64), ("abi_version", C.c_uint32), ("a", C.c_void_p), ("b", C.c_void_p),
                ("c", C.c_void_p), ("workspace", C.c_void_p)]


vp = C.c_void_p
i64 = C.c_int64
u64 = C.c_uint64
u32 = C.c_uint32
u16 = C.c_uint16
P = C.POINTER

# name -> (restype, argtypes). Pointer arguments are passed as void*/ints so
# numpy arrays and device pointers can be handed over directly.
SIGNATURES = {
    "rns8_status_string": (C.c_char_p, [c_status]),
    "rns8_default_modulus_count": (u32, []),
    "rns8_default_modulus": (u16, [u32]),
    "rns8_prefix_range_bits": (C.c_double, [u32]),
    "rns8_validate_default_moduli": (c_status, []),
    "rns8_create_context": (c_status, [C.c_int, vp, P(vp)]),
    "rns8_destroy_context": (c_status, [vp]),
    "rns8_get_device_info": (c_status, [vp, vp]),
    "rns8_get_backend_capability_info": (c_status, [c_enum, vp]),
    "rns8_create_plan": (c_status, [vp, vp, P(vp)]),
    "rns8_destroy_plan": (c_status, [vp]),
    "rns8_get_plan_schedule_info": (c_status, [vp, vp]),
    "rns8_get_plan_tile_schedule": (c_status, [vp, vp, u64, P(u64)]),
    "rns8_get_plan_backend_info": (c_status, [vp, vp]),
    "rns8_get_plan_packing_info": (c_status, [vp, vp]),
    "rns8_get_grouped_dispatch_contract_info": (c_status, [vp, u32, vp]),
    "rns8_create_workspace": (c_status, [vp, vp, P(vp)]),
    "rns8_destroy_workspace": (c_status, [vp]),
    "rns8_create_matrix": (c_status, [vp, vp, P(vp)]),
    "rns8_destroy_matrix": (c_status, [vp]),
    "rns8_get_matrix_storage_info": (c_status, [vp, vp]),
    "rns8_get_resident_lifetime_info": (c_status, [vp, vp, vp, c_enum, vp]),
    "rns8_pack_i64": (c_status, [vp, vp, vp, i64, u64]),
    "rns8_pack_u64": (c_status, [vp, vp, vp, i64, u64]),
    "rns8_pack_finite_u8": (c_status, [vp, vp, u16, vp, i64, u64]),
    "rns8_gemm_rns": (c_status, [vp, vp, vp, vp, vp, vp]),
    "rns8_gemm_rns_grouped": (c_status, [vp, vp, vp, u32]),
    "rns8_gemm_finite_u8": (c_status, [vp, vp, u16, vp, vp, vp, vp]),
    "rns8_gemm_finite_u8_grouped": (c_status, [vp, vp, u16, vp, u32]),
    "rns8_export_i64": (c_status, [vp, vp, vp, vp, i64]),
    "rns8_export_u64": (c_status, [vp, vp, vp, vp, i64]),
    "rns8_export_finite_u8": (c_status, [vp, vp, u16, vp, vp, i64]),
    "rns8_export_exact_wide_signed_limbs": (c_status, [vp, vp, vp, vp, i64, u32]),
    "rns8_export_exact_wide_unsigned_limbs": (c_status, [vp, vp, vp, vp, i64, u32]),
    "rns8_gemm_i64_oneshot": (c_status, [vp, vp, vp, i64, vp, i64, vp, i64]),
    "rns8_gemm_u64_oneshot": (c_status, [vp, vp, vp, i64, vp, i64, vp, i64]),
    "rns8_gemm_wrap_u64": (c_status, [vp, vp, vp, vp, vp, vp]),
    "rns8_export_wrap_u64": (c_status, [vp, vp, vp, vp, i64]),
    "rns8_gemm_wrap_u64_oneshot": (c_status, [vp, vp, vp, i64, vp, i64, vp, i64]),
    "rns8_gemm_finite_ring_u8_oneshot": (c_status, [vp, vp, u16, vp, i64, vp, i64, vp, i64]),
    "rns8_gemm_finite_field_u8_oneshot": (c_status, [vp, vp, u16, vp, i64, vp, i64, vp, i64]),
    # device-pointer seam (include/rns8/rns8_cuda.h)
    "rns8_cuda_pack_i64_device": (c_status, [C.c_int, vp, i64, i64, i64, u32, vp, vp]),
    "rns8_cuda_pack_u64_device": (c_status, [C.c_int, vp, i64, i64, i64, u32, vp, vp]),
    "rns8_cuda_pack_finite_u8_device": (c_status, [C.c_int, vp, i64, i64, i64, u16, vp, vp]),
    "rns8_cuda_gemm_rns_scratch_bytes": (u64, [C.c_int, i64, i64, i64, u32]),
    "rns8_cuda_gemm_rns_device": (c_status, [C.c_int, vp, vp, vp, i64, i64, i64, u32, u32, vp, u64, vp, vp]),
    "rns8_cuda_gemm_export_bounded_scratch_bytes": (u64, [C.c_int, i64, i64, i64, u32]),
    "rns8_cuda_gemm_export_bounded_device": (c_status, [C.c_int, vp, vp, i64, i64, i64, u32, u32, u64, vp, i64, vp,
                                                        u64, vp, vp]),
    "rns8_cuda_gemm_finite_u8_scratch_bytes": (u64, [C.c_int, i64, i64, i64, u32]),
    "rns8_cuda_gemm_finite_u8_grouped_device": (c_status, [C.c_int, vp, vp, vp, u32, i64, i64, i64, u16, u32, vp,
                                                           u64, vp, vp]),
    "rns8_cuda_export_i64_device": (c_status, [C.c_int, vp, i64, i64, u32, u64, vp, i64, vp, vp]),
    "rns8_cuda_export_u64_device": (c_status, [C.c_int, vp, i64, i64, u32, u64, vp, i64, vp, vp]),
    "rns8_cuda_export_limbs_device": (c_status, [C.c_int, vp, i64, i64, u32, u32, u32, vp, i64, vp, vp]),
    "rns8_cuda_export_finite_u8_device": (c_status, [C.c_int, vp, i64, i64, u16, vp, i64, vp]),
    "rns8_cuda_plan_probe": (c_status, [vp, P(u32), P(u32), P(u64)]),
    "rns8_cuda_plan_tile_schedule_probe": (c_status, [vp, vp, u64, P(u64), vp]),
    "rns8_cuda_exact_gemm_bound_device": (c_status, [C.c_int, vp, vp, i64, i64, i64, u32, vp, vp, vp, vp, vp, vp]),
    "rns8_cuda_pack_wrap_u64_device": (c_status, [C.c_int, vp, i64, i64, i64, vp, vp]),
    "rns8_cuda_gemm_wrap_u64_device": (c_status, [C.c_int, vp, vp, vp, i64, i64, i64, u32, vp, vp]),
    "rns8_cuda_export_wrap_u64_device": (c_status, [C.c_int, vp, i64, i64, vp, i64, vp]),
    "rns8_cuda_pack_i64_planes_device": (c_status, [C.c_int, vp, i64, i64, i64, vp, u32, vp, vp]),
    "rns8_cuda_pack_u64_planes_device": (c_status, [C.c_int, vp, i64, i64, i64, vp, u32, vp, vp]),
    "rns8_cuda_gemm_rns_slabs_scratch_bytes": (u64, [C.c_int, i64, i64, i64, u32, u32]),
    "rns8_cuda_gemm_rns_slabs_device": (c_status, [C.c_int, vp, vp, i64, i64, i64, vp, u32, vp, u32, i64, u32, vp,
                                                   u64, vp, vp, vp]),
    "rns8_cuda_ipc_alloc": (c_status, [C.c_int, u64, P(vp), vp]),
    "rns8_cuda_ipc_free": (c_status, [C.c_int, vp]),
    "rns8_cuda_ipc_open": (c_status, [C.c_int, vp, P(vp)]),
    "rns8_cuda_ipc_close": (c_status, [C.c_int, vp]),
    "rns8_cuda_wait_probe": (c_status, [C.c_int, u32, u64, vp, vp]),
}

_LIB: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load librns8.so (built in-tree by rns8_b200.build). Raises if absent."""
    global _LIB
    if _LIB is None:
        path = Path(os.environ.get("RNS8_LIBRARY", LIB_PATH))
        if not path.exists():
            raise RuntimeError(f"{path} is missing: build it with `python -m rns8_b200.build`")
        handle = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError if the symbol is not exported
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def status_string(status: int) -> str:
    return lib().rns8_status_string(status).decode()
