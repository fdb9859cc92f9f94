"""rns8_b200: the RNS8 exact-integer GEMM hot path on NVIDIA B200 (sm_100a).

librns8.so (built from rns8_b200/csrc by rns8_b200.build) implements the
reference's include/rns8 C ABI: pack int64/uint64/uint8 into centered int8
residue planes, per-plane int8 GEMM on tcgen05 tensor cores with a modular
epilogue, and CRT/Garner export. This package only loads and wraps it.
"""

from .abi import (Backend, BoundKind, GEMM_AUTO, GEMM_SIMT, GEMM_TENSOR_CORE, Layout, PLAN_FORCE_FIXED_PREFIX,
                  Semantics, Status, lib)
from .api import (Context, Error, Matrix, Plan, Workspace, check, export_exact_wide_limbs, export_finite_u8,
                  export_i64, export_u64, gemm_desc, gemm_finite_u8, gemm_finite_u8_grouped,
                  gemm_finite_u8_oneshot, gemm_i64_oneshot, gemm_rns, gemm_rns_grouped, gemm_u64_oneshot,
                  gemm_wrap_u64, gemm_wrap_u64_oneshot, export_wrap_u64, plan_probe)

LADDER = (256, 255, 253, 251, 247, 239, 233, 229, 227, 223, 217, 211, 199, 197,
          193, 191, 181, 179, 173, 167, 163, 157, 151, 149, 139, 137, 131, 127)
