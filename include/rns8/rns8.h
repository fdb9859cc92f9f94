/* rns8 public C ABI: handles, descriptors, introspection structs and every
 * exported entry point.
 *
 * Interface source: include/rns8/rns8.h of the RNS8 reference (structs at
 * lines 17-647, functions at lines 661-1358). Field order, field types and
 * function signatures are the binary contract shared with existing callers and
 * are therefore identical; the comments are this library's own.
 *
 * Conventions (reference rns8.h:654-660):
 *   - every struct starts with {uint64_t struct_size; uint32_t abi_version};
 *     a struct is accepted when abi_version == RNS8_ABI_VERSION and
 *     struct_size >= sizeof(struct);
 *   - reserved flags must be zero;
 *   - malformed descriptors and unknown enum values return
 *     RNS8_INVALID_ARGUMENT before any backend is consulted; well-formed
 *     requests for a backend this library does not provide return
 *     RNS8_UNSUPPORTED_BACKEND;
 *   - calls are synchronous; callers serialise use of each handle.
 *
 * Backend: this library implements RNS8_BACKEND_CUDA_SM100 only (AUTO maps to
 * it). There is no CPU fallback: a context request for any other backend
 * returns RNS8_UNSUPPORTED_BACKEND. */
#ifndef RNS8_RNS8_H
#define RNS8_RNS8_H

#include <stdint.h>

#include "rns8/abi.h"
#include "rns8/bounds.h"
#include "rns8/moduli.h"
#include "rns8/semantics.h"
#include "rns8/status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct rns8_context rns8_context;
typedef struct rns8_plan rns8_plan;
typedef struct rns8_matrix rns8_matrix;
typedef struct rns8_sparse_matrix rns8_sparse_matrix;
typedef struct rns8_workspace rns8_workspace;
typedef struct rns8_prepack_cache rns8_prepack_cache;
typedef struct rns8_result_cache rns8_result_cache;

typedef struct rns8_context_options {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind requested_backend;
  uint32_t flags; /* reserved, must be zero */
} rns8_context_options;

typedef struct rns8_device_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  int32_t device_id;
  /* Historical field names kept for ABI compatibility: on this backend they
   * report CUDA availability and the CUDA runtime/driver versions, and
   * gcn_arch carries the compute capability ("sm_100a"). */
  uint32_t hip_available;
  uint32_t hip_runtime_version;
  uint32_t hip_driver_version;
  uint64_t global_mem_bytes;
  char name[128];
  char gcn_arch[64];
  char detail[256];
} rns8_device_info;

/* rns8_gemm_desc.flags. By default max_prefix is an upper budget and the plan
 * runs the smallest prefix whose modulus product covers the declared bound;
 * FORCE_FIXED_PREFIX runs exactly max_prefix planes. The two zero-skip flags
 * are only valid with per-tile bounds and caller-supplied proofs. */
#define RNS8_PLAN_FORCE_FIXED_PREFIX 0x00000001u
#define RNS8_PLAN_ALLOW_PROVEN_ZERO_TILE_SKIPS 0x00000002u
#define RNS8_PLAN_ALLOW_PROVEN_ZERO_ROW_COL_SKIPS 0x00000004u

/* Per-tile schedule flags (rns8_plan_schedule_info / tile entries). */
#define RNS8_TILE_SCHEDULE_ZERO_OUTPUT 0x00000001u
#define RNS8_TILE_SCHEDULE_ZERO_ROW_COL_PRODUCT 0x00000002u

typedef struct rns8_gemm_desc {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_semantics semantics;
  rns8_bound_kind bound_kind;
  rns8_backend_kind requested_backend;
  int64_t m;
  int64_t n;
  int64_t k;
  uint64_t bound;
  uint32_t max_prefix;
  uint32_t tile_m;
  uint32_t tile_n;
  /* Finite modulus for FINITE_RING_U8 / FINITE_FIELD_U8 plans; zero otherwise. */
  uint32_t finite_modulus;
  uint32_t flags; /* RNS8_PLAN_* */
  const uint64_t* tile_bounds;
  uint64_t tile_bounds_count;
  /* Per-operand magnitude bounds for RNS8_BOUND_INPUT_RANGE_AND_K; the plan
   * derives the output bound k * lhs_bound * rhs_bound. */
  uint64_t lhs_bound;
  uint64_t rhs_bound;
  const uint8_t* zero_a_rows;
  uint64_t zero_a_rows_count;
  const uint8_t* zero_b_cols;
  uint64_t zero_b_cols_count;
} rns8_gemm_desc;

typedef struct rns8_matrix_desc {
  uint64_t struct_size;
  uint32_t abi_version;
  int64_t rows;
  int64_t cols;
  int64_t logical_ld;
  rns8_semantics semantics;
  rns8_layout logical_layout;
  rns8_bound_kind bound_kind;
  uint32_t tile_m;
  uint32_t tile_n;
  uint32_t max_prefix;
  uint32_t flags; /* reserved, must be zero */
} rns8_matrix_desc;

typedef enum rns8_sparse_contract RNS8_ENUM_BASE {
  RNS8_SPARSE_NONE = 0,
  RNS8_SPARSE_A_4_TO_2_STRUCTURED_K = 1
} rns8_sparse_contract;

typedef enum rns8_sparse_operand RNS8_ENUM_BASE {
  RNS8_SPARSE_OPERAND_A = 1
} rns8_sparse_operand;

typedef enum rns8_sparse_index_layout RNS8_ENUM_BASE {
  RNS8_SPARSE_INDEX_LAYOUT_NONE = 0,
  RNS8_SPARSE_INDEX_LAYOUT_CANONICAL_2BIT_K_GROUPS_V1 = 1
} rns8_sparse_index_layout;

typedef enum rns8_sparse_value_signedness RNS8_ENUM_BASE {
  RNS8_SPARSE_VALUE_SIGNEDNESS_UNSPECIFIED = 0,
  RNS8_SPARSE_VALUE_SIGNEDNESS_SIGNED_I8 = 1,
  RNS8_SPARSE_VALUE_SIGNEDNESS_UNSIGNED_U8 = 2
} rns8_sparse_value_signedness;

typedef struct rns8_sparse_matrix_desc {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_semantics semantics;
  rns8_bound_kind bound_kind;
  rns8_sparse_contract contract;
  rns8_sparse_operand sparse_operand;
  rns8_sparse_index_layout index_layout;
  rns8_sparse_value_signedness value_signedness;
  int64_t rows;
  int64_t expanded_k;
  uint32_t group_size;
  uint32_t nonzeros_per_group;
  uint32_t max_prefix;
  uint32_t finite_modulus;
  uint32_t flags; /* reserved, must be zero */
  uint32_t reserved0;
} rns8_sparse_matrix_desc;

typedef struct rns8_sparse_matrix_storage_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  rns8_semantics semantics;
  rns8_bound_kind bound_kind;
  rns8_sparse_contract contract;
  rns8_sparse_operand sparse_operand;
  rns8_sparse_index_layout index_layout;
  rns8_sparse_value_signedness value_signedness;
  int64_t rows;
  int64_t expanded_k;
  uint32_t group_size;
  uint32_t nonzeros_per_group;
  uint32_t max_prefix;
  uint32_t finite_modulus;
  uint64_t matrix_instance_id;
  uint64_t source_version;
  uint64_t group_count;
  uint64_t packed_value_count;
  uint64_t host_packed_value_bytes;
  uint64_t host_packed_index_bytes;
  uint64_t device_packed_value_bytes;
  uint64_t device_packed_index_bytes;
  uint32_t host_current;
  uint32_t device_current;
  int32_t hip_device_id;
  uint32_t flags;
  char layout_version[96];
  char cache_key[512];
  char detail[256];
} rns8_sparse_matrix_storage_info;

typedef struct rns8_plan_schedule_info {
  uint64_t struct_size;
  uint32_t abi_version;
  uint32_t tile_m;
  uint32_t tile_n;
  uint64_t tile_rows;
  uint64_t tile_cols;
  uint64_t tile_count;
  uint32_t min_required_prefix;
  uint32_t max_required_prefix;
  uint32_t min_selected_prefix;
  uint32_t max_selected_prefix;
  uint32_t prefix_group_count;
  uint32_t adaptive_prefix_active;
  uint32_t adaptive_skip_active;
  uint32_t range_bit_length;
  uint32_t flags;
  rns8_bound_kind bound_kind;
  uint32_t reserved0;
  uint64_t effective_bound;
  uint64_t lhs_bound;
  uint64_t rhs_bound;
  uint64_t zero_a_row_count;
  uint64_t zero_b_col_count;
  uint64_t zero_row_col_product_count;
  char bound_contract[96];
} rns8_plan_schedule_info;

typedef struct rns8_plan_tile_schedule_entry {
  uint64_t struct_size;
  uint32_t abi_version;
  uint32_t flags;
  uint64_t tile_row;
  uint64_t tile_col;
  int64_t row_offset;
  int64_t col_offset;
  int64_t row_extent;
  int64_t col_extent;
  uint32_t required_prefix;
  uint32_t selected_prefix;
  uint32_t group_index;
  uint32_t range_bit_length;
} rns8_plan_tile_schedule_entry;

typedef struct rns8_backend_capability_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  uint32_t is_accelerator;
  uint32_t is_available;
  uint32_t is_correctness_backend;
  uint32_t is_matrix_engine_backend;
  uint32_t supports_bounded_rns;
  uint32_t supports_exact_wide_rns;
  uint32_t supports_finite_u8;
  uint32_t supports_wrap64;
  uint32_t requires_feature_detection;
  uint32_t enable_flag_fail_fast;
  uint32_t candidate_evidence_only;
  uint32_t compiled_kernel_available;
  uint32_t exact_differential_validated;
  uint32_t performance_validated;
  uint32_t flags;
  char backend_name[64];
  char selected_kernel[128];
  char library_name[64];
  char library_version[64];
  char enable_flag[64];
  char epilogue_mode[96];
  char workspace_mode[96];
  char isa_evidence[128];
  char status[128];
  char detail[256];
} rns8_backend_capability_info;

typedef struct rns8_plan_backend_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  uint32_t is_accelerator;
  uint32_t is_correctness_backend;
  uint32_t is_matrix_engine_backend;
  uint32_t compiled_kernel_available;
  uint32_t exact_differential_validated;
  uint32_t performance_validated;
  uint32_t flags;
  uint64_t workspace_required_bytes;
  char selected_kernel[128];
  char accelerator_library[64];
  char accelerator_version[64];
  char capability_status[128];
  char epilogue_mode[96];
  char workspace_mode[96];
  char isa_evidence[128];
  char autotune_key[1024];
  uint64_t accumulator_k_block_size;
  uint64_t accumulator_k_block_cap;
  uint64_t accumulator_modulus;
  uint64_t accumulator_max_lhs_abs;
  uint64_t accumulator_max_rhs_abs;
  uint64_t accumulator_max_product;
  uint32_t accumulator_uses_int32_inner_product;
  uint32_t accumulator_safe_for_k_block;
  char accumulator_input_domain[64];
  char accumulator_signedness[64];
  char accumulator_type[64];
  char accumulator_modulus_policy[128];
  char accumulator_safety_status[128];
} rns8_plan_backend_info;

typedef enum rns8_output_domain RNS8_ENUM_BASE {
  RNS8_OUTPUT_DOMAIN_RNS_RESIDUE = 1,
  RNS8_OUTPUT_DOMAIN_NATIVE_I64_U64 = 2,
  RNS8_OUTPUT_DOMAIN_FINITE_U8 = 3,
  RNS8_OUTPUT_DOMAIN_WRAP64_BYTE_LIMB = 4
} rns8_output_domain;

typedef enum rns8_next_op_flags RNS8_ENUM_BASE {
  RNS8_NEXT_OP_FINAL_EXPORT = 1u << 0,
  RNS8_NEXT_OP_RNS_GEMM = 1u << 1,
  RNS8_NEXT_OP_NATIVE_GEMM = 1u << 2,
  RNS8_NEXT_OP_NATIVE_TO_RNS_CONVERTIBLE = 1u << 3,
  RNS8_NEXT_OP_REUSABLE_B_PREPACK = 1u << 4
} rns8_next_op_flags;

#define RNS8_PLAN_PACKING_SOURCE_VERSIONED_INPUTS 0x00000001u
#define RNS8_PLAN_PACKING_SAME_SOURCE_VERSION_PACK_ELISION 0x00000002u

typedef struct rns8_plan_packing_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  rns8_semantics semantics;
  uint32_t uses_resident_matrix_inputs;
  uint32_t uses_transient_pack_workspace;
  uint32_t uses_matrix_engine_pack_layout;
  uint32_t reusable_prepack_cache_available;
  uint32_t production_prepack_cache_available;
  uint32_t flags;
  rns8_output_domain input_domain;
  rns8_output_domain output_domain;
  uint32_t output_host_current;
  uint32_t output_device_current;
  uint32_t next_op_flags;
  uint32_t reserved0;
  uint64_t a_pack_workspace_bytes;
  uint64_t b_pack_workspace_bytes;
  uint64_t accumulator_workspace_bytes;
  uint64_t library_workspace_bytes;
  uint64_t total_transient_workspace_bytes;
  char input_domain_name[64];
  char output_domain_name[64];
  char next_op_hint[160];
  char a_layout_version[96];
  char b_layout_version[96];
  char output_layout_version[96];
  char prepack_cache_scope[96];
  char detail[256];
} rns8_plan_packing_info;

#define RNS8_GROUPED_DISPATCH_CONTRACT_SAME_SHAPE_REQUIRED 0x00000001u
#define RNS8_GROUPED_DISPATCH_CONTRACT_COMPACT_ROW_MAJOR_REQUIRED 0x00000002u
#define RNS8_GROUPED_DISPATCH_CONTRACT_UNIQUE_TASK_HANDLES_REQUIRED 0x00000004u
#define RNS8_GROUPED_DISPATCH_CONTRACT_ONE_WORKSPACE_PER_TASK_REQUIRED 0x00000008u
#define RNS8_GROUPED_DISPATCH_CONTRACT_SAME_DEVICE_REQUIRED 0x00000010u
#define RNS8_GROUPED_DISPATCH_CONTRACT_PER_TASK_SOURCE_VERSION_REQUIRED 0x00000020u
#define RNS8_GROUPED_DISPATCH_CONTRACT_DEVICE_CURRENT_OUTPUT_REQUIRED 0x00000040u
#define RNS8_GROUPED_DISPATCH_CONTRACT_BENCHMARK_ONLY_EXECUTION 0x00000080u
#define RNS8_GROUPED_DISPATCH_CONTRACT_PUBLIC_PACK_EXPLICIT 0x00000100u
#define RNS8_GROUPED_DISPATCH_CONTRACT_PUBLIC_EXPORT_EXPLICIT 0x00000200u
#define RNS8_GROUPED_DISPATCH_CONTRACT_GENERIC_BUCKETING_UNAVAILABLE 0x00000400u
#define RNS8_GROUPED_DISPATCH_CONTRACT_AUTO_ROUTING_DISABLED 0x00000800u

typedef struct rns8_grouped_dispatch_contract_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  rns8_semantics semantics;
  uint32_t task_count;
  uint32_t descriptor_contract_supported;
  uint32_t public_execution_available;
  uint32_t same_shape_required;
  uint32_t same_semantics_required;
  uint32_t compact_row_major_required;
  uint32_t unique_matrix_handles_required;
  uint32_t unique_workspace_handles_required;
  uint32_t same_plan_fingerprint_required;
  uint32_t same_device_required;
  uint32_t device_resident_inputs_required;
  uint32_t per_task_source_versions_required;
  uint32_t produces_device_current_output;
  uint32_t final_export_required_for_host_output;
  uint32_t per_task_status_required;
  uint32_t checksum_policy_required;
  uint32_t descriptor_reuse_validated;
  uint32_t flags;
  char descriptor_layout[96];
  char bucket_policy[96];
  char source_version_policy[96];
  char workspace_policy[96];
  char matrix_ownership_policy[128];
  char descriptor_reuse_policy[128];
  char stride_policy[128];
  char output_currentness_policy[128];
  char lifetime_policy[128];
  char checksum_policy[96];
  char status_policy[96];
  char device_descriptor_policy[96];
  char output_domain[64];
  char unsupported_reason[160];
  char detail[256];
} rns8_grouped_dispatch_contract_info;

typedef struct rns8_grouped_gemm_task {
  uint64_t struct_size;
  uint32_t abi_version;
  const rns8_matrix* a;
  const rns8_matrix* b;
  rns8_matrix* c;
  rns8_workspace* workspace;
} rns8_grouped_gemm_task;

typedef struct rns8_matrix_storage_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  rns8_semantics semantics;
  rns8_layout logical_layout;
  rns8_bound_kind bound_kind;
  int64_t rows;
  int64_t cols;
  int64_t logical_ld;
  uint32_t max_prefix;
  uint32_t finite_modulus;
  uint64_t matrix_instance_id;
  uint64_t source_version;
  uint32_t host_residues_current;
  uint32_t device_residues_current;
  uint32_t host_byte_limbs_current;
  uint32_t device_byte_limbs_current;
  uint32_t host_native_current;
  uint32_t device_native_current;
  uint32_t uses_residue_storage;
  uint32_t uses_byte_limb_storage;
  uint32_t uses_native_storage;
  int32_t hip_device_id;
  uint32_t flags;
  uint64_t host_residue_bytes;
  uint64_t device_residue_bytes;
  uint64_t host_byte_limb_bytes;
  uint64_t device_byte_limb_bytes;
  uint64_t host_native_bytes;
  uint64_t device_native_bytes;
  char layout_version[96];
  char storage_scope[96];
  char detail[256];
} rns8_matrix_storage_info;

#define RNS8_RESULT_CACHE_CONTRACT_OUTPUT_RECTANGLES 0x00000001u
#define RNS8_RESULT_CACHE_CONTRACT_DIRECT_HIP_ONLY 0x00000002u
#define RNS8_RESULT_CACHE_CONTRACT_FULL_K_RECOMPUTE 0x00000004u
#define RNS8_RESULT_CACHE_CONTRACT_EXPLICIT_OPT_IN 0x00000008u

#define RNS8_RESULT_CACHE_FLAG_INITIALIZED 0x00000001u
#define RNS8_RESULT_CACHE_FLAG_LAST_CALL_HIT 0x00000002u
#define RNS8_RESULT_CACHE_FLAG_LAST_CALL_MISS 0x00000004u
#define RNS8_RESULT_CACHE_FLAG_LAST_CALL_PARTIAL_RECOMPUTE 0x00000008u
#define RNS8_RESULT_CACHE_FLAG_LAST_CALL_FULL_FALLBACK 0x00000010u
#define RNS8_RESULT_CACHE_FLAG_LAST_CALL_STALE_REJECTED 0x00000020u

typedef struct rns8_result_cache_desc {
  uint64_t struct_size;
  uint32_t abi_version;
  uint32_t flags;
  uint32_t max_dirty_regions;
  uint32_t reserved0;
} rns8_result_cache_desc;

typedef struct rns8_dirty_region {
  uint64_t struct_size;
  uint32_t abi_version;
  uint32_t flags;
  int64_t row_offset;
  int64_t col_offset;
  int64_t row_extent;
  int64_t col_extent;
} rns8_dirty_region;

typedef struct rns8_result_cache_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  rns8_semantics semantics;
  rns8_bound_kind bound_kind;
  int64_t m;
  int64_t n;
  int64_t k;
  uint32_t max_prefix;
  uint32_t finite_modulus;
  uint32_t flags;
  int32_t hip_device_id;
  uint32_t initialized;
  uint32_t max_dirty_regions;
  uint32_t last_dirty_region_count;
  uint32_t last_recomputed_region_count;
  uint32_t last_full_fallback;
  uint32_t last_cache_hit;
  uint32_t last_cache_miss;
  uint32_t last_stale_rejection;
  uint64_t plan_fingerprint;
  uint64_t workspace_fingerprint;
  uint64_t result_cache_key_hash;
  uint64_t a_matrix_instance_id;
  uint64_t b_matrix_instance_id;
  uint64_t c_matrix_instance_id;
  uint64_t a_source_version;
  uint64_t b_source_version;
  uint64_t c_source_version;
  uint64_t snapshot_device_bytes;
  uint64_t copied_from_cache_bytes;
  uint64_t recomputed_cell_count;
  uint64_t cache_allocation_bytes;
  char target_id[128];
  char selected_backend[64];
  char selected_kernel[128];
  char dirty_region_contract[128];
  char source_identity_policy[128];
  char source_version_policy[128];
  char result_lifetime_policy[128];
  char stale_reason[160];
  char fallback_reason[160];
  char detail[256];
} rns8_result_cache_info;

typedef enum rns8_resident_matrix_role RNS8_ENUM_BASE {
  RNS8_RESIDENT_MATRIX_ROLE_UNKNOWN = 0,
  RNS8_RESIDENT_MATRIX_ROLE_A = 1,
  RNS8_RESIDENT_MATRIX_ROLE_B = 2,
  RNS8_RESIDENT_MATRIX_ROLE_C = 3
} rns8_resident_matrix_role;

typedef struct rns8_resident_lifetime_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  rns8_semantics semantics;
  rns8_layout logical_layout;
  rns8_bound_kind bound_kind;
  rns8_resident_matrix_role matrix_role;
  rns8_output_domain current_output_domain;
  int64_t rows;
  int64_t cols;
  int64_t logical_ld;
  uint32_t max_prefix;
  uint32_t finite_modulus;
  uint64_t source_version;
  uint64_t plan_fingerprint;
  uint64_t workspace_fingerprint;
  int32_t hip_device_id;
  uint32_t source_version_valid;
  uint32_t host_current;
  uint32_t device_current;
  uint32_t device_resident;
  uint32_t plan_binding_available;
  uint32_t plan_binding_matches;
  uint32_t workspace_binding_available;
  uint32_t workspace_identity_matches;
  uint32_t workspace_schedule_matches;
  uint32_t workspace_backend_matches;
  uint32_t workspace_binding_matches;
  uint32_t device_id_matches;
  uint32_t can_feed_rns_gemm;
  uint32_t can_feed_native_gemm;
  uint32_t can_feed_final_export;
  uint32_t flags;
  char current_domain[64];
  char matrix_role_name[32];
  char source_version_policy[96];
  char workspace_binding_policy[128];
  char output_currentness_policy[128];
  char lifetime_policy[128];
  char mismatch_policy[160];
  char detail[256];
} rns8_resident_lifetime_info;

typedef enum rns8_operand_role RNS8_ENUM_BASE {
  RNS8_OPERAND_A = 1,
  RNS8_OPERAND_B = 2
} rns8_operand_role;

typedef struct rns8_prepack_cache_key_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  rns8_semantics semantics;
  rns8_operand_role operand_role;
  uint32_t cache_key_valid;
  uint32_t reusable_prepack_cache_available;
  uint32_t production_prepack_cache_available;
  uint32_t flags;
  int32_t hip_device_id;
  uint32_t reserved0;
  int64_t matrix_rows;
  int64_t matrix_cols;
  uint32_t max_prefix;
  uint32_t finite_modulus;
  uint64_t source_version;
  uint64_t plan_fingerprint;
  uint64_t cache_key_hash;
  char matrix_layout_version[96];
  char operand_layout_version[96];
  char cache_scope[96];
  char cache_key[512];
  char detail[256];
} rns8_prepack_cache_key_info;

typedef struct rns8_prepack_cache_info {
  uint64_t struct_size;
  uint32_t abi_version;
  rns8_backend_kind backend;
  rns8_semantics semantics;
  rns8_operand_role operand_role;
  uint32_t cache_key_valid;
  uint32_t reusable_prepack_cache_available;
  uint32_t production_prepack_cache_available;
  uint32_t flags;
  int32_t hip_device_id;
  uint32_t reserved0;
  int64_t matrix_rows;
  int64_t matrix_cols;
  int64_t k;
  uint32_t max_prefix;
  uint32_t finite_modulus;
  uint64_t source_version;
  uint64_t plan_fingerprint;
  uint64_t cache_key_hash;
  uint64_t device_bytes;
  uint64_t operand_pack_bytes;
  char matrix_layout_version[96];
  char operand_layout_version[96];
  char cache_scope[96];
  char cache_key[512];
  char detail[256];
} rns8_prepack_cache_info;

/* ---- context ---------------------------------------------------------- */
/* device_id < 0 selects device 0. options may be NULL (AUTO). */
RNS8_API rns8_status rns8_create_context(int device_id, const rns8_context_options* options, rns8_context** out);
RNS8_API rns8_status rns8_destroy_context(rns8_context* ctx);
RNS8_API rns8_status rns8_get_device_info(rns8_context* ctx, rns8_device_info* out);
RNS8_API rns8_status rns8_get_backend_capability_info(rns8_backend_kind backend, rns8_backend_capability_info* out);

/* ---- plan ------------------------------------------------------------- */
RNS8_API rns8_status rns8_create_plan(rns8_context* ctx, const rns8_gemm_desc* desc, rns8_plan** out);
RNS8_API rns8_status rns8_destroy_plan(rns8_plan* plan);
RNS8_API rns8_status rns8_get_plan_schedule_info(const rns8_plan* plan, rns8_plan_schedule_info* out);
RNS8_API rns8_status rns8_get_plan_tile_schedule(const rns8_plan* plan, rns8_plan_tile_schedule_entry* entries,
                                                 uint64_t capacity, uint64_t* written);
RNS8_API rns8_status rns8_get_plan_backend_info(const rns8_plan* plan, rns8_plan_backend_info* out);
RNS8_API rns8_status rns8_get_plan_packing_info(const rns8_plan* plan, rns8_plan_packing_info* out);
RNS8_API rns8_status rns8_get_grouped_dispatch_contract_info(const rns8_plan* plan, uint32_t task_count,
                                                             rns8_grouped_dispatch_contract_info* out);

/* ---- workspace and resident matrices ----------------------------------- */
RNS8_API rns8_status rns8_create_workspace(rns8_context* ctx, const rns8_plan* plan, rns8_workspace** out);
RNS8_API rns8_status rns8_destroy_workspace(rns8_workspace* workspace);
RNS8_API rns8_status rns8_create_matrix(rns8_context* ctx, const rns8_matrix_desc* desc, rns8_matrix** out);
RNS8_API rns8_status rns8_destroy_matrix(rns8_matrix* matrix);
RNS8_API rns8_status rns8_get_matrix_storage_info(const rns8_matrix* matrix, rns8_matrix_storage_info* out);
RNS8_API rns8_status rns8_get_resident_lifetime_info(const rns8_matrix* matrix, const rns8_plan* plan,
                                                     const rns8_workspace* workspace,
                                                     rns8_resident_matrix_role matrix_role,
                                                     rns8_resident_lifetime_info* out);

/* ---- prepack / result caches (not provided by this backend) ----------- */
RNS8_API rns8_status rns8_get_prepack_cache_key_info(const rns8_plan* plan, const rns8_matrix* matrix,
                                                     rns8_operand_role operand_role,
                                                     rns8_prepack_cache_key_info* out);
RNS8_API rns8_status rns8_create_prepack_cache(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* matrix,
                                               rns8_operand_role operand_role, rns8_prepack_cache** out);
RNS8_API rns8_status rns8_create_b_prepack_cache_i64(rns8_context* ctx, const rns8_plan* plan, const int64_t* values,
                                                     int64_t ld, uint64_t source_version, rns8_prepack_cache** out);
RNS8_API rns8_status rns8_create_b_prepack_cache_u64(rns8_context* ctx, const rns8_plan* plan, const uint64_t* values,
                                                     int64_t ld, uint64_t source_version, rns8_prepack_cache** out);
RNS8_API rns8_status rns8_get_prepack_cache_info(const rns8_prepack_cache* cache, rns8_prepack_cache_info* out);
RNS8_API rns8_status rns8_destroy_prepack_cache(rns8_prepack_cache* cache);
RNS8_API rns8_status rns8_create_result_cache(rns8_context* ctx, const rns8_plan* plan,
                                              const rns8_result_cache_desc* desc, rns8_result_cache** out);
RNS8_API rns8_status rns8_destroy_result_cache(rns8_result_cache* cache);
RNS8_API rns8_status rns8_get_result_cache_info(const rns8_result_cache* cache, rns8_result_cache_info* out);
RNS8_API rns8_status rns8_invalidate_result_cache(rns8_result_cache* cache);

/* ---- pack: native host values -> resident centered int8 residue planes -- */
/* ld is in elements; source_version != 0 lets a repeated pack of the same
 * source skip the upload and conversion. */
RNS8_API rns8_status rns8_pack_i64(rns8_context* ctx, rns8_matrix* matrix, const int64_t* src, int64_t ld,
                                   uint64_t source_version);
RNS8_API rns8_status rns8_pack_u64(rns8_context* ctx, rns8_matrix* matrix, const uint64_t* src, int64_t ld,
                                   uint64_t source_version);
RNS8_API rns8_status rns8_lift_exact_wide_cpu(rns8_context* ctx, rns8_matrix* matrix, uint32_t target_prefix,
                                              uint64_t max_staged_residue_bytes);
/* Finite u8: modulus in [2,256] (ring) or prime <= 251 (field). */
RNS8_API rns8_status rns8_pack_finite_u8(rns8_context* ctx, rns8_matrix* matrix, uint16_t modulus,
                                         const uint8_t* src, int64_t ld, uint64_t source_version);

/* ---- 4:2 structured-sparse A (not provided by this backend) ------------ */
RNS8_API rns8_status rns8_sparse_a_4_to_2_layout_counts(const rns8_sparse_matrix_desc* desc, uint64_t* group_count,
                                                        uint64_t* packed_value_count);
RNS8_API rns8_status rns8_pack_sparse_a_4_to_2_u8(const rns8_sparse_matrix_desc* desc, const uint8_t* dense_a,
                                                  int64_t dense_ld, uint8_t* packed_values, uint8_t* packed_indices);
RNS8_API rns8_status rns8_expand_sparse_a_4_to_2_u8(const rns8_sparse_matrix_desc* desc,
                                                    const uint8_t* packed_values, const uint8_t* packed_indices,
                                                    uint8_t* dense_a, int64_t dense_ld);
RNS8_API rns8_status rns8_create_sparse_matrix(rns8_context* ctx, const rns8_sparse_matrix_desc* desc,
                                               rns8_sparse_matrix** out);
RNS8_API rns8_status rns8_destroy_sparse_matrix(rns8_sparse_matrix* matrix);
RNS8_API rns8_status rns8_get_sparse_matrix_storage_info(const rns8_sparse_matrix* matrix,
                                                         rns8_sparse_matrix_storage_info* out);
RNS8_API rns8_status rns8_pack_sparse_a_4_to_2_matrix_u8(rns8_context* ctx, rns8_sparse_matrix* matrix,
                                                         const uint8_t* dense_a_planes, int64_t dense_ld,
                                                         uint64_t source_version);
RNS8_API rns8_status rns8_expand_sparse_a_4_to_2_matrix_u8(const rns8_sparse_matrix* matrix, uint8_t* dense_a_planes,
                                                           int64_t dense_ld);
RNS8_API rns8_status rns8_gemm_rns_sparse_a(rns8_context* ctx, const rns8_plan* plan, const rns8_sparse_matrix* A,
                                            const rns8_matrix* B, rns8_matrix* C, rns8_workspace* workspace);

/* ---- GEMM over resident residue planes --------------------------------- */
/* Per plane p: C_p = (A_p x B_p) mod m_p, int32 accumulation reduced modulo
 * m_p at least every RNS8_SAFE_INT32_K_BLOCK products. Exact-wide inputs
 * carry range proofs; an insufficient prefix returns RNS8_RANGE_ERROR before
 * C is touched. */
RNS8_API rns8_status rns8_gemm_rns(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* A,
                                   const rns8_matrix* B, rns8_matrix* C, rns8_workspace* workspace);
RNS8_API rns8_status rns8_gemm_exact_wide_cpu_auto(rns8_context* ctx, const rns8_plan* plan, rns8_matrix* A,
                                                   rns8_matrix* B, rns8_matrix* C, rns8_workspace* workspace,
                                                   uint64_t max_staged_residue_bytes, uint32_t* out_selected_prefix);
RNS8_API rns8_status rns8_gemm_rns_incremental(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* A,
                                               const rns8_matrix* B, rns8_matrix* C, rns8_workspace* workspace,
                                               rns8_result_cache* cache, const rns8_dirty_region* dirty_regions,
                                               uint32_t dirty_region_count);
/* Same-shape batch of resident RNS GEMMs executed as one persistent launch. */
RNS8_API rns8_status rns8_gemm_rns_grouped(rns8_context* ctx, const rns8_plan* plan,
                                           const rns8_grouped_gemm_task* tasks, uint32_t task_count);
RNS8_API rns8_status rns8_gemm_rns_prepacked_b(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* A,
                                               const rns8_prepack_cache* B, rns8_matrix* C,
                                               rns8_workspace* workspace);
RNS8_API rns8_status rns8_gemm_wrap_u64(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* A,
                                        const rns8_matrix* B, rns8_matrix* C, rns8_workspace* workspace);
RNS8_API rns8_status rns8_gemm_finite_u8(rns8_context* ctx, const rns8_plan* plan, uint16_t modulus,
                                         const rns8_matrix* A, const rns8_matrix* B, rns8_matrix* C,
                                         rns8_workspace* workspace);
RNS8_API rns8_status rns8_gemm_finite_u8_sparse_a(rns8_context* ctx, const rns8_plan* plan, uint16_t modulus,
                                                  const rns8_sparse_matrix* A, const rns8_matrix* B, rns8_matrix* C,
                                                  rns8_workspace* workspace);
RNS8_API rns8_status rns8_gemm_finite_u8_incremental(rns8_context* ctx, const rns8_plan* plan, uint16_t modulus,
                                                     const rns8_matrix* A, const rns8_matrix* B, rns8_matrix* C,
                                                     rns8_workspace* workspace, rns8_result_cache* cache,
                                                     const rns8_dirty_region* dirty_regions,
                                                     uint32_t dirty_region_count);
/* Same-shape batch of resident finite-u8 GEMMs executed as one persistent launch. */
RNS8_API rns8_status rns8_gemm_finite_u8_grouped(rns8_context* ctx, const rns8_plan* plan, uint16_t modulus,
                                                 const rns8_grouped_gemm_task* tasks, uint32_t task_count);

/* ---- export: residue planes -> native host values ----------------------- */
/* Bounded exports stage every cell and return RNS8_RANGE_ERROR, with dst
 * untouched, if any reconstructed value violates the plan's bound. */
RNS8_API rns8_status rns8_export_i64(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* C, int64_t* dst,
                                     int64_t ld);
RNS8_API rns8_status rns8_export_u64(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* C, uint64_t* dst,
                                     int64_t ld);
RNS8_API rns8_status rns8_export_wrap_u64(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* C,
                                          uint64_t* dst, int64_t ld);
/* Canonical residues in [0, modulus) (full byte for 256); padded columns
 * beyond n are left untouched. */
RNS8_API rns8_status rns8_export_finite_u8(rns8_context* ctx, const rns8_plan* plan, uint16_t modulus,
                                           const rns8_matrix* C, uint8_t* dst, int64_t ld);
/* dst[((row * ld) + col) * limb_count + limb], little-endian 64-bit limbs,
 * limb_count in [1,32]. Signed: two's complement of the centered CRT value;
 * unsigned: the canonical value. A value that does not fit returns
 * RNS8_RANGE_ERROR with dst untouched; nothing is ever truncated. */
RNS8_API rns8_status rns8_export_exact_wide_signed_limbs(rns8_context* ctx, const rns8_plan* plan,
                                                         const rns8_matrix* C, uint64_t* dst, int64_t ld,
                                                         uint32_t limb_count);
RNS8_API rns8_status rns8_export_exact_wide_unsigned_limbs(rns8_context* ctx, const rns8_plan* plan,
                                                           const rns8_matrix* C, uint64_t* dst, int64_t ld,
                                                           uint32_t limb_count);

/* ---- one-shot host-to-host GEMMs --------------------------------------- */
RNS8_API rns8_status rns8_gemm_i64_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc, const int64_t* A,
                                           int64_t lda, const int64_t* B, int64_t ldb, int64_t* C, int64_t ldc);
RNS8_API rns8_status rns8_gemm_u64_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc, const uint64_t* A,
                                           int64_t lda, const uint64_t* B, int64_t ldb, uint64_t* C, int64_t ldc);
RNS8_API rns8_status rns8_gemm_wrap_u64_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc, const uint64_t* A,
                                                int64_t lda, const uint64_t* B, int64_t ldb, uint64_t* C,
                                                int64_t ldc);
RNS8_API rns8_status rns8_gemm_finite_ring_u8_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc,
                                                      uint16_t modulus, const uint8_t* A, int64_t lda,
                                                      const uint8_t* B, int64_t ldb, uint8_t* C, int64_t ldc);
RNS8_API rns8_status rns8_gemm_finite_field_u8_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc,
                                                       uint16_t modulus, const uint8_t* A, int64_t lda,
                                                       const uint8_t* B, int64_t ldb, uint8_t* C, int64_t ldc);

/* ---- research placeholders: always RNS8_UNSUPPORTED_BACKEND ------------- */
RNS8_API rns8_status rns8_ozaki_decompose_i64(rns8_context* ctx, const int64_t* src, int64_t rows, int64_t cols,
                                              int64_t ld, int8_t** out_components, int64_t* out_component_ld,
                                              int* out_split_count);
RNS8_API rns8_status rns8_strassen_gemm_research(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* A,
                                                 const rns8_matrix* B, rns8_matrix* C, rns8_workspace* workspace,
                                                 int strassen_level, double* out_memory_overhead_ratio);
RNS8_API rns8_status rns8_freivalds_verify(rns8_context* ctx, const rns8_matrix* A, const rns8_matrix* B,
                                           const rns8_matrix* C, uint64_t random_seed, int repetition_count,
                                           double* out_failure_probability);

#ifdef __cplusplus
}
#endif

#endif /* RNS8_RNS8_H */
