// Entry points of the rns8 C ABI that this backend does not provide: prepack
// and result caches, incremental GEMM, 4:2 structured sparsity, strict
// mod 2^64 byte-limb GEMM, CPU-only exact-wide lifting and the research
// placeholders. They exist so the library is link-compatible with every
// caller of the reference ABI; each returns RNS8_UNSUPPORTED_BACKEND without
// touching its outputs, as the reference does for a backend that lacks a
// surface (include/rns8/rns8.h:1314-1347, src/core/accelerator_backend.cpp:77-101).
// Creation functions clear *out first; destroy functions accept NULL.
#include "api_internal.hpp"

#define RNS8_UNSUPPORTED return RNS8_UNSUPPORTED_BACKEND

extern "C" {

rns8_status rns8_get_prepack_cache_key_info(const rns8_plan*, const rns8_matrix*, rns8_operand_role,
                                            rns8_prepack_cache_key_info*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_create_prepack_cache(rns8_context*, const rns8_plan*, const rns8_matrix*, rns8_operand_role,
                                      rns8_prepack_cache** out) {
  if (out) *out = nullptr;
  RNS8_UNSUPPORTED;
}
rns8_status rns8_create_b_prepack_cache_i64(rns8_context*, const rns8_plan*, const int64_t*, int64_t, uint64_t,
                                            rns8_prepack_cache** out) {
  if (out) *out = nullptr;
  RNS8_UNSUPPORTED;
}
rns8_status rns8_create_b_prepack_cache_u64(rns8_context*, const rns8_plan*, const uint64_t*, int64_t, uint64_t,
                                            rns8_prepack_cache** out) {
  if (out) *out = nullptr;
  RNS8_UNSUPPORTED;
}
rns8_status rns8_get_prepack_cache_info(const rns8_prepack_cache*, rns8_prepack_cache_info*) { RNS8_UNSUPPORTED; }
rns8_status rns8_destroy_prepack_cache(rns8_prepack_cache* cache) {
  return cache ? RNS8_UNSUPPORTED_BACKEND : RNS8_SUCCESS;
}
rns8_status rns8_create_result_cache(rns8_context*, const rns8_plan*, const rns8_result_cache_desc*,
                                     rns8_result_cache** out) {
  if (out) *out = nullptr;
  RNS8_UNSUPPORTED;
}
rns8_status rns8_destroy_result_cache(rns8_result_cache* cache) {
  return cache ? RNS8_UNSUPPORTED_BACKEND : RNS8_SUCCESS;
}
rns8_status rns8_get_result_cache_info(const rns8_result_cache*, rns8_result_cache_info*) { RNS8_UNSUPPORTED; }
rns8_status rns8_invalidate_result_cache(rns8_result_cache*) { RNS8_UNSUPPORTED; }

rns8_status rns8_lift_exact_wide_cpu(rns8_context*, rns8_matrix*, uint32_t, uint64_t) { RNS8_UNSUPPORTED; }

rns8_status rns8_sparse_a_4_to_2_layout_counts(const rns8_sparse_matrix_desc*, uint64_t*, uint64_t*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_pack_sparse_a_4_to_2_u8(const rns8_sparse_matrix_desc*, const uint8_t*, int64_t, uint8_t*,
                                         uint8_t*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_expand_sparse_a_4_to_2_u8(const rns8_sparse_matrix_desc*, const uint8_t*, const uint8_t*, uint8_t*,
                                           int64_t) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_create_sparse_matrix(rns8_context*, const rns8_sparse_matrix_desc*, rns8_sparse_matrix** out) {
  if (out) *out = nullptr;
  RNS8_UNSUPPORTED;
}
rns8_status rns8_destroy_sparse_matrix(rns8_sparse_matrix* matrix) {
  return matrix ? RNS8_UNSUPPORTED_BACKEND : RNS8_SUCCESS;
}
rns8_status rns8_get_sparse_matrix_storage_info(const rns8_sparse_matrix*, rns8_sparse_matrix_storage_info*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_pack_sparse_a_4_to_2_matrix_u8(rns8_context*, rns8_sparse_matrix*, const uint8_t*, int64_t,
                                                uint64_t) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_expand_sparse_a_4_to_2_matrix_u8(const rns8_sparse_matrix*, uint8_t*, int64_t) { RNS8_UNSUPPORTED; }
rns8_status rns8_gemm_rns_sparse_a(rns8_context*, const rns8_plan*, const rns8_sparse_matrix*, const rns8_matrix*,
                                   rns8_matrix*, rns8_workspace*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_gemm_finite_u8_sparse_a(rns8_context*, const rns8_plan*, uint16_t, const rns8_sparse_matrix*,
                                         const rns8_matrix*, rns8_matrix*, rns8_workspace*) {
  RNS8_UNSUPPORTED;
}

rns8_status rns8_gemm_exact_wide_cpu_auto(rns8_context*, const rns8_plan*, rns8_matrix*, rns8_matrix*, rns8_matrix*,
                                          rns8_workspace*, uint64_t, uint32_t*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_gemm_rns_incremental(rns8_context*, const rns8_plan*, const rns8_matrix*, const rns8_matrix*,
                                      rns8_matrix*, rns8_workspace*, rns8_result_cache*, const rns8_dirty_region*,
                                      uint32_t) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_gemm_finite_u8_incremental(rns8_context*, const rns8_plan*, uint16_t, const rns8_matrix*,
                                            const rns8_matrix*, rns8_matrix*, rns8_workspace*, rns8_result_cache*,
                                            const rns8_dirty_region*, uint32_t) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_gemm_rns_prepacked_b(rns8_context*, const rns8_plan*, const rns8_matrix*, const rns8_prepack_cache*,
                                      rns8_matrix*, rns8_workspace*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_ozaki_decompose_i64(rns8_context*, const int64_t*, int64_t, int64_t, int64_t, int8_t**, int64_t*,
                                     int*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_strassen_gemm_research(rns8_context*, const rns8_plan*, const rns8_matrix*, const rns8_matrix*,
                                        rns8_matrix*, rns8_workspace*, int, double*) {
  RNS8_UNSUPPORTED;
}
rns8_status rns8_freivalds_verify(rns8_context*, const rns8_matrix*, const rns8_matrix*, const rns8_matrix*, uint64_t,
                                  int, double*) {
  RNS8_UNSUPPORTED;
}

}  // extern "C"
