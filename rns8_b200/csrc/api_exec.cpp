// Pack, plane GEMM, export and one-shot entry points of the rns8 C ABI on the
// sm_100a kernels.
//
// Reference behaviour followed here:
//   src/core/api_pack.cpp:31-305      argument checks, same-source-version elision,
//                                     exact-wide input proofs before packing
//   src/core/api_gemm.cpp:1-345,838-1143,1267-1450
//                                     operand validation, exact-wide admission,
//                                     grouped execution, finite GEMM
//   src/core/api_export.cpp:1-803     export validation; a RANGE_ERROR leaves dst untouched
//   src/core/api_oneshot.cpp:61-677   one-shot contracts and orchestration
// Host buffers are copied with cudaMemcpy2DAsync so caller leading dimensions
// never reach the kernels, and every call ends with a stream synchronisation.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <future>
#include <limits>
#include <thread>
#include <utility>
#include <vector>

#include "api_internal.hpp"

namespace rns8host {
namespace {

rns8_status sync(rns8_context& ctx) { return cuda_status(cudaStreamSynchronize(ctx.stream)); }

uint64_t combine_source_versions(uint64_t a, uint64_t b) {
  if (a == 0 || b == 0) return 0;
  uint64_t h = 1469598103934665603ull;
  h = (h ^ a) * 1099511628211ull;
  h = (h ^ b) * 1099511628211ull;
  return h == 0 ? 1 : h;
}

// Device status word: zero, run, read back.
rns8_status read_status(rns8_context& ctx, uint32_t* out) {
  const cudaError_t e = cudaMemcpyAsync(out, ctx.dev_status, sizeof(uint32_t), cudaMemcpyDeviceToHost, ctx.stream);
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  return sync(ctx);
}
rns8_status clear_status(rns8_context& ctx) {
  return cuda_status(cudaMemsetAsync(ctx.dev_status, 0, 4 * sizeof(uint32_t), ctx.stream));
}
rns8_status status_from_device(uint32_t word) {
  if (word == 0) return RNS8_SUCCESS;
  if (word & rns8cuda::kDevWaitTimeout) return RNS8_BACKEND_FAILURE;
  return RNS8_RANGE_ERROR;
}

rns8_status copy_in_2d(rns8_context& ctx, void* dst, const void* src, int64_t rows, int64_t cols, int64_t ld,
                       size_t elem) {
  return cuda_status(cudaMemcpy2DAsync(dst, static_cast<size_t>(cols) * elem, src, static_cast<size_t>(ld) * elem,
                                       static_cast<size_t>(cols) * elem, static_cast<size_t>(rows),
                                       cudaMemcpyHostToDevice, ctx.stream));
}
rns8_status copy_out_2d(rns8_context& ctx, void* dst, int64_t ld, const void* src, int64_t rows, int64_t cols,
                        size_t elem) {
  return cuda_status(cudaMemcpy2DAsync(dst, static_cast<size_t>(ld) * elem, src, static_cast<size_t>(cols) * elem,
                                       static_cast<size_t>(cols) * elem, static_cast<size_t>(rows),
                                       cudaMemcpyDeviceToHost, ctx.stream));
}

bool plan_context_ok(const rns8_context& ctx, const rns8_plan& plan) {
  return plan.backend == ctx.backend && plan.device_id == ctx.device_id;
}

// validate_plan_context_workspace (api_workspace_contracts_resources.inc:222-247).
rns8_status validate_workspace(const rns8_context& ctx, const rns8_plan& plan, const rns8_workspace& ws) {
  if (!plan_context_ok(ctx, plan) || ws.backend != plan.backend) return RNS8_INVALID_ARGUMENT;
  if (ws.semantics != plan.desc.semantics || ws.bound_kind != plan.desc.bound_kind) return RNS8_INVALID_ARGUMENT;
  if (ws.m != plan.desc.m || ws.n != plan.desc.n || ws.k != plan.desc.k || ws.prefix != plan.prefix)
    return RNS8_WORKSPACE_TOO_SMALL;
  if (ws.plan_fingerprint != plan.fingerprint || ws.device_id != ctx.device_id) return RNS8_INVALID_ARGUMENT;
  return RNS8_SUCCESS;
}

// matrix_descriptor_matches (api_matrix_currentness_storage.inc:1-23).
// Wrap64 and per-tile matrices also carry the plan's tile dimensions.
bool descriptor_matches(const rns8_matrix& mtx, rns8_semantics s, rns8_bound_kind bk, int64_t rows, int64_t cols,
                        uint32_t prefix, const rns8_plan& plan) {
  if (mtx.desc.semantics != s || mtx.desc.bound_kind != bk || mtx.desc.rows != rows || mtx.desc.cols != cols ||
      mtx.desc.logical_layout != RNS8_LAYOUT_ROW_MAJOR || mtx.desc.logical_ld < mtx.desc.cols ||
      mtx.desc.flags != 0 || mtx.prefix < prefix || mtx.desc.max_prefix < prefix)
    return false;
  if (prefix == 0 && (mtx.prefix != 0 || mtx.desc.max_prefix != 0)) return false;
  if ((s == RNS8_WRAP_U64_MOD_2_64 || bk == RNS8_BOUND_PER_TILE_MAX_ABS || bk == RNS8_BOUND_PER_TILE_MAX_UNSIGNED) &&
      (mtx.desc.tile_m != plan.desc.tile_m || mtx.desc.tile_n != plan.desc.tile_n))
    return false;
  return mtx.residues != nullptr;
}

rns8_status validate_rns_operands(const rns8_context& ctx, const rns8_plan& plan, const rns8_matrix& A,
                                  const rns8_matrix& B, const rns8_matrix& C) {
  if (!uses_rns_storage(plan.desc.semantics) || plan.prefix == 0) return RNS8_INVALID_ARGUMENT;
  if (A.device_id != ctx.device_id || B.device_id != ctx.device_id || C.device_id != ctx.device_id)
    return RNS8_INVALID_ARGUMENT;
  const rns8_bound_kind bk = storage_bound_kind(plan);
  const auto& d = plan.desc;
  const uint32_t sp = plan.storage_prefix();
  if (!descriptor_matches(A, d.semantics, bk, d.m, d.k, sp, plan) ||
      !descriptor_matches(B, d.semantics, bk, d.k, d.n, sp, plan) || !descriptor_matches(C, d.semantics, bk, d.m, d.n, sp, plan))
    return RNS8_INVALID_ARGUMENT;
  if (!A.device_current || !B.device_current) return RNS8_INVALID_ARGUMENT;
  if (exact_wide(d.semantics) && (&A == &C || &B == &C)) return RNS8_INVALID_ARGUMENT;
  return RNS8_SUCCESS;
}

rns8_status validate_finite_operands(const rns8_context& ctx, const rns8_plan& plan, uint16_t modulus,
                                     const rns8_matrix& A, const rns8_matrix& B, const rns8_matrix& C) {
  if (!uses_finite_storage(plan.desc.semantics) ||
      !valid_finite_modulus_for_semantics(plan.desc.semantics, modulus) || plan.desc.finite_modulus != modulus)
    return RNS8_INVALID_ARGUMENT;
  if (A.device_id != ctx.device_id || B.device_id != ctx.device_id || C.device_id != ctx.device_id)
    return RNS8_INVALID_ARGUMENT;
  const auto& d = plan.desc;
  if (!descriptor_matches(A, d.semantics, RNS8_BOUND_NONE, d.m, d.k, 0, plan) ||
      !descriptor_matches(B, d.semantics, RNS8_BOUND_NONE, d.k, d.n, 0, plan) ||
      !descriptor_matches(C, d.semantics, RNS8_BOUND_NONE, d.m, d.n, 0, plan))
    return RNS8_INVALID_ARGUMENT;
  if (!A.device_current || !B.device_current || A.finite_modulus != modulus || B.finite_modulus != modulus)
    return RNS8_INVALID_ARGUMENT;
  return RNS8_SUCCESS;
}

rns8_status run_plane_gemm(rns8_context& ctx, const rns8cuda::PlaneGemmProblem& prob, rns8_workspace* ws) {
  const uint64_t need = rns8cuda::plane_gemm_scratch_bytes(prob, ctx.sm_count);
  void* scratch = nullptr;
  if (need) {
    if (!ws) return RNS8_INVALID_ARGUMENT;
    const rns8_status s = ws->scratch.ensure(ctx.device_id, need);
    if (s != RNS8_SUCCESS) return s;
    scratch = ws->scratch.ptr;
  }
  rns8_status s = clear_status(ctx);
  if (s != RNS8_SUCCESS) return s;
  s = cuda_status(rns8cuda::plane_gemm(prob, rns8cuda::GemmPath::Auto, ctx.sm_count, scratch, need, ctx.dev_status,
                                       ctx.stream));
  if (s != RNS8_SUCCESS) return s;
  uint32_t word = 0;
  s = read_status(ctx, &word);
  if (s != RNS8_SUCCESS) return s;
  return word == 0 ? RNS8_SUCCESS : RNS8_BACKEND_FAILURE;
}

// Per-tile schedule in kernel form: the selected prefix of every schedule
// tile, | 0x80 for proven-zero outputs. A per-tile plan whose schedule
// collapsed runs every tile at the plan prefix.
struct KernelSchedule {
  std::vector<uint8_t> sel;
  rns8cuda::PlaneSchedule view{};
};
KernelSchedule kernel_schedule(const rns8_plan& plan) {
  KernelSchedule ks;
  ks.sel.assign(static_cast<size_t>(plan.tile_count), static_cast<uint8_t>(plan.prefix));
  for (size_t t = 0; t < plan.tile_schedule.size() && t < ks.sel.size(); ++t) {
    const auto& e = plan.tile_schedule[t];
    ks.sel[t] = static_cast<uint8_t>(e.selected_prefix | ((e.flags & RNS8_TILE_SCHEDULE_ZERO_OUTPUT) ? 0x80u : 0u));
  }
  ks.view.tile_m = plan.desc.tile_m;
  ks.view.tile_n = plan.desc.tile_n;
  ks.view.tile_rows = plan.tile_rows;
  ks.view.tile_cols = plan.tile_cols;
  ks.view.tile_sel = ks.sel.data();
  return ks;
}

// rns8_gemm_rns under a tile schedule (reference cpu_reference.cpp:221-260).
rns8_status run_plane_gemm_scheduled(rns8_context& ctx, const rns8_plan& plan,
                                     const rns8cuda::PlaneGemmProblem& prob, rns8_workspace* ws) {
  const KernelSchedule ks = kernel_schedule(plan);
  const uint64_t need = rns8cuda::plane_gemm_scheduled_scratch_bytes(prob, ks.view, ctx.sm_count);
  if (!ws) return RNS8_INVALID_ARGUMENT;
  rns8_status s = ws->scratch.ensure(ctx.device_id, need);
  if (s != RNS8_SUCCESS) return s;
  if ((s = clear_status(ctx)) != RNS8_SUCCESS) return s;
  s = cuda_status(rns8cuda::plane_gemm_scheduled(prob, ks.view, ctx.sm_count, ws->scratch.ptr, need, ctx.dev_status,
                                                 ctx.stream));
  if (s != RNS8_SUCCESS) return s;
  uint32_t word = 0;
  if ((s = read_status(ctx, &word)) != RNS8_SUCCESS) return s;
  return word == 0 ? RNS8_SUCCESS : RNS8_BACKEND_FAILURE;
}

rns8cuda::PlaneGemmProblem rns_problem(const rns8_plan& plan, uint32_t planes, const rns8cuda::PlaneGemmTask* tasks,
                                       uint32_t count, uint16_t finite_modulus) {
  rns8cuda::PlaneGemmProblem prob{};
  prob.m = plan.desc.m;
  prob.n = plan.desc.n;
  prob.k = plan.desc.k;
  prob.planes = planes;
  for (uint32_t p = 0; p < planes; ++p) prob.moduli[p] = finite_modulus ? finite_modulus : kLadder[p];
  prob.task_count = count;
  prob.tasks = tasks;
  return prob;
}

// ---- WRAP_U64_MOD_2_64 (byte-limb storage) ------------------------------------
// wrap_matrix_storage_matches (api_gemm.cpp:190-193): eight byte planes of a
// rows x cols row-major wrap64 matrix, no CRT prefix.
bool wrap_storage_ok(const rns8_matrix& m, int64_t rows, int64_t cols) {
  return m.desc.semantics == RNS8_WRAP_U64_MOD_2_64 && m.desc.bound_kind == RNS8_BOUND_NONE && m.desc.rows == rows &&
         m.desc.cols == cols && m.desc.logical_layout == RNS8_LAYOUT_ROW_MAJOR && m.prefix == 0 &&
         m.desc.max_prefix == 0 && m.residues != nullptr &&
         m.residue_bytes == static_cast<uint64_t>(rows) * static_cast<uint64_t>(cols) * 8;
}

// rns8_pack_u64 on a wrap64 matrix (api_pack.cpp:178-208): upload, then the
// byte planes; a repeated non-zero source version skips the work.
rns8_status pack_wrap(rns8_context* ctx, rns8_matrix* matrix, const uint64_t* src, int64_t ld,
                      uint64_t source_version) {
  if (ctx->backend != matrix->backend || matrix->device_id != ctx->device_id ||
      !wrap_storage_ok(*matrix, matrix->desc.rows, matrix->desc.cols))
    return RNS8_INVALID_ARGUMENT;
  if (source_version != 0 && matrix->source_version == source_version && matrix->device_current)
    return RNS8_SUCCESS;
  DeviceScope dev(ctx->device_id);
  if (!dev.ok) return RNS8_BACKEND_FAILURE;
  const int64_t rows = matrix->desc.rows, cols = matrix->desc.cols;
  rns8_status st = matrix->upload.ensure(ctx->device_id, static_cast<uint64_t>(rows) * cols * sizeof(uint64_t));
  if (st != RNS8_SUCCESS) return st;
  if ((st = copy_in_2d(*ctx, matrix->upload.ptr, src, rows, cols, ld, sizeof(uint64_t))) != RNS8_SUCCESS) return st;
  matrix->device_current = false;
  if (rns8cuda::wrap_pack_u64(static_cast<const uint64_t*>(matrix->upload.ptr), rows, cols, cols,
                              reinterpret_cast<uint8_t*>(matrix->residues), ctx->stream) != cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  if ((st = sync(*ctx)) != RNS8_SUCCESS) return st;
  matrix->device_current = true;
  matrix->source_version = source_version;
  return RNS8_SUCCESS;
}

// validate_wrap_gemm_operands (api_gemm.cpp:158-198).
rns8_status validate_wrap_operands(const rns8_context& ctx, const rns8_plan& plan, const rns8_matrix& A,
                                   const rns8_matrix& B, const rns8_matrix& C) {
  if (plan.desc.semantics != RNS8_WRAP_U64_MOD_2_64 || plan.prefix != 0) return RNS8_INVALID_ARGUMENT;
  if (A.backend != plan.backend || B.backend != plan.backend || C.backend != plan.backend) return RNS8_INVALID_ARGUMENT;
  if (A.device_id != ctx.device_id || B.device_id != ctx.device_id || C.device_id != ctx.device_id)
    return RNS8_INVALID_ARGUMENT;
  const auto& d = plan.desc;
  if (!wrap_storage_ok(A, d.m, d.k) || !wrap_storage_ok(B, d.k, d.n) || !wrap_storage_ok(C, d.m, d.n))
    return RNS8_INVALID_ARGUMENT;
  for (const rns8_matrix* mtx : {&A, &B, &C})  // wrap64 matrices carry the plan's tile dimensions
    if (mtx->desc.tile_m != d.tile_m || mtx->desc.tile_n != d.tile_n) return RNS8_INVALID_ARGUMENT;
  if (!A.device_current || !B.device_current) return RNS8_INVALID_ARGUMENT;
  return RNS8_SUCCESS;
}

// C = A x B mod 2^64 into the uint64 buffer c (m x n), then c's byte planes
// into `planes` when given. Reads the status word (a wait that ran out is a
// backend failure).
rns8_status run_wrap_gemm(rns8_context& ctx, const uint8_t* a, const uint8_t* b, uint64_t* c, int64_t m, int64_t n,
                          int64_t k, uint8_t* planes) {
  rns8_status st = clear_status(ctx);
  if (st != RNS8_SUCCESS) return st;
  if (rns8cuda::wrap_gemm(a, b, c, m, n, k, rns8cuda::GemmPath::Auto, ctx.sm_count, ctx.dev_status, ctx.stream) !=
      cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  if (planes && rns8cuda::wrap_pack_u64(c, m, n, n, planes, ctx.stream) != cudaSuccess) return RNS8_BACKEND_FAILURE;
  uint32_t word = 0;
  if ((st = read_status(ctx, &word)) != RNS8_SUCCESS) return st;
  return status_from_device(word);
}

template <typename T>
rns8_status pack_native(rns8_context* ctx, rns8_matrix* matrix, const T* src, int64_t ld, uint64_t source_version) {
  constexpr bool kSigned = std::numeric_limits<T>::is_signed;
  if (!ctx || !matrix || !src || !valid_matrix_access(matrix->desc.rows, matrix->desc.cols, ld))
    return RNS8_INVALID_ARGUMENT;
  const rns8_semantics s = matrix->desc.semantics;
  if (kSigned ? (s != RNS8_BOUNDED_I64 && s != RNS8_EXACT_WIDE_SIGNED)
              : (s != RNS8_BOUNDED_U64 && s != RNS8_EXACT_WIDE_UNSIGNED && s != RNS8_WRAP_U64_MOD_2_64))
    return RNS8_INVALID_ARGUMENT;
  if constexpr (!kSigned) {
    if (s == RNS8_WRAP_U64_MOD_2_64) return pack_wrap(ctx, matrix, src, ld, source_version);
  }
  if (ctx->backend != matrix->backend || matrix->device_id != ctx->device_id || matrix->prefix == 0)
    return RNS8_INVALID_ARGUMENT;
  const bool same_source = source_version != 0 && matrix->source_version == source_version && matrix->device_current;
  if (same_source) {
    if (exact_wide(s) && !exact_range_fits(s, matrix->exact_max_magnitude, modulus_product(matrix->prefix)))
      return RNS8_RANGE_ERROR;
    return RNS8_SUCCESS;
  }
  DeviceScope dev(ctx->device_id);
  if (!dev.ok) return RNS8_BACKEND_FAILURE;
  const int64_t rows = matrix->desc.rows, cols = matrix->desc.cols;
  rns8_status st = matrix->upload.ensure(ctx->device_id, static_cast<uint64_t>(rows) * cols * sizeof(T));
  if (st != RNS8_SUCCESS) return st;
  st = copy_in_2d(*ctx, matrix->upload.ptr, src, rows, cols, ld, sizeof(T));
  if (st != RNS8_SUCCESS) return st;
  // Exact-wide admission (exact_range.hpp:51-77): the row and column
  // summaries of the uploaded values, before the residues are touched, so a
  // RANGE_ERROR leaves the matrix as it was.
  i256 exact_bound;
  ExactRanges ranges;
  if (exact_wide(s)) {
    st = device_exact_ranges(*ctx, matrix->upload.ptr, kSigned, rows, cols, ranges, exact_bound);
    if (st != RNS8_SUCCESS) return st;
    if (!exact_range_fits(s, exact_bound, modulus_product(matrix->prefix))) return RNS8_RANGE_ERROR;
  }
  matrix->device_current = false;
  const cudaError_t e =
      kSigned ? rns8cuda::pack_i64(reinterpret_cast<const int64_t*>(matrix->upload.ptr), rows, cols, cols,
                                   matrix->prefix, matrix->residues, ctx->stream)
              : rns8cuda::pack_u64(reinterpret_cast<const uint64_t*>(matrix->upload.ptr), rows, cols, cols,
                                   matrix->prefix, matrix->residues, ctx->stream);
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  st = sync(*ctx);
  if (st != RNS8_SUCCESS) return st;
  matrix->device_current = true;
  if (exact_wide(s)) {
    matrix->exact_max_magnitude = exact_bound;
    matrix->exact_axes.rows.swap(ranges.rows);
    matrix->exact_axes.cols.swap(ranges.cols);
    matrix->exact_deferred = DeferredExactRange{};
    matrix->exact_range_prefix = matrix->prefix;
  }
  matrix->source_version = source_version;
  return RNS8_SUCCESS;
}

// validate_export_matrix (api_export.cpp:5-52) for RNS outputs.
rns8_status validate_rns_export(const rns8_context& ctx, const rns8_plan& plan, const rns8_matrix& C,
                                rns8_semantics semantics) {
  if (!plan_context_ok(ctx, plan) || plan.desc.semantics != semantics) return RNS8_INVALID_ARGUMENT;
  if (C.device_id != ctx.device_id || C.backend != plan.backend) return RNS8_INVALID_ARGUMENT;
  if (!descriptor_matches(C, semantics, storage_bound_kind(plan), plan.desc.m, plan.desc.n, plan.storage_prefix(), plan))
    return RNS8_INVALID_ARGUMENT;
  if (!C.device_current) return RNS8_INVALID_ARGUMENT;
  if (exact_wide(semantics) && C.exact_range_prefix != 0 &&
      (C.exact_range_prefix < plan.prefix || !exact_range_fits(semantics, C.exact_max_magnitude, plan.modulus_product)))
    return RNS8_RANGE_ERROR;
  return RNS8_SUCCESS;
}

enum class ExportKind { I64, U64, LimbsS, LimbsU };

// Reconstruct into the matrix's staging buffer, check the status word, and
// only then copy to the caller's buffer (dst untouched on RANGE_ERROR).
rns8_status export_rns(rns8_context& ctx, const rns8_plan& plan, const rns8_matrix& Cc, void* dst, int64_t ld,
                       ExportKind kind, uint32_t limbs) {
  rns8_matrix& C = const_cast<rns8_matrix&>(Cc);  // export staging is a documented mutable cache
  DeviceScope dev(ctx.device_id);
  if (!dev.ok) return RNS8_BACKEND_FAILURE;
  const int64_t m = plan.desc.m, n = plan.desc.n;
  const uint64_t per_cell = (kind == ExportKind::LimbsS || kind == ExportKind::LimbsU) ? 8ull * limbs : 8ull;
  rns8_status st = C.staging.ensure(ctx.device_id, static_cast<uint64_t>(m) * n * per_cell);
  if (st != RNS8_SUCCESS) return st;
  st = clear_status(ctx);
  if (st != RNS8_SUCCESS) return st;
  cudaError_t e = cudaSuccess;
  if (!plan.tile_bounds.empty() && (kind == ExportKind::I64 || kind == ExportKind::U64)) {
    // Per-tile plans: each tile's selected prefix and bound (api_export.cpp:365-391).
    const KernelSchedule ks = kernel_schedule(plan);
    const uint64_t jb = rns8cuda::export_scheduled_scratch_bytes(ks.view);
    if ((st = C.export_jobs.ensure(ctx.device_id, jb)) != RNS8_SUCCESS) return st;
    e = rns8cuda::export_scheduled(C.residues, m, n, kind == ExportKind::I64, ks.view, plan.tile_bounds.data(),
                                   C.staging.ptr, ctx.dev_status, C.export_jobs.ptr, jb, ctx.stream);
  } else {
  switch (kind) {
    case ExportKind::I64:
      e = rns8cuda::export_i64(C.residues, m, n, plan.prefix, plan.desc.bound, static_cast<int64_t*>(C.staging.ptr), n,
                               ctx.dev_status, ctx.stream);
      break;
    case ExportKind::U64:
      e = rns8cuda::export_u64(C.residues, m, n, plan.prefix, plan.desc.bound, static_cast<uint64_t*>(C.staging.ptr),
                               n, ctx.dev_status, ctx.stream);
      break;
    case ExportKind::LimbsS:
    case ExportKind::LimbsU:
      e = rns8cuda::export_limbs(C.residues, m, n, plan.prefix, kind == ExportKind::LimbsS, limbs,
                                 static_cast<uint64_t*>(C.staging.ptr), n, ctx.dev_status, ctx.stream);
      break;
  }
  }
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  uint32_t word = 0;
  st = read_status(ctx, &word);
  if (st != RNS8_SUCCESS) return st;
  st = status_from_device(word);
  if (st != RNS8_SUCCESS) return st;
  st = copy_out_2d(ctx, dst, ld * static_cast<int64_t>(per_cell / 8), C.staging.ptr, m, n * static_cast<int64_t>(per_cell / 8),
                   sizeof(uint64_t));
  if (st != RNS8_SUCCESS) return st;
  return sync(ctx);
}

bool valid_limb_export_access(int64_t rows, int64_t cols, int64_t ld, uint32_t limbs) {
  if (!valid_matrix_access(rows, cols, ld) || limbs == 0 || limbs > 32) return false;
  const int64_t max = std::numeric_limits<int64_t>::max();
  if (ld > max / static_cast<int64_t>(limbs)) return false;
  return rows <= max / (ld * static_cast<int64_t>(limbs));
}

// ---- one-shot device arena -------------------------------------------------
struct Carve {
  uint8_t* base;
  uint64_t off = 0;
  void* take(uint64_t bytes) {
    void* p = base + off;
    off += (bytes + 255) & ~uint64_t(255);
    return p;
  }
};
uint64_t round256(uint64_t b) { return (b + 255) & ~uint64_t(255); }

// validate_typed_oneshot_contract (api_oneshot.cpp:440-466).
rns8_status validate_typed_oneshot(const rns8_gemm_desc& d, rns8_semantics expected, int64_t lda, int64_t ldb,
                                   int64_t ldc) {
  if (!valid_abi(d.struct_size, d.abi_version, sizeof(d)) || d.semantics != expected) return RNS8_INVALID_ARGUMENT;
  const uint32_t prefix = d.max_prefix == 0 ? default_prefix_for_semantics(d.semantics) : d.max_prefix;
  const rns8_status v = validate_gemm_desc(d, prefix);
  if (v != RNS8_SUCCESS) return v;
  if (!valid_matrix_access(d.m, d.k, lda) || !valid_matrix_access(d.k, d.n, ldb) || !valid_matrix_access(d.m, d.n, ldc))
    return RNS8_INVALID_ARGUMENT;
  if (!backend_request_ok(d.requested_backend)) return RNS8_UNSUPPORTED_BACKEND;
  return RNS8_SUCCESS;
}

// One-shot with the upload overlapped with compute: B, then A
// in row slabs, go up on the context's copy stream, each slab followed by an
// event; the compute stream packs B, then for every slab waits for its event
// and runs pack, plane GEMM and export into device staging. Copies and compute
// are enqueued interleaved, so pageable host memory (whose copies return only
// when done) overlaps too. The result goes down only after every slab passed
// the range check, so a RANGE_ERROR leaves C untouched.
// Processes on this host that run one-shots at the same time, and so share
// its memory bandwidth: RNS8_CUDA_HOST_RANKS when set, else the launcher's
// local world size (LOCAL_WORLD_SIZE from torchrun,
// OMPI_COMM_WORLD_LOCAL_SIZE from Open MPI), else 1. The count of GPUs this
// process can see says nothing about it: ranks started with one visible GPU
// each still share the host.
int host_ranks() {
  for (const char* name : {"RNS8_CUDA_HOST_RANKS", "LOCAL_WORLD_SIZE", "OMPI_COMM_WORLD_LOCAL_SIZE"}) {
    const char* v = std::getenv(name);
    if (!v || !*v) continue;
    char* end = nullptr;
    const long n = std::strtol(v, &end, 10);
    if (end && *end == '\0' && n >= 1 && n <= 4096) return static_cast<int>(n);
  }
  return 1;
}

// Largest |x| of a row-major host matrix (x itself for uint64), over up to
// 16 host threads, the host's cores divided among `host_ranks` processes; the
// scan gives up (returns ~0) once *stop is set.
template <typename T>
uint64_t host_max_magnitude(const T* src, int64_t rows, int64_t cols, int64_t ld, int host_ranks,
                            const std::atomic<bool>* stop) {
  auto scan = [=](int64_t r0, int64_t r1) {
    uint64_t mx = 0;
    for (int64_t r = r0; r < r1; ++r) {
      if (stop->load(std::memory_order_relaxed)) return ~uint64_t{0};
      const T* row = src + r * ld;
      for (int64_t c = 0; c < cols; ++c) {
        uint64_t v;
        if constexpr (std::numeric_limits<T>::is_signed)
          v = row[c] < 0 ? uint64_t{0} - static_cast<uint64_t>(row[c]) : static_cast<uint64_t>(row[c]);
        else
          v = static_cast<uint64_t>(row[c]);
        mx = v > mx ? v : mx;
      }
    }
    return mx;
  };
  const int64_t hw = std::max<int64_t>(1, std::thread::hardware_concurrency() / std::max(1, host_ranks));
  const int64_t parts = std::min<int64_t>({std::max<int64_t>(hw, 2), 16, rows});
  std::vector<std::future<uint64_t>> futures;
  const int64_t per = (rows + parts - 1) / parts;
  for (int64_t r0 = per; r0 < rows; r0 += per)
    futures.push_back(std::async(std::launch::async, scan, r0, std::min(rows, r0 + per)));
  uint64_t mx = scan(0, std::min(rows, per));
  for (auto& f : futures) mx = std::max(mx, f.get());
  return mx;
}

// True when no cell of A x B can exceed the bound: |C_ij| <= K max|A| max|B|.
bool bound_proven(uint64_t max_a, uint64_t max_b, int64_t k, uint64_t bound) {
  const unsigned __int128 prod = static_cast<unsigned __int128>(max_a) * max_b;
  return prod <= static_cast<unsigned __int128>(bound / static_cast<uint64_t>(k));
}

template <typename T>
rns8_status bounded_oneshot_pipelined(rns8_context* ctx, const rns8_plan& plan, const T* A, int64_t lda, const T* B,
                                      int64_t ldb, T* C, int64_t ldc, int slabs) {
  constexpr bool kSigned = std::numeric_limits<T>::is_signed;
  const int64_t m = plan.desc.m, n = plan.desc.n, k = plan.desc.k;
  const uint32_t P = plan.prefix;
  const int64_t rows = (m + slabs - 1) / slabs;
  const int64_t slab_rows = (rows + 127) / 128 * 128;  // whole 128-row tiles per slab
  int8_t* const fake = reinterpret_cast<int8_t*>(256);
  rns8cuda::PlaneGemmTask task{fake, fake, fake};
  rns8cuda::PlaneGemmProblem prob = rns_problem(plan, P, &task, 1, 0);
  // Split-K scratch of the largest slab and of the last, shorter one (fewer
  // tiles can mean more K splits).
  const int64_t last_rows = m - (m - 1) / slab_rows * slab_rows;
  prob.m = last_rows;
  const uint64_t scratch_last = rns8cuda::plane_gemm_scratch_bytes(prob, ctx->sm_count);
  prob.m = std::min<int64_t>(slab_rows, m);
  const uint64_t scratch = std::max(rns8cuda::plane_gemm_scratch_bytes(prob, ctx->sm_count), scratch_last);
  const uint64_t a_nat = static_cast<uint64_t>(m) * k * sizeof(T), b_nat = static_cast<uint64_t>(k) * n * sizeof(T);
  const uint64_t a_res = static_cast<uint64_t>(P) * prob.m * k, b_res = static_cast<uint64_t>(P) * k * n;
  const uint64_t c_res = static_cast<uint64_t>(P) * prob.m * n, c_nat = static_cast<uint64_t>(m) * n * sizeof(T);
  const uint64_t total = round256(a_nat) + round256(b_nat) + round256(a_res) + round256(b_res) + round256(c_res) +
                         round256(c_nat) + round256(scratch) + 256;
  std::unique_lock<std::mutex> lock(ctx->oneshot_mutex, std::try_to_lock);
  DevBuf local;
  DevBuf& arena = lock.owns_lock() ? ctx->oneshot_arena : local;
  rns8_status st = arena.ensure(ctx->device_id, total);
  if (st != RNS8_SUCCESS) return st;
  Carve cv{static_cast<uint8_t*>(arena.ptr)};
  T* dA = static_cast<T*>(cv.take(a_nat));
  T* dB = static_cast<T*>(cv.take(b_nat));
  int8_t* rA = static_cast<int8_t*>(cv.take(a_res));
  int8_t* rB = static_cast<int8_t*>(cv.take(b_res));
  int8_t* rC = static_cast<int8_t*>(cv.take(c_res));
  T* dC = static_cast<T*>(cv.take(c_nat));
  void* dS = cv.take(scratch);
  auto* d_max_b = static_cast<uint64_t*>(cv.take(sizeof(uint64_t)));
  auto pack = [&](const T* src, int64_t r, int64_t c, int8_t* planes) {
    return kSigned ? rns8cuda::pack_i64(reinterpret_cast<const int64_t*>(src), r, c, c, P, planes, ctx->stream)
                   : rns8cuda::pack_u64(reinterpret_cast<const uint64_t*>(src), r, c, c, P, planes, ctx->stream);
  };
  // While the copies and kernels run, check whether the inputs alone prove
  // the bound (max|A| on host threads, max|B| on the device once B is in). If
  // they do, no cell can be a RANGE_ERROR, so each slab of C goes back to the
  // host as soon as it is exported, overlapping the uploads still in flight
  // (C stays untouched only on a RANGE_ERROR, which is then impossible);
  // otherwise C is copied after the status check. When more than four
  // processes on this host run one-shots at once, this is skipped and the
  // scan never starts: host memory is then the shared limit and the scan's
  // extra reads of A cost more than the overlap gains (8 ranks: 100.5 ms per
  // rank step against 90.4 ms; 2 ranks: 25.8 ms against 37.7 ms).
  const int ranks = host_ranks();
  const bool try_early = ranks <= 4;
  std::atomic<bool> stop_scan{!try_early};
  std::future<uint64_t> max_a;
  if (try_early)
    max_a = std::async(std::launch::async, [&stop_scan, A, m, k, lda, ranks] {
      return host_max_magnitude(A, m, k, lda, ranks, &stop_scan);
    });
  std::vector<cudaEvent_t> events(2 * static_cast<size_t>(slabs) + 1, nullptr);
  int last_slab = -1;  // the last slab whose export was issued
  auto destroy = [&] {
    for (cudaEvent_t& e : events)
      if (e) cudaEventDestroy(e);
  };
  for (cudaEvent_t& e : events)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      stop_scan.store(true);  // the scan's future joins on return
      destroy();
      return RNS8_BACKEND_FAILURE;
    }
  auto upload = [&](void* dst, const T* src, int64_t r, int64_t c, int64_t ld, cudaEvent_t done) {
    return cudaMemcpy2DAsync(dst, static_cast<size_t>(c) * sizeof(T), src, static_cast<size_t>(ld) * sizeof(T),
                             static_cast<size_t>(c) * sizeof(T), static_cast<size_t>(r), cudaMemcpyHostToDevice,
                             ctx->copy_stream) == cudaSuccess &&
           cudaEventRecord(done, ctx->copy_stream) == cudaSuccess;
  };
  bool ok = clear_status(*ctx) == RNS8_SUCCESS && upload(dB, B, k, n, ldb, events[0]) &&
            cudaStreamWaitEvent(ctx->stream, events[0], 0) == cudaSuccess && pack(dB, k, n, rB) == cudaSuccess;
  for (int i = 0; ok && i < slabs; ++i) {
    const int64_t r0 = i * slab_rows;
    if (r0 >= m) break;
    const int64_t r = std::min<int64_t>(slab_rows, m - r0);
    ok = upload(dA + r0 * k, A + r0 * lda, r, k, lda, events[i + 1]) &&
         cudaStreamWaitEvent(ctx->stream, events[i + 1], 0) == cudaSuccess &&
         pack(dA + r0 * k, r, k, rA) == cudaSuccess;
    if (!ok) break;
    task = {rA, rB, rC};
    prob.m = r;
    ok = rns8cuda::plane_gemm(prob, rns8cuda::GemmPath::Auto, ctx->sm_count, dS, scratch, ctx->dev_status,
                              ctx->stream) == cudaSuccess;
    if (ok)
      ok = (kSigned ? rns8cuda::export_i64(rC, r, n, P, plan.desc.bound, reinterpret_cast<int64_t*>(dC) + r0 * n, n,
                                           ctx->dev_status, ctx->stream)
                    : rns8cuda::export_u64(rC, r, n, P, plan.desc.bound, reinterpret_cast<uint64_t*>(dC) + r0 * n, n,
                                           ctx->dev_status, ctx->stream)) == cudaSuccess &&
           cudaEventRecord(events[slabs + 1 + i], ctx->stream) == cudaSuccess;
    if (ok) last_slab = i;
  }
  uint64_t max_b = ~uint64_t{0};
  bool early_ok = ok && try_early && cudaStreamWaitEvent(ctx->out_stream, events[0], 0) == cudaSuccess &&
                  rns8cuda::max_magnitude(dB, k * n, kSigned, d_max_b, ctx->sm_count, ctx->out_stream) ==
                      cudaSuccess &&
                  cudaMemcpyAsync(&max_b, d_max_b, sizeof(uint64_t), cudaMemcpyDeviceToHost, ctx->out_stream) ==
                      cudaSuccess &&
                  cudaStreamSynchronize(ctx->out_stream) == cudaSuccess;
  // The proof is only worth waiting for while slabs are still being
  // computed: once the last slab is exported, the checked path is as fast.
  if (!try_early) {
    // no scan was started
  } else if (!early_ok || last_slab < 0) {
    stop_scan.store(true);
  } else {
    const cudaEvent_t last_export = events[static_cast<size_t>(slabs + 1 + last_slab)];
    while (max_a.wait_for(std::chrono::microseconds(200)) != std::future_status::ready) {
      if (cudaEventQuery(last_export) != cudaErrorNotReady) {
        stop_scan.store(true);
        break;
      }
    }
    (void)cudaGetLastError();  // a not-ready query leaves a non-sticky error behind
  }
  // C written while A is still uploading must not overlap either input.
  auto span = [](const void* p, int64_t rows, int64_t cols, int64_t ld) {
    const auto lo = reinterpret_cast<uintptr_t>(p);
    return std::make_pair(lo, lo + static_cast<uintptr_t>((rows - 1) * ld + cols) * sizeof(T));
  };
  auto overlap = [](std::pair<uintptr_t, uintptr_t> x, std::pair<uintptr_t, uintptr_t> y) {
    return x.first < y.second && y.first < x.second;
  };
  const auto c_span = span(C, m, n, ldc);
  const bool disjoint = !overlap(c_span, span(A, m, k, lda)) && !overlap(c_span, span(B, k, n, ldb));
  const bool early = try_early && early_ok && disjoint && bound_proven(max_a.get(), max_b, k, plan.desc.bound);
  if (ok && early) {
    for (int i = 0; early_ok && i < slabs; ++i) {
      const int64_t r0 = i * slab_rows;
      if (r0 >= m) break;
      const int64_t r = std::min<int64_t>(slab_rows, m - r0);
      early_ok = cudaStreamWaitEvent(ctx->out_stream, events[slabs + 1 + i], 0) == cudaSuccess &&
                 cudaMemcpy2DAsync(C + r0 * ldc, static_cast<size_t>(ldc) * sizeof(T), dC + r0 * n,
                                   static_cast<size_t>(n) * sizeof(T), static_cast<size_t>(n) * sizeof(T),
                                   static_cast<size_t>(r), cudaMemcpyDeviceToHost, ctx->out_stream) == cudaSuccess;
    }
  }
  // Every stream finishes before the events go and before any result is read.
  const bool copies_ok = cudaStreamSynchronize(ctx->copy_stream) == cudaSuccess &&
                         cudaStreamSynchronize(ctx->out_stream) == cudaSuccess;
  uint32_t word = 0;
  st = read_status(*ctx, &word);
  destroy();
  if (!ok || !copies_ok || (early && !early_ok)) return RNS8_BACKEND_FAILURE;
  if (st != RNS8_SUCCESS) return st;
  if ((st = status_from_device(word)) != RNS8_SUCCESS) return st;
  if (early) return RNS8_SUCCESS;
  if ((st = copy_out_2d(*ctx, C, ldc, dC, m, n, sizeof(T))) != RNS8_SUCCESS) return st;
  return sync(*ctx);
}

// One-shot under a per-tile bound plan: pack the storage prefix, the
// scheduled plane GEMM, the per-tile export, all in the context's arena.
template <typename T>
rns8_status bounded_oneshot_per_tile(rns8_context* ctx, const rns8_plan& plan, const T* A, int64_t lda, const T* B,
                                     int64_t ldb, T* C, int64_t ldc) {
  constexpr bool kSigned = std::numeric_limits<T>::is_signed;
  const int64_t m = plan.desc.m, n = plan.desc.n, k = plan.desc.k;
  const uint32_t P = plan.storage_prefix();
  const KernelSchedule ks = kernel_schedule(plan);
  int8_t* const fake = reinterpret_cast<int8_t*>(256);  // shape-only problem for the scratch sizes
  rns8cuda::PlaneGemmTask task{fake, fake, fake};
  rns8cuda::PlaneGemmProblem prob = rns_problem(plan, P, &task, 1, 0);
  const bool scheduled = !plan.tile_schedule.empty();
  const uint64_t gemm_scratch = scheduled ? rns8cuda::plane_gemm_scheduled_scratch_bytes(prob, ks.view, ctx->sm_count)
                                          : rns8cuda::plane_gemm_scratch_bytes(prob, ctx->sm_count);
  const uint64_t jobs = rns8cuda::export_scheduled_scratch_bytes(ks.view);
  const uint64_t a_nat = static_cast<uint64_t>(m) * k * 8, b_nat = static_cast<uint64_t>(k) * n * 8;
  const uint64_t a_res = static_cast<uint64_t>(P) * m * k, b_res = static_cast<uint64_t>(P) * k * n;
  const uint64_t c_res = static_cast<uint64_t>(P) * m * n, c_nat = static_cast<uint64_t>(m) * n * 8;
  const uint64_t total = round256(a_nat) + round256(b_nat) + round256(a_res) + round256(b_res) + round256(c_res) +
                         round256(c_nat) + round256(gemm_scratch) + round256(jobs);
  std::unique_lock<std::mutex> lock(ctx->oneshot_mutex, std::try_to_lock);
  DevBuf local;
  DevBuf& arena = lock.owns_lock() ? ctx->oneshot_arena : local;
  rns8_status st = arena.ensure(ctx->device_id, total);
  if (st != RNS8_SUCCESS) return st;
  Carve cv{static_cast<uint8_t*>(arena.ptr)};
  T* dA = static_cast<T*>(cv.take(a_nat));
  T* dB = static_cast<T*>(cv.take(b_nat));
  int8_t* rA = static_cast<int8_t*>(cv.take(a_res));
  int8_t* rB = static_cast<int8_t*>(cv.take(b_res));
  int8_t* rC = static_cast<int8_t*>(cv.take(c_res));
  void* dC = cv.take(c_nat);
  void* dS = cv.take(gemm_scratch);
  void* dJ = cv.take(jobs);
  if ((st = copy_in_2d(*ctx, dA, A, m, k, lda, sizeof(T))) != RNS8_SUCCESS) return st;
  if ((st = copy_in_2d(*ctx, dB, B, k, n, ldb, sizeof(T))) != RNS8_SUCCESS) return st;
  // A fresh C is zero in every plane, as a newly created matrix is.
  if (cudaMemsetAsync(rC, 0, c_res, ctx->stream) != cudaSuccess) return RNS8_BACKEND_FAILURE;
  cudaError_t e = kSigned ? rns8cuda::pack_i64(reinterpret_cast<const int64_t*>(dA), m, k, k, P, rA, ctx->stream)
                          : rns8cuda::pack_u64(reinterpret_cast<const uint64_t*>(dA), m, k, k, P, rA, ctx->stream);
  if (e == cudaSuccess)
    e = kSigned ? rns8cuda::pack_i64(reinterpret_cast<const int64_t*>(dB), k, n, n, P, rB, ctx->stream)
                : rns8cuda::pack_u64(reinterpret_cast<const uint64_t*>(dB), k, n, n, P, rB, ctx->stream);
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  if ((st = clear_status(*ctx)) != RNS8_SUCCESS) return st;
  task = {rA, rB, rC};
  e = scheduled ? rns8cuda::plane_gemm_scheduled(prob, ks.view, ctx->sm_count, dS, gemm_scratch, ctx->dev_status,
                                                 ctx->stream)
                : rns8cuda::plane_gemm(prob, rns8cuda::GemmPath::Auto, ctx->sm_count, dS, gemm_scratch,
                                       ctx->dev_status, ctx->stream);
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  uint32_t word = 0;
  if ((st = read_status(*ctx, &word)) != RNS8_SUCCESS) return st;
  if (word != 0) return RNS8_BACKEND_FAILURE;
  if ((st = clear_status(*ctx)) != RNS8_SUCCESS) return st;
  if (rns8cuda::export_scheduled(rC, m, n, kSigned, ks.view, plan.tile_bounds.data(), dC, ctx->dev_status, dJ, jobs,
                                 ctx->stream) != cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  if ((st = read_status(*ctx, &word)) != RNS8_SUCCESS) return st;
  if ((st = status_from_device(word)) != RNS8_SUCCESS) return st;
  if ((st = copy_out_2d(*ctx, C, ldc, dC, m, n, sizeof(T))) != RNS8_SUCCESS) return st;
  return sync(*ctx);
}

template <typename T>
rns8_status bounded_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc, const T* A, int64_t lda, const T* B,
                            int64_t ldb, T* C, int64_t ldc) {
  constexpr bool kSigned = std::numeric_limits<T>::is_signed;
  if (!ctx || !desc || !A || !B || !C) return RNS8_INVALID_ARGUMENT;
  rns8_status st = validate_typed_oneshot(*desc, kSigned ? RNS8_BOUNDED_I64 : RNS8_BOUNDED_U64, lda, ldb, ldc);
  if (st != RNS8_SUCCESS) return st;
  rns8_plan plan;
  plan.device_id = ctx->device_id;
  st = build_plan(*desc, plan);
  if (st != RNS8_SUCCESS) return st;
  DeviceScope dev(ctx->device_id);
  if (!dev.ok) return RNS8_BACKEND_FAILURE;
  if (!plan.tile_bounds.empty()) return bounded_oneshot_per_tile<T>(ctx, plan, A, lda, B, ldb, C, ldc);
  // Large calls overlap the upload with pack, GEMM and export, slab by slab.
  if (plan.desc.m >= 1024 && static_cast<uint64_t>(plan.desc.m) * plan.desc.k * 8 >= (uint64_t{64} << 20)) {
    const int slabs = static_cast<int>(std::min<int64_t>(16, plan.desc.m / 512));
    return bounded_oneshot_pipelined<T>(ctx, plan, A, lda, B, ldb, C, ldc, slabs);
  }
  const int64_t m = plan.desc.m, n = plan.desc.n, k = plan.desc.k;
  const uint32_t P = plan.prefix;
  const uint64_t a_nat = static_cast<uint64_t>(m) * k * 8, b_nat = static_cast<uint64_t>(k) * n * 8;
  const uint64_t a_res = static_cast<uint64_t>(P) * m * k, b_res = static_cast<uint64_t>(P) * k * n;
  const uint64_t c_nat = static_cast<uint64_t>(m) * n * 8;
  // Scratch size depends only on shape and alignment; the arena keeps 256-byte alignment.
  rns8cuda::PlaneGemmTask task{reinterpret_cast<const int8_t*>(256), reinterpret_cast<const int8_t*>(256), nullptr};
  rns8cuda::PlaneGemmProblem prob = rns_problem(plan, P, &task, 1, 0);
  const uint64_t scratch = rns8cuda::gemm_export_bounded_scratch_bytes(prob, ctx->sm_count);
  const uint64_t total = round256(a_nat) + round256(b_nat) + round256(a_res) + round256(b_res) + round256(c_nat) +
                         round256(scratch);
  std::unique_lock<std::mutex> lock(ctx->oneshot_mutex, std::try_to_lock);
  DevBuf local;
  DevBuf& arena = lock.owns_lock() ? ctx->oneshot_arena : local;
  st = arena.ensure(ctx->device_id, total);
  if (st != RNS8_SUCCESS) return st;
  Carve cv{static_cast<uint8_t*>(arena.ptr)};
  T* dA = static_cast<T*>(cv.take(a_nat));
  T* dB = static_cast<T*>(cv.take(b_nat));
  int8_t* rA = static_cast<int8_t*>(cv.take(a_res));
  int8_t* rB = static_cast<int8_t*>(cv.take(b_res));
  T* dC = static_cast<T*>(cv.take(c_nat));
  void* dS = cv.take(scratch);
  if ((st = copy_in_2d(*ctx, dA, A, m, k, lda, sizeof(T))) != RNS8_SUCCESS) return st;
  if ((st = copy_in_2d(*ctx, dB, B, k, n, ldb, sizeof(T))) != RNS8_SUCCESS) return st;
  cudaError_t e = kSigned ? rns8cuda::pack_i64(reinterpret_cast<const int64_t*>(dA), m, k, k, P, rA, ctx->stream)
                          : rns8cuda::pack_u64(reinterpret_cast<const uint64_t*>(dA), m, k, k, P, rA, ctx->stream);
  if (e == cudaSuccess)
    e = kSigned ? rns8cuda::pack_i64(reinterpret_cast<const int64_t*>(dB), k, n, n, P, rB, ctx->stream)
                : rns8cuda::pack_u64(reinterpret_cast<const uint64_t*>(dB), k, n, n, P, rB, ctx->stream);
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  if ((st = clear_status(*ctx)) != RNS8_SUCCESS) return st;
  // Plane GEMM into arena planes, then the bounded export.
  task = {rA, rB, nullptr};
  e = rns8cuda::gemm_export_bounded(prob, kSigned, plan.desc.bound, dC, n, ctx->sm_count, dS, scratch, ctx->dev_status,
                                    ctx->stream);
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  uint32_t word = 0;
  if ((st = read_status(*ctx, &word)) != RNS8_SUCCESS) return st;
  if ((st = status_from_device(word)) != RNS8_SUCCESS) return st;
  if ((st = copy_out_2d(*ctx, C, ldc, dC, m, n, sizeof(T))) != RNS8_SUCCESS) return st;
  return sync(*ctx);
}

// validate_finite_u8_oneshot_contract (api_oneshot.cpp:78-106).
rns8_status finite_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc, rns8_semantics expected, uint16_t modulus,
                           const uint8_t* A, int64_t lda, const uint8_t* B, int64_t ldb, uint8_t* C, int64_t ldc) {
  if (!ctx || !desc || !A || !B || !C) return RNS8_INVALID_ARGUMENT;
  const rns8_gemm_desc& d = *desc;
  if (!valid_abi(d.struct_size, d.abi_version, sizeof(d)) || d.semantics != expected) return RNS8_INVALID_ARGUMENT;
  if (!valid_finite_modulus_for_semantics(expected, modulus) || d.m <= 0 || d.n <= 0 || d.k <= 0 ||
      d.bound_kind != RNS8_BOUND_NONE || d.bound != 0 || d.max_prefix != 0 || d.finite_modulus != modulus ||
      d.flags != 0 || d.tile_bounds || d.tile_bounds_count != 0 || d.lhs_bound != 0 || d.rhs_bound != 0 ||
      !valid_tile_size(d.tile_m) || !valid_tile_size(d.tile_n))
    return RNS8_INVALID_ARGUMENT;
  if (!valid_matrix_access(d.m, d.k, lda) || !valid_matrix_access(d.k, d.n, ldb) || !valid_matrix_access(d.m, d.n, ldc))
    return RNS8_INVALID_ARGUMENT;
  if (!backend_request_ok(d.requested_backend)) return RNS8_UNSUPPORTED_BACKEND;
  DeviceScope dev(ctx->device_id);
  if (!dev.ok) return RNS8_BACKEND_FAILURE;
  const int64_t m = d.m, n = d.n, k = d.k;
  const uint64_t a = static_cast<uint64_t>(m) * k, b = static_cast<uint64_t>(k) * n, c = static_cast<uint64_t>(m) * n;
  rns8_plan plan;
  plan.desc = d;
  rns8cuda::PlaneGemmTask task{reinterpret_cast<const int8_t*>(256), reinterpret_cast<const int8_t*>(256),
                               reinterpret_cast<int8_t*>(256)};
  rns8cuda::PlaneGemmProblem prob = rns_problem(plan, 1, &task, 1, modulus);
  const uint64_t scratch = rns8cuda::plane_gemm_scratch_bytes(prob, ctx->sm_count);
  const uint64_t total =
      2 * round256(a) + 2 * round256(b) + 2 * round256(c) + round256(scratch);
  std::unique_lock<std::mutex> lock(ctx->oneshot_mutex, std::try_to_lock);
  DevBuf local;
  DevBuf& arena = lock.owns_lock() ? ctx->oneshot_arena : local;
  rns8_status st = arena.ensure(ctx->device_id, total);
  if (st != RNS8_SUCCESS) return st;
  Carve cv{static_cast<uint8_t*>(arena.ptr)};
  uint8_t* dA = static_cast<uint8_t*>(cv.take(a));
  uint8_t* dB = static_cast<uint8_t*>(cv.take(b));
  int8_t* rA = static_cast<int8_t*>(cv.take(a));
  int8_t* rB = static_cast<int8_t*>(cv.take(b));
  int8_t* rC = static_cast<int8_t*>(cv.take(c));
  uint8_t* dC = static_cast<uint8_t*>(cv.take(c));
  void* dS = scratch ? cv.take(scratch) : nullptr;
  if ((st = copy_in_2d(*ctx, dA, A, m, k, lda, 1)) != RNS8_SUCCESS) return st;
  if ((st = copy_in_2d(*ctx, dB, B, k, n, ldb, 1)) != RNS8_SUCCESS) return st;
  cudaError_t e = rns8cuda::pack_finite_u8(dA, m, k, k, modulus, rA, ctx->stream);
  if (e == cudaSuccess) e = rns8cuda::pack_finite_u8(dB, k, n, n, modulus, rB, ctx->stream);
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  if ((st = clear_status(*ctx)) != RNS8_SUCCESS) return st;
  task = {rA, rB, rC};
  e = rns8cuda::plane_gemm(prob, rns8cuda::GemmPath::Auto, ctx->sm_count, dS, scratch, ctx->dev_status, ctx->stream);
  if (e == cudaSuccess) e = rns8cuda::export_finite_u8(rC, m, n, modulus, dC, n, ctx->stream);
  if (e != cudaSuccess) return RNS8_BACKEND_FAILURE;
  uint32_t word = 0;
  if ((st = read_status(*ctx, &word)) != RNS8_SUCCESS) return st;
  if (word != 0) return RNS8_BACKEND_FAILURE;
  if ((st = copy_out_2d(*ctx, C, ldc, dC, m, n, 1)) != RNS8_SUCCESS) return st;
  return sync(*ctx);
}

rns8_status grouped_gemm(rns8_context* ctx, const rns8_plan* plan, const rns8_grouped_gemm_task* tasks,
                         uint32_t count, bool finite, uint16_t modulus) {
  if (!ctx || !plan) return RNS8_INVALID_ARGUMENT;
  if ((finite && (!uses_finite_storage(plan->desc.semantics) || plan->desc.finite_modulus != modulus ||
                  !valid_finite_modulus_for_semantics(plan->desc.semantics, modulus))) ||
      (!finite && !uses_rns_storage(plan->desc.semantics)))
    return RNS8_INVALID_ARGUMENT;
  if (!tasks || count <= 1) return RNS8_INVALID_ARGUMENT;
  for (uint32_t i = 0; i < count; ++i) {
    const auto& t = tasks[i];
    if (!valid_abi(t.struct_size, t.abi_version, sizeof(t)) || !t.a || !t.b || !t.c || !t.workspace)
      return RNS8_INVALID_ARGUMENT;
    const rns8_status ws = validate_workspace(*ctx, *plan, *t.workspace);
    if (ws != RNS8_SUCCESS) return ws;
  }
  std::vector<i256> bounds(exact_wide(plan->desc.semantics) ? count : 0);
  std::vector<ExactRanges> ranges(bounds.size());
  std::vector<DeferredExactRange> deferred(bounds.size());
  for (uint32_t i = 0; i < count; ++i) {
    const auto& t = tasks[i];
    const rns8_status v = finite ? validate_finite_operands(*ctx, *plan, modulus, *t.a, *t.b, *t.c)
                                 : validate_rns_operands(*ctx, *plan, *t.a, *t.b, *t.c);
    if (v != RNS8_SUCCESS) return v;
    // Outputs are written concurrently: no output may alias an input or another output.
    for (uint32_t j = 0; j < count; ++j) {
      if (t.c == tasks[j].a || t.c == tasks[j].b || (i != j && t.c == tasks[j].c)) return RNS8_INVALID_ARGUMENT;
    }
    if (!bounds.empty()) {
      const rns8_status r = exact_gemm_range(*ctx, *plan, *t.a, *t.b, bounds[i], &ranges[i], &deferred[i]);
      if (r != RNS8_SUCCESS) return r;
    }
  }
  DeviceScope dev(ctx->device_id);
  if (!dev.ok) return RNS8_BACKEND_FAILURE;
  std::vector<rns8cuda::PlaneGemmTask> list(count);
  for (uint32_t i = 0; i < count; ++i) list[i] = {tasks[i].a->residues, tasks[i].b->residues, tasks[i].c->residues};
  for (uint32_t i = 0; i < count; ++i) tasks[i].c->device_current = false;
  if (!finite && !plan->tile_schedule.empty()) {
    // Scheduled plans run task by task with the plan's tile schedule.
    for (uint32_t i = 0; i < count; ++i) {
      const rns8cuda::PlaneGemmProblem one = rns_problem(*plan, plan->storage_prefix(), &list[i], 1, 0);
      const rns8_status st = run_plane_gemm_scheduled(*ctx, *plan, one, tasks[i].workspace);
      if (st != RNS8_SUCCESS) return st;
    }
  } else {
    const rns8cuda::PlaneGemmProblem prob =
        rns_problem(*plan, finite ? 1 : plan->prefix, list.data(), count, finite ? modulus : 0);
    const rns8_status st = run_plane_gemm(*ctx, prob, tasks[0].workspace);
    if (st != RNS8_SUCCESS) return st;
  }
  for (uint32_t i = 0; i < count; ++i) {
    rns8_matrix& C = *tasks[i].c;
    C.device_current = true;
    C.source_version = combine_source_versions(tasks[i].a->source_version, tasks[i].b->source_version);
    if (finite) C.finite_modulus = modulus;
    if (!bounds.empty()) commit_exact_range(C, *plan, bounds[i], &ranges[i], &deferred[i]);
  }
  return RNS8_SUCCESS;
}

}  // namespace
}  // namespace rns8host

using namespace rns8host;

extern "C" rns8_status rns8_pack_i64(rns8_context* ctx, rns8_matrix* matrix, const int64_t* src, int64_t ld,
                                     uint64_t source_version) {
  return guard([&] { return pack_native<int64_t>(ctx, matrix, src, ld, source_version); });
}

extern "C" rns8_status rns8_pack_u64(rns8_context* ctx, rns8_matrix* matrix, const uint64_t* src, int64_t ld,
                                     uint64_t source_version) {
  return guard([&] { return pack_native<uint64_t>(ctx, matrix, src, ld, source_version); });
}

extern "C" rns8_status rns8_pack_finite_u8(rns8_context* ctx, rns8_matrix* matrix, uint16_t modulus,
                                           const uint8_t* src, int64_t ld, uint64_t source_version) {
  return guard([&]() -> rns8_status {
    if (!ctx || !matrix || !src || !valid_matrix_access(matrix->desc.rows, matrix->desc.cols, ld) ||
        !valid_finite_modulus_for_semantics(matrix->desc.semantics, modulus))
      return RNS8_INVALID_ARGUMENT;
    if (ctx->backend != matrix->backend || matrix->device_id != ctx->device_id) return RNS8_INVALID_ARGUMENT;
    if (!uses_finite_storage(matrix->desc.semantics) || matrix->prefix != 0) return RNS8_INVALID_ARGUMENT;
    if (source_version != 0 && matrix->source_version == source_version && matrix->finite_modulus == modulus &&
        matrix->device_current)
      return RNS8_SUCCESS;
    DeviceScope dev(ctx->device_id);
    if (!dev.ok) return RNS8_BACKEND_FAILURE;
    const int64_t rows = matrix->desc.rows, cols = matrix->desc.cols;
    rns8_status st = matrix->upload.ensure(ctx->device_id, static_cast<uint64_t>(rows) * cols);
    if (st != RNS8_SUCCESS) return st;
    matrix->device_current = false;
    if ((st = copy_in_2d(*ctx, matrix->upload.ptr, src, rows, cols, ld, 1)) != RNS8_SUCCESS) return st;
    if (rns8cuda::pack_finite_u8(static_cast<const uint8_t*>(matrix->upload.ptr), rows, cols, cols, modulus,
                                 matrix->residues, ctx->stream) != cudaSuccess)
      return RNS8_BACKEND_FAILURE;
    if ((st = sync(*ctx)) != RNS8_SUCCESS) return st;
    matrix->device_current = true;
    matrix->finite_modulus = modulus;
    matrix->source_version = source_version;
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_gemm_rns(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* A,
                                     const rns8_matrix* B, rns8_matrix* C, rns8_workspace* workspace) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !A || !B || !C || !workspace) return RNS8_INVALID_ARGUMENT;
    rns8_status st = validate_workspace(*ctx, *plan, *workspace);
    if (st != RNS8_SUCCESS) return st;
    st = validate_rns_operands(*ctx, *plan, *A, *B, *C);
    if (st != RNS8_SUCCESS) return st;
    i256 bound;
    ExactRanges ranges;
    DeferredExactRange defer;
    if (exact_wide(plan->desc.semantics)) {
      st = exact_gemm_range(*ctx, *plan, *A, *B, bound, &ranges, &defer);
      if (st != RNS8_SUCCESS) return st;
    }
    DeviceScope dev(ctx->device_id);
    if (!dev.ok) return RNS8_BACKEND_FAILURE;
    C->device_current = false;
    rns8cuda::PlaneGemmTask task{A->residues, B->residues, C->residues};
    const rns8cuda::PlaneGemmProblem prob = rns_problem(*plan, plan->storage_prefix(), &task, 1, 0);
    st = plan->tile_schedule.empty() ? run_plane_gemm(*ctx, prob, workspace)
                                     : run_plane_gemm_scheduled(*ctx, *plan, prob, workspace);
    if (st != RNS8_SUCCESS) return st;
    C->device_current = true;
    C->source_version = combine_source_versions(A->source_version, B->source_version);
    if (exact_wide(plan->desc.semantics)) commit_exact_range(*C, *plan, bound, &ranges, &defer);
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_gemm_rns_grouped(rns8_context* ctx, const rns8_plan* plan,
                                             const rns8_grouped_gemm_task* tasks, uint32_t task_count) {
  return guard([&] { return grouped_gemm(ctx, plan, tasks, task_count, false, 0); });
}

extern "C" rns8_status rns8_gemm_finite_u8(rns8_context* ctx, const rns8_plan* plan, uint16_t modulus,
                                           const rns8_matrix* A, const rns8_matrix* B, rns8_matrix* C,
                                           rns8_workspace* workspace) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !A || !B || !C || !workspace) return RNS8_INVALID_ARGUMENT;
    rns8_status st = validate_workspace(*ctx, *plan, *workspace);
    if (st != RNS8_SUCCESS) return st;
    st = validate_finite_operands(*ctx, *plan, modulus, *A, *B, *C);
    if (st != RNS8_SUCCESS) return st;
    DeviceScope dev(ctx->device_id);
    if (!dev.ok) return RNS8_BACKEND_FAILURE;
    C->device_current = false;
    rns8cuda::PlaneGemmTask task{A->residues, B->residues, C->residues};
    const rns8cuda::PlaneGemmProblem prob = rns_problem(*plan, 1, &task, 1, modulus);
    st = run_plane_gemm(*ctx, prob, workspace);
    if (st != RNS8_SUCCESS) return st;
    C->device_current = true;
    C->finite_modulus = modulus;
    C->source_version = combine_source_versions(A->source_version, B->source_version);
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_gemm_finite_u8_grouped(rns8_context* ctx, const rns8_plan* plan, uint16_t modulus,
                                                   const rns8_grouped_gemm_task* tasks, uint32_t task_count) {
  return guard([&] { return grouped_gemm(ctx, plan, tasks, task_count, true, modulus); });
}

extern "C" rns8_status rns8_export_i64(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* C, int64_t* dst,
                                       int64_t ld) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !C || !dst || !valid_matrix_access(plan->desc.m, plan->desc.n, ld))
      return RNS8_INVALID_ARGUMENT;
    const rns8_status v = validate_rns_export(*ctx, *plan, *C, RNS8_BOUNDED_I64);
    if (v != RNS8_SUCCESS) return v;
    return export_rns(*ctx, *plan, *C, dst, ld, ExportKind::I64, 1);
  });
}

extern "C" rns8_status rns8_export_u64(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* C, uint64_t* dst,
                                       int64_t ld) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !C || !dst || !valid_matrix_access(plan->desc.m, plan->desc.n, ld))
      return RNS8_INVALID_ARGUMENT;
    const rns8_status v = validate_rns_export(*ctx, *plan, *C, RNS8_BOUNDED_U64);
    if (v != RNS8_SUCCESS) return v;
    return export_rns(*ctx, *plan, *C, dst, ld, ExportKind::U64, 1);
  });
}

extern "C" rns8_status rns8_export_exact_wide_signed_limbs(rns8_context* ctx, const rns8_plan* plan,
                                                           const rns8_matrix* C, uint64_t* dst, int64_t ld,
                                                           uint32_t limb_count) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !C || !dst || !valid_limb_export_access(plan->desc.m, plan->desc.n, ld, limb_count))
      return RNS8_INVALID_ARGUMENT;
    const rns8_status v = validate_rns_export(*ctx, *plan, *C, RNS8_EXACT_WIDE_SIGNED);
    if (v != RNS8_SUCCESS) return v;
    return export_rns(*ctx, *plan, *C, dst, ld, ExportKind::LimbsS, limb_count);
  });
}

extern "C" rns8_status rns8_export_exact_wide_unsigned_limbs(rns8_context* ctx, const rns8_plan* plan,
                                                             const rns8_matrix* C, uint64_t* dst, int64_t ld,
                                                             uint32_t limb_count) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !C || !dst || !valid_limb_export_access(plan->desc.m, plan->desc.n, ld, limb_count))
      return RNS8_INVALID_ARGUMENT;
    const rns8_status v = validate_rns_export(*ctx, *plan, *C, RNS8_EXACT_WIDE_UNSIGNED);
    if (v != RNS8_SUCCESS) return v;
    return export_rns(*ctx, *plan, *C, dst, ld, ExportKind::LimbsU, limb_count);
  });
}

extern "C" rns8_status rns8_export_finite_u8(rns8_context* ctx, const rns8_plan* plan, uint16_t modulus,
                                             const rns8_matrix* Cc, uint8_t* dst, int64_t ld) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !Cc || !dst || !valid_matrix_access(plan->desc.m, plan->desc.n, ld))
      return RNS8_INVALID_ARGUMENT;
    if (!uses_finite_storage(plan->desc.semantics) ||
        !valid_finite_modulus_for_semantics(plan->desc.semantics, modulus) || plan->desc.finite_modulus != modulus)
      return RNS8_INVALID_ARGUMENT;
    if (!plan_context_ok(*ctx, *plan) || Cc->device_id != ctx->device_id) return RNS8_INVALID_ARGUMENT;
    if (!descriptor_matches(*Cc, plan->desc.semantics, RNS8_BOUND_NONE, plan->desc.m, plan->desc.n, 0, *plan) ||
        !Cc->device_current || Cc->finite_modulus != modulus)
      return RNS8_INVALID_ARGUMENT;
    rns8_matrix& C = const_cast<rns8_matrix&>(*Cc);
    DeviceScope dev(ctx->device_id);
    if (!dev.ok) return RNS8_BACKEND_FAILURE;
    const int64_t m = plan->desc.m, n = plan->desc.n;
    rns8_status st = C.staging.ensure(ctx->device_id, static_cast<uint64_t>(m) * n);
    if (st != RNS8_SUCCESS) return st;
    if (rns8cuda::export_finite_u8(C.residues, m, n, modulus, static_cast<uint8_t*>(C.staging.ptr), n, ctx->stream) !=
        cudaSuccess)
      return RNS8_BACKEND_FAILURE;
    if ((st = copy_out_2d(*ctx, dst, ld, C.staging.ptr, m, n, 1)) != RNS8_SUCCESS) return st;
    return sync(*ctx);
  });
}

extern "C" rns8_status rns8_gemm_i64_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc, const int64_t* A,
                                             int64_t lda, const int64_t* B, int64_t ldb, int64_t* C, int64_t ldc) {
  return guard([&] { return bounded_oneshot<int64_t>(ctx, desc, A, lda, B, ldb, C, ldc); });
}

extern "C" rns8_status rns8_gemm_u64_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc, const uint64_t* A,
                                             int64_t lda, const uint64_t* B, int64_t ldb, uint64_t* C, int64_t ldc) {
  return guard([&] { return bounded_oneshot<uint64_t>(ctx, desc, A, lda, B, ldb, C, ldc); });
}

extern "C" rns8_status rns8_gemm_finite_ring_u8_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc,
                                                        uint16_t modulus, const uint8_t* A, int64_t lda,
                                                        const uint8_t* B, int64_t ldb, uint8_t* C, int64_t ldc) {
  return guard([&] { return finite_oneshot(ctx, desc, RNS8_FINITE_RING_U8, modulus, A, lda, B, ldb, C, ldc); });
}

extern "C" rns8_status rns8_gemm_finite_field_u8_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc,
                                                         uint16_t modulus, const uint8_t* A, int64_t lda,
                                                         const uint8_t* B, int64_t ldb, uint8_t* C, int64_t ldc) {
  return guard([&] { return finite_oneshot(ctx, desc, RNS8_FINITE_FIELD_U8, modulus, A, lda, B, ldb, C, ldc); });
}

extern "C" rns8_status rns8_gemm_wrap_u64(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* A,
                                         const rns8_matrix* B, rns8_matrix* C, rns8_workspace* workspace) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !A || !B || !C || !workspace) return RNS8_INVALID_ARGUMENT;
    rns8_status st = validate_workspace(*ctx, *plan, *workspace);
    if (st != RNS8_SUCCESS) return st;
    if ((st = validate_wrap_operands(*ctx, *plan, *A, *B, *C)) != RNS8_SUCCESS) return st;
    DeviceScope dev(ctx->device_id);
    if (!dev.ok) return RNS8_BACKEND_FAILURE;
    const int64_t m = plan->desc.m, n = plan->desc.n, k = plan->desc.k;
    if ((st = workspace->scratch.ensure(ctx->device_id, static_cast<uint64_t>(m) * n * sizeof(uint64_t))) !=
        RNS8_SUCCESS)
      return st;
    C->device_current = false;
    st = run_wrap_gemm(*ctx, reinterpret_cast<const uint8_t*>(A->residues), reinterpret_cast<const uint8_t*>(B->residues),
                       static_cast<uint64_t*>(workspace->scratch.ptr), m, n, k, reinterpret_cast<uint8_t*>(C->residues));
    if (st != RNS8_SUCCESS) return st;
    C->device_current = true;
    C->source_version = combine_source_versions(A->source_version, B->source_version);
    return RNS8_SUCCESS;
  });
}

// rns8_export_wrap_u64 (api_export.cpp:534-585): the low 64 bits of every cell.
extern "C" rns8_status rns8_export_wrap_u64(rns8_context* ctx, const rns8_plan* plan, const rns8_matrix* C,
                                           uint64_t* dst, int64_t ld) {
  return guard([&]() -> rns8_status {
    if (!ctx || !plan || !C || !dst || !valid_matrix_access(plan->desc.m, plan->desc.n, ld))
      return RNS8_INVALID_ARGUMENT;
    if (!plan_context_ok(*ctx, *plan) || plan->desc.semantics != RNS8_WRAP_U64_MOD_2_64 || plan->prefix != 0)
      return RNS8_INVALID_ARGUMENT;
    if (C->device_id != ctx->device_id || C->backend != plan->backend ||
        !wrap_storage_ok(*C, plan->desc.m, plan->desc.n) || !C->device_current)
      return RNS8_INVALID_ARGUMENT;
    DeviceScope dev(ctx->device_id);
    if (!dev.ok) return RNS8_BACKEND_FAILURE;
    const int64_t m = plan->desc.m, n = plan->desc.n;
    rns8_matrix& mc = const_cast<rns8_matrix&>(*C);  // export staging is a documented mutable cache
    rns8_status st = mc.staging.ensure(ctx->device_id, static_cast<uint64_t>(m) * n * sizeof(uint64_t));
    if (st != RNS8_SUCCESS) return st;
    if (rns8cuda::wrap_export_u64(reinterpret_cast<const uint8_t*>(C->residues), m, n,
                                  static_cast<uint64_t*>(mc.staging.ptr), n, ctx->stream) != cudaSuccess)
      return RNS8_BACKEND_FAILURE;
    if ((st = copy_out_2d(*ctx, dst, ld, mc.staging.ptr, m, n, sizeof(uint64_t))) != RNS8_SUCCESS) return st;
    return sync(*ctx);
  });
}

// rns8_gemm_wrap_u64_oneshot (api_oneshot.cpp:588-618): pack, GEMM and export
// through the context's one-shot arena.
extern "C" rns8_status rns8_gemm_wrap_u64_oneshot(rns8_context* ctx, const rns8_gemm_desc* desc, const uint64_t* A,
                                                 int64_t lda, const uint64_t* B, int64_t ldb, uint64_t* C,
                                                 int64_t ldc) {
  return guard([&]() -> rns8_status {
    if (!ctx || !desc || !A || !B || !C) return RNS8_INVALID_ARGUMENT;
    rns8_status st = validate_typed_oneshot(*desc, RNS8_WRAP_U64_MOD_2_64, lda, ldb, ldc);
    if (st != RNS8_SUCCESS) return st;
    rns8_plan plan;
    plan.device_id = ctx->device_id;
    if ((st = build_plan(*desc, plan)) != RNS8_SUCCESS) return st;
    DeviceScope dev(ctx->device_id);
    if (!dev.ok) return RNS8_BACKEND_FAILURE;
    const int64_t m = plan.desc.m, n = plan.desc.n, k = plan.desc.k;
    const uint64_t a_bytes = static_cast<uint64_t>(m) * k * 8, b_bytes = static_cast<uint64_t>(k) * n * 8;
    const uint64_t c_bytes = static_cast<uint64_t>(m) * n * 8;
    const uint64_t total = 2 * round256(a_bytes) + 2 * round256(b_bytes) + round256(c_bytes);
    std::unique_lock<std::mutex> lock(ctx->oneshot_mutex, std::try_to_lock);
    DevBuf local;
    DevBuf& arena = lock.owns_lock() ? ctx->oneshot_arena : local;
    if ((st = arena.ensure(ctx->device_id, total)) != RNS8_SUCCESS) return st;
    Carve cv{static_cast<uint8_t*>(arena.ptr)};
    auto* dA = static_cast<uint64_t*>(cv.take(a_bytes));
    auto* dB = static_cast<uint64_t*>(cv.take(b_bytes));
    auto* lA = static_cast<uint8_t*>(cv.take(a_bytes));
    auto* lB = static_cast<uint8_t*>(cv.take(b_bytes));
    auto* dC = static_cast<uint64_t*>(cv.take(c_bytes));
    if ((st = copy_in_2d(*ctx, dA, A, m, k, lda, 8)) != RNS8_SUCCESS) return st;
    if ((st = copy_in_2d(*ctx, dB, B, k, n, ldb, 8)) != RNS8_SUCCESS) return st;
    if (rns8cuda::wrap_pack_u64(dA, m, k, k, lA, ctx->stream) != cudaSuccess ||
        rns8cuda::wrap_pack_u64(dB, k, n, n, lB, ctx->stream) != cudaSuccess)
      return RNS8_BACKEND_FAILURE;
    if ((st = run_wrap_gemm(*ctx, lA, lB, dC, m, n, k, nullptr)) != RNS8_SUCCESS) return st;
    if ((st = copy_out_2d(*ctx, C, ldc, dC, m, n, 8)) != RNS8_SUCCESS) return st;
    return sync(*ctx);
  });
}
