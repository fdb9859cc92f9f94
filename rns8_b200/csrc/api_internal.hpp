// Host-side state behind the rns8 C ABI handles (reference counterpart:
// src/core/internal.hpp:13-251). Device buffers are plain cudaMalloc
// allocations owned by the handle that created them.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <exception>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "kernels.hpp"
#include "ladder.hpp"
#include "rns8/rns8.h"
#include "rns8/rns8_cuda.h"
#include "wide_int.hpp"

namespace rns8host {

using rns8ladder::kLadder;

// One growable device allocation.
struct DevBuf {
  void* ptr = nullptr;
  uint64_t bytes = 0;
  int device = -1;
  rns8_status ensure(int dev, uint64_t need);
  void release();
  ~DevBuf() { release(); }
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
};

// Exact-wide range proof of one axis (row or column), reference
// src/core/internal.hpp:74-87. Magnitudes and sums of int64/uint64 values
// over at most 2^63 elements fit in 128 bits; products fit in 256 bits.
struct AxisRange {
  i256 max_magnitude, absolute_sum, sum, minimum, maximum, deviation_sum;
  bool sum_known = false;
};
struct ExactRanges {
  std::vector<AxisRange> rows, cols;
};
// The per-cell bound pass of an exact-wide GEMM whose cheap bound
// K * max|A| * max|B| already fitted the prefix: its only results are the
// output's recorded bound and row/column records, which no decision needs
// until the output feeds another exact-wide GEMM. The pass's inputs are kept
// here and it runs then (resolve_exact_range), with the same result.
struct DeferredExactRange {
  bool pending = false;
  int64_t m = 0, n = 0, k = 0;
  i256 a_max, b_max;
  bool a_rows_known = false, b_cols_known = false;
  std::vector<AxisRange> a_rows, b_cols;
};

}  // namespace rns8host

struct rns8_context {
  rns8_backend_kind backend = RNS8_BACKEND_CUDA_SM100;
  int device_id = 0;
  int sm_count = 148;
  cudaStream_t stream = nullptr;
  cudaStream_t copy_stream = nullptr;  // host-to-device uploads overlapped with `stream`
  cudaStream_t out_stream = nullptr;   // device-to-host results overlapped with both
  rns8_device_info info{};
  uint32_t* dev_status = nullptr;  // 4 status words
  // Device arena reused by the one-shot entry points (serialised by the mutex).
  std::mutex oneshot_mutex;
  rns8host::DevBuf oneshot_arena;
  // Device scratch of the exact-wide admission proofs (serialised by the mutex).
  std::mutex admission_mutex;
  rns8host::DevBuf admission;
};

struct rns8_plan {
  rns8_gemm_desc desc{};          // normalised: tile sizes and max_prefix filled in, pointers dropped
  uint32_t prefix = 0;            // selected prefix (0 for finite / wrap)
  uint32_t requested_max_prefix = 0;
  rns8host::i256 modulus_product;
  rns8_backend_kind backend = RNS8_BACKEND_CUDA_SM100;
  int device_id = 0;
  uint64_t tile_rows = 0, tile_cols = 0, tile_count = 0;
  uint32_t min_required = 0, max_required = 0, min_selected = 0, max_selected = 0;
  uint32_t group_count = 0, range_bit_length = 0, adaptive_prefix = 0, adaptive_skip = 0, schedule_flags = 0;
  uint64_t fingerprint = 0;
  // Per-tile bound plans (api_plan_schedule.inc:109-261): one entry per
  // tile_m x tile_n output tile, empty when every tile runs the plan prefix.
  std::vector<uint64_t> tile_bounds;
  std::vector<rns8_plan_tile_schedule_entry> tile_schedule;
  std::vector<uint8_t> zero_a_rows, zero_b_cols;
  uint64_t zero_a_row_count = 0, zero_b_col_count = 0, zero_row_col_product_count = 0;
  // Residue planes the plan's matrices must hold: the largest selected prefix.
  uint32_t storage_prefix() const {
    return !tile_schedule.empty() && max_selected > 0 ? max_selected : prefix;
  }
};

struct rns8_matrix {
  rns8_matrix_desc desc{};
  rns8_backend_kind backend = RNS8_BACKEND_CUDA_SM100;
  uint64_t id = 0;
  uint32_t prefix = 0;          // allocated planes (1 for finite storage)
  uint16_t finite_modulus = 0;  // stamped by finite pack / GEMM
  uint64_t source_version = 0;
  int device_id = 0;
  int8_t* residues = nullptr;   // device, prefix * rows * cols bytes
  uint64_t residue_bytes = 0;
  bool device_current = false;
  rns8host::DevBuf upload;      // native input staging
  rns8host::DevBuf staging;     // export staging
  rns8host::DevBuf export_jobs; // per-tile export descriptors (scheduled plans)
  // Exact-wide proof (reference internal.hpp:96-99); zero prefix = unknown.
  // Mutable: a GEMM output's records may be completed lazily when it is read
  // as an operand (DeferredExactRange).
  mutable rns8host::i256 exact_max_magnitude;
  uint32_t exact_range_prefix = 0;
  mutable rns8host::ExactRanges exact_axes;
  mutable rns8host::DeferredExactRange exact_deferred;
};

struct rns8_workspace {
  rns8_backend_kind backend = RNS8_BACKEND_CUDA_SM100;
  int device_id = 0;
  uint64_t plan_fingerprint = 0;
  rns8_semantics semantics = RNS8_BOUNDED_I64;
  rns8_bound_kind bound_kind = RNS8_BOUND_NONE;
  int64_t m = 0, n = 0, k = 0;
  uint32_t prefix = 0;
  rns8host::DevBuf scratch;  // split-K partial sums
};

namespace rns8host {

// Runs body, mapping exceptions to RNS8_INTERNAL_ERROR (reference guard_api,
// src/core/api_internal.hpp:34-42).
template <typename F>
rns8_status guard(F&& body) {
  try {
    return body();
  } catch (const std::bad_alloc&) {
    return RNS8_INTERNAL_ERROR;
  } catch (...) {
    return RNS8_INTERNAL_ERROR;
  }
}

bool valid_abi(uint64_t struct_size, uint32_t abi_version, size_t expected);
void set_text(char* dst, size_t cap, const std::string& s);
rns8_status cuda_status(cudaError_t e);

// Makes `dev` the calling thread's current device for the life of the scope
// and puts the caller's current device back when it ends, so that no entry
// point leaves the thread on another device than it found it on. `ok` is
// false when `dev` is negative or cannot be made current.
class DeviceScope {
 public:
  explicit DeviceScope(int dev) {
    if (cudaGetDevice(&prev_) != cudaSuccess) {
      (void)cudaGetLastError();
      prev_ = -1;
    }
    if (dev < 0) return;
    if (prev_ == dev) {
      ok = true;
      return;
    }
    ok = cudaSetDevice(dev) == cudaSuccess;
    switched_ = ok;
    if (!ok) (void)cudaGetLastError();
  }
  ~DeviceScope() {
    if (switched_ && prev_ >= 0) (void)cudaSetDevice(prev_);
  }
  DeviceScope(const DeviceScope&) = delete;
  DeviceScope& operator=(const DeviceScope&) = delete;
  bool ok = false;

 private:
  int prev_ = -1;
  bool switched_ = false;
};

// Number of CUDA devices visible to this process (0 when none or on error).
int visible_device_count();

// Contract arithmetic (reference src/core/moduli.cpp).
i256 modulus_product(uint32_t prefix);
uint32_t required_prefix_for_range(const i256& range);
uint32_t default_prefix_for_semantics(rns8_semantics s);
bool known_semantics(uint32_t s);
bool known_bound_kind(uint32_t b);
bool known_layout(uint32_t l);
bool valid_tile_size(uint32_t v);
bool valid_finite_modulus_for_semantics(rns8_semantics s, uint32_t m);
bool uses_rns_storage(rns8_semantics s);
bool uses_finite_storage(rns8_semantics s);
bool exact_wide(rns8_semantics s);
bool input_range_output_bound(const rns8_gemm_desc& d, uint64_t& out);
rns8_status validate_bound_contract(rns8_semantics s, rns8_bound_kind bk, uint64_t bound, uint32_t prefix);
rns8_status validate_gemm_desc(const rns8_gemm_desc& d, uint32_t prefix);
rns8_status validate_matrix_desc(const rns8_matrix_desc& d, uint32_t prefix);
rns8_bound_kind storage_bound_kind(const rns8_plan& plan);
bool valid_matrix_access(int64_t rows, int64_t cols, int64_t ld);
bool backend_request_ok(rns8_backend_kind requested);

// Plan construction shared by rns8_create_plan and rns8_cuda_plan_probe.
rns8_status build_plan(const rns8_gemm_desc& desc, rns8_plan& plan);

// Exact-wide proofs (reference src/core/exact_range.hpp), computed on the
// context's device. device_exact_ranges summarises a compact native matrix
// already in device memory; maximum = the largest |v|.
rns8_status device_exact_ranges(rns8_context& ctx, const void* d_src, bool is_signed, int64_t rows, int64_t cols,
                                ExactRanges& out, i256& maximum);
bool exact_range_fits(rns8_semantics s, const i256& bound, const i256& product);
// The admission bound of an m x n x k product from A's row records (or its
// largest |a| alone when a_rows is null) and B's column records; out_ranges
// receives the per-row and per-column maxima and sums of the cell bounds.
rns8_status exact_gemm_bound(rns8_context& ctx, int64_t m, int64_t n, int64_t k, const i256& a_max,
                             const std::vector<AxisRange>* a_rows, const i256& b_max,
                             const std::vector<AxisRange>* b_cols, i256& bound, ExactRanges* out_ranges);
rns8_status exact_gemm_range(rns8_context& ctx, const rns8_plan& plan, const rns8_matrix& A, const rns8_matrix& B,
                             i256& bound, ExactRanges* out_ranges, DeferredExactRange* defer = nullptr);
// Runs a matrix's deferred per-cell bound pass, if any.
rns8_status resolve_exact_range(rns8_context& ctx, const rns8_matrix& M);
void commit_exact_range(rns8_matrix& C, const rns8_plan& plan, i256& bound, ExactRanges* ranges,
                        DeferredExactRange* defer = nullptr);

uint64_t next_matrix_id();
uint64_t plan_fingerprint(const rns8_plan& plan);

}  // namespace rns8host
