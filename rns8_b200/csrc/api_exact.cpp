// Exact-wide admission proofs (reference src/core/exact_range.hpp:12-168).
//
// Packing an exact-wide matrix records per-row and per-column summaries of
// the native values (max |v|, sum |v|, sum v, min, max, sum |v - center|).
// A GEMM derives an output bound per cell from the row of A and the column of
// B, keeps the smallest of several valid bounds, and rejects the GEMM with
// RNS8_RANGE_ERROR unless the largest cell bound fits the prefix (signed:
// 2*bound < P; unsigned: bound < P). The arithmetic is exact: 128-bit
// accumulators for the summaries, 256-bit for products, with cpp_int's
// truncation toward zero for the axis centers. The summaries and the cell
// bounds run on the device (exact_range.cu); the host keeps the per-axis
// records and the final comparisons.
#include <algorithm>
#include <vector>

#include "api_internal.hpp"

namespace rns8host {
namespace {

AxisRange to_axis(const rns8cuda::AxisSummary& s) {
  AxisRange a;
  a.max_magnitude = i256::from_u128(s.max_mag);
  a.absolute_sum = i256::from_u128(s.abs_sum);
  a.sum = i256::from_i128(s.sum);
  a.minimum = i256::from_i128(s.minimum);
  a.maximum = i256::from_i128(s.maximum);
  a.deviation_sum = i256::from_u128(s.dev_sum);
  a.sum_known = s.any != 0;
  return a;
}

void put(uint64_t (&dst)[4], const i256& v) {
  for (int l = 0; l < 4; ++l) dst[l] = v.w[l];
}
i256 get(const uint64_t (&src)[4]) {
  i256 v;
  for (int l = 0; l < 4; ++l) v.w[l] = src[l];
  return v;
}

// Per-axis quantities reused for every cell (exact_range.hpp:79-98).
rns8cuda::AxisBoundInput bound_input(const AxisRange& a) {
  rns8cuda::AxisBoundInput in{};
  put(in.max_mag, a.max_magnitude);
  put(in.abs_sum, a.absolute_sum);
  put(in.sum, a.sum);
  put(in.dev_sum, a.deviation_sum);
  in.sum_known = a.sum_known ? 1 : 0;
  if (a.sum_known) {
    const i256 center = half_trunc(a.minimum + a.maximum);
    put(in.center, center);
    put(in.dev_max, max(abs(a.minimum - center), abs(a.maximum - center)));
  }
  return in;
}

AxisRange uniform_axis(const i256& maximum, int64_t length) {
  AxisRange a;
  a.max_magnitude = maximum;
  a.absolute_sum = i256::from_i64(length) * maximum;
  a.sum_known = false;
  return a;
}

uint64_t round256(uint64_t v) { return (v + 255) / 256 * 256; }

// Carves consecutive 256-byte aligned pieces out of the context's admission
// buffer; the caller holds admission_mutex.
struct AdmissionArena {
  rns8_context& ctx;
  uint8_t* base = nullptr;
  uint64_t used = 0;
  rns8_status reserve(uint64_t bytes) {
    const rns8_status st = ctx.admission.ensure(ctx.device_id, bytes);
    base = static_cast<uint8_t*>(ctx.admission.ptr);
    return st;
  }
  void* take(uint64_t bytes) {
    void* p = base + used;
    used += round256(bytes);
    return p;
  }
};

}  // namespace

bool exact_range_fits(rns8_semantics s, const i256& bound, const i256& product) {
  if (bound.neg()) return false;
  return s == RNS8_EXACT_WIDE_SIGNED ? (bound * i256::from_u64(2)) < product : bound < product;
}

rns8_status device_exact_ranges(rns8_context& ctx, const void* d_src, bool is_signed, int64_t rows, int64_t cols,
                                ExactRanges& out, i256& maximum) {
  DeviceScope scope(ctx.device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  std::lock_guard<std::mutex> lock(ctx.admission_mutex);
  using rns8cuda::AxisSummary;
  const uint64_t row_bytes = static_cast<uint64_t>(rows) * sizeof(AxisSummary);
  const uint64_t col_bytes = static_cast<uint64_t>(cols) * sizeof(AxisSummary);
  const uint64_t scratch = rns8cuda::axis_summaries_scratch_bytes(rows, cols);
  AdmissionArena arena{ctx};
  rns8_status st = arena.reserve(round256(row_bytes) + round256(col_bytes) + round256(scratch));
  if (st != RNS8_SUCCESS) return st;
  auto* d_rows = static_cast<AxisSummary*>(arena.take(row_bytes));
  auto* d_cols = static_cast<AxisSummary*>(arena.take(col_bytes));
  void* d_scratch = arena.take(scratch);
  if (rns8cuda::axis_summaries(d_src, is_signed, rows, cols, d_rows, d_cols, d_scratch, scratch, ctx.stream) !=
      cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  std::vector<AxisSummary> h_rows(static_cast<size_t>(rows)), h_cols(static_cast<size_t>(cols));
  if (cudaMemcpyAsync(h_rows.data(), d_rows, row_bytes, cudaMemcpyDeviceToHost, ctx.stream) != cudaSuccess ||
      cudaMemcpyAsync(h_cols.data(), d_cols, col_bytes, cudaMemcpyDeviceToHost, ctx.stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx.stream) != cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  out.rows.resize(static_cast<size_t>(rows));
  out.cols.resize(static_cast<size_t>(cols));
  unsigned __int128 best = 0;
  for (int64_t r = 0; r < rows; ++r) {
    out.rows[r] = to_axis(h_rows[r]);
    best = std::max(best, h_rows[r].max_mag);
  }
  for (int64_t c = 0; c < cols; ++c) out.cols[c] = to_axis(h_cols[c]);
  maximum = i256::from_u128(best);
  return RNS8_SUCCESS;
}

// exact_gemm_bound (exact_range.hpp:109-144).
rns8_status exact_gemm_bound(rns8_context& ctx, int64_t m, int64_t n, int64_t k, const i256& a_max,
                             const std::vector<AxisRange>* a_rows, const i256& b_max,
                             const std::vector<AxisRange>* b_cols, i256& bound, ExactRanges* out_ranges) {
  const i256 kk = i256::from_i64(k);
  bound = kk * a_max * b_max;
  if (out_ranges) {
    out_ranges->rows.clear();
    out_ranges->cols.clear();
  }
  if (!a_rows && !b_cols) return RNS8_SUCCESS;
  using rns8cuda::AxisBoundInput;
  using rns8cuda::BoundStats;
  std::vector<AxisBoundInput> h_in(static_cast<size_t>(m + n));
  const AxisRange fa = uniform_axis(a_max, k);
  const AxisRange fb = uniform_axis(b_max, k);
  for (int64_t r = 0; r < m; ++r) h_in[r] = bound_input(a_rows ? (*a_rows)[r] : fa);
  for (int64_t c = 0; c < n; ++c) h_in[m + c] = bound_input(b_cols ? (*b_cols)[c] : fb);
  DeviceScope scope(ctx.device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  std::lock_guard<std::mutex> lock(ctx.admission_mutex);
  const uint64_t in_bytes = static_cast<uint64_t>(m + n) * sizeof(AxisBoundInput);
  const uint64_t stat_bytes = static_cast<uint64_t>(m + n) * sizeof(BoundStats);
  const uint64_t scratch = rns8cuda::cell_bounds_scratch_bytes(m, n);
  AdmissionArena arena{ctx};
  rns8_status st = arena.reserve(round256(in_bytes) + round256(stat_bytes) + round256(scratch));
  if (st != RNS8_SUCCESS) return st;
  auto* d_in = static_cast<AxisBoundInput*>(arena.take(in_bytes));
  auto* d_stats = static_cast<BoundStats*>(arena.take(stat_bytes));
  void* d_scratch = arena.take(scratch);
  if (cudaMemcpyAsync(d_in, h_in.data(), in_bytes, cudaMemcpyHostToDevice, ctx.stream) != cudaSuccess ||
      rns8cuda::cell_bounds(d_in, m, d_in + m, n, k, d_stats, d_stats + m, d_scratch, scratch, ctx.stream) !=
          cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  std::vector<BoundStats> h_stats(static_cast<size_t>(m + n));
  if (cudaMemcpyAsync(h_stats.data(), d_stats, stat_bytes, cudaMemcpyDeviceToHost, ctx.stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx.stream) != cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  i256 maximum;
  for (int64_t r = 0; r < m; ++r) maximum = max(maximum, get(h_stats[r].max));
  if (out_ranges) {
    out_ranges->rows.resize(static_cast<size_t>(m));
    out_ranges->cols.resize(static_cast<size_t>(n));
    for (int64_t r = 0; r < m; ++r) {
      out_ranges->rows[r].max_magnitude = get(h_stats[r].max);
      out_ranges->rows[r].absolute_sum = get(h_stats[r].sum);
    }
    for (int64_t c = 0; c < n; ++c) {
      out_ranges->cols[c].max_magnitude = get(h_stats[m + c].max);
      out_ranges->cols[c].absolute_sum = get(h_stats[m + c].sum);
    }
  }
  if (maximum < bound) bound = maximum;
  return RNS8_SUCCESS;
}

// exact_gemm_range (exact_range.hpp:146-154): the bound must fit the plan's prefix.
// With `defer`, a GEMM whose cheap bound K * max|A| * max|B| already fits the
// prefix is admitted at once: the per-cell pass could only lower the bound,
// and its results (the output's tightened bound and row/column records) are
// produced on demand by resolve_exact_range, from the inputs kept in *defer.
rns8_status exact_gemm_range(rns8_context& ctx, const rns8_plan& plan, const rns8_matrix& A, const rns8_matrix& B,
                             i256& bound, ExactRanges* out_ranges, DeferredExactRange* defer) {
  if (!exact_wide(plan.desc.semantics)) return RNS8_SUCCESS;
  if (A.exact_range_prefix < plan.prefix || B.exact_range_prefix < plan.prefix) return RNS8_RANGE_ERROR;
  rns8_status st = resolve_exact_range(ctx, A);
  if (st == RNS8_SUCCESS) st = resolve_exact_range(ctx, B);
  if (st != RNS8_SUCCESS) return st;
  const int64_t m = plan.desc.m, n = plan.desc.n;
  const bool a_rows = A.exact_axes.rows.size() == static_cast<size_t>(m);
  const bool b_cols = B.exact_axes.cols.size() == static_cast<size_t>(n);
  if (defer && (a_rows || b_cols)) {
    const i256 cheap = i256::from_i64(plan.desc.k) * A.exact_max_magnitude * B.exact_max_magnitude;
    if (exact_range_fits(plan.desc.semantics, cheap, plan.modulus_product)) {
      bound = cheap;
      if (out_ranges) {
        out_ranges->rows.clear();
        out_ranges->cols.clear();
      }
      defer->pending = true;
      defer->m = m;
      defer->n = n;
      defer->k = plan.desc.k;
      defer->a_max = A.exact_max_magnitude;
      defer->b_max = B.exact_max_magnitude;
      defer->a_rows_known = a_rows;
      defer->b_cols_known = b_cols;
      defer->a_rows = a_rows ? A.exact_axes.rows : std::vector<AxisRange>{};
      defer->b_cols = b_cols ? B.exact_axes.cols : std::vector<AxisRange>{};
      return RNS8_SUCCESS;
    }
  }
  st = exact_gemm_bound(ctx, m, n, plan.desc.k, A.exact_max_magnitude, a_rows ? &A.exact_axes.rows : nullptr,
                        B.exact_max_magnitude, b_cols ? &B.exact_axes.cols : nullptr, bound, out_ranges);
  if (st != RNS8_SUCCESS) return st;
  return exact_range_fits(plan.desc.semantics, bound, plan.modulus_product) ? RNS8_SUCCESS : RNS8_RANGE_ERROR;
}

rns8_status resolve_exact_range(rns8_context& ctx, const rns8_matrix& M) {
  DeferredExactRange& d = M.exact_deferred;
  if (!d.pending) return RNS8_SUCCESS;
  i256 bound;
  ExactRanges ranges;
  const rns8_status st = exact_gemm_bound(ctx, d.m, d.n, d.k, d.a_max, d.a_rows_known ? &d.a_rows : nullptr,
                                          d.b_max, d.b_cols_known ? &d.b_cols : nullptr, bound, &ranges);
  if (st != RNS8_SUCCESS) return st;
  M.exact_max_magnitude = bound;
  M.exact_axes.rows.swap(ranges.rows);
  M.exact_axes.cols.swap(ranges.cols);
  M.exact_deferred = DeferredExactRange{};
  return RNS8_SUCCESS;
}

void commit_exact_range(rns8_matrix& C, const rns8_plan& plan, i256& bound, ExactRanges* ranges,
                        DeferredExactRange* defer) {
  if (!exact_wide(plan.desc.semantics)) return;
  C.exact_max_magnitude = bound;
  C.exact_axes.rows.clear();
  C.exact_axes.cols.clear();
  if (ranges) {
    C.exact_axes.rows.swap(ranges->rows);
    C.exact_axes.cols.swap(ranges->cols);
  }
  C.exact_deferred = DeferredExactRange{};
  if (defer && defer->pending) std::swap(C.exact_deferred, *defer);
  C.exact_range_prefix = plan.prefix;
}

}  // namespace rns8host

using namespace rns8host;

extern "C" rns8_status rns8_cuda_exact_gemm_bound_device(int device_id, const void* d_a, const void* d_b, int64_t m,
                                                         int64_t n, int64_t k, uint32_t is_signed, uint64_t* out_bound,
                                                         uint64_t* out_a_max, uint64_t* out_b_max,
                                                         uint64_t* out_row_stats, uint64_t* out_col_stats,
                                                         void* stream) {
  return guard([&]() -> rns8_status {
    if (!d_a || !d_b || !out_bound || m <= 0 || n <= 0 || k <= 0 || is_signed > 1 ||
        !valid_matrix_access(m, k, k) || !valid_matrix_access(k, n, n))
      return RNS8_INVALID_ARGUMENT;
    if (device_id < 0) return RNS8_INVALID_ARGUMENT;
    rns8_context scope;  // device, stream and admission scratch of this call
    scope.device_id = device_id;
    scope.stream = static_cast<cudaStream_t>(stream);
    ExactRanges ra, rb, rc;
    i256 a_max, b_max, bound;
    rns8_status st = device_exact_ranges(scope, d_a, is_signed != 0, m, k, ra, a_max);
    if (st == RNS8_SUCCESS) st = device_exact_ranges(scope, d_b, is_signed != 0, k, n, rb, b_max);
    if (st == RNS8_SUCCESS) st = exact_gemm_bound(scope, m, n, k, a_max, &ra.rows, b_max, &rb.cols, bound, &rc);
    if (st != RNS8_SUCCESS) return st;
    for (int l = 0; l < 4; ++l) {
      out_bound[l] = bound.w[l];
      if (out_a_max) out_a_max[l] = a_max.w[l];
      if (out_b_max) out_b_max[l] = b_max.w[l];
    }
    auto write_stats = [](uint64_t* dst, const std::vector<AxisRange>& axes) {
      for (size_t i = 0; i < axes.size(); ++i)
        for (int l = 0; l < 4; ++l) {
          dst[8 * i + l] = axes[i].max_magnitude.w[l];
          dst[8 * i + 4 + l] = axes[i].absolute_sum.w[l];
        }
    };
    if (out_row_stats) write_stats(out_row_stats, rc.rows);
    if (out_col_stats) write_stats(out_col_stats, rc.cols);
    return RNS8_SUCCESS;
  });
}
