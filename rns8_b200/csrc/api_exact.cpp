// Exact-wide admission proofs (reference src/core/exact_range.hpp:12-168).
//
// Packing an exact-wide matrix records per-row and per-column summaries of
// the native values (max |v|, sum |v|, sum v, min, max, sum |v - center|).
// A GEMM derives an output bound per cell from the row of A and the column of
// B, keeps the smallest of several valid bounds, and rejects the GEMM with
// RNS8_RANGE_ERROR unless the largest cell bound fits the prefix (signed:
// 2*bound < P; unsigned: bound < P). The arithmetic is exact: 128-bit
// accumulators for the summaries, 256-bit for products, with cpp_int's
// truncation toward zero for the axis centers. Work is split over host
// threads by rows.
#include <algorithm>
#include <thread>
#include <vector>

#include "api_internal.hpp"

namespace rns8host {
namespace {

unsigned worker_count(int64_t units) {
  unsigned hw = std::thread::hardware_concurrency();
  if (hw == 0) hw = 4;
  if (hw > 32) hw = 32;
  const int64_t by_work = units / 4096 + 1;
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(hw, by_work)));
}

template <typename F>
void parallel_rows(int64_t rows, F&& body) {
  const unsigned workers = worker_count(rows * 64);
  if (workers <= 1) {
    body(0, rows, 0u);
    return;
  }
  std::vector<std::thread> pool;
  const int64_t chunk = (rows + workers - 1) / workers;
  for (unsigned w = 0; w < workers; ++w) {
    const int64_t r0 = w * chunk, r1 = std::min(rows, r0 + chunk);
    if (r0 >= r1) break;
    pool.emplace_back([&body, r0, r1, w] { body(r0, r1, w); });
  }
  for (auto& t : pool) t.join();
}

// 128-bit accumulation of one axis while scanning.
struct Acc {
  unsigned __int128 max_mag = 0, abs_sum = 0, dev_sum = 0;
  __int128 sum = 0, minimum = 0, maximum = 0;
  bool any = false;
  void add(__int128 v) {
    const unsigned __int128 mag = v < 0 ? static_cast<unsigned __int128>(-v) : static_cast<unsigned __int128>(v);
    if (mag > max_mag) max_mag = mag;
    abs_sum += mag;
    sum += v;
    if (!any) {
      minimum = maximum = v;
      any = true;
    } else {
      if (v < minimum) minimum = v;
      if (v > maximum) maximum = v;
    }
  }
  void merge(const Acc& o) {
    if (!o.any) return;
    if (o.max_mag > max_mag) max_mag = o.max_mag;
    abs_sum += o.abs_sum;
    sum += o.sum;
    dev_sum += o.dev_sum;
    if (!any) {
      minimum = o.minimum;
      maximum = o.maximum;
      any = true;
    } else {
      minimum = std::min(minimum, o.minimum);
      maximum = std::max(maximum, o.maximum);
    }
  }
  // (min + max) / 2 rounded toward zero.
  __int128 center() const { return (minimum + maximum) / 2; }
  AxisRange to_axis() const {
    AxisRange a;
    a.max_magnitude = i256::from_u128(max_mag);
    a.absolute_sum = i256::from_u128(abs_sum);
    a.sum = i256::from_i128(sum);
    a.minimum = i256::from_i128(minimum);
    a.maximum = i256::from_i128(maximum);
    a.deviation_sum = i256::from_u128(dev_sum);
    a.sum_known = any;
    return a;
  }
};

inline unsigned __int128 absdiff(__int128 a, __int128 b) {
  return a >= b ? static_cast<unsigned __int128>(a - b) : static_cast<unsigned __int128>(b - a);
}

i256 axis_center(const AxisRange& a) { return half_trunc(a.minimum + a.maximum); }
i256 axis_dev_max(const AxisRange& a, const i256& c) { return max(abs(a.minimum - c), abs(a.maximum - c)); }
void tighten(i256& bound, const i256& cand) {
  if (cand < bound) bound = cand;
}

// Per-axis quantities reused for every cell (exact_range.hpp:79-98).
struct AxisPre {
  const AxisRange* axis;
  i256 center, dev_max;
};
AxisPre precompute(const AxisRange& a) {
  AxisPre p;
  p.axis = &a;
  if (a.sum_known) {
    p.center = axis_center(a);
    p.dev_max = axis_dev_max(a, p.center);
  }
  return p;
}

i256 axis_product_bound(const AxisPre& pa, const AxisPre& pb, const i256& k) {
  const AxisRange& a = *pa.axis;
  const AxisRange& b = *pb.axis;
  i256 bound = k * a.max_magnitude * b.max_magnitude;
  tighten(bound, a.absolute_sum * b.max_magnitude);
  tighten(bound, a.max_magnitude * b.absolute_sum);
  if (a.sum_known && b.sum_known) {
    i256 rem = k * pa.dev_max * pb.dev_max;
    tighten(rem, a.deviation_sum * pb.dev_max);
    tighten(rem, pa.dev_max * b.deviation_sum);
    // dot(a,b) = ca*sum(b) + cb*sum(a) - K*ca*cb + dot(a-ca, b-cb)
    const i256 center_term = pa.center * b.sum + pb.center * a.sum - k * pa.center * pb.center;
    tighten(bound, abs(center_term) + rem);
  }
  return bound;
}

AxisRange uniform_axis(const i256& maximum, int64_t length) {
  AxisRange a;
  a.max_magnitude = maximum;
  a.absolute_sum = i256::from_i64(length) * maximum;
  a.sum_known = false;
  return a;
}

}  // namespace

bool exact_range_fits(rns8_semantics s, const i256& bound, const i256& product) {
  if (bound.neg()) return false;
  return s == RNS8_EXACT_WIDE_SIGNED ? (bound * i256::from_u64(2)) < product : bound < product;
}

template <typename T>
void native_exact_ranges(const T* src, int64_t rows, int64_t cols, int64_t ld, ExactRanges& out, i256& maximum) {
  std::vector<Acc> row_acc(static_cast<size_t>(rows));
  const unsigned workers = worker_count(rows * 64);
  std::vector<std::vector<Acc>> col_part(workers, std::vector<Acc>(static_cast<size_t>(cols)));
  parallel_rows(rows, [&](int64_t r0, int64_t r1, unsigned w) {
    auto& cp = col_part[w];
    for (int64_t r = r0; r < r1; ++r) {
      Acc& ra = row_acc[r];
      const T* line = src + r * ld;
      for (int64_t c = 0; c < cols; ++c) {
        const __int128 v = static_cast<__int128>(line[c]);
        ra.add(v);
        cp[c].add(v);
      }
    }
  });
  std::vector<Acc> col_acc(static_cast<size_t>(cols));
  for (auto& cp : col_part)
    for (int64_t c = 0; c < cols; ++c) col_acc[c].merge(cp[c]);
  // Second scan: L1 distance of every value from its row and column centers.
  for (auto& cp : col_part)
    for (auto& a : cp) a.dev_sum = 0;
  std::vector<__int128> col_center(static_cast<size_t>(cols));
  for (int64_t c = 0; c < cols; ++c) col_center[c] = col_acc[c].center();
  parallel_rows(rows, [&](int64_t r0, int64_t r1, unsigned w) {
    auto& cp = col_part[w];
    for (int64_t r = r0; r < r1; ++r) {
      Acc& ra = row_acc[r];
      const __int128 rc = ra.center();
      const T* line = src + r * ld;
      for (int64_t c = 0; c < cols; ++c) {
        const __int128 v = static_cast<__int128>(line[c]);
        ra.dev_sum += absdiff(v, rc);
        cp[c].dev_sum += absdiff(v, col_center[c]);
      }
    }
  });
  for (int64_t c = 0; c < cols; ++c) {
    unsigned __int128 d = 0;
    for (auto& cp : col_part) d += cp[c].dev_sum;
    col_acc[c].dev_sum = d;
  }
  out.rows.resize(static_cast<size_t>(rows));
  out.cols.resize(static_cast<size_t>(cols));
  unsigned __int128 best = 0;
  for (int64_t r = 0; r < rows; ++r) {
    out.rows[r] = row_acc[r].to_axis();
    best = std::max(best, row_acc[r].max_mag);
  }
  for (int64_t c = 0; c < cols; ++c) out.cols[c] = col_acc[c].to_axis();
  maximum = i256::from_u128(best);
}

template void native_exact_ranges<int64_t>(const int64_t*, int64_t, int64_t, int64_t, ExactRanges&, i256&);
template void native_exact_ranges<uint64_t>(const uint64_t*, int64_t, int64_t, int64_t, ExactRanges&, i256&);

// exact_gemm_bound + exact_gemm_range (exact_range.hpp:109-154).
rns8_status exact_gemm_range(const rns8_plan& plan, const rns8_matrix& A, const rns8_matrix& B, i256& bound,
                             ExactRanges* out_ranges) {
  if (!exact_wide(plan.desc.semantics)) return RNS8_SUCCESS;
  if (A.exact_range_prefix < plan.prefix || B.exact_range_prefix < plan.prefix) return RNS8_RANGE_ERROR;
  const int64_t m = plan.desc.m, n = plan.desc.n;
  const i256 k = i256::from_i64(plan.desc.k);
  const bool a_rows = A.exact_axes.rows.size() == static_cast<size_t>(m);
  const bool b_cols = B.exact_axes.cols.size() == static_cast<size_t>(n);
  bound = k * A.exact_max_magnitude * B.exact_max_magnitude;
  if (out_ranges) {
    out_ranges->rows.clear();
    out_ranges->cols.clear();
  }
  if (a_rows || b_cols) {
    const AxisRange fa = uniform_axis(A.exact_max_magnitude, plan.desc.k);
    const AxisRange fb = uniform_axis(B.exact_max_magnitude, plan.desc.k);
    std::vector<AxisPre> pa(static_cast<size_t>(m)), pb(static_cast<size_t>(n));
    for (int64_t r = 0; r < m; ++r) pa[r] = precompute(a_rows ? A.exact_axes.rows[r] : fa);
    for (int64_t c = 0; c < n; ++c) pb[c] = precompute(b_cols ? B.exact_axes.cols[c] : fb);
    const unsigned workers = worker_count(m * 64);
    std::vector<i256> part_max(workers);
    std::vector<std::vector<AxisRange>> col_part(out_ranges ? workers : 0, std::vector<AxisRange>(static_cast<size_t>(n)));
    if (out_ranges) out_ranges->rows.resize(static_cast<size_t>(m));
    parallel_rows(m, [&](int64_t r0, int64_t r1, unsigned w) {
      i256 best;
      for (int64_t r = r0; r < r1; ++r) {
        AxisRange rr;
        for (int64_t c = 0; c < n; ++c) {
          const i256 b = axis_product_bound(pa[r], pb[c], k);
          best = max(best, b);
          if (out_ranges) {
            rr.max_magnitude = max(rr.max_magnitude, b);
            rr.absolute_sum = rr.absolute_sum + b;
            AxisRange& cr = col_part[w][c];
            cr.max_magnitude = max(cr.max_magnitude, b);
            cr.absolute_sum = cr.absolute_sum + b;
          }
        }
        if (out_ranges) out_ranges->rows[r] = rr;
      }
      part_max[w] = best;
    });
    i256 maximum;
    for (const auto& v : part_max) maximum = max(maximum, v);
    if (out_ranges) {
      out_ranges->cols.resize(static_cast<size_t>(n));
      for (auto& cp : col_part)
        for (int64_t c = 0; c < n; ++c) {
          out_ranges->cols[c].max_magnitude = max(out_ranges->cols[c].max_magnitude, cp[c].max_magnitude);
          out_ranges->cols[c].absolute_sum = out_ranges->cols[c].absolute_sum + cp[c].absolute_sum;
        }
    }
    tighten(bound, maximum);
  }
  return exact_range_fits(plan.desc.semantics, bound, plan.modulus_product) ? RNS8_SUCCESS : RNS8_RANGE_ERROR;
}

void commit_exact_range(rns8_matrix& C, const rns8_plan& plan, i256& bound, ExactRanges* ranges) {
  if (!exact_wide(plan.desc.semantics)) return;
  C.exact_max_magnitude = bound;
  C.exact_axes.rows.clear();
  C.exact_axes.cols.clear();
  if (ranges) {
    C.exact_axes.rows.swap(ranges->rows);
    C.exact_axes.cols.swap(ranges->cols);
  }
  C.exact_range_prefix = plan.prefix;
}

}  // namespace rns8host
