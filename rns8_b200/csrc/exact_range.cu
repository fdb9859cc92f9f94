// Exact-wide admission proofs on the device (reference
// src/core/exact_range.hpp:51-154).
//
// Packing an exact-wide matrix summarises every row and column of its native
// values; a GEMM bounds every output cell from the summaries of its row of A
// and column of B. Both are exact integer reductions (max and sum of 128- and
// 256-bit values), so the order in which the device combines partial results
// does not change them: they equal the reference's cpp_int results.
//
//   axis_summaries: two passes over the matrix. Pass 1 gives max |v|, sum |v|,
//     sum v, min and max per row (one warp per row) and per column (one
//     thread per column over a chunk of rows, then a reduction over chunks);
//     pass 2 gives sum |v - center| around the centers from pass 1.
//   cell_bounds: one thread per output column of a 256-column tile, looping
//     over the rows given to its block; each cell bound is folded into the
//     thread's column maximum and sum and, by a warp and block reduction,
//     into per-tile row partials that a second kernel combines.
#include "kernels.hpp"
#include "wide_int.hpp"

namespace rns8cuda {
namespace {

using u128 = unsigned __int128;
using i128 = __int128;
using rns8host::i256;

static_assert(sizeof(AxisSummary) == 112, "AxisSummary layout is shared with host code");

// ---- axis summaries -------------------------------------------------------------
struct Acc {
  u128 max_mag, abs_sum, dev_sum;
  i128 sum, mn, mx;
  bool any;
};

__device__ __forceinline__ Acc acc_zero() {
  Acc a;
  a.max_mag = a.abs_sum = a.dev_sum = 0;
  a.sum = a.mn = a.mx = 0;
  a.any = false;
  return a;
}

__device__ __forceinline__ void acc_add(Acc& a, i128 v) {
  const u128 mag = v < 0 ? static_cast<u128>(-v) : static_cast<u128>(v);
  if (mag > a.max_mag) a.max_mag = mag;
  a.abs_sum += mag;
  a.sum += v;
  if (!a.any) {
    a.mn = a.mx = v;
    a.any = true;
  } else {
    if (v < a.mn) a.mn = v;
    if (v > a.mx) a.mx = v;
  }
}

__device__ __forceinline__ void acc_merge(Acc& a, const Acc& o) {
  if (!o.any) return;
  if (o.max_mag > a.max_mag) a.max_mag = o.max_mag;
  a.abs_sum += o.abs_sum;
  a.sum += o.sum;
  a.dev_sum += o.dev_sum;
  if (!a.any) {
    a.mn = o.mn;
    a.mx = o.mx;
    a.any = true;
  } else {
    if (o.mn < a.mn) a.mn = o.mn;
    if (o.mx > a.mx) a.mx = o.mx;
  }
}

__device__ __forceinline__ u128 shfl_down_u128(u128 v, int off) {
  const uint64_t lo = __shfl_down_sync(0xFFFFFFFFu, static_cast<uint64_t>(v), off);
  const uint64_t hi = __shfl_down_sync(0xFFFFFFFFu, static_cast<uint64_t>(v >> 64), off);
  return (static_cast<u128>(hi) << 64) | lo;
}

__device__ __forceinline__ Acc warp_reduce(Acc a) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Acc o;
    o.max_mag = shfl_down_u128(a.max_mag, off);
    o.abs_sum = shfl_down_u128(a.abs_sum, off);
    o.dev_sum = shfl_down_u128(a.dev_sum, off);
    o.sum = static_cast<i128>(shfl_down_u128(static_cast<u128>(a.sum), off));
    o.mn = static_cast<i128>(shfl_down_u128(static_cast<u128>(a.mn), off));
    o.mx = static_cast<i128>(shfl_down_u128(static_cast<u128>(a.mx), off));
    o.any = __shfl_down_sync(0xFFFFFFFFu, a.any ? 1 : 0, off) != 0;
    acc_merge(a, o);
  }
  return a;
}

__device__ __forceinline__ u128 absdiff(i128 a, i128 b) {
  return a >= b ? static_cast<u128>(a - b) : static_cast<u128>(b - a);
}

// (min + max) / 2 rounded toward zero, as cpp_int division does.
__device__ __forceinline__ i128 center_of(const AxisSummary& s) { return (s.minimum + s.maximum) / 2; }

__device__ __forceinline__ void store(AxisSummary& s, const Acc& a) {
  s.max_mag = a.max_mag;
  s.abs_sum = a.abs_sum;
  s.dev_sum = a.dev_sum;
  s.sum = a.sum;
  s.minimum = a.mn;
  s.maximum = a.mx;
  s.any = a.any ? 1 : 0;
  s.pad = 0;
}

__device__ __forceinline__ Acc load(const AxisSummary& s) {
  Acc a;
  a.max_mag = s.max_mag;
  a.abs_sum = s.abs_sum;
  a.dev_sum = s.dev_sum;
  a.sum = s.sum;
  a.mn = s.minimum;
  a.mx = s.maximum;
  a.any = s.any != 0;
  return a;
}

// One warp per row. Pass 1 writes the row's summary; pass 2 adds the
// deviation sum around the row's center.
template <typename T, bool kDeviation>
__global__ void __launch_bounds__(256) row_summary_kernel(const T* __restrict__ src, int64_t rows, int64_t cols,
                                                          AxisSummary* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const T* line = src + r * cols;
    if constexpr (!kDeviation) {
      Acc a = acc_zero();
      for (int64_t c = lane; c < cols; c += 32) acc_add(a, static_cast<i128>(line[c]));
      a = warp_reduce(a);
      if (lane == 0) store(out[r], a);
    } else {
      const i128 center = center_of(out[r]);
      u128 d = 0;
      for (int64_t c = lane; c < cols; c += 32) d += absdiff(static_cast<i128>(line[c]), center);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) d += shfl_down_u128(d, off);
      if (lane == 0) out[r].dev_sum = d;
    }
  }
}

// One thread per column over rows [chunk * rows_per_chunk, ...): partial
// summaries (pass 1) or partial deviation sums (pass 2) per chunk.
template <typename T, bool kDeviation>
__global__ void __launch_bounds__(256) col_partial_kernel(const T* __restrict__ src, int64_t rows, int64_t cols,
                                                          int64_t rows_per_chunk, const AxisSummary* __restrict__ cols_final,
                                                          AxisSummary* __restrict__ part) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_chunk;
  const int64_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  AxisSummary& p = part[static_cast<int64_t>(blockIdx.y) * cols + c];
  if constexpr (!kDeviation) {
    Acc a = acc_zero();
#pragma unroll 4
    for (int64_t r = r0; r < r1; ++r) acc_add(a, static_cast<i128>(src[r * cols + c]));
    store(p, a);
  } else {
    const i128 center = center_of(cols_final[c]);
    u128 d = 0;
#pragma unroll 4
    for (int64_t r = r0; r < r1; ++r) d += absdiff(static_cast<i128>(src[r * cols + c]), center);
    p.dev_sum = d;
  }
}

template <bool kDeviation>
__global__ void __launch_bounds__(256) col_reduce_kernel(const AxisSummary* __restrict__ part, int64_t chunks,
                                                         int64_t cols, AxisSummary* __restrict__ out) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  if constexpr (!kDeviation) {
    Acc a = acc_zero();
    for (int64_t ch = 0; ch < chunks; ++ch) acc_merge(a, load(part[ch * cols + c]));
    a.dev_sum = 0;
    store(out[c], a);
  } else {
    u128 d = 0;
    for (int64_t ch = 0; ch < chunks; ++ch) d += part[ch * cols + c].dev_sum;
    out[c].dev_sum = d;
  }
}

// Chunks of rows for the column partials: at least 256 rows each, at most
// 64 chunks, and at most 256 MiB of partials.
int64_t summary_chunks(int64_t rows, int64_t cols) {
  int64_t c = (rows + 255) / 256;
  const int64_t budget = (int64_t{256} << 20) / (cols * static_cast<int64_t>(sizeof(AxisSummary)));
  if (c > budget) c = budget;
  if (c > 64) c = 64;
  if (c < 1) c = 1;
  return c;
}

template <typename T>
cudaError_t launch_summaries(const T* src, int64_t rows, int64_t cols, AxisSummary* d_rows, AxisSummary* d_cols,
                             AxisSummary* part, cudaStream_t stream) {
  const int64_t chunks = summary_chunks(rows, cols);
  const int64_t per_chunk = (rows + chunks - 1) / chunks;
  int64_t row_blocks = (rows * 32 + 255) / 256;
  if (row_blocks > 148 * 16) row_blocks = 148 * 16;
  const dim3 col_grid(static_cast<unsigned>((cols + 255) / 256), static_cast<unsigned>(chunks));
  const unsigned col_blocks = static_cast<unsigned>((cols + 255) / 256);
  row_summary_kernel<T, false><<<static_cast<unsigned>(row_blocks), 256, 0, stream>>>(src, rows, cols, d_rows);
  col_partial_kernel<T, false><<<col_grid, 256, 0, stream>>>(src, rows, cols, per_chunk, nullptr, part);
  col_reduce_kernel<false><<<col_blocks, 256, 0, stream>>>(part, chunks, cols, d_cols);
  row_summary_kernel<T, true><<<static_cast<unsigned>(row_blocks), 256, 0, stream>>>(src, rows, cols, d_rows);
  col_partial_kernel<T, true><<<col_grid, 256, 0, stream>>>(src, rows, cols, per_chunk, d_cols, part);
  col_reduce_kernel<true><<<col_blocks, 256, 0, stream>>>(part, chunks, cols, d_cols);
  return cudaGetLastError();
}

// ---- cell bounds ----------------------------------------------------------------
constexpr int kBoundRows = 32;  // rows staged per block iteration

__device__ __forceinline__ i256 ld256(const uint64_t (&w)[4]) {
  i256 r;
  r.w[0] = w[0];
  r.w[1] = w[1];
  r.w[2] = w[2];
  r.w[3] = w[3];
  return r;
}

__device__ __forceinline__ void tighten(i256& bound, const i256& cand) {
  if (cand < bound) bound = cand;
}

// exact_range.hpp:79-98: the smallest of the product bounds of one row of A
// and one column of B, and (when both sums are known) of the centered
// decomposition dot(a, b) = ca*sum(b) + cb*sum(a) - K*ca*cb + dot(a-ca, b-cb).
__device__ i256 cell_bound(const AxisBoundInput& a, const AxisBoundInput& b, const i256& k) {
  const i256 amax = ld256(a.max_mag), bmax = ld256(b.max_mag);
  i256 bound = k * amax * bmax;
  tighten(bound, ld256(a.abs_sum) * bmax);
  tighten(bound, amax * ld256(b.abs_sum));
  if (a.sum_known && b.sum_known) {
    const i256 adev = ld256(a.dev_max), bdev = ld256(b.dev_max);
    i256 rem = k * adev * bdev;
    tighten(rem, ld256(a.dev_sum) * bdev);
    tighten(rem, adev * ld256(b.dev_sum));
    const i256 ca = ld256(a.center), cb = ld256(b.center);
    const i256 center_term = ca * ld256(b.sum) + cb * ld256(a.sum) - k * ca * cb;
    tighten(bound, rns8host::abs(center_term) + rem);
  }
  return bound;
}

__device__ __forceinline__ i256 shfl_down_i256(const i256& v, int off) {
  i256 r;
#pragma unroll
  for (int l = 0; l < 4; ++l) r.w[l] = __shfl_down_sync(0xFFFFFFFFu, v.w[l], off);
  return r;
}

__device__ __forceinline__ void put(BoundStats& s, const i256& mx, const i256& sum) {
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    s.max[l] = mx.w[l];
    s.sum[l] = sum.w[l];
  }
}

// grid.x: 256-column tiles of the stripe [c0, c0 + width); grid.y: row
// groups (block y takes rows y*32.., then every gridDim.y*32 rows).
// row_part[tile][m], col_part[grid.y][width]. Cell bounds are >= 0, so zero
// is neutral for both the maximum and the sum (columns past the stripe).
__global__ void __launch_bounds__(256) cell_bounds_kernel(const AxisBoundInput* __restrict__ rows_in, int64_t m,
                                                          const AxisBoundInput* __restrict__ cols_in, int64_t c0,
                                                          int64_t width, i256 k, BoundStats* __restrict__ row_part,
                                                          BoundStats* __restrict__ col_part) {
  __shared__ AxisBoundInput srow[kBoundRows];
  __shared__ BoundStats swarp[kBoundRows][8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t cl = static_cast<int64_t>(blockIdx.x) * 256 + tid;
  const bool valid = cl < width;
  const AxisBoundInput* col = cols_in + c0 + (valid ? cl : 0);
  i256 cmax, csum;
  for (int64_t rb = static_cast<int64_t>(blockIdx.y) * kBoundRows; rb < m;
       rb += static_cast<int64_t>(gridDim.y) * kBoundRows) {
    const int rcount = m - rb < kBoundRows ? static_cast<int>(m - rb) : kBoundRows;
    __syncthreads();
    if (tid < rcount) srow[tid] = rows_in[rb + tid];
    __syncthreads();
    for (int i = 0; i < rcount; ++i) {
      i256 b;
      if (valid) b = cell_bound(srow[i], *col, k);
      cmax = rns8host::max(cmax, b);
      csum = csum + b;
      i256 wmax = b, wsum = b;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        wmax = rns8host::max(wmax, shfl_down_i256(wmax, off));
        wsum = wsum + shfl_down_i256(wsum, off);
      }
      if (lane == 0) put(swarp[i][warp], wmax, wsum);
    }
    __syncthreads();
    if (tid < rcount) {
      i256 mx, sm;
      for (int w = 0; w < 8; ++w) {
        mx = rns8host::max(mx, ld256(swarp[tid][w].max));
        sm = sm + ld256(swarp[tid][w].sum);
      }
      put(row_part[static_cast<int64_t>(blockIdx.x) * m + rb + tid], mx, sm);
    }
  }
  if (valid) put(col_part[static_cast<int64_t>(blockIdx.y) * width + cl], cmax, csum);
}

__global__ void __launch_bounds__(256) row_stats_kernel(const BoundStats* __restrict__ row_part, int64_t tiles,
                                                        int64_t m, bool first, BoundStats* __restrict__ row_stats) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= m) return;
  i256 mx, sm;
  if (!first) {
    mx = ld256(row_stats[r].max);
    sm = ld256(row_stats[r].sum);
  }
  for (int64_t t = 0; t < tiles; ++t) {
    mx = rns8host::max(mx, ld256(row_part[t * m + r].max));
    sm = sm + ld256(row_part[t * m + r].sum);
  }
  put(row_stats[r], mx, sm);
}

__global__ void __launch_bounds__(256) col_stats_kernel(const BoundStats* __restrict__ col_part, int64_t groups,
                                                        int64_t width, BoundStats* __restrict__ col_stats) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= width) return;
  i256 mx, sm;
  for (int64_t g = 0; g < groups; ++g) {
    mx = rns8host::max(mx, ld256(col_part[g * width + c].max));
    sm = sm + ld256(col_part[g * width + c].sum);
  }
  put(col_stats[c], mx, sm);
}

// Columns per launch: row partials (width/256 per row) stay below about
// 1 GiB / 64; at least one tile, at most 8192 columns.
int64_t stripe_width(int64_t m, int64_t n) {
  int64_t s = (int64_t{1} << 30) / (64 * (m > 0 ? m : 1)) * 256;
  if (s > 8192) s = 8192;
  if (s < 256) s = 256;
  const int64_t n_up = (n + 255) / 256 * 256;
  return s < n_up ? s : n_up;
}

int64_t row_groups(int64_t m) {
  const int64_t g = (m + kBoundRows - 1) / kBoundRows;
  return g < 64 ? g : 64;
}

}  // namespace

uint64_t axis_summaries_scratch_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return static_cast<uint64_t>(summary_chunks(rows, cols)) * cols * sizeof(AxisSummary);
}

cudaError_t axis_summaries(const void* src, bool is_signed, int64_t rows, int64_t cols, AxisSummary* d_rows,
                           AxisSummary* d_cols, void* scratch, uint64_t scratch_bytes, cudaStream_t stream) {
  if (rows <= 0 || cols <= 0 || !src || !d_rows || !d_cols) return cudaErrorInvalidValue;
  if (scratch_bytes < axis_summaries_scratch_bytes(rows, cols) || !scratch) return cudaErrorInvalidValue;
  auto* part = static_cast<AxisSummary*>(scratch);
  return is_signed ? launch_summaries(static_cast<const int64_t*>(src), rows, cols, d_rows, d_cols, part, stream)
                   : launch_summaries(static_cast<const uint64_t*>(src), rows, cols, d_rows, d_cols, part, stream);
}

uint64_t cell_bounds_scratch_bytes(int64_t m, int64_t n) {
  if (m <= 0 || n <= 0) return 0;
  const int64_t s = stripe_width(m, n);
  return (static_cast<uint64_t>(s / 256) * m + static_cast<uint64_t>(row_groups(m)) * s) * sizeof(BoundStats);
}

cudaError_t cell_bounds(const AxisBoundInput* d_rows, int64_t m, const AxisBoundInput* d_cols, int64_t n, int64_t k,
                        BoundStats* d_row_stats, BoundStats* d_col_stats, void* scratch, uint64_t scratch_bytes,
                        cudaStream_t stream) {
  if (m <= 0 || n <= 0 || k <= 0 || !d_rows || !d_cols || !d_row_stats || !d_col_stats) return cudaErrorInvalidValue;
  if (!scratch || scratch_bytes < cell_bounds_scratch_bytes(m, n)) return cudaErrorInvalidValue;
  const int64_t s = stripe_width(m, n);
  const int64_t groups = row_groups(m);
  auto* row_part = static_cast<BoundStats*>(scratch);
  BoundStats* col_part = row_part + (s / 256) * m;
  const i256 kk = i256::from_i64(k);
  for (int64_t c0 = 0; c0 < n; c0 += s) {
    const int64_t width = n - c0 < s ? n - c0 : s;
    const int64_t tiles = (width + 255) / 256;
    cell_bounds_kernel<<<dim3(static_cast<unsigned>(tiles), static_cast<unsigned>(groups)), 256, 0, stream>>>(
        d_rows, m, d_cols, c0, width, kk, row_part, col_part);
    row_stats_kernel<<<static_cast<unsigned>((m + 255) / 256), 256, 0, stream>>>(row_part, tiles, m, c0 == 0,
                                                                                 d_row_stats);
    col_stats_kernel<<<static_cast<unsigned>((width + 255) / 256), 256, 0, stream>>>(col_part, groups, width,
                                                                                     d_col_stats + c0);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace rns8cuda
