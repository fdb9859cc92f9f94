// Internal launch API of the sm_100a kernels. Every function enqueues work on
// `stream` and returns the launch's cudaError_t; none synchronises. Pointers
// are device pointers. Residue planes are modulus-major and compact:
// plane p of an R x C matrix holds int8 centered residues at
// base[p * R * C + r * C + c].
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace rns8cuda {

// Maximum number of same-shape tasks one grouped plane-GEMM launch covers.
constexpr int kMaxGroupTasks = 32;

// Error codes kernels OR into their device status word.
constexpr uint32_t kDevOk = 0;
constexpr uint32_t kDevRangeError = 5;       // == RNS8_RANGE_ERROR
constexpr uint32_t kDevWaitTimeout = 0x100;  // a bounded device wait ran out

// ---- pack (native -> centered int8 residue planes) ------------------------
// *out = the largest |x| over count contiguous int64 (is_signed) or uint64
// values; *out must be 8-byte aligned device memory.
cudaError_t max_magnitude(const void* src, int64_t count, bool is_signed, uint64_t* out, int sm_count,
                          cudaStream_t stream);
cudaError_t pack_i64(const int64_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* planes,
                     cudaStream_t stream);
cudaError_t pack_u64(const uint64_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* planes,
                     cudaStream_t stream);
cudaError_t pack_finite_u8(const uint8_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t modulus,
                           int8_t* residues, cudaStream_t stream);

// Pack of selected planes only: plane j of `planes` holds the residues modulo
// ladder entry plane_index[j] (host array, plane_count entries, each < 20).
// A GPU that computes a subset of the planes (plane sharding) packs just those.
cudaError_t pack_planes_i64(const int64_t* src, int64_t rows, int64_t cols, int64_t ld, const uint32_t* plane_index,
                            uint32_t plane_count, int8_t* planes, cudaStream_t stream);
cudaError_t pack_planes_u64(const uint64_t* src, int64_t rows, int64_t cols, int64_t ld, const uint32_t* plane_index,
                            uint32_t plane_count, int8_t* planes, cudaStream_t stream);

// ---- plane GEMM -------------------------------------------------------------
// One GEMM family: tasks[t] x planes[p]; every plane of every task has the
// same shape. Plane p reduces modulo moduli[p].
struct PlaneGemmTask {
  const int8_t* a;  // plane 0 of A (m x k), planes at stride m*k
  const int8_t* b;  // plane 0 of B (k x n), planes at stride k*n
  int8_t* c;        // plane 0 of C (m x n), planes at stride m*n
};
struct PlaneGemmProblem {
  int64_t m, n, k;
  uint32_t planes;
  uint16_t moduli[20];
  uint32_t task_count;
  const PlaneGemmTask* tasks;  // host array of task_count entries
};
enum class GemmPath : int { Auto = 0, TensorCore = 1, Simt = 2 };

// Per-tile prefix schedule of a plan (reference api_plan_schedule.inc:109-261)
// for scheduled GEMM and export: tile_sel[tile_row * tile_cols + tile_col] is
// the tile's selected prefix, | 0x80 when its output is proven zero.
struct PlaneSchedule {
  uint32_t tile_m, tile_n;  // powers of two in [64, 512]
  uint64_t tile_rows, tile_cols;
  const uint8_t* tile_sel;  // host array
};
// Plane GEMM of one task under a schedule (cpu_reference.cpp:221-260): each
// schedule tile gets the planes below its selected prefix; proven-zero tiles
// are zero-filled there; planes at or above a tile's prefix are not written.
uint64_t plane_gemm_scheduled_scratch_bytes(const PlaneGemmProblem& prob, const PlaneSchedule& sched, int sm_count);
cudaError_t plane_gemm_scheduled(const PlaneGemmProblem& prob, const PlaneSchedule& sched, int sm_count,
                                 void* scratch, uint64_t scratch_bytes, uint32_t* dev_status, cudaStream_t stream);
// Bounded export under a per-tile schedule (api_export.cpp:365-414): each
// cell is reconstructed from its tile's selected prefix and checked against
// its tile's bound (tile_bounds, host array); proven-zero tiles export 0.
// dst is uint64 m x n (ld = n); range errors are ORed into *dev_status.
uint64_t export_scheduled_scratch_bytes(const PlaneSchedule& sched);
cudaError_t export_scheduled(const int8_t* planes, int64_t m, int64_t n, bool is_signed, const PlaneSchedule& sched,
                             const uint64_t* tile_bounds, void* dst, uint32_t* dev_status, void* scratch,
                             uint64_t scratch_bytes, cudaStream_t stream);

// Scratch the tensor-core path needs for split-K (int32 per output element
// of the largest chunk). Returns 0 when the problem runs without split-K.
uint64_t plane_gemm_scratch_bytes(const PlaneGemmProblem& prob, int sm_count);
// Runs the plane GEMM. scratch may be null when plane_gemm_scratch_bytes()
// is 0. dev_status receives kDevWaitTimeout if a bounded wait ran out.
cudaError_t plane_gemm(const PlaneGemmProblem& prob, GemmPath path, int sm_count, void* scratch,
                       uint64_t scratch_bytes, uint32_t* dev_status, cudaStream_t stream, GemmPath* used = nullptr);
bool tensor_core_path_supported(const PlaneGemmProblem& prob);

// Plane GEMM into scratch planes followed by export_i64/u64 (one task).
// scratch must hold gemm_export_bounded_scratch_bytes().
uint64_t gemm_export_bounded_scratch_bytes(const PlaneGemmProblem& prob, int sm_count);
cudaError_t gemm_export_bounded(const PlaneGemmProblem& prob, bool is_signed, uint64_t bound, void* out, int64_t ld,
                                int sm_count, void* scratch, uint64_t scratch_bytes, uint32_t* dev_status,
                                cudaStream_t stream);

// Plane GEMM whose output rows are split into row slabs, each slab going to
// its own destination (this GPU's memory or a peer GPU's, mapped into this
// process): the plane-sharded exchange, where every GPU computes some planes
// of all of C and every GPU then needs all planes of its own row slab.
// Slab s covers rows [s * slab_rows, min(m, (s + 1) * slab_rows)); its
// destination holds planes at stride rows_s * n, and local plane p lands in
// plane slot dst_plane[p]. Fused: the GEMM epilogue stores straight into the
// destinations (peer stores over NVLink, ordered by a system fence before the
// kernel completes). Copy: the GEMM writes local planes into scratch and one
// device-to-device copy per (plane, slab) moves them. The fused form needs the
// tensor-core path without split-K; otherwise the copy form runs.
constexpr int kMaxSlabs = 8;
struct SlabScatter {
  int8_t* const* slab_dst;    // host array of slab_count device pointers
  int64_t slab_rows;
  uint32_t slab_count;
  const uint32_t* dst_plane;  // host array, one plane slot per local plane
};
bool plane_gemm_scatter_fusable(const PlaneGemmProblem& prob, int sm_count);
uint64_t plane_gemm_scatter_scratch_bytes(const PlaneGemmProblem& prob, int sm_count, bool copy_exchange);
cudaError_t plane_gemm_scatter(const PlaneGemmProblem& prob, const SlabScatter& scatter, bool copy_exchange,
                               int sm_count, void* scratch, uint64_t scratch_bytes, uint32_t* dev_status,
                               cudaStream_t stream, bool* fused_used = nullptr);

// ---- export (residue planes -> native values) ------------------------------
// Bounded i64: every cell must reconstruct to a value v with |v| <= bound;
// otherwise *dev_status is set to kDevRangeError (dst contents unspecified).
cudaError_t export_i64(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, uint64_t bound, int64_t* dst,
                       int64_t ld, uint32_t* dev_status, cudaStream_t stream);
cudaError_t export_u64(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, uint64_t bound, uint64_t* dst,
                       int64_t ld, uint32_t* dev_status, cudaStream_t stream);
// Exact-wide: limb_count 64-bit limbs per element at dst[(r*ld + c)*limbs + l].
cudaError_t export_limbs(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, bool is_signed,
                         uint32_t limb_count, uint64_t* dst, int64_t ld, uint32_t* dev_status, cudaStream_t stream);
cudaError_t export_finite_u8(const int8_t* residues, int64_t m, int64_t n, uint32_t modulus, uint8_t* dst, int64_t ld,
                             cudaStream_t stream);

// ---- WRAP_U64_MOD_2_64 (reference src/backend_wrap64/) -----------------------------
// uint64 (row-major, ld >= cols) -> 8 limb-major byte planes [8][rows][cols].
cudaError_t wrap_pack_u64(const uint64_t* src, int64_t rows, int64_t cols, int64_t ld, uint8_t* planes,
                          cudaStream_t stream);
// 8 byte planes -> uint64 dst[row * ld + col].
cudaError_t wrap_export_u64(const uint8_t* planes, int64_t rows, int64_t cols, uint64_t* dst, int64_t ld,
                            cudaStream_t stream);
bool wrap_tensor_core_supported(const uint8_t* a, const uint8_t* b, const uint64_t* c, int64_t m, int64_t n,
                                int64_t k);
// c (m x n uint64, compact row-major) = A x B mod 2^64 from byte planes. The
// tensor-core path ORs kDevWaitTimeout into *dev_status if a wait runs out.
cudaError_t wrap_gemm(const uint8_t* a_limbs, const uint8_t* b_limbs, uint64_t* c, int64_t m, int64_t n, int64_t k,
                      GemmPath path, int sm_count, uint32_t* dev_status, cudaStream_t stream,
                      GemmPath* used = nullptr);

// ---- exact-wide admission (reference src/core/exact_range.hpp:51-154) ------------
// Summary of one row or column of native int64/uint64 values: max |v|, sum |v|,
// sum v, min, max and sum |v - center| with center = (min + max) / 2
// truncated toward zero. 128-bit fields hold sums of up to 2^63 values.
struct AxisSummary {
  unsigned __int128 max_mag, abs_sum, dev_sum;
  __int128 sum, minimum, maximum;
  uint64_t any;
  uint64_t pad;
};
// Scratch for axis_summaries on a rows x cols matrix.
uint64_t axis_summaries_scratch_bytes(int64_t rows, int64_t cols);
// Row and column summaries of a compact (ld == cols) int64 (is_signed) or
// uint64 matrix in device memory into d_rows[rows] and d_cols[cols].
cudaError_t axis_summaries(const void* src, bool is_signed, int64_t rows, int64_t cols, AxisSummary* d_rows,
                           AxisSummary* d_cols, void* scratch, uint64_t scratch_bytes, cudaStream_t stream);

// Per-axis inputs of the cell bound (exact_range.hpp:79-98), 256-bit
// little-endian two's complement limbs.
struct AxisBoundInput {
  uint64_t max_mag[4], abs_sum[4], sum[4], center[4], dev_max[4], dev_sum[4];
  uint64_t sum_known;
};
// Maximum and sum of the cell bounds along one output row or column.
struct BoundStats {
  uint64_t max[4];
  uint64_t sum[4];
};
uint64_t cell_bounds_scratch_bytes(int64_t m, int64_t n);
// For every output cell (r, c) of an m x n exact-wide product with inner
// dimension k, the smallest of the admission bounds of row r of A and
// column c of B; d_row_stats[m] and d_col_stats[n] receive their maxima and
// sums along rows and columns.
cudaError_t cell_bounds(const AxisBoundInput* d_rows, int64_t m, const AxisBoundInput* d_cols, int64_t n, int64_t k,
                        BoundStats* d_row_stats, BoundStats* d_col_stats, void* scratch, uint64_t scratch_bytes,
                        cudaStream_t stream);

}  // namespace rns8cuda
