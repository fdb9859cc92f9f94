// Shared declarations between the plane-GEMM implementations.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "kernels.hpp"

namespace rns8cuda {

struct PlaneModuli {
  uint16_t m[20];
};

cudaError_t simt_plane_gemm(const PlaneGemmProblem& prob, cudaStream_t stream);

// Narrow outputs (1 <= n < 16): B^T staging in scratch, then a dp4a stream
// over A's planes (gemm_skinny.cu).
bool skinny_path_supported(const PlaneGemmProblem& prob);
uint64_t skinny_scratch_bytes(const PlaneGemmProblem& prob);
cudaError_t skinny_plane_gemm(const PlaneGemmProblem& prob, void* scratch, uint64_t scratch_bytes,
                              cudaStream_t stream,
                              int sm_count_hint);

// Split-K decomposition chosen for the tensor-core kernel.
struct TcSchedule {
  uint32_t m_tiles, n_tiles, total_kb, splits, kb_per_split;
  uint64_t units;
};
TcSchedule tc_schedule(const PlaneGemmProblem& prob, int sm_count);

// Scheduled (per-tile prefix) runs of the tensor-core kernel: the explicit
// unit list and the per-schedule-tile mask, both in device memory.
struct TcScheduleUnits {
  const uint64_t* units_dev;
  uint64_t unit_count;
  const uint8_t* tile_sel_dev;
  uint32_t shift_m, shift_n, cols;
};
// A proven-zero schedule tile: planes [0, planes) of its cells are zero.
struct ZeroTile {
  int64_t row0, col0, rows, cols;
  uint32_t planes, pad;
};
// With `scatter`, C's rows go to the slab destinations instead of tasks[0].c
// (one task, no split-K).
cudaError_t tc_plane_gemm(const PlaneGemmProblem& prob, int sm_count, void* scratch, uint64_t scratch_bytes,
                          uint32_t* dev_status, cudaStream_t stream, const TcScheduleUnits* sched = nullptr,
                          const SlabScatter* scatter = nullptr);

// wrap64 on the tensor cores: c (m x n uint64, row-major) = A x B mod 2^64 from
// 8 byte planes each (k % 16 == 0, n % 16 == 0, 16-byte aligned planes).
bool tma_encode_available();
// Compact residue planes [plane_count][cells] as a (cell in chunk, plane,
// 128-cell chunk) byte tensor with the 128-byte swizzle; a box is box_chunks
// consecutive chunks of box_rows planes (a multiple of 8, at most 32; planes
// past plane_count read as zero), chunk-major. Needs 16-byte aligned planes
// and cells % 128 == 0.
bool encode_plane_cells(CUtensorMap* map, const void* planes, uint64_t cells, uint32_t plane_count,
                        uint32_t box_rows, uint32_t box_chunks);
cudaError_t tc_wrap64_gemm(const uint8_t* a_limbs, const uint8_t* b_limbs, uint64_t* c, int64_t m, int64_t n,
                           int64_t k, int sm_count, uint32_t* dev_status, cudaStream_t stream);

}  // namespace rns8cuda
