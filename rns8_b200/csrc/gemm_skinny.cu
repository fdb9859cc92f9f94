// Narrow plane GEMM: C_p = (A_p x B_p) mod m_p for outputs fewer than 16
// columns wide (GEMV-like shapes, reference hip_direct_gemm_tiled_kernels.cuh:
// 298-434 serves them with dedicated small tiles). The work is a stream over
// A's planes, so the kernel is built to read A once at full width:
//
//   pass 1  each B plane is transposed into B^T (NP x Kp bytes, NP = n rounded
//           up to 4, 8 or 16 with zero rows, Kp = K rounded up to 16 with zero
//           columns) in scratch, so that 16 consecutive k of one column are one
//           16-byte word;
//   pass 2  one warp per 4 rows of A: each lane loads 16 bytes of each row and
//           the matching 16 bytes of every B^T row (L1-resident), and folds
//           them with dp4a into 4 x NP int32 sums. Every 65536 products the
//           warp adds its lanes' sums and reduces them to centered residues
//           (|sum| <= 65536 * 128 * 128 = 2^30 stays exact in int32), and the
//           residues of the segments are summed and reduced at the end. Sums of
//           per-block residues are congruent to the reference's folded running
//           residue (cpu_reference.cpp:171-174), so the bytes are identical.
#include "device_common.cuh"
#include <algorithm>

#include "gemm_internal.hpp"

namespace rns8cuda {
namespace {

constexpr int64_t kSegment = 65536;  // products per exact int32 segment

// Rows per warp: every B^T word loaded serves R rows; 16 columns keep 2 rows
// so that the R x NP sums and residues stay in registers.
template <int NP>
constexpr int rows_per_warp() { return NP == 16 ? 2 : 4; }

__global__ void __launch_bounds__(256) transpose_b_kernel(const int8_t* __restrict__ b, int64_t k, int64_t n,
                                                          uint32_t np, int64_t kp, int8_t* __restrict__ bt) {
  const uint32_t p = blockIdx.y;
  const int8_t* src = b + static_cast<int64_t>(p) * k * n;
  int8_t* dst = bt + static_cast<int64_t>(p) * np * kp;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < static_cast<int64_t>(np) * kp;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = i / kp, kk = i - j * kp;
    dst[i] = (j < n && kk < k) ? src[kk * n + j] : int8_t{0};
  }
}

struct SkinnyParams {
  const int8_t* a;
  const int8_t* bt;  // B^T planes, np x kp each
  int8_t* c;
  int64_t m, n, k, kp;
  PlaneModuli moduli;
};

__device__ __forceinline__ int32_t warp_sum(int32_t v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
  return v;
}

// Four bytes of A at row r, k..k+3 (zero past K or past the last row).
__device__ __forceinline__ uint32_t load_a4(const int8_t* a, int64_t k_total, int64_t kk, bool row_ok) {
  if (!row_ok) return 0;
  uint32_t w = 0;
#pragma unroll
  for (int q = 0; q < 4; ++q)
    if (kk + q < k_total) w |= (static_cast<uint32_t>(static_cast<uint8_t>(a[kk + q])) << (8 * q));
  return w;
}

// kVec: K % 16 == 0 and 16-byte aligned planes: each lane takes 16 bytes of
// a row per step. Otherwise 4 bytes per step with bounds checks.
template <int NP, bool kVec>
__global__ void __launch_bounds__(256) skinny_kernel(const SkinnyParams prm) {
  constexpr int R = rows_per_warp<NP>();
  constexpr int kRowsPerBlock = R * 8;  // 8 warps
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t p = blockIdx.y;
  const int64_t m = prm.m, n = prm.n, k = prm.k, kp = prm.kp;
  const int8_t* a = prm.a + static_cast<int64_t>(p) * m * k;
  const int8_t* bt = prm.bt + static_cast<int64_t>(p) * NP * kp;
  int8_t* c = prm.c + static_cast<int64_t>(p) * m * n;
  const ModConst mc = make_mod_const(prm.moduli.m[p]);
  constexpr int kStep = kVec ? 16 : 4;  // bytes of k per lane per step
  for (int64_t rb = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock; rb < m;
       rb += static_cast<int64_t>(gridDim.x) * kRowsPerBlock) {
    const int64_t r0 = rb + warp * R;
    if (r0 >= m) continue;  // whole warp idle: no shuffles below are reached by half a warp
    int32_t res[R][NP];
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int j = 0; j < NP; ++j) res[i][j] = 0;
    for (int64_t s0 = 0; s0 < k; s0 += kSegment) {
      const int64_t s1 = s0 + kSegment < k ? s0 + kSegment : k;
      int32_t acc[R][NP];
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < NP; ++j) acc[i][j] = 0;
      for (int64_t kk = s0 + static_cast<int64_t>(lane) * kStep; kk < s1; kk += 32 * kStep) {
        if constexpr (kVec) {
          uint4 aw[R];
#pragma unroll
          for (int i = 0; i < R; ++i)
            aw[i] = (r0 + i < m) ? __ldcs(reinterpret_cast<const uint4*>(a + (r0 + i) * k + kk)) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int j = 0; j < NP; ++j) {
            const uint4 bw = __ldg(reinterpret_cast<const uint4*>(bt + j * kp + kk));
#pragma unroll
            for (int i = 0; i < R; ++i) {
              int32_t v = acc[i][j];
              v = __dp4a(static_cast<int>(aw[i].x), static_cast<int>(bw.x), v);
              v = __dp4a(static_cast<int>(aw[i].y), static_cast<int>(bw.y), v);
              v = __dp4a(static_cast<int>(aw[i].z), static_cast<int>(bw.z), v);
              v = __dp4a(static_cast<int>(aw[i].w), static_cast<int>(bw.w), v);
              acc[i][j] = v;
            }
          }
        } else {
          uint32_t aw[R];
#pragma unroll
          for (int i = 0; i < R; ++i) aw[i] = load_a4(a + (r0 + i < m ? r0 + i : 0) * k, k, kk, r0 + i < m);
#pragma unroll
          for (int j = 0; j < NP; ++j) {
            const uint32_t bw = *reinterpret_cast<const uint32_t*>(bt + j * kp + kk);
#pragma unroll
            for (int i = 0; i < R; ++i) acc[i][j] = __dp4a(static_cast<int>(aw[i]), static_cast<int>(bw), acc[i][j]);
          }
        }
      }
      // The segment's exact sums -> centered residues, added up across segments.
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < NP; ++j) res[i][j] += reduce_i32_centered(warp_sum(acc[i][j]), mc);
    }
    // Every lane holds the totals; lane j writes column j of the warp's rows.
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int64_t r = r0 + i;
#pragma unroll
      for (int j = 0; j < NP; ++j)
        if (lane == j && j < n && r < m) c[r * n + j] = static_cast<int8_t>(reduce_i32_centered(res[i][j], mc));
    }
  }
}

int padded_np(int64_t n) { return n <= 4 ? 4 : (n <= 8 ? 8 : 16); }

// ---- few rows: K split across warps ----------------------------------------------
// With few rows (a GEMV, or an output of a handful of cells) the row-parallel
// kernel above runs one warp per row group down the whole of K, which leaves
// the GPU idle and the call latency-bound (1 x 1 x 65536: 146 us). Here each
// warp takes a row group and one K chunk of at most 65536 products: its exact
// int32 sums are reduced to centered residues and added (atomically) into an
// int32 accumulator per output cell; a finalize pass reduces each
// accumulator. The accumulated residues of the chunks are congruent to the
// reference's folded running residue, so the bytes are identical.
constexpr int64_t kSplitMaxRows = 1024;  // the accumulator area is reserved up to this many rows

template <int NP, bool kVec>
__global__ void __launch_bounds__(256) skinny_split_kernel(const SkinnyParams prm, int64_t chunk, int64_t chunks,
                                                           int32_t* __restrict__ acc_out) {
  constexpr int R = rows_per_warp<NP>();
  constexpr int kStep = kVec ? 16 : 4;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t ci = static_cast<int64_t>(blockIdx.x) * 8 + warp;  // this warp's K chunk
  if (ci >= chunks) return;  // whole warp: the shuffles below are never reached by part of one
  const uint32_t p = blockIdx.y;
  const int64_t m = prm.m, n = prm.n, k = prm.k, kp = prm.kp;
  const int64_t r0 = static_cast<int64_t>(blockIdx.z) * R;
  const int8_t* a = prm.a + static_cast<int64_t>(p) * m * k;
  const int8_t* bt = prm.bt + static_cast<int64_t>(p) * NP * kp;
  const ModConst mc = make_mod_const(prm.moduli.m[p]);
  const int64_t s0 = ci * chunk, s1 = s0 + chunk < k ? s0 + chunk : k;
  int32_t acc[R][NP];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int j = 0; j < NP; ++j) acc[i][j] = 0;
  for (int64_t kk = s0 + static_cast<int64_t>(lane) * kStep; kk < s1; kk += 32 * kStep) {
    if constexpr (kVec) {
      uint4 aw[R];
#pragma unroll
      for (int i = 0; i < R; ++i)
        aw[i] = (r0 + i < m) ? __ldcs(reinterpret_cast<const uint4*>(a + (r0 + i) * k + kk)) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const uint4 bw = __ldg(reinterpret_cast<const uint4*>(bt + j * kp + kk));
#pragma unroll
        for (int i = 0; i < R; ++i) {
          int32_t v = acc[i][j];
          v = __dp4a(static_cast<int>(aw[i].x), static_cast<int>(bw.x), v);
          v = __dp4a(static_cast<int>(aw[i].y), static_cast<int>(bw.y), v);
          v = __dp4a(static_cast<int>(aw[i].z), static_cast<int>(bw.z), v);
          v = __dp4a(static_cast<int>(aw[i].w), static_cast<int>(bw.w), v);
          acc[i][j] = v;
        }
      }
    } else {
      uint32_t aw[R];
#pragma unroll
      for (int i = 0; i < R; ++i) aw[i] = load_a4(a + (r0 + i < m ? r0 + i : 0) * k, k, kk, r0 + i < m);
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        const uint32_t bw = *reinterpret_cast<const uint32_t*>(bt + j * kp + kk);
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i][j] = __dp4a(static_cast<int>(aw[i]), static_cast<int>(bw), acc[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const int32_t res = reduce_i32_centered(warp_sum(acc[i][j]), mc);
      if (lane == j && j < n && r0 + i < m) atomicAdd(acc_out + (static_cast<int64_t>(p) * m + r0 + i) * n + j, res);
    }
}

__global__ void __launch_bounds__(256) skinny_finalize_kernel(const int32_t* __restrict__ acc, int64_t cells,
                                                              PlaneModuli moduli, int8_t* __restrict__ c) {
  const uint32_t p = blockIdx.y;
  const ModConst mc = make_mod_const(moduli.m[p]);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < cells;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    c[static_cast<int64_t>(p) * cells + i] = static_cast<int8_t>(reduce_i32_centered(acc[static_cast<int64_t>(p) * cells + i], mc));
}

uint64_t round256(uint64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

bool skinny_path_supported(const PlaneGemmProblem& prob) {
  return prob.n >= 1 && prob.n < 16 && prob.m > 0 && prob.k > 0 && prob.planes >= 1 && prob.planes <= 20;
}

uint64_t skinny_scratch_bytes(const PlaneGemmProblem& prob) {
  if (!skinny_path_supported(prob)) return 0;
  const int64_t kp = (prob.k + 15) / 16 * 16;
  const uint64_t bt = round256(static_cast<uint64_t>(prob.planes) * padded_np(prob.n) * kp);
  const uint64_t acc = prob.m <= kSplitMaxRows ? static_cast<uint64_t>(prob.planes) * prob.m * prob.n * 4 : 0;
  return bt + acc;
}

cudaError_t skinny_plane_gemm(const PlaneGemmProblem& prob, void* scratch, uint64_t scratch_bytes,
                              cudaStream_t stream, int sm_count_hint) {
  if (!skinny_path_supported(prob) || !scratch || scratch_bytes < skinny_scratch_bytes(prob))
    return cudaErrorInvalidValue;
  const int np = padded_np(prob.n);
  const int64_t kp = (prob.k + 15) / 16 * 16;
  PlaneModuli pm{};
  for (uint32_t p = 0; p < prob.planes; ++p) pm.m[p] = prob.moduli[p];
  int8_t* bt = static_cast<int8_t*>(scratch);
  for (uint32_t t = 0; t < prob.task_count; ++t) {
    const PlaneGemmTask& task = prob.tasks[t];
    const int64_t tb = (static_cast<int64_t>(np) * kp + 255) / 256;
    transpose_b_kernel<<<dim3(static_cast<unsigned>(tb < 4096 ? tb : 4096), prob.planes), 256, 0, stream>>>(
        task.b, prob.k, prob.n, static_cast<uint32_t>(np), kp, bt);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    SkinnyParams prm{task.a, bt, task.c, prob.m, prob.n, prob.k, kp, pm};
    const bool vec = prob.k % 16 == 0 && reinterpret_cast<uintptr_t>(task.a) % 16 == 0;
    const int64_t rows_per_block = 8 * (np == 16 ? 2 : 4);
    const int64_t blocks = (prob.m + rows_per_block - 1) / rows_per_block;
    if (prob.m <= kSplitMaxRows && blocks * prob.planes < sm_count_hint) {
      // Few rows: split K so that about 4 x 148 x 8 warps share the work.
      const int R = np == 16 ? 2 : 4;
      const int64_t groups = (prob.m + R - 1) / R;
      const int64_t step = 32 * (vec ? 16 : 4);  // K one warp covers per iteration
      const int64_t want = std::max<int64_t>(1, (4 * 8 * static_cast<int64_t>(sm_count_hint)) /
                                                    (groups * static_cast<int64_t>(prob.planes)));
      int64_t chunk = (prob.k + want - 1) / want;
      chunk = (chunk + step - 1) / step * step;
      if (chunk > kSegment) chunk = kSegment;  // exact int32 sums
      const int64_t chunks = (prob.k + chunk - 1) / chunk;
      int32_t* acc = reinterpret_cast<int32_t*>(static_cast<int8_t*>(scratch) +
                                                round256(static_cast<uint64_t>(prob.planes) * np * kp));
      const int64_t cells = prob.m * prob.n;
      e = cudaMemsetAsync(acc, 0, static_cast<size_t>(cells) * prob.planes * sizeof(int32_t), stream);
      if (e != cudaSuccess) return e;
      const dim3 sgrid(static_cast<unsigned>((chunks + 7) / 8), prob.planes, static_cast<unsigned>(groups));
#define RNS8_SPLIT(NP)                                                                                        \
  (vec ? (skinny_split_kernel<NP, true><<<sgrid, 256, 0, stream>>>(prm, chunk, chunks, acc), cudaGetLastError()) \
       : (skinny_split_kernel<NP, false><<<sgrid, 256, 0, stream>>>(prm, chunk, chunks, acc), cudaGetLastError()))
      e = np == 4 ? RNS8_SPLIT(4) : (np == 8 ? RNS8_SPLIT(8) : RNS8_SPLIT(16));
#undef RNS8_SPLIT
      if (e != cudaSuccess) return e;
      const int64_t fb = (cells + 255) / 256;
      skinny_finalize_kernel<<<dim3(static_cast<unsigned>(fb < 1024 ? fb : 1024), prob.planes), 256, 0, stream>>>(
          acc, cells, pm, task.c);
      e = cudaGetLastError();
      if (e != cudaSuccess) return e;
      continue;
    }
    const dim3 grid(static_cast<unsigned>(blocks < (int64_t{1} << 30) ? blocks : (int64_t{1} << 30)), prob.planes);
#define RNS8_SKINNY(NP)                                                          \
  (vec ? (skinny_kernel<NP, true><<<grid, 256, 0, stream>>>(prm), cudaGetLastError()) \
       : (skinny_kernel<NP, false><<<grid, 256, 0, stream>>>(prm), cudaGetLastError()))
    e = np == 4 ? RNS8_SKINNY(4) : (np == 8 ? RNS8_SKINNY(8) : RNS8_SKINNY(16));
#undef RNS8_SKINNY
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace rns8cuda
