// SIMT plane GEMM: C_p = (A_p x B_p) mod m_p for shapes the tensor-core
// kernel does not take (K or N not a multiple of 16, i.e. rows the TMA cannot
// address). Same arithmetic contract as the reference CPU ring GEMM
// (src/cpu/cpu_reference.cpp:156-206): exact int32 sums over runs of at most
// RNS8_SAFE_INT32_K_BLOCK products, each run folded into the running
// centered residue.
#include "device_common.cuh"
#include "gemm_internal.hpp"

namespace rns8cuda {
namespace {

constexpr int kTile = 64;   // output tile edge
constexpr int kChunk = 32;  // K slice staged in shared memory

__global__ void __launch_bounds__(256) simt_plane_gemm_kernel(const int8_t* __restrict__ A, const int8_t* __restrict__ B,
                                                              int8_t* __restrict__ C, int64_t m, int64_t n, int64_t k,
                                                              PlaneModuli moduli) {
  __shared__ int8_t As[kTile][kChunk + 4];
  __shared__ int8_t Bs[kChunk][kTile + 4];
  const int p = blockIdx.z;
  const int8_t* a = A + static_cast<int64_t>(p) * m * k;
  const int8_t* b = B + static_cast<int64_t>(p) * k * n;
  int8_t* c = C + static_cast<int64_t>(p) * m * n;
  const ModConst mc = make_mod_const(moduli.m[p]);
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * kTile;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kTile;
  const int tr = threadIdx.x / 16, tc = threadIdx.x % 16;  // 16 x 16 threads, 4 x 4 cells each

  int residue[4][4];
  int32_t acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) residue[i][j] = 0, acc[i][j] = 0;

  int64_t run = 0;  // products accumulated since the last fold
  for (int64_t k0 = 0; k0 < k; k0 += kChunk) {
    for (int idx = threadIdx.x; idx < kTile * kChunk; idx += 256) {
      const int r = idx / kChunk, kk = idx % kChunk;
      const int64_t gr = row0 + r, gk = k0 + kk;
      As[r][kk] = (gr < m && gk < k) ? a[gr * k + gk] : int8_t{0};
    }
    for (int idx = threadIdx.x; idx < kChunk * kTile; idx += 256) {
      const int kk = idx / kTile, cc = idx % kTile;
      const int64_t gk = k0 + kk, gc = col0 + cc;
      Bs[kk][cc] = (gk < k && gc < n) ? b[gk * n + gc] : int8_t{0};
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kChunk; ++kk) {
      int av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[tr * 4 + i][kk];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tc * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += av[i] * bv[j];
    }
    __syncthreads();
    run += kChunk;
    // kChunk divides the safe block, so runs end exactly on 65536 boundaries.
    if (run == kSafeKBlock || k0 + kChunk >= k) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          residue[i][j] = reduce_i32_centered(acc[i][j] + residue[i][j], mc);
          acc[i][j] = 0;
        }
      run = 0;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gr = row0 + tr * 4 + i;
    if (gr >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gc = col0 + tc * 4 + j;
      if (gc < n) c[gr * n + gc] = static_cast<int8_t>(residue[i][j]);
    }
  }
}

}  // namespace

cudaError_t simt_plane_gemm(const PlaneGemmProblem& prob, cudaStream_t stream) {
  PlaneModuli pm{};
  for (uint32_t p = 0; p < prob.planes; ++p) pm.m[p] = prob.moduli[p];
  const dim3 grid(static_cast<unsigned>((prob.n + kTile - 1) / kTile), static_cast<unsigned>((prob.m + kTile - 1) / kTile),
                  prob.planes);
  if (grid.y > 65535u || prob.planes == 0 || prob.planes > 20) return cudaErrorInvalidValue;
  for (uint32_t t = 0; t < prob.task_count; ++t) {
    simt_plane_gemm_kernel<<<grid, 256, 0, stream>>>(prob.tasks[t].a, prob.tasks[t].b, prob.tasks[t].c, prob.m, prob.n,
                                                     prob.k, pm);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace rns8cuda
