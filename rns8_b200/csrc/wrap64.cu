// WRAP_U64_MOD_2_64: C = A x B modulo 2^64 over uint64 matrices stored as
// eight unsigned byte planes (reference src/backend_wrap64/, README.md:1-81).
//
// Storage is limb-major: byte l of cell (r, c) of an R x C matrix is
// planes[l*R*C + r*C + c], so each byte plane is a u8 matrix the tensor-core
// kernel can load with TMA (the reference keeps the eight bytes of a cell
// together, cell*8 + limb, wrap64_reference.cpp:20-24; only the byte count is
// observable, 8*R*C either way).
//
//   pack:   uint64 (row-major, leading dimension ld) -> 8 byte planes
//   gemm:   byte planes -> uint64 C (row-major, compact): tensor cores when
//           K and N are multiples of 16 (gemm_tc.cu), else the SIMT kernel
//           below, which multiplies the reassembled uint64 values directly
//           (uint64 arithmetic wraps modulo 2^64, wrap64_reference.cpp:254-290)
//   export: 8 byte planes -> uint64 (leading dimension ld)
#include "gemm_internal.hpp"
#include "kernels.hpp"

namespace rns8cuda {
namespace {

// 4 x 4 byte transpose: out[j] byte i = in[i] byte j. Used both ways: four
// cells' words -> four planes' words, and back.
__device__ __forceinline__ void transpose4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t (&o)[4]) {
  const uint32_t a_lo = __byte_perm(w0, w1, 0x5140);  // w0.b0 w1.b0 w0.b1 w1.b1
  const uint32_t a_hi = __byte_perm(w0, w1, 0x7362);  // w0.b2 w1.b2 w0.b3 w1.b3
  const uint32_t b_lo = __byte_perm(w2, w3, 0x5140);
  const uint32_t b_hi = __byte_perm(w2, w3, 0x7362);
  o[0] = __byte_perm(a_lo, b_lo, 0x5410);
  o[1] = __byte_perm(a_lo, b_lo, 0x7632);
  o[2] = __byte_perm(a_hi, b_hi, 0x5410);
  o[3] = __byte_perm(a_hi, b_hi, 0x7632);
}

// 4 cells per thread: two 16-byte loads, one 4-byte store per plane.
// grid.x over groups of 4 columns, grid.y over rows (a contiguous matrix is
// passed as one row), so no division per group.
__global__ void __launch_bounds__(256) wrap_pack_vec4_kernel(const uint64_t* __restrict__ src, int64_t rows,
                                                             int64_t cols, int64_t ld, int64_t plane_elems,
                                                             uint8_t* __restrict__ planes) {
  const int64_t groups = cols >> 2;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const uint4* s = reinterpret_cast<const uint4*>(src + row * ld);
    uint8_t* out = planes + row * cols;
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const uint4 v0 = __ldcs(s + 2 * g);
      const uint4 v1 = __ldcs(s + 2 * g + 1);
      uint32_t lo[4], hi[4];
      transpose4(v0.x, v0.z, v1.x, v1.z, lo);  // low words of cells 0..3: bytes 0..3
      transpose4(v0.y, v0.w, v1.y, v1.w, hi);  // high words: bytes 4..7
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        reinterpret_cast<uint32_t*>(out + l * plane_elems)[g] = lo[l];
        reinterpret_cast<uint32_t*>(out + (l + 4) * plane_elems)[g] = hi[l];
      }
    }
  }
}

__global__ void __launch_bounds__(256) wrap_pack_scalar_kernel(const uint64_t* __restrict__ src, int64_t rows,
                                                               int64_t cols, int64_t ld, int64_t plane_elems,
                                                               uint8_t* __restrict__ planes) {
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y)
    for (int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; col < cols;
         col += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const uint64_t v = src[row * ld + col];
#pragma unroll
      for (int l = 0; l < 8; ++l) planes[l * plane_elems + row * cols + col] = static_cast<uint8_t>(v >> (8 * l));
    }
}

__global__ void __launch_bounds__(256) wrap_export_vec4_kernel(const uint8_t* __restrict__ planes, int64_t rows,
                                                               int64_t cols, int64_t plane_elems,
                                                               uint64_t* __restrict__ dst, int64_t ld) {
  const int64_t groups = cols >> 2;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const uint8_t* in = planes + row * cols;
    uint4* d = reinterpret_cast<uint4*>(dst + row * ld);
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      uint32_t p[8];
#pragma unroll
      for (int l = 0; l < 8; ++l) p[l] = __ldcs(reinterpret_cast<const uint32_t*>(in + l * plane_elems) + g);
      uint32_t lo[4], hi[4];
      transpose4(p[0], p[1], p[2], p[3], lo);  // bytes 0..3 of cells 0..3
      transpose4(p[4], p[5], p[6], p[7], hi);  // bytes 4..7
      __stcs(d + 2 * g, make_uint4(lo[0], hi[0], lo[1], hi[1]));
      __stcs(d + 2 * g + 1, make_uint4(lo[2], hi[2], lo[3], hi[3]));
    }
  }
}

__global__ void __launch_bounds__(256) wrap_export_scalar_kernel(const uint8_t* __restrict__ planes, int64_t rows,
                                                                 int64_t cols, int64_t plane_elems,
                                                                 uint64_t* __restrict__ dst, int64_t ld) {
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y)
    for (int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; col < cols;
         col += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      uint64_t v = 0;
#pragma unroll
      for (int l = 0; l < 8; ++l) v |= static_cast<uint64_t>(planes[l * plane_elems + row * cols + col]) << (8 * l);
      dst[row * ld + col] = v;
    }
}

__device__ __forceinline__ uint64_t gather_u64(const uint8_t* __restrict__ planes, int64_t plane_elems, int64_t idx) {
  uint64_t v = 0;
#pragma unroll
  for (int l = 0; l < 8; ++l) v |= static_cast<uint64_t>(planes[l * plane_elems + idx]) << (8 * l);
  return v;
}

// 16 x 16 output tile per block, K in steps of 16 through shared memory.
__global__ void __launch_bounds__(256) wrap_simt_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b,
                                                        uint64_t* __restrict__ c, int64_t m, int64_t n, int64_t k) {
  __shared__ uint64_t sa[16][17];
  __shared__ uint64_t sb[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  for (int64_t bm = blockIdx.y; bm * 16 < m; bm += gridDim.y) {
    for (int64_t bn = blockIdx.x; bn * 16 < n; bn += gridDim.x) {
      const int64_t row = bm * 16 + ty, col = bn * 16 + tx;
      uint64_t acc = 0;
      for (int64_t k0 = 0; k0 < k; k0 += 16) {
        sa[ty][tx] = (row < m && k0 + tx < k) ? gather_u64(a, m * k, row * k + k0 + tx) : 0;
        sb[ty][tx] = (k0 + ty < k && col < n) ? gather_u64(b, k * n, (k0 + ty) * n + col) : 0;
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) acc += sa[ty][kk] * sb[kk][tx];
        __syncthreads();
      }
      if (row < m && col < n) c[row * n + col] = acc;
    }
  }
}

dim3 grid_2d(int64_t rows, int64_t per_row) {
  const int64_t by = rows < 65535 ? rows : 65535;
  int64_t bx = (per_row + 255) / 256;
  const int64_t max_x = (148 * 16 + by - 1) / by;
  if (bx > max_x) bx = max_x;
  if (bx < 1) bx = 1;
  return dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by));
}

}  // namespace

cudaError_t wrap_pack_u64(const uint64_t* src, int64_t rows, int64_t cols, int64_t ld, uint8_t* planes,
                          cudaStream_t stream) {
  if (rows <= 0 || cols <= 0 || ld < cols || !src || !planes) return cudaErrorInvalidValue;
  const int64_t plane_elems = rows * cols;
  if (ld == cols) {  // contiguous: one long row
    cols *= rows;
    ld = cols;
    rows = 1;
  }
  const bool vec = cols % 4 == 0 && ld % 2 == 0 && reinterpret_cast<uintptr_t>(src) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(planes) % 4 == 0 && plane_elems % 4 == 0;
  if (vec)
    wrap_pack_vec4_kernel<<<grid_2d(rows, cols / 4), 256, 0, stream>>>(src, rows, cols, ld, plane_elems, planes);
  else
    wrap_pack_scalar_kernel<<<grid_2d(rows, cols), 256, 0, stream>>>(src, rows, cols, ld, plane_elems, planes);
  return cudaGetLastError();
}

cudaError_t wrap_export_u64(const uint8_t* planes, int64_t rows, int64_t cols, uint64_t* dst, int64_t ld,
                            cudaStream_t stream) {
  if (rows <= 0 || cols <= 0 || ld < cols || !planes || !dst) return cudaErrorInvalidValue;
  const int64_t plane_elems = rows * cols;
  if (ld == cols) {
    cols *= rows;
    ld = cols;
    rows = 1;
  }
  const bool vec = cols % 4 == 0 && ld % 2 == 0 && reinterpret_cast<uintptr_t>(dst) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(planes) % 4 == 0 && plane_elems % 4 == 0;
  if (vec)
    wrap_export_vec4_kernel<<<grid_2d(rows, cols / 4), 256, 0, stream>>>(planes, rows, cols, plane_elems, dst, ld);
  else
    wrap_export_scalar_kernel<<<grid_2d(rows, cols), 256, 0, stream>>>(planes, rows, cols, plane_elems, dst, ld);
  return cudaGetLastError();
}

bool wrap_tensor_core_supported(const uint8_t* a, const uint8_t* b, const uint64_t* c, int64_t m, int64_t n,
                                int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0 || k % 16 != 0 || n % 16 != 0) return false;
  if (m > (int64_t(1) << 31) || n > (int64_t(1) << 31) || k > (int64_t(1) << 31)) return false;
  if (reinterpret_cast<uintptr_t>(a) % 16 || reinterpret_cast<uintptr_t>(b) % 16 ||
      reinterpret_cast<uintptr_t>(c) % 16)
    return false;
  return tma_encode_available();
}

cudaError_t wrap_gemm(const uint8_t* a_limbs, const uint8_t* b_limbs, uint64_t* c, int64_t m, int64_t n, int64_t k,
                      GemmPath path, int sm_count, uint32_t* dev_status, cudaStream_t stream, GemmPath* used) {
  if (m <= 0 || n <= 0 || k <= 0 || !a_limbs || !b_limbs || !c) return cudaErrorInvalidValue;
  const bool tc_ok = wrap_tensor_core_supported(a_limbs, b_limbs, c, m, n, k);
  if (path == GemmPath::TensorCore && !tc_ok) return cudaErrorInvalidValue;
  if (path == GemmPath::Simt || !tc_ok) {
    if (used) *used = GemmPath::Simt;
    const int64_t gx = (n + 15) / 16, gy = (m + 15) / 16;
    const dim3 grid(static_cast<unsigned>(gx < 65535 ? gx : 65535), static_cast<unsigned>(gy < 65535 ? gy : 65535));
    wrap_simt_kernel<<<grid, 256, 0, stream>>>(a_limbs, b_limbs, c, m, n, k);
    return cudaGetLastError();
  }
  if (used) *used = GemmPath::TensorCore;
  return tc_wrap64_gemm(a_limbs, b_limbs, c, m, n, k, sm_count, dev_status, stream);
}

}  // namespace rns8cuda
