// Pack kernels: native int64 / uint64 / uint8 matrices -> centered int8
// residue planes (reference behaviour: src/cpu/cpu_reference.cpp:26-130,
// layout res[p*rows*cols + r*cols + c] from :46-51).
//
// Reduction of a 64-bit value u modulo a ladder modulus m (m <= 256):
// u = d3*2^48 + d2*2^32 + d1*2^16 + d0 with 16-bit digits, so
// u = d0 + d1*w1 + d2*w2 + d3*w3 (mod m) with w_j = 2^(16j) mod m < 256.
// The folded sum is below 2^26 and one mul-hi reduction finishes it. A signed
// value x < 0 is u - 2^64, so its residue adds (-2^64) mod m. The digits are
// computed once per element and shared by every plane; the per-plane
// constants fold to immediates because the prefix is a template parameter.
#include "device_common.cuh"
#include "kernels.hpp"

namespace rns8cuda {
namespace {

__host__ __device__ __forceinline__ uint32_t ladder_modulus(int i) {
  switch (i) {
    case 0: return 256; case 1: return 255; case 2: return 253; case 3: return 251; case 4: return 247;
    case 5: return 239; case 6: return 233; case 7: return 229; case 8: return 227; case 9: return 223;
    case 10: return 217; case 11: return 211; case 12: return 199; case 13: return 197; case 14: return 193;
    case 15: return 191; case 16: return 181; case 17: return 179; case 18: return 173; case 19: return 167;
    default: return 1;
  }
}

struct Digits {
  uint32_t d0, d1, d2, d3, neg;
};

template <typename T>
__device__ __forceinline__ Digits split_digits(T v) {
  const uint64_t u = static_cast<uint64_t>(v);
  const uint32_t lo = static_cast<uint32_t>(u), hi = static_cast<uint32_t>(u >> 32);
  Digits d;
  d.d0 = lo & 0xFFFFu;
  d.d1 = lo >> 16;
  d.d2 = hi & 0xFFFFu;
  d.d3 = hi >> 16;
  d.neg = (static_cast<T>(-1) < 0) ? (hi >> 31) : 0u;
  return d;
}

// Centered residue of the element with digits d modulo ladder entry p.
template <bool kSigned>
__device__ __forceinline__ int residue_of(const Digits& d, int p) {
  const uint32_t m = ladder_modulus(p);
  const uint32_t w1 = static_cast<uint32_t>((1ull << 16) % m);
  const uint32_t w2 = static_cast<uint32_t>((1ull << 32) % m);
  const uint32_t w3 = static_cast<uint32_t>((1ull << 48) % m);
  // (-2^64) mod m, computed without 128-bit arithmetic: 2^64 mod m = (w3 * 2^16) mod m.
  const uint32_t t64 = static_cast<uint32_t>((static_cast<uint64_t>(w3) << 16) % m);
  const uint32_t wneg = (m - t64) % m;
  uint32_t s = d.d0 + d.d1 * w1 + d.d2 * w2 + d.d3 * w3;
  if (kSigned) s += d.neg * wneg;
  return center_residue(umod_u32(s, m, floor_magic(m)), m);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

// Vector path: each thread converts 8 consecutive elements of one row
// (four 128-bit loads) and writes 8 bytes to each of the P planes.
// Requires cols % 8 == 0 and ld % 2 == 0 so every access is aligned.
template <int P, typename T>
__global__ void __launch_bounds__(256) pack_vec8_kernel(const T* __restrict__ src, int64_t rows, int64_t cols,
                                                         int64_t ld, int8_t* __restrict__ planes) {
  constexpr bool kSigned = static_cast<T>(-1) < 0;
  const int64_t groups_per_row = cols >> 3;
  const int64_t total = rows * groups_per_row;
  const int64_t plane_elems = rows * cols;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = g / groups_per_row;
    const int64_t col = (g - row * groups_per_row) << 3;
    const int4* in = reinterpret_cast<const int4*>(src + row * ld + col);
    Digits d[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int4 v = __ldcs(in + q);  // streamed once: do not keep in L1/L2
      const uint64_t e0 = (static_cast<uint64_t>(static_cast<uint32_t>(v.y)) << 32) | static_cast<uint32_t>(v.x);
      const uint64_t e1 = (static_cast<uint64_t>(static_cast<uint32_t>(v.w)) << 32) | static_cast<uint32_t>(v.z);
      d[2 * q] = split_digits<T>(static_cast<T>(e0));
      d[2 * q + 1] = split_digits<T>(static_cast<T>(e1));
    }
    int8_t* out = planes + row * cols + col;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      uint2 w;
      w.x = pack4(residue_of<kSigned>(d[0], p), residue_of<kSigned>(d[1], p), residue_of<kSigned>(d[2], p),
                  residue_of<kSigned>(d[3], p));
      w.y = pack4(residue_of<kSigned>(d[4], p), residue_of<kSigned>(d[5], p), residue_of<kSigned>(d[6], p),
                  residue_of<kSigned>(d[7], p));
      *reinterpret_cast<uint2*>(out + static_cast<int64_t>(p) * plane_elems) = w;
    }
  }
}

// Generic path: one element per thread, any shape and leading dimension.
template <int P, typename T>
__global__ void __launch_bounds__(256) pack_scalar_kernel(const T* __restrict__ src, int64_t rows, int64_t cols,
                                                           int64_t ld, int8_t* __restrict__ planes) {
  constexpr bool kSigned = static_cast<T>(-1) < 0;
  const int64_t total = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / cols, col = i - row * cols;
    const Digits d = split_digits<T>(src[row * ld + col]);
#pragma unroll
    for (int p = 0; p < P; ++p) planes[static_cast<int64_t>(p) * total + i] = static_cast<int8_t>(residue_of<kSigned>(d, p));
  }
}

template <int P, typename T>
cudaError_t launch_pack(const T* src, int64_t rows, int64_t cols, int64_t ld, int8_t* planes, cudaStream_t stream) {
  const bool vec = (cols % 8 == 0) && (ld % 2 == 0) && (reinterpret_cast<uintptr_t>(src) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(planes) % 8 == 0);
  const int64_t work = vec ? rows * (cols / 8) : rows * cols;
  const int threads = 256;
  int64_t blocks = (work + threads - 1) / threads;
  if (blocks > 148 * 16) blocks = 148 * 16;  // grid-stride beyond 16 blocks per SM
  if (blocks < 1) blocks = 1;
  if (vec)
    pack_vec8_kernel<P, T><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(src, rows, cols, ld, planes);
  else
    pack_scalar_kernel<P, T><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(src, rows, cols, ld, planes);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_pack(const T* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* planes,
                          cudaStream_t stream) {
  switch (prefix) {
#define RNS8_PACK_CASE(P) \
  case P: return launch_pack<P, T>(src, rows, cols, ld, planes, stream);
    RNS8_PACK_CASE(1) RNS8_PACK_CASE(2) RNS8_PACK_CASE(3) RNS8_PACK_CASE(4) RNS8_PACK_CASE(5)
    RNS8_PACK_CASE(6) RNS8_PACK_CASE(7) RNS8_PACK_CASE(8) RNS8_PACK_CASE(9) RNS8_PACK_CASE(10)
    RNS8_PACK_CASE(11) RNS8_PACK_CASE(12) RNS8_PACK_CASE(13) RNS8_PACK_CASE(14) RNS8_PACK_CASE(15)
    RNS8_PACK_CASE(16) RNS8_PACK_CASE(17) RNS8_PACK_CASE(18) RNS8_PACK_CASE(19) RNS8_PACK_CASE(20)
#undef RNS8_PACK_CASE
    default: return cudaErrorInvalidValue;
  }
}

// Finite u8: residues of bytes modulo an arbitrary m in [2, 256].
__global__ void __launch_bounds__(256) pack_u8_vec16_kernel(const uint8_t* __restrict__ src, int64_t rows,
                                                            int64_t cols, int64_t ld, uint32_t m, uint32_t magic,
                                                            int8_t* __restrict__ out) {
  const int64_t groups_per_row = cols >> 4;
  const int64_t total = rows * groups_per_row;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = g / groups_per_row;
    const int64_t col = (g - row * groups_per_row) << 4;
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src + row * ld + col));
    uint32_t words[4] = {v.x, v.y, v.z, v.w};
    uint4 o;
    uint32_t* ow = &o.x;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      int r[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) r[b] = center_residue(umod_u32((words[w] >> (8 * b)) & 0xFFu, m, magic), m);
      ow[w] = pack4(r[0], r[1], r[2], r[3]);
    }
    *reinterpret_cast<uint4*>(out + row * cols + col) = o;
  }
}
__global__ void __launch_bounds__(256) pack_u8_scalar_kernel(const uint8_t* __restrict__ src, int64_t rows,
                                                             int64_t cols, int64_t ld, uint32_t m, uint32_t magic,
                                                             int8_t* __restrict__ out) {
  const int64_t total = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / cols, col = i - row * cols;
    out[i] = static_cast<int8_t>(center_residue(umod_u32(src[row * ld + col], m, magic), m));
  }
}

}  // namespace

cudaError_t pack_i64(const int64_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* planes,
                     cudaStream_t stream) {
  return dispatch_pack<int64_t>(src, rows, cols, ld, prefix, planes, stream);
}
cudaError_t pack_u64(const uint64_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* planes,
                     cudaStream_t stream) {
  return dispatch_pack<uint64_t>(src, rows, cols, ld, prefix, planes, stream);
}
cudaError_t pack_finite_u8(const uint8_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t modulus,
                           int8_t* residues, cudaStream_t stream) {
  if (modulus < 2 || modulus > 256) return cudaErrorInvalidValue;
  const uint32_t magic = floor_magic(modulus);
  const bool vec = (cols % 16 == 0) && (ld % 16 == 0) && (reinterpret_cast<uintptr_t>(src) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(residues) % 16 == 0);
  const int64_t work = vec ? rows * (cols / 16) : rows * cols;
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  if (vec)
    pack_u8_vec16_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, rows, cols, ld, modulus, magic,
                                                                            residues);
  else
    pack_u8_scalar_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, rows, cols, ld, modulus, magic,
                                                                             residues);
  return cudaGetLastError();
}

}  // namespace rns8cuda
