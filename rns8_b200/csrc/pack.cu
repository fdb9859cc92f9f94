// Pack kernels: native int64 / uint64 / uint8 matrices -> centered int8
// residue planes (reference behaviour: src/cpu/cpu_reference.cpp:26-130,
// layout res[p*rows*cols + r*cols + c] from :46-51).
//
// Reduction of a 64-bit value modulo a ladder modulus m (m <= 256): with the
// eight bytes b_j of an unsigned 64-bit u,
//   u = sum_j b_j * 2^(8j)  =  sum_j b_j * w_j  (mod m),  w_j = 2^(8j) mod m < 256,
// which is two dp4a instructions. A signed x is packed as u = x + 2^63 (its
// top bit flipped), and the constant (-2^63) mod m starts the dp4a sum, so
// both signs take the same path. With h = floor(m/2) added to that start
// constant the sum s = t + h is below 2^20, where q = mulhi(s, ceil(2^32/m))
// is the exact quotient of s by m, and s - (q*m + h) is the centered residue
// (in [-h, m - 1 - h]): two dp4a, one mul-hi, one multiply-add and one add
// per residue. Modulus 256 is the low byte itself (two's complement). The
// byte split is shared by every plane; per-plane constants are immediates
// because the prefix is a template parameter.
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

struct Words {
  uint32_t lo, hi;  // the value as unsigned 64 bits (signed: x + 2^63)
};

template <typename T>
__device__ __forceinline__ Words split_words(T v) {
  const uint64_t u = static_cast<uint64_t>(v);
  constexpr uint32_t kBias = (static_cast<T>(-1) < 0) ? 0x80000000u : 0u;
  return Words{static_cast<uint32_t>(u), static_cast<uint32_t>(u >> 32) ^ kBias};
}

// Low byte of the centered residue of the element modulo ladder entry p.
template <bool kSigned>
__device__ __forceinline__ uint32_t residue_byte(const Words& w, int p) {
  const uint32_t m = ladder_modulus(p);
  if (m == 256) return w.lo;  // the low byte; the signed bias only touches bit 63
  const uint32_t h = m / 2;
  uint32_t wl = 0, wh = 0;
  uint64_t pow = 1;  // 2^(8j) mod m
  uint64_t pow56 = 1;
  for (int j = 0; j < 8; ++j) {
    if (j < 4)
      wl |= static_cast<uint32_t>(pow) << (8 * j);
    else
      wh |= static_cast<uint32_t>(pow) << (8 * (j - 4));
    if (j == 7) pow56 = pow;
    pow = (pow * 256) % m;
  }
  const uint32_t pow63 = static_cast<uint32_t>((pow56 * 128) % m);  // 2^63 mod m
  const uint32_t start = kSigned ? (m - pow63) % m : 0u;           // (-2^63) mod m
  const uint32_t magic = static_cast<uint32_t>(((1ull << 32) + m - 1) / m);
  uint32_t t = __dp4a(w.hi, wh, start + h);  // + h: the centering shift rides in the start constant
  t = __dp4a(w.lo, wl, t);
  const uint32_t q = __umulhi(t, magic);
  return t - (q * m + h);  // low byte = centered residue
}

// Bytes 0 of a, b, c, d -> one word.
__device__ __forceinline__ uint32_t pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
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
    Words d[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int4 v = __ldcs(in + q);  // streamed once: do not keep in L1/L2
      const uint64_t e0 = (static_cast<uint64_t>(static_cast<uint32_t>(v.y)) << 32) | static_cast<uint32_t>(v.x);
      const uint64_t e1 = (static_cast<uint64_t>(static_cast<uint32_t>(v.w)) << 32) | static_cast<uint32_t>(v.z);
      d[2 * q] = split_words<T>(static_cast<T>(e0));
      d[2 * q + 1] = split_words<T>(static_cast<T>(e1));
    }
    int8_t* out = planes + row * cols + col;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      uint2 w;
      w.x = pack4(residue_byte<kSigned>(d[0], p), residue_byte<kSigned>(d[1], p), residue_byte<kSigned>(d[2], p),
                  residue_byte<kSigned>(d[3], p));
      w.y = pack4(residue_byte<kSigned>(d[4], p), residue_byte<kSigned>(d[5], p), residue_byte<kSigned>(d[6], p),
                  residue_byte<kSigned>(d[7], p));
      __stcs(reinterpret_cast<uint2*>(out + static_cast<int64_t>(p) * plane_elems), w);
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
    const Words d = split_words<T>(src[row * ld + col]);
#pragma unroll
    for (int p = 0; p < P; ++p)
      planes[static_cast<int64_t>(p) * total + i] = static_cast<int8_t>(residue_byte<kSigned>(d, p) & 0xFFu);
  }
}

// ---- streamed pack (compact or row-tiled sources) ---------------------------------------------
// A persistent CTA per SM: one producer warp streams 4096-element tiles of
// the source (32 KiB) into a ring of shared-memory stages with 1-D bulk
// copies; 16 consumer warps convert eight elements per lane and store eight
// bytes to each plane. The copies run up to kStages tiles ahead of the
// integer arithmetic, which the register-fed kernel above cannot do (its
// loads wait behind its own multiply chains). A lane's 64 source bytes are
// read as four 16-byte chunks starting at chunk (lane / 2) mod 4, which puts
// the 32 lanes of each read on distinct bank groups; the eight output bytes
// of each plane are rotated back into place with two byte permutes.
constexpr int kPackWarps = 16;
constexpr int kPackThreads = 32 * (kPackWarps + 1);
constexpr int kPackTile = kPackWarps * 32 * 8;
constexpr int kPackStages = 4;

// Source element offset of tile t: the tiles of a row lie side by side
// (row_tiles of them per row, rows ld elements apart); a compact source is one
// row of all tiles. Plane offsets are always t * kPackTile (planes are compact).
__device__ __forceinline__ int64_t tile_source(int64_t t, int64_t row_tiles, int64_t ld) {
  const int64_t row = t / row_tiles;
  return row * ld + (t - row * row_tiles) * kPackTile;
}

// The pack has no status word, so a bounded wait that runs out cannot be
// reported; instead it cannot change the result: the warp that gives up sets
// a block-wide flag, the producer stops issuing, and every consumer warp
// reads its remaining tiles straight from global memory. The producer then
// waits (bounded) for the copies it already issued before the block exits.
template <int P, typename T>
__device__ __forceinline__ void pack8_store(const int4 (&v)[4], int8_t* out, int64_t elems, uint32_t sel_lo,
                                           uint32_t sel_hi) {
  constexpr bool kSigned = static_cast<T>(-1) < 0;
  Words d[8];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    d[2 * q] = split_words<T>(static_cast<T>((static_cast<uint64_t>(static_cast<uint32_t>(v[q].y)) << 32) |
                                             static_cast<uint32_t>(v[q].x)));
    d[2 * q + 1] = split_words<T>(static_cast<T>((static_cast<uint64_t>(static_cast<uint32_t>(v[q].w)) << 32) |
                                                 static_cast<uint32_t>(v[q].z)));
  }
#pragma unroll
  for (int p = 0; p < P; ++p) {
    const uint32_t lo = pack4(residue_byte<kSigned>(d[0], p), residue_byte<kSigned>(d[1], p),
                              residue_byte<kSigned>(d[2], p), residue_byte<kSigned>(d[3], p));
    const uint32_t hi = pack4(residue_byte<kSigned>(d[4], p), residue_byte<kSigned>(d[5], p),
                              residue_byte<kSigned>(d[6], p), residue_byte<kSigned>(d[7], p));
    __stcs(reinterpret_cast<uint2*>(out + static_cast<int64_t>(p) * elems),
           make_uint2(__byte_perm(lo, hi, sel_lo), __byte_perm(lo, hi, sel_hi)));
  }
}

template <int P, typename T>
__global__ void __launch_bounds__(kPackThreads, 1) pack_ws_kernel(const T* __restrict__ src, int64_t elems,
                                                                  int8_t* __restrict__ planes, int64_t row_tiles,
                                                                  int64_t ld) {
  constexpr bool kSigned = static_cast<T>(-1) < 0;
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[kPackStages], empty[kPackStages];
  __shared__ int gave_up;
  const int64_t tiles = elems / kPackTile;
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPackStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kPackWarps);
    }
    gave_up = 0;
    fence_barrier_init();
  }
  __syncthreads();
  volatile int* stop = &gave_up;
  int64_t mine = 0;  // tiles b, b + grid, ... of this CTA
  if (blockIdx.x < tiles) mine = (tiles - 1 - blockIdx.x) / gridDim.x + 1;
  if (warp == kPackWarps) {
    if (lane != 0) return;
    int64_t issued = 0;
    for (int64_t j = 0; j < mine && !*stop; ++j, ++issued) {
      const int s = static_cast<int>(j % kPackStages);
      if (j >= kPackStages && !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(((j / kPackStages) - 1) & 1))) {
        *stop = 1;
        break;
      }
      const int64_t tile = blockIdx.x + j * gridDim.x;
      mbar_arrive_expect_tx(&full[s], kPackTile * 8);
      bulk_load_1d(ring + static_cast<size_t>(s) * kPackTile * 8, src + tile_source(tile, row_tiles, ld),
                   kPackTile * 8, &full[s]);
    }
    for (int64_t j = issued > kPackStages ? issued - kPackStages : 0; j < issued; ++j)
      (void)mbar_wait_bounded(&full[j % kPackStages], static_cast<uint32_t>((j / kPackStages) & 1));
    return;
  }
  const int rot = (lane >> 1) & 3;
  uint32_t sel_lo = 0, sel_hi = 0;  // rotate the 8 output bytes left by 2 * rot
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sel_lo |= static_cast<uint32_t>((j - 2 * rot) & 7) << (4 * j);
    sel_hi |= static_cast<uint32_t>((j + 4 - 2 * rot) & 7) << (4 * j);
  }
  const int tid = warp * 32 + lane;
  for (int64_t j = 0; j < mine; ++j) {
    const int s = static_cast<int>(j % kPackStages);
    const int64_t tile = blockIdx.x + j * gridDim.x;
    bool direct = *stop != 0;
    if (!direct) direct = !mbar_wait_bounded(&full[s], static_cast<uint32_t>((j / kPackStages) & 1));
    direct = __any_sync(0xFFFFFFFFu, direct);
    int4 v[4];
    if (direct) {  // a wait ran out somewhere in this block: read the tile from global memory
      *stop = 1;
      const int4* gp = reinterpret_cast<const int4*>(src + tile_source(tile, row_tiles, ld)) + tid * 4;
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = gp[(q + rot) & 3];
    } else {
      const int4* sp = reinterpret_cast<const int4*>(ring + static_cast<size_t>(s) * kPackTile * 8) + tid * 4;
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = sp[(q + rot) & 3];  // slot q holds chunk (q + rot) mod 4
      release_stage_reads();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    pack8_store<P, T>(v, planes + tile * kPackTile + tid * 8, elems, sel_lo, sel_hi);
  }
  // The last, partial tile: one CTA, one element per thread.
  if (blockIdx.x == tiles % gridDim.x) {
    for (int64_t i = tiles * kPackTile + tid; i < elems; i += kPackWarps * 32) {
      const Words d = split_words<T>(src[i]);
#pragma unroll
      for (int p = 0; p < P; ++p)
        planes[static_cast<int64_t>(p) * elems + i] = static_cast<int8_t>(residue_byte<kSigned>(d, p) & 0xFFu);
    }
  }
}

// Compact sources of at least one tile with a 16-byte aligned start and
// 8-byte aligned planes take the streamed kernel.
// Strided sources take it when every row is a whole number of tiles (a
// column slab of B 4096 or 8192 wide, say) and rows start on 16 bytes.
template <int P, typename T>
bool launch_pack_ws(const T* src, int64_t elems, int8_t* planes, cudaStream_t stream, cudaError_t* err,
                    int64_t row_tiles = 0, int64_t ld = 0) {
  if (elems < kPackTile || elems % 8 != 0 || reinterpret_cast<uintptr_t>(src) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(planes) % 8 != 0 || (row_tiles > 0 && ld % 2 != 0))
    return false;
  if (row_tiles == 0) row_tiles = (elems + kPackTile - 1) / kPackTile;  // compact: one row of tiles
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    *err = cudaGetLastError();
    return true;
  }
  constexpr int smem = kPackStages * kPackTile * 8;
  auto kernel = pack_ws_kernel<P, T>;
  static std::atomic<uint64_t> configured{0};
  *err = raise_smem_limit_once(kernel, smem, configured);
  if (*err != cudaSuccess) return true;
  const int64_t tiles = elems / kPackTile;
  kernel<<<static_cast<unsigned>(tiles < sms ? tiles : sms), kPackThreads, smem, stream>>>(src, elems, planes,
                                                                                           row_tiles, ld);
  *err = cudaGetLastError();
  return true;
}

template <int P, typename T>
cudaError_t launch_pack(const T* src, int64_t rows, int64_t cols, int64_t ld, int8_t* planes, cudaStream_t stream) {
  if (ld == cols) {  // compact source: one long row, so any column count can take the vector path
    cols *= rows;
    ld = cols;
    rows = 1;
    cudaError_t err = cudaSuccess;
    if (launch_pack_ws<P, T>(src, cols, planes, stream, &err)) return err;
  } else if (cols % kPackTile == 0) {
    cudaError_t err = cudaSuccess;
    if (launch_pack_ws<P, T>(src, rows * cols, planes, stream, &err, cols / kPackTile, ld)) return err;
  }
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

// ---- selected planes (plane sharding) -------------------------------------------
// The same arithmetic as residue_byte with the per-plane constants read from
// the kernel parameters instead of immediates; modulus 256 needs no special
// case (weights 1,0,...; start 0; magic 2^24 gives q = (b0 + 128) >> 8).
constexpr int kSubsetMax = 10;  // planes per launch; larger subsets take two launches

struct SubsetConsts {
  uint32_t wl[kSubsetMax], wh[kSubsetMax], start[kSubsetMax], magic[kSubsetMax], m[kSubsetMax];
  uint64_t hmagic[kSubsetMax];  // floor(m / 2) * magic
};

template <bool kSigned>
SubsetConsts subset_consts(const uint32_t* plane_index, uint32_t count) {
  SubsetConsts c{};
  for (uint32_t j = 0; j < count; ++j) {
    const uint32_t m = ladder_modulus(static_cast<int>(plane_index[j]));
    uint64_t pow = 1, pow56 = 1;
    for (int b = 0; b < 8; ++b) {
      if (b < 4)
        c.wl[j] |= static_cast<uint32_t>(pow) << (8 * b);
      else
        c.wh[j] |= static_cast<uint32_t>(pow) << (8 * (b - 4));
      if (b == 7) pow56 = pow;
      pow = (pow * 256) % m;
    }
    const uint32_t pow63 = static_cast<uint32_t>((pow56 * 128) % m);
    c.start[j] = kSigned ? (m - pow63) % m : 0u;
    c.magic[j] = static_cast<uint32_t>(((1ull << 32) + m - 1) / m);
    c.m[j] = m;
    c.hmagic[j] = static_cast<uint64_t>(m / 2) * c.magic[j];
  }
  return c;
}

__device__ __forceinline__ uint32_t residue_byte_rt(const Words& w, const SubsetConsts& c, int j) {
  uint32_t t = __dp4a(w.hi, c.wh[j], c.start[j]);
  t = __dp4a(w.lo, c.wl[j], t);
  const uint32_t q = static_cast<uint32_t>((static_cast<uint64_t>(t) * c.magic[j] + c.hmagic[j]) >> 32);
  return t - q * c.m[j];
}

template <int NP, typename T>
__global__ void __launch_bounds__(256) pack_subset_vec8_kernel(const T* __restrict__ src, int64_t rows, int64_t cols,
                                                                int64_t ld, int8_t* __restrict__ planes,
                                                                const __grid_constant__ SubsetConsts c) {
  const int64_t groups_per_row = cols >> 3;
  const int64_t total = rows * groups_per_row;
  const int64_t plane_elems = rows * cols;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = g / groups_per_row;
    const int64_t col = (g - row * groups_per_row) << 3;
    const int4* in = reinterpret_cast<const int4*>(src + row * ld + col);
    Words d[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int4 v = __ldcs(in + q);
      d[2 * q] = split_words<T>(static_cast<T>((static_cast<uint64_t>(static_cast<uint32_t>(v.y)) << 32) |
                                               static_cast<uint32_t>(v.x)));
      d[2 * q + 1] = split_words<T>(static_cast<T>((static_cast<uint64_t>(static_cast<uint32_t>(v.w)) << 32) |
                                                   static_cast<uint32_t>(v.z)));
    }
    int8_t* out = planes + row * cols + col;
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      uint2 w;
      w.x = pack4(residue_byte_rt(d[0], c, j), residue_byte_rt(d[1], c, j), residue_byte_rt(d[2], c, j),
                  residue_byte_rt(d[3], c, j));
      w.y = pack4(residue_byte_rt(d[4], c, j), residue_byte_rt(d[5], c, j), residue_byte_rt(d[6], c, j),
                  residue_byte_rt(d[7], c, j));
      __stcs(reinterpret_cast<uint2*>(out + static_cast<int64_t>(j) * plane_elems), w);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) pack_subset_scalar_kernel(const T* __restrict__ src, int64_t rows,
                                                                  int64_t cols, int64_t ld, uint32_t count,
                                                                  int8_t* __restrict__ planes,
                                                                  const __grid_constant__ SubsetConsts c) {
  const int64_t total = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / cols, col = i - row * cols;
    const Words d = split_words<T>(src[row * ld + col]);
    for (uint32_t j = 0; j < count; ++j)
      planes[static_cast<int64_t>(j) * total + i] = static_cast<int8_t>(residue_byte_rt(d, c, static_cast<int>(j)) & 0xFFu);
  }
}

template <typename T>
cudaError_t launch_subset(const T* src, int64_t rows, int64_t cols, int64_t ld, const uint32_t* plane_index,
                          uint32_t count, int8_t* planes, cudaStream_t stream) {
  constexpr bool kSigned = static_cast<T>(-1) < 0;
  const SubsetConsts c = subset_consts<kSigned>(plane_index, count);
  if (ld == cols) {  // compact source: one long row
    cols *= rows;
    ld = cols;
    rows = 1;
  }
  const bool vec = (cols % 8 == 0) && (ld % 2 == 0) && (reinterpret_cast<uintptr_t>(src) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(planes) % 8 == 0);
  const int64_t work = vec ? rows * (cols / 8) : rows * cols;
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  const unsigned grid = static_cast<unsigned>(blocks);
  if (!vec) {
    pack_subset_scalar_kernel<T><<<grid, 256, 0, stream>>>(src, rows, cols, ld, count, planes, c);
    return cudaGetLastError();
  }
  switch (count) {
#define RNS8_SUBSET_CASE(NP)   case NP: pack_subset_vec8_kernel<NP, T><<<grid, 256, 0, stream>>>(src, rows, cols, ld, planes, c); break;
    RNS8_SUBSET_CASE(1) RNS8_SUBSET_CASE(2) RNS8_SUBSET_CASE(3) RNS8_SUBSET_CASE(4) RNS8_SUBSET_CASE(5)
    RNS8_SUBSET_CASE(6) RNS8_SUBSET_CASE(7) RNS8_SUBSET_CASE(8) RNS8_SUBSET_CASE(9) RNS8_SUBSET_CASE(10)
#undef RNS8_SUBSET_CASE
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_subset(const T* src, int64_t rows, int64_t cols, int64_t ld, const uint32_t* plane_index,
                            uint32_t count, int8_t* planes, cudaStream_t stream) {
  if (!plane_index || count == 0 || count > 20) return cudaErrorInvalidValue;
  for (uint32_t j = 0; j < count; ++j)
    if (plane_index[j] >= 20) return cudaErrorInvalidValue;
  const int64_t plane_elems = rows * cols;
  for (uint32_t j0 = 0; j0 < count; j0 += kSubsetMax) {
    const uint32_t n = count - j0 < static_cast<uint32_t>(kSubsetMax) ? count - j0 : static_cast<uint32_t>(kSubsetMax);
    const cudaError_t e = launch_subset<T>(src, rows, cols, ld, plane_index + j0, n, planes + j0 * plane_elems, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Finite u8: residues of bytes modulo an arbitrary m in [2, 256].
enum class U8Kind : int {
  General = 0,   // m < 128: magic-multiply modulo per byte
  OneStep = 1,   // 128 <= m < 171: a byte needs at most one subtraction of m
  Identity = 2,  // m = 256: the byte read as int8 is the centered residue
  Centered = 3,  // 171 <= m < 256: x >= ceil(m/2) ? x - m : x, one compare per byte
};

template <U8Kind kKind>
__device__ __forceinline__ uint32_t residues4(uint32_t x, uint32_t m, uint32_t magic, uint32_t m4, uint32_t h4) {
  if constexpr (kKind == U8Kind::Identity) {
    return x;
  } else if constexpr (kKind == U8Kind::Centered) {
    // For m >= 171 a byte x >= m is below ceil(m/2) after one subtraction, so
    // the centered residue is x - m exactly when x >= h = ceil(m/2) (h in
    // [86, 128]). Bit 7 of (x & 0x7F) + (128 - h) flags 7-bit values >= h;
    // OR x's own bit 7 (x >= 128 >= h). The flagged bytes take m (no byte
    // overflows: m < 256), subtracted bytewise without borrows between bytes.
    constexpr uint32_t kHigh = 0x80808080u;
    const uint32_t t = (x & 0x7F7F7F7Fu) + h4;  // h4 holds 128 - h per byte here
    const uint32_t sub = (((t | x) & kHigh) >> 7) * m;
    return ((x | kHigh) - (sub & ~kHigh)) ^ ((x ^ ~sub) & kHigh);
  } else if constexpr (kKind == U8Kind::OneStep) {
    // Per byte: t = x >= m ? x - m : x, then t >= ceil(m/2) ? t - m : t
    // (mod 256, i.e. the int8 of the centered residue).
    const uint32_t t = __vsub4(x, __vcmpgeu4(x, m4) & m4);
    return __vsub4(t, __vcmpgeu4(t, h4) & m4);
  } else {
    uint32_t r[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) r[b] = static_cast<uint32_t>(center_residue(umod_u32((x >> (8 * b)) & 0xFFu, m, magic), m));
    return pack4(r[0], r[1], r[2], r[3]);
  }
}

// 16 bytes per thread; grid.x over the 16-byte groups of a row, grid.y over
// rows (a contiguous matrix is passed as one row), so no division per group.
template <U8Kind kKind>
__global__ void __launch_bounds__(256) pack_u8_vec16_kernel(const uint8_t* __restrict__ src, int64_t rows,
                                                            int64_t cols, int64_t ld, uint32_t m, uint32_t magic,
                                                            int8_t* __restrict__ out) {
  const int64_t groups = cols >> 4;
  const uint32_t m4 = (m & 0xFFu) * 0x01010101u;
  const uint32_t h4 = kKind == U8Kind::Centered ? (128u - (m + 1) / 2) * 0x01010101u  // 128 - ceil(m/2)
                                                : ((m + 1) / 2) * 0x01010101u;        // ceil(m/2)
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const uint4* s = reinterpret_cast<const uint4*>(src + row * ld);
    uint4* o = reinterpret_cast<uint4*>(out + row * cols);
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      uint4 v = __ldcs(s + g);
      v.x = residues4<kKind>(v.x, m, magic, m4, h4);
      v.y = residues4<kKind>(v.y, m, magic, m4, h4);
      v.z = residues4<kKind>(v.z, m, magic, m4, h4);
      v.w = residues4<kKind>(v.w, m, magic, m4, h4);
      __stcs(o + g, v);
    }
  }
}

__global__ void __launch_bounds__(256) pack_u8_scalar_kernel(const uint8_t* __restrict__ src, int64_t rows,
                                                             int64_t cols, int64_t ld, uint32_t m, uint32_t magic,
                                                             int8_t* __restrict__ out) {
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    for (int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; col < cols;
         col += static_cast<int64_t>(gridDim.x) * blockDim.x)
      out[row * cols + col] = static_cast<int8_t>(center_residue(umod_u32(src[row * ld + col], m, magic), m));
  }
}

// Largest |x| (x for unsigned) of count contiguous 64-bit values into *out
// (zeroed first), by a grid-stride sweep and one atomicMax per warp.
__global__ void __launch_bounds__(256) max_magnitude_kernel(const uint64_t* __restrict__ src, int64_t count,
                                                            bool is_signed, unsigned long long* out) {
  unsigned long long mx = 0;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count; i += step) {
    const uint64_t v = __ldcs(src + i);
    const uint64_t mag = (is_signed && (v >> 63)) ? 0 - v : v;
    mx = mag > mx ? mag : mx;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
    mx = other > mx ? other : mx;
  }
  if ((threadIdx.x & 31) == 0 && mx != 0) atomicMax(out, mx);
}

}  // namespace

cudaError_t max_magnitude(const void* src, int64_t count, bool is_signed, uint64_t* out, int sm_count,
                          cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(uint64_t), stream);
  if (e != cudaSuccess || count <= 0) return e;
  int64_t blocks = (count + 255) / 256;
  if (blocks > static_cast<int64_t>(sm_count) * 8) blocks = static_cast<int64_t>(sm_count) * 8;
  max_magnitude_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      static_cast<const uint64_t*>(src), count, is_signed, reinterpret_cast<unsigned long long*>(out));
  return cudaGetLastError();
}

cudaError_t pack_i64(const int64_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* planes,
                     cudaStream_t stream) {
  return dispatch_pack<int64_t>(src, rows, cols, ld, prefix, planes, stream);
}
cudaError_t pack_u64(const uint64_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* planes,
                     cudaStream_t stream) {
  return dispatch_pack<uint64_t>(src, rows, cols, ld, prefix, planes, stream);
}
cudaError_t pack_planes_i64(const int64_t* src, int64_t rows, int64_t cols, int64_t ld, const uint32_t* plane_index,
                            uint32_t plane_count, int8_t* planes, cudaStream_t stream) {
  return dispatch_subset<int64_t>(src, rows, cols, ld, plane_index, plane_count, planes, stream);
}
cudaError_t pack_planes_u64(const uint64_t* src, int64_t rows, int64_t cols, int64_t ld, const uint32_t* plane_index,
                            uint32_t plane_count, int8_t* planes, cudaStream_t stream) {
  return dispatch_subset<uint64_t>(src, rows, cols, ld, plane_index, plane_count, planes, stream);
}
cudaError_t pack_finite_u8(const uint8_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t modulus,
                           int8_t* residues, cudaStream_t stream) {
  if (modulus < 2 || modulus > 256) return cudaErrorInvalidValue;
  const uint32_t magic = floor_magic(modulus);
  if (ld == cols) {  // contiguous: one long row
    cols *= rows;
    ld = cols;
    rows = 1;
  }
  const bool vec = (cols % 16 == 0) && (ld % 16 == 0) && (reinterpret_cast<uintptr_t>(src) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(residues) % 16 == 0);
  const int64_t per_row = vec ? cols / 16 : cols;
  int64_t bx = (per_row + 255) / 256;
  const int64_t by = rows < 65535 ? rows : 65535;
  const int64_t max_x = (148 * 16 + by - 1) / by;  // about 16 blocks per SM in all
  if (bx > max_x) bx = max_x;
  if (bx < 1) bx = 1;
  const dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(by));
  if (!vec)
    pack_u8_scalar_kernel<<<grid, 256, 0, stream>>>(src, rows, cols, ld, modulus, magic, residues);
  else if (modulus == 256)
    pack_u8_vec16_kernel<U8Kind::Identity><<<grid, 256, 0, stream>>>(src, rows, cols, ld, modulus, magic, residues);
  else if (modulus >= 171)
    pack_u8_vec16_kernel<U8Kind::Centered><<<grid, 256, 0, stream>>>(src, rows, cols, ld, modulus, magic, residues);
  else if (modulus >= 128)
    pack_u8_vec16_kernel<U8Kind::OneStep><<<grid, 256, 0, stream>>>(src, rows, cols, ld, modulus, magic, residues);
  else
    pack_u8_vec16_kernel<U8Kind::General><<<grid, 256, 0, stream>>>(src, rows, cols, ld, modulus, magic, residues);
  return cudaGetLastError();
}

}  // namespace rns8cuda
