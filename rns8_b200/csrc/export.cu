// Export kernels: centered residue planes -> bounded int64 / uint64, or
// fixed-width little-endian limbs (exact-wide), or canonical finite u8.
//
// Reference behaviour: src/reconstruct/crt.cpp:54-170 (Garner order,
// centering at ceil(P/2), fits checks, two's-complement limbs) and
// src/core/api_export.cpp:307-803 (a failing cell makes the whole export a
// RANGE_ERROR). The device status word replaces the reference's
// atomicCAS(status, 0, 5) (hip_direct_export_kernels.cuh:137-177).
//
// The digit recurrence and Horner rebuild live in garner.cuh.
#include <algorithm>
#include <vector>

#include <cstring>

#include "garner.cuh"
#include "gemm_internal.hpp"
#include "kernels.hpp"

namespace rns8cuda {
namespace {

using namespace garner;

enum class Mode : int { I64 = 0, U64 = 1, LimbsSigned = 2, LimbsUnsigned = 3 };

struct ExportArgs {
  const int8_t* planes;
  int64_t m, n;
  int64_t ld;
  BoundedLimits lim;              // I64 / U64
  FracLimits frac;                // I64 / U64 fast path
  uint32_t limb_count;            // limb modes
  void* dst;
  uint32_t* status;
};

__device__ __forceinline__ int64_t dst_index(const ExportArgs& a, int64_t cell) {
  if (a.ld == a.n) return cell;
  const int64_t row = cell / a.n;
  return row * a.ld + (cell - row * a.n);
}

// Writes a cell's limbs from its 192-bit value w32 (two's complement for the
// signed mode, the canonical value for the unsigned one): limb_count limbs,
// sign (or zero) filled above 192 bits; false when the value does not fit.
template <Mode kMode>
__device__ __forceinline__ bool store_limbs(const ExportArgs& a, int64_t cell, const uint32_t (&w32)[6]) {
  uint64_t v[3];
#pragma unroll
  for (int l = 0; l < 3; ++l) v[l] = static_cast<uint64_t>(w32[2 * l]) | (static_cast<uint64_t>(w32[2 * l + 1]) << 32);
  const uint32_t limbs = a.limb_count;
  const uint64_t sign_fill = (kMode == Mode::LimbsSigned && (v[2] >> 63)) ? ~0ull : 0ull;
  if (limbs == 1) {
    const uint64_t ext = (kMode == Mode::LimbsSigned && (v[0] >> 63)) ? ~0ull : 0ull;
    if (v[1] != ext || v[2] != ext) return false;
  } else if (limbs == 2) {
    const uint64_t ext = (kMode == Mode::LimbsSigned && (v[1] >> 63)) ? ~0ull : 0ull;
    if (v[2] != ext) return false;
  }
  uint64_t* out = static_cast<uint64_t*>(a.dst) + dst_index(a, cell) * static_cast<int64_t>(limbs);
  out[0] = v[0];
  if (limbs > 1) out[1] = v[1];
  if (limbs > 2) out[2] = v[2];
  for (uint32_t l = 3; l < limbs; ++l) out[l] = sign_fill;
  return true;
}

// Reconstructs one cell into dst (one int64/uint64, or limb_count limbs).
template <int P, Mode kMode>
__device__ __forceinline__ bool export_cell(const ExportArgs& a, int64_t cell, const int (&r)[P]) {
  if constexpr (kMode == Mode::I64 || kMode == Mode::U64) {
    uint64_t v;
    if (!reconstruct_bounded<P, kMode == Mode::I64>(r, a.lim, &v)) return false;
    static_cast<uint64_t*>(a.dst)[dst_index(a, cell)] = v;
    return true;
  } else {
    constexpr int L = limbs32_for<P>();
    constexpr GarnerTable<P> T = make_table<P>();
    uint32_t c[P];
    uint32_t cp[(P + 3) / 4];
    garner_digits<P>(r, cp, c);
    uint32_t x[L];
    horner32<P, L>(c, x);
    // 192-bit two's-complement working value in 64-bit limbs.
    uint32_t w32[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int l = 0; l < L; ++l) w32[l] = x[l];
    if (kMode == Mode::LimbsSigned && geq32<L>(x, T.half)) {
      uint64_t borrow = 0;
#pragma unroll
      for (int l = 0; l < 6; ++l) {
        const uint64_t sub = static_cast<uint64_t>(l < kLimbs32 ? T.product[l] : 0u) + borrow;
        const uint64_t cur = w32[l];
        borrow = cur < sub ? 1 : 0;
        w32[l] = static_cast<uint32_t>(cur - sub);
      }
    }
    return store_limbs<kMode>(a, cell, w32);
  }
}

// Exact-wide limbs by the fractional CRT (garner.cuh, wide_frac_reconstruct):
// each thread takes 4 consecutive cells (one 32-bit load per plane), turns
// the P plane words into 4-plane cell words with byte permutes, reconstructs
// every cell with dp4a byte-slice sums, and sends the rare cells whose
// quotient is in doubt (|v| within rounding error of M/2) to the exact
// Garner path.
template <int P, Mode kMode>
__global__ void __launch_bounds__(256) export_limbs_frac_kernel(ExportArgs a) {
  constexpr int kG = (P + 3) / 4;
  constexpr GarnerTable<P> GT = make_table<P>();
  const int64_t cells = a.m * a.n;
  const int64_t groups = cells / 4;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  bool bad = false;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += step) {
    uint32_t w[4 * kG];
#pragma unroll
    for (int p = 0; p < 4 * kG; ++p)
      w[p] = p < P ? (__ldcs(reinterpret_cast<const uint32_t*>(a.planes + static_cast<int64_t>(p) * cells) + g) ^
                      0x80808080u)
                   : 0u;
    uint32_t cw[4][kG];
#pragma unroll
    for (int q = 0; q < kG; ++q) {  // 4 x 4 byte transpose: plane words -> cell words
      const uint32_t t0 = __byte_perm(w[4 * q], w[4 * q + 1], 0x5140);
      const uint32_t t1 = __byte_perm(w[4 * q + 2], w[4 * q + 3], 0x5140);
      const uint32_t t2 = __byte_perm(w[4 * q], w[4 * q + 1], 0x7362);
      const uint32_t t3 = __byte_perm(w[4 * q + 2], w[4 * q + 3], 0x7362);
      cw[0][q] = __byte_perm(t0, t1, 0x5410);
      cw[1][q] = __byte_perm(t0, t1, 0x7632);
      cw[2][q] = __byte_perm(t2, t3, 0x5410);
      cw[3][q] = __byte_perm(t2, t3, 0x7632);
    }
    uint32_t undecided = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t v[6];
      if (!wide_frac_reconstruct<P>(cw[c], v)) {
        undecided |= 1u << c;
        continue;
      }
      if constexpr (kMode == Mode::LimbsUnsigned) {
        if (v[5] >> 31) {  // centered value below zero: the canonical value is v + M
          uint64_t carry = 0;
#pragma unroll
          for (int l = 0; l < 6; ++l) {
            const uint64_t t = static_cast<uint64_t>(v[l]) + (l < kLimbs32 ? GT.product[l] : 0u) + carry;
            v[l] = static_cast<uint32_t>(t);
            carry = t >> 32;
          }
        }
      }
      bad |= !store_limbs<kMode>(a, 4 * g + c, v);
    }
    while (undecided != 0) {
      const int c = __ffs(undecided) - 1;
      undecided &= undecided - 1;
      int r[P];
#pragma unroll
      for (int p = 0; p < P; ++p) r[p] = static_cast<int>((w[p] >> (8 * c)) & 0xFFu) - 128;
      bad |= !export_cell<P, kMode>(a, 4 * g + c, r);
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicOr(a.status, kDevRangeError);
}

// Each thread reconstructs 4 consecutive cells (one 32-bit load per plane).
template <int P, Mode kMode, bool kVec4>
__global__ void __launch_bounds__(256) export_kernel(ExportArgs a) {
  const int64_t cells = a.m * a.n;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  bool bad = false;
  if (kVec4) {
    const int64_t groups = cells >> 2;
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += step) {
      uint32_t w[P];
#pragma unroll
      for (int p = 0; p < P; ++p) w[p] = __ldcs(reinterpret_cast<const uint32_t*>(a.planes + static_cast<int64_t>(p) * cells) + g);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int r[P];
#pragma unroll
        for (int p = 0; p < P; ++p) r[p] = static_cast<int>(static_cast<int8_t>(w[p] >> (8 * e)));
        bad |= !export_cell<P, kMode>(a, 4 * g + e, r);
      }
    }
  } else {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < cells; i += step) {
      int r[P];
#pragma unroll
      for (int p = 0; p < P; ++p) r[p] = a.planes[static_cast<int64_t>(p) * cells + i];
      bad |= !export_cell<P, kMode>(a, i, r);
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicOr(a.status, kDevRangeError);
}

template <int kCells>
__device__ __forceinline__ void load_plane_words(const int8_t* src, uint32_t (&w)[kCells / 4]) {
  if constexpr (kCells == 4) {
    w[0] = __ldcs(reinterpret_cast<const unsigned int*>(src));
  } else if constexpr (kCells == 8) {
    const uint2 v = __ldcs(reinterpret_cast<const uint2*>(src));
    w[0] = v.x;
    w[1] = v.y;
  } else {
    const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src));
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  }
}

// Bounded int64 / uint64 export, kCells consecutive cells per thread: one
// kCells-byte load per plane, the fractional CRT per cell, 16-byte streaming
// stores when the destination is contiguous (ld == n, 16-byte aligned).
template <int P, bool kSigned, int kCells, bool kContig>
__global__ void __launch_bounds__(256) export_bounded_kernel(ExportArgs a) {
  const int64_t cells = a.m * a.n;
  const int64_t groups = cells / kCells;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  bool bad = false;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += step) {
    uint32_t w[P][kCells / 4];
#pragma unroll
    for (int p = 0; p < P; ++p) {
      load_plane_words<kCells>(a.planes + static_cast<int64_t>(p) * cells + g * kCells, w[p]);
#pragma unroll
      for (int j = 0; j < kCells / 4; ++j) w[p][j] ^= 0x80808080u;  // r + 128 in every byte
    }
    // Fast path: the fractional CRT. Cells it cannot decide are flagged and
    // redone by the exact Garner path below, after the vector stores.
    uint32_t undecided = a.frac.enabled ? 0u : (1u << kCells) - 1u;
    const int64_t first = g * kCells;
    if (a.frac.enabled) {
#pragma unroll
      for (int e = 0; e < kCells; e += 2) {
        uint64_t v[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t u[P];
#pragma unroll
          for (int p = 0; p < P; ++p)
            u[p] = __byte_perm(w[p][(e + h) / 4], 0u, 0x4440u | static_cast<uint32_t>((e + h) & 3));
          const int verdict = frac_reconstruct<P>(u, a.frac, &v[h]);
          bad |= verdict == 0;
          undecided |= verdict < 0 ? (1u << (e + h)) : 0u;
        }
        if constexpr (kContig) {
          __stcs(reinterpret_cast<ulonglong2*>(static_cast<uint64_t*>(a.dst) + first + e),
                 make_ulonglong2(static_cast<unsigned long long>(v[0]), static_cast<unsigned long long>(v[1])));
        } else {
          static_cast<uint64_t*>(a.dst)[dst_index(a, first + e)] = v[0];
          static_cast<uint64_t*>(a.dst)[dst_index(a, first + e + 1)] = v[1];
        }
      }
    }
    while (undecided != 0) {
      const int e = __ffs(undecided) - 1;
      undecided &= undecided - 1;
      int r[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        uint32_t word = w[p][0];
#pragma unroll
        for (int j = 1; j < kCells / 4; ++j) word = (e >> 2) == j ? w[p][j] : word;
        r[p] = static_cast<int>((word >> (8 * (e & 3))) & 0xFFu) - 128;
      }
      uint64_t v;
      if (reconstruct_bounded<P, kSigned>(r, a.lim, &v))
        static_cast<uint64_t*>(a.dst)[dst_index(a, first + e)] = v;
      else
        bad = true;
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && (threadIdx.x & 31) == 0) atomicOr(a.status, kDevRangeError);
}

// ---- bounded export, streamed (contiguous destinations) --------------------------
// A persistent CTA per SM: one producer warp streams each tile's slice of
// every plane (4096 cells, so P copies of 4 KiB) into a ring of shared-memory
// stages with 1-D bulk copies, and 16 consumer warps reconstruct eight cells
// per lane from shared memory with the two-plane dp2a sums (PairTable). The
// copies run ahead of the arithmetic by up to kStages tiles whatever the
// consumers are doing, which is what the register-fed kernel above cannot
// do: its loads wait behind its own multiply chains. full[s] completes when
// a stage's copies have landed; empty[s] when all consumer warps have read it.
constexpr int kWsConsumerWarps = 16;
constexpr int kWsThreads = 32 * (kWsConsumerWarps + 1);
constexpr int kWsTileCells = kWsConsumerWarps * 32 * 8;

// Eight consecutive cells from their P plane words (signed residues, cells
// 4j..4j+3 in word j): fractional CRT by the dp2a sums, 16-byte streaming
// stores, then the exact path for cells the fraction leaves undecided.
template <int P, bool kSigned>
__device__ __forceinline__ void pair_reconstruct8(const ExportArgs& a, uint64_t s_init,
                                                  uint32_t (&w)[2 * PairTable<P>::kPairs][2], int64_t first,
                                                  bool& bad) {
  constexpr PairTable<P> K = make_pair_table<P>();
  constexpr int kPairs = PairTable<P>::kPairs;
  if constexpr (P % 2 != 0) {
    w[P][0] = 0;
    w[P][1] = 0;
  }
  uint32_t undecided = 0;
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    int32_t f0[2] = {0, 0}, f1[2] = {0, 0}, g0[2] = {0, 0}, g1[2] = {0, 0}, g2[2] = {0, 0}, g3[2] = {0, 0};
    constexpr uint32_t kSel[2] = {0x5140u, 0x7362u};  // bytes (j, 4+j, j+1, 5+j) for j = 0, 2
    const uint32_t sel = kSel[(e & 3) >> 1];
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
      const int x = static_cast<int>(__byte_perm(w[2 * q][e / 4], w[2 * q + 1][e / 4], sel));
      f0[0] = __dp2a_lo(static_cast<int>(K.f[q][0]), x, f0[0]);
      f1[0] = __dp2a_lo(static_cast<int>(K.f[q][1]), x, f1[0]);
      g0[0] = __dp2a_lo(static_cast<int>(K.g[q][0]), x, g0[0]);
      g1[0] = __dp2a_lo(static_cast<int>(K.g[q][1]), x, g1[0]);
      g2[0] = __dp2a_lo(static_cast<int>(K.g[q][2]), x, g2[0]);
      g3[0] = __dp2a_lo(static_cast<int>(K.g[q][3]), x, g3[0]);
      f0[1] = __dp2a_hi(static_cast<int>(K.f[q][0]), x, f0[1]);
      f1[1] = __dp2a_hi(static_cast<int>(K.f[q][1]), x, f1[1]);
      g0[1] = __dp2a_hi(static_cast<int>(K.g[q][0]), x, g0[1]);
      g1[1] = __dp2a_hi(static_cast<int>(K.g[q][1]), x, g1[1]);
      g2[1] = __dp2a_hi(static_cast<int>(K.g[q][2]), x, g2[1]);
      g3[1] = __dp2a_hi(static_cast<int>(K.g[q][3]), x, g3[1]);
    }
    uint64_t v[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint64_t s = s_init + static_cast<uint64_t>(static_cast<int64_t>(f0[h])) +
                         (static_cast<uint64_t>(static_cast<int64_t>(f1[h])) << 16);
      const uint32_t s_lo = static_cast<uint32_t>(s);
      const uint32_t q = __funnelshift_r(s_lo, static_cast<uint32_t>(s >> 32), 31);
      const int32_t frac = static_cast<int32_t>(s_lo & 0x7FFFFFFFu) - (1 << 30);
      const uint32_t afrac = static_cast<uint32_t>(frac < 0 ? -frac : frac);
      bad |= afrac >= a.frac.t_out;
      undecided |= (afrac > a.frac.t_in && afrac < a.frac.t_out) ? (1u << (e + h)) : 0u;
      const uint64_t sum = static_cast<uint64_t>(static_cast<int64_t>(g0[h])) +
                           (static_cast<uint64_t>(static_cast<int64_t>(g1[h])) << 16) +
                           (static_cast<uint64_t>(static_cast<int64_t>(g2[h])) << 32) +
                           (static_cast<uint64_t>(static_cast<int64_t>(g3[h])) << 48);
      v[h] = sum + K.bias_m64 - static_cast<uint64_t>(q) * K.m64;
    }
    __stcs(reinterpret_cast<ulonglong2*>(static_cast<uint64_t*>(a.dst) + first + e),
           make_ulonglong2(static_cast<unsigned long long>(v[0]), static_cast<unsigned long long>(v[1])));
  }
  while (undecided != 0) {
    const int e = __ffs(undecided) - 1;
    undecided &= undecided - 1;
    int r[P];
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const uint32_t word = (e >> 2) ? w[p][1] : w[p][0];
      r[p] = static_cast<int>(static_cast<int8_t>((word >> (8 * (e & 3))) & 0xFFu));
    }
    uint64_t v;
    if (reconstruct_bounded<P, kSigned>(r, a.lim, &v))
      static_cast<uint64_t*>(a.dst)[first + e] = v;
    else
      bad = true;
  }
}

template <int P, bool kSigned, int kStages>
__global__ void __launch_bounds__(kWsThreads, 1) export_bounded_ws_kernel(ExportArgs a) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[kStages], empty[kStages];
  const int64_t cells = a.m * a.n;
  const int64_t tiles = cells / kWsTileCells;
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWsConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  int64_t mine = 0;  // tiles b, b + grid, ... of this CTA
  if (blockIdx.x < tiles) mine = (tiles - 1 - blockIdx.x) / gridDim.x + 1;
  if (warp == kWsConsumerWarps) {
    if (lane != 0) return;
    int64_t issued = 0;
    for (int64_t j = 0; j < mine; ++j, ++issued) {
      const int s = static_cast<int>(j % kStages);
      if (j >= kStages && !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(((j / kStages) - 1) & 1))) {
        atomicOr(a.status, kDevWaitTimeout);
        break;
      }
      const int64_t tile = blockIdx.x + j * gridDim.x;
      mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(P * kWsTileCells));
#pragma unroll
      for (int p = 0; p < P; ++p)
        bulk_load_1d(ring + (s * P + p) * kWsTileCells, a.planes + static_cast<int64_t>(p) * cells + tile * kWsTileCells,
                     kWsTileCells, &full[s]);
    }
    // Leave no copy in flight: wait (bounded) for the last stages issued.
    for (int64_t j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
      if (!mbar_wait_bounded(&full[j % kStages], static_cast<uint32_t>((j / kStages) & 1)))
        atomicOr(a.status, kDevWaitTimeout);
    return;
  }
  const uint64_t s_init = a.frac.s_init + make_pair_table<P>().sumF128;  // residues r, not r + 128
  bool bad = false;
  const int off = (warp * 32 + lane) * 8;
  for (int64_t j = 0; j < mine; ++j) {
    const int s = static_cast<int>(j % kStages);
    if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>((j / kStages) & 1))) {
      if (lane == 0) atomicOr(a.status, kDevWaitTimeout);
      break;
    }
    uint32_t w[2 * PairTable<P>::kPairs][2];
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const uint2 v = *reinterpret_cast<const uint2*>(ring + (s * P + p) * kWsTileCells + off);
      w[p][0] = v.x;
      w[p][1] = v.y;
    }
    release_stage_reads();  // the stage is refilled once every warp has arrived on empty[s]
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    pair_reconstruct8<P, kSigned>(a, s_init, w, (blockIdx.x + j * gridDim.x) * kWsTileCells + off, bad);
  }
  // The last, partial tile (fewer than 4096 cells): one CTA, exact path.
  if (blockIdx.x == tiles % gridDim.x) {
    for (int64_t c = tiles * kWsTileCells + warp * 32 + lane; c < cells; c += kWsConsumerWarps * 32) {
      int r[P];
#pragma unroll
      for (int p = 0; p < P; ++p) r[p] = a.planes[static_cast<int64_t>(p) * cells + c];
      uint64_t v;
      if (reconstruct_bounded<P, kSigned>(r, a.lim, &v))
        static_cast<uint64_t*>(a.dst)[c] = v;
      else
        bad = true;
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(a.status, kDevRangeError);
}

// ---- exact-wide limb export, streamed ---------------------------------------------
// The same producer / consumer ring as the bounded export, with tiles of 2048
// cells (each lane takes four consecutive cells, one 32-bit word per plane)
// and the wide fractional CRT of export_limbs_frac_kernel per cell. With
// three limbs and a contiguous, 16-byte aligned destination, a lane's four
// cells are twelve consecutive limbs, written as six 16-byte stores.
constexpr int kLimbTileCells = kWsConsumerWarps * 32 * 4;

template <int P, Mode kMode>
__device__ __forceinline__ void limbs_from_words(const ExportArgs& a, uint32_t (&w)[4 * ((P + 3) / 4)], int64_t first,
                                                 bool vec3, bool& bad) {
  constexpr int kG = (P + 3) / 4;
  constexpr GarnerTable<P> GT = make_table<P>();
#pragma unroll
  for (int p = 0; p < 4 * kG; ++p) w[p] = p < P ? (w[p] ^ 0x80808080u) : 0u;
  uint32_t cw[4][kG];
#pragma unroll
  for (int q = 0; q < kG; ++q) {  // 4 x 4 byte transpose: plane words -> cell words
    const uint32_t t0 = __byte_perm(w[4 * q], w[4 * q + 1], 0x5140);
    const uint32_t t1 = __byte_perm(w[4 * q + 2], w[4 * q + 3], 0x5140);
    const uint32_t t2 = __byte_perm(w[4 * q], w[4 * q + 1], 0x7362);
    const uint32_t t3 = __byte_perm(w[4 * q + 2], w[4 * q + 3], 0x7362);
    cw[0][q] = __byte_perm(t0, t1, 0x5410);
    cw[1][q] = __byte_perm(t0, t1, 0x7632);
    cw[2][q] = __byte_perm(t2, t3, 0x5410);
    cw[3][q] = __byte_perm(t2, t3, 0x7632);
  }
  uint32_t undecided = 0;
  uint64_t limbs[4][3];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t v[6];
    if (!wide_frac_reconstruct<P>(cw[c], v)) {
      undecided |= 1u << c;
      limbs[c][0] = limbs[c][1] = limbs[c][2] = 0;
      continue;
    }
    if constexpr (kMode == Mode::LimbsUnsigned) {
      if (v[5] >> 31) {  // centered value below zero: the canonical value is v + M
        uint64_t carry = 0;
#pragma unroll
        for (int l = 0; l < 6; ++l) {
          const uint64_t t = static_cast<uint64_t>(v[l]) + (l < kLimbs32 ? GT.product[l] : 0u) + carry;
          v[l] = static_cast<uint32_t>(t);
          carry = t >> 32;
        }
      }
    }
    if (vec3) {
#pragma unroll
      for (int l = 0; l < 3; ++l)
        limbs[c][l] = static_cast<uint64_t>(v[2 * l]) | (static_cast<uint64_t>(v[2 * l + 1]) << 32);
    } else {
      bad |= !store_limbs<kMode>(a, first + c, v);
    }
  }
  if (vec3) {  // 12 limbs of 4 cells, 96 contiguous bytes
    ulonglong2* out = reinterpret_cast<ulonglong2*>(static_cast<uint64_t*>(a.dst) + first * 3);
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      const int i0 = 2 * j, i1 = 2 * j + 1;
      __stcs(out + j, make_ulonglong2(static_cast<unsigned long long>(limbs[i0 / 3][i0 % 3]),
                                      static_cast<unsigned long long>(limbs[i1 / 3][i1 % 3])));
    }
  }
  while (undecided != 0) {  // rewrites the placeholder limbs of undecided cells
    const int c = __ffs(undecided) - 1;
    undecided &= undecided - 1;
    int r[P];
#pragma unroll
    for (int p = 0; p < P; ++p) r[p] = static_cast<int>((w[p] >> (8 * c)) & 0xFFu) - 128;
    bad |= !export_cell<P, kMode>(a, first + c, r);
  }
}

template <int P, Mode kMode, int kStages>
__global__ void __launch_bounds__(kWsThreads, 1) export_limbs_ws_kernel(ExportArgs a) {
  constexpr int kG = (P + 3) / 4;
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[kStages], empty[kStages];
  const int64_t cells = a.m * a.n;
  const int64_t tiles = cells / kLimbTileCells;
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWsConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  int64_t mine = 0;
  if (blockIdx.x < tiles) mine = (tiles - 1 - blockIdx.x) / gridDim.x + 1;
  if (warp == kWsConsumerWarps) {
    if (lane != 0) return;
    int64_t issued = 0;
    for (int64_t j = 0; j < mine; ++j, ++issued) {
      const int s = static_cast<int>(j % kStages);
      if (j >= kStages && !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(((j / kStages) - 1) & 1))) {
        atomicOr(a.status, kDevWaitTimeout);
        break;
      }
      const int64_t tile = blockIdx.x + j * gridDim.x;
      mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(P * kLimbTileCells));
#pragma unroll
      for (int p = 0; p < P; ++p)
        bulk_load_1d(ring + (s * P + p) * kLimbTileCells,
                     a.planes + static_cast<int64_t>(p) * cells + tile * kLimbTileCells, kLimbTileCells, &full[s]);
    }
    for (int64_t j = issued > kStages ? issued - kStages : 0; j < issued; ++j)
      if (!mbar_wait_bounded(&full[j % kStages], static_cast<uint32_t>((j / kStages) & 1)))
        atomicOr(a.status, kDevWaitTimeout);
    return;
  }
  const bool vec3 = a.limb_count == 3 && a.ld == a.n && reinterpret_cast<uintptr_t>(a.dst) % 16 == 0;
  bool bad = false;
  const int off = (warp * 32 + lane) * 4;
  for (int64_t j = 0; j < mine; ++j) {
    const int s = static_cast<int>(j % kStages);
    if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>((j / kStages) & 1))) {
      if (lane == 0) atomicOr(a.status, kDevWaitTimeout);
      break;
    }
    uint32_t w[4 * kG];
#pragma unroll
    for (int p = 0; p < P; ++p) w[p] = *reinterpret_cast<const uint32_t*>(ring + (s * P + p) * kLimbTileCells + off);
    release_stage_reads();  // the stage is refilled once every warp has arrived on empty[s]
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    limbs_from_words<P, kMode>(a, w, (blockIdx.x + j * gridDim.x) * kLimbTileCells + off, vec3, bad);
  }
  // The last, partial tile (fewer than 2048 cells): one CTA, exact path.
  if (blockIdx.x == tiles % gridDim.x) {
    for (int64_t c = tiles * kLimbTileCells + warp * 32 + lane; c < cells; c += kWsConsumerWarps * 32) {
      int r[P];
#pragma unroll
      for (int p = 0; p < P; ++p) r[p] = a.planes[static_cast<int64_t>(p) * cells + c];
      bad |= !export_cell<P, kMode>(a, c, r);
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(a.status, kDevRangeError);
}

template <int P>
constexpr int limb_ws_stages() {
  constexpr int by_smem = (224 * 1024) / (P * kLimbTileCells);
  return by_smem > 4 ? 4 : by_smem;
}

template <int P, Mode kMode>
bool launch_limbs_ws(const ExportArgs& a, cudaStream_t stream, cudaError_t* err) {
  constexpr int kStages = limb_ws_stages<P>();
  const int64_t cells = a.m * a.n;
  if (kStages < 2 || P < 2 || reinterpret_cast<uintptr_t>(a.planes) % 16 != 0 || cells % 16 != 0 ||
      cells < kLimbTileCells)
    return false;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    *err = cudaGetLastError();
    return true;
  }
  const int smem = kStages * P * kLimbTileCells;
  auto kernel = export_limbs_ws_kernel<P, kMode, kStages>;
  static std::atomic<uint64_t> configured{0};
  *err = raise_smem_limit_once(kernel, smem, configured);
  if (*err != cudaSuccess) return true;
  const int64_t tiles = cells / kLimbTileCells;
  kernel<<<static_cast<unsigned>(tiles < sms ? tiles : sms), kWsThreads, smem, stream>>>(a);
  *err = cudaGetLastError();
  return true;
}

// ---- exact-wide limb export on the tensor cores ----------------------------------
// The wide fractional CRT's sums over the residue planes, sum_i r_i * F_i (the
// quotient and fraction) and sum_i r_i * G_i (the value mod 2^192), split into
// 8-bit digit columns, form an int8 product of the planes (cells x planes)
// with a constant table (planes x 32 digit columns). One tcgen05 MMA per 128
// cells (M = 128 cells read MN-major by TMA straight from the compact planes;
// K = 32 planes; N = 32 digit columns from a table in shared memory) leaves
// every cell's digit sums in tensor memory, and the epilogue thread that owns
// the cell combines them, which takes the dp4a work off the integer pipe.
// F_i and G_i are written in signed 8-bit digits (x = sum_c d_c 2^(8c),
// d_c in [-128, 127]) so that both operands are s8 like the stored centered
// residues; with r_i in place of u_i = r_i + 128 the value is
// v = S + bias*M - q*M, S = sum_c T_c 2^(8c). Each digit sum has
// |T_c| <= 20 * 128 * 128 < 2^19, so two neighbouring sums combine in 32 bits
// (|T_c + 256 T_c+1| < 2^28) and a 32-bit limb of v is one signed 64-bit
// accumulation (carry + limb of bias*M + two pairs - q * limb of M, q < 2^14,
// every term below 2^47). A box holds roundup(P, 8) plane rows; the MMA
// always reads 32 rows, and table rows past P are zero, so the rows it reads
// beyond the box (the next box, or the table) add nothing. (The bounded
// int64 export built the same way, with 16 digit columns, ran at 342 us
// against 200 us for the streamed dp2a kernel at 8192^2 x 9: with little
// arithmetic per cell, the MMA -> tensor memory -> epilogue latency and the
// cells that tensor memory can hold in flight set its rate.)
constexpr int kTcFDigits = 5;  // F_i < 2^31 in signed digits (a carry can reach the fifth)
constexpr int kTcBoxCells = 128;
constexpr int kTcEpiWarps = 16;                // four groups of one warp per tensor-memory lane quarter
constexpr int kTcThreads = 32 * (2 + kTcEpiWarps);
constexpr uint32_t kTcTableBytes = 32 * 128;  // up to 32 rows of 128 bytes (K-major, swizzled)
constexpr int kTcMaxStages = 24;

template <int P, Mode kMode>
struct TcShape {
  static_assert(kMode == Mode::LimbsSigned || kMode == Mode::LimbsUnsigned, "limb exports only");
  static constexpr int kGDigits = wide_bytes<P>() + 1 > 24 ? 24 : wide_bytes<P>() + 1;
  static constexpr int kN = 32;  // digit columns (MMA N)
  // A stage is kBoxes consecutive 128-cell boxes, loaded by one TMA (each
  // plane's kBoxes * 128 bytes in one piece) and multiplied by kBoxes MMAs.
  static constexpr int kBoxes = 4;
  static constexpr int kUnitCells = kBoxes * kTcBoxCells;
  static constexpr int kBatch = 2;  // boxes an epilogue thread holds at once
  static constexpr int kBoxRows = (P + 7) / 8 * 8;
  static constexpr uint32_t kBoxBytes = kBoxRows * 128;
  static constexpr uint32_t kStageBytes = kBoxes * kBoxBytes;
  static constexpr int kStages = (192 * 1024) / kStageBytes > kTcMaxStages ? kTcMaxStages : (192 * 1024) / kStageBytes;
  // Accumulators of several stages in flight (all 512 columns of tensor
  // memory): with two, the MMA -> epilogue -> MMA hand-off latency capped
  // the rate at about one stage per 0.5 us.
  static constexpr int kAccBufs = 512 / (kBoxes * kN) > 8 ? 8 : 512 / (kBoxes * kN);
  static constexpr uint32_t kTmemCols = kAccBufs * kBoxes * kN;
  static_assert(kAccBufs % 4 == 0, "each accumulator buffer must belong to one epilogue group");
  static constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + kTcTableBytes + 1024;
  static_assert(kTcFDigits + kGDigits <= kN, "digit columns exceed N");
};

struct TcExportParams {
  CUtensorMap tm;  // planes as (cells, P, 1), box {128, roundup(P, 8), 1}, 128-byte swizzle
  ExportArgs a;
  int8_t digits[32][32];  // column c, plane i
  uint32_t nc0[6];        // bias * M (< 2^168)
  uint32_t product[kLimbs32];
  uint64_t s_init;
  uint32_t t_dec;  // limbs: the quotient is certain when |frac| <= t_dec
  int64_t units;
};

// Signed digits of the little-endian 32-bit-limb value x (six limbs).
inline void signed_digits(const uint64_t (&x)[6], int count, int8_t* out) {
  int carry = 0;
  for (int c = 0; c < count; ++c) {
    const int byte = static_cast<int>((x[c / 4] >> (8 * (c % 4))) & 0xFFu) + carry;
    if (byte >= 128) {
      out[c] = static_cast<int8_t>(byte - 256);
      carry = 1;
    } else {
      out[c] = static_cast<int8_t>(byte);
      carry = 0;
    }
  }
}

template <int P, Mode kMode>
void make_tc_export_params(TcExportParams& prm) {
  using S = TcShape<P, kMode>;
  std::memset(prm.digits, 0, sizeof(prm.digits));
  uint64_t M[6] = {1, 0, 0, 0, 0, 0};
  for (int i = 0; i < P; ++i) {
    uint64_t carry = 0;
    for (int l = 0; l < 6; ++l) {
      const uint64_t v = M[l] * rns8ladder::kLadder[i] + carry;
      M[l] = v & 0xFFFFFFFFull;
      carry = v >> 32;
    }
  }
  for (int l = 0; l < kLimbs32; ++l) prm.product[l] = static_cast<uint32_t>(M[l]);
  for (int i = 0; i < P; ++i) {
    const uint32_t mi = rns8ladder::kLadder[i];
    uint64_t E[6] = {1, 0, 0, 0, 0, 0};  // M / m_i
    uint32_t emod = 1;
    for (int j = 0; j < P; ++j) {
      if (j == i) continue;
      uint64_t carry = 0;
      for (int l = 0; l < 6; ++l) {
        const uint64_t v = E[l] * rns8ladder::kLadder[j] + carry;
        E[l] = v & 0xFFFFFFFFull;
        carry = v >> 32;
      }
      emod = (emod * rns8ladder::kLadder[j]) % mi;
    }
    const uint32_t inv = inv_mod(emod, mi);
    uint64_t G[6] = {0, 0, 0, 0, 0, 0}, carry = 0;  // E_i * inv_i < M
    for (int l = 0; l < 6; ++l) {
      const uint64_t v = E[l] * inv + carry;
      G[l] = v & 0xFFFFFFFFull;
      carry = v >> 32;
    }
    const uint64_t F = ((static_cast<uint64_t>(inv) << 31) + mi / 2) / mi;  // < 2^31
    const uint64_t Fx[6] = {F & 0xFFFFFFFFull, F >> 32, 0, 0, 0, 0};
    int8_t d[32];
    signed_digits(Fx, kTcFDigits, d);
    for (int c = 0; c < kTcFDigits; ++c) prm.digits[c][i] = d[c];
    signed_digits(G, S::kGDigits, d);  // mod 2^192
    for (int c = 0; c < S::kGDigits; ++c) prm.digits[kTcFDigits + c][i] = d[c];
  }
  uint64_t carry = 0;  // bias * M
  for (int l = 0; l < 6; ++l) {
    const uint64_t v = M[l] * static_cast<uint64_t>(kQuotientBias) + carry;
    prm.nc0[l] = static_cast<uint32_t>(v & 0xFFFFFFFFull);
    carry = v >> 32;
  }
  constexpr WideFracTable<P> kWide = make_wide_frac_table<P>();
  prm.s_init = (1ull << 30) + (static_cast<uint64_t>(kQuotientBias) << 31);
  prm.t_dec = kWide.t_dec;
}

// T_c + 256 * T_c+1 (or T_c alone): two digit sums in one 32-bit value.
template <int kCols>
__device__ __forceinline__ int32_t digit_pair(const uint32_t (&t)[kCols], int c, bool both) {
  const int32_t lo = static_cast<int32_t>(t[c]);
  return both ? lo + static_cast<int32_t>(t[c + 1]) * 256 : lo;
}

// s = s_init + sum_{c<5} T_c 2^(8c): the biased quotient above bit 31, the
// fraction below.
template <int kCols>
__device__ __forceinline__ int64_t tc_fraction_sum(uint64_t s_init, const uint32_t (&t)[kCols]) {
  return static_cast<int64_t>(s_init) + digit_pair(t, 0, true) + (static_cast<int64_t>(digit_pair(t, 2, true)) << 16) +
         (static_cast<int64_t>(static_cast<int32_t>(t[4])) << 32);
}

template <int P, Mode kMode>
__device__ __forceinline__ void tc_limb_cell(const TcExportParams& prm, int64_t cell, const uint32_t (&t)[32],
                                             bool vec3, bool& bad) {
  constexpr int kGD = TcShape<P, kMode>::kGDigits;
  const ExportArgs& a = prm.a;
  const int64_t s = tc_fraction_sum(prm.s_init, t);
  const int32_t frac = static_cast<int32_t>(static_cast<uint32_t>(s) & 0x7FFFFFFFu) - (1 << 30);
  if (static_cast<uint32_t>(frac < 0 ? -frac : frac) > prm.t_dec) {  // quotient in doubt: exact path
    const int64_t cells = a.m * a.n;
    int r[P];
#pragma unroll
    for (int p = 0; p < P; ++p) r[p] = a.planes[static_cast<int64_t>(p) * cells + cell];
    bad |= !export_cell<P, kMode>(a, cell, r);
    return;
  }
  const uint32_t q = static_cast<uint32_t>(static_cast<uint64_t>(s) >> 31);
  uint32_t v[6];
  int64_t carry = 0;
#pragma unroll
  for (int l = 0; l < 6; ++l) {  // v = S + bias * M - q * M  (mod 2^192)
    int64_t acc = carry + static_cast<int64_t>(prm.nc0[l]) -
                  static_cast<int64_t>(q) * static_cast<int64_t>(l < kLimbs32 ? prm.product[l] : 0u);
    const int c = kTcFDigits + 4 * l;
    if (4 * l < kGD) acc += digit_pair(t, c, 4 * l + 1 < kGD);
    if (4 * l + 2 < kGD) acc += static_cast<int64_t>(digit_pair(t, c + 2, 4 * l + 3 < kGD)) << 16;
    v[l] = static_cast<uint32_t>(acc);
    carry = acc >> 32;
  }
  if constexpr (kMode == Mode::LimbsUnsigned) {  // centered value below zero: the canonical value is v + M
    const uint32_t neg = static_cast<uint32_t>(static_cast<int32_t>(v[5]) >> 31);
    uint64_t c = 0;
#pragma unroll
    for (int l = 0; l < 6; ++l) {
      const uint64_t x = static_cast<uint64_t>(v[l]) + ((l < kLimbs32 ? prm.product[l] : 0u) & neg) + c;
      v[l] = static_cast<uint32_t>(x);
      c = x >> 32;
    }
  }
  if (vec3) {
    uint64_t* out = static_cast<uint64_t*>(a.dst) + cell * 3;
#pragma unroll
    for (int l = 0; l < 3; ++l)
      __stcs(reinterpret_cast<unsigned long long*>(out + l),
             static_cast<unsigned long long>(v[2 * l]) | (static_cast<unsigned long long>(v[2 * l + 1]) << 32));
  } else {
    bad |= !store_limbs<kMode>(a, cell, v);
  }
}

template <int P, Mode kMode>
__global__ void __launch_bounds__(kTcThreads, 1) export_tc_kernel(const __grid_constant__ TcExportParams prm) {
  using S = TcShape<P, kMode>;
  constexpr int kN = S::kN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* table = smem + S::kStages * S::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(table + kTcTableBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* acc_full = empty + S::kStages;
  uint64_t* acc_empty = acc_full + S::kAccBufs;
  uint64_t* drain = acc_empty + S::kAccBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const ExportArgs& a = prm.a;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  // Digit table as the B operand: row c (a digit column), logical byte i
  // (a plane), K-major with the 128-byte swizzle (16-byte chunk i/16 of row
  // c stored at chunk (i/16) ^ (c % 8)); the MMA reads bytes 0..31 of a row.
  for (int e = threadIdx.x; e < kN * 32; e += blockDim.x) {
    const int c = e >> 5, i = e & 31;
    table[c * 128 + ((((i >> 4) ^ (c & 7)) << 4) | (i & 15))] = static_cast<uint8_t>(prm.digits[c][i]);
  }
  release_stage_reads();  // the table is read through the async proxy by the MMA
  if (threadIdx.x == 0) {
    for (int st = 0; st < S::kStages; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], 1);
    }
    for (int b = 0; b < S::kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4 * 32);  // the group that drains the buffer
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&prm.tm);
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  auto give_up = [&] {  // a bounded wait ran out: every role stops at its next check
    if (!*abort_flag) {
      *abort_flag = 1;
      atomicOr(a.status, kDevWaitTimeout);
    }
  };

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer ----------------
      uint32_t pending = 0, pending_parity = 0;
      int64_t j = 0;
      for (int64_t u = blockIdx.x; u < prm.units; u += gridDim.x, ++j) {
        const int st = static_cast<int>(j % S::kStages);
        const uint32_t phase = static_cast<uint32_t>((j / S::kStages) & 1);
        if (*abort_flag || !mbar_wait_bounded(&empty[st], phase ^ 1u)) {
          give_up();
          break;
        }
        mbar_arrive_expect_tx(&full[st], S::kStageBytes);
        tma_load_3d(smem + st * S::kStageBytes, &prm.tm, &full[st], 0, 0, static_cast<int32_t>(u * S::kBoxes));
        pending |= 1u << st;
        pending_parity = (pending_parity & ~(1u << st)) | (phase << st);
      }
      // Loads issued but never consumed (abort path) land before exit.
      for (int st = 0; st < S::kStages; ++st)
        if (pending & (1u << st)) (void)mbar_wait_bounded(&full[st], (pending_parity >> st) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = make_idesc_i8_mn_a(128, kN);
      const uint64_t bdesc = make_smem_desc_sw128(smem_u32(table), 16, 1024);
      int64_t j = 0;
      for (int64_t u = blockIdx.x; u < prm.units; u += gridDim.x, ++j) {
        const int st = static_cast<int>(j % S::kStages);
        const uint32_t phase = static_cast<uint32_t>((j / S::kStages) & 1);
        const uint32_t acc = static_cast<uint32_t>(j % S::kAccBufs);
        const uint32_t acc_phase = static_cast<uint32_t>((j / S::kAccBufs) & 1);
        if (*abort_flag || !mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u) ||
            !mbar_wait_bounded(&full[st], phase)) {
          give_up();
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + st * S::kStageBytes);
#pragma unroll
        for (int b = 0; b < S::kBoxes; ++b) {
          // A: plane rows of 128 cells, 8-row swizzle atoms 1 KiB apart.
          const uint64_t adesc = make_smem_desc_sw128(sa + b * S::kBoxBytes, S::kBoxBytes, 1024);
          tc_mma_i8(tmem_base + acc * (S::kBoxes * kN) + b * kN, adesc, bdesc, idesc, 0u);
        }
        tc_commit(&empty[st]);
        tc_commit(&acc_full[acc]);
      }
      tc_commit(drain);
      (void)mbar_wait_bounded(drain, 0);
    }
  } else {  // ---------------- epilogue (warps 2..17) ----------------
    // Group g (warps 2+4g .. 5+4g, one per lane quarter) drains the stages
    // j = g, g+4, ... of this CTA: four cells per thread and stage, and four
    // stages in flight across the groups (kAccBufs is a multiple of four, so
    // a buffer always belongs to one group). One cell per thread and stage
    // left the epilogue latency-bound at about one stage per 0.5 us.
    const uint32_t quarter = static_cast<uint32_t>(warp & 3);
    const int group = (warp - 2) >> 2;
    const int64_t cells = a.m * a.n;
    const bool vec3 = a.limb_count == 3 && a.ld == a.n;
    bool bad = false;
    for (int64_t j = group, u = blockIdx.x + group * static_cast<int64_t>(gridDim.x); u < prm.units;
         j += 4, u += 4 * static_cast<int64_t>(gridDim.x)) {
      const uint32_t acc = static_cast<uint32_t>(j % S::kAccBufs);
      const uint32_t acc_phase = static_cast<uint32_t>((j / S::kAccBufs) & 1);
      if (*abort_flag || !mbar_wait_bounded(&acc_full[acc], acc_phase)) {
        give_up();
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + acc * (S::kBoxes * kN);
      const int64_t cell = u * S::kUnitCells + quarter * 32 + lane;  // + box * 128
#pragma unroll
      for (int h = 0; h < S::kBoxes / S::kBatch; ++h) {
        uint32_t t[S::kBatch][kN];
#pragma unroll
        for (int b = 0; b < S::kBatch; ++b) tmem_ld_32x32b_x32(taddr + (h * S::kBatch + b) * kN, t[b]);
#pragma unroll
        for (int b = 0; b < S::kBatch; ++b) tmem_wait_ld(t[b]);
        if (h == S::kBoxes / S::kBatch - 1) {  // every box of the stage is in registers
          tc_fence_before();
          mbar_arrive(&acc_empty[acc]);
        }
#pragma unroll
        for (int b = 0; b < S::kBatch; ++b) {
          const int64_t c = cell + (h * S::kBatch + b) * kTcBoxCells;
          if (c < cells) tc_limb_cell<P, kMode>(prm, c, t[b], vec3, bad);
        }
      }
    }
    if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(a.status, kDevRangeError);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// The tensor-core limb export: 16-byte aligned planes, whole 128-cell chunks,
// at least one stage of cells, TMA coordinates within int32.
template <int P, Mode kMode>
bool launch_export_tc(const ExportArgs& a, cudaStream_t stream, cudaError_t* err) {
  using S = TcShape<P, kMode>;
  const int64_t cells = a.m * a.n;
  if (P < 2 || cells % kTcBoxCells != 0 || reinterpret_cast<uintptr_t>(a.planes) % 16 != 0 ||
      cells < S::kUnitCells || cells / kTcBoxCells > (int64_t{1} << 30))
    return false;
  static thread_local TcExportParams prm;
  std::memset(&prm, 0, sizeof(prm));
  if (!encode_plane_cells(&prm.tm, a.planes, static_cast<uint64_t>(cells), static_cast<uint32_t>(P),
                          static_cast<uint32_t>(S::kBoxRows), static_cast<uint32_t>(S::kBoxes)))
    return false;
  prm.a = a;
  make_tc_export_params<P, kMode>(prm);
  prm.units = (cells + S::kUnitCells - 1) / S::kUnitCells;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
    *err = cudaGetLastError();
    return true;
  }
  auto kernel = export_tc_kernel<P, kMode>;
  static std::atomic<uint64_t> configured{0};
  *err = raise_smem_limit_once(kernel, static_cast<int>(S::kSmemBytes), configured);
  if (*err != cudaSuccess) return true;
  const int64_t grid = prm.units < sms ? prm.units : sms;
  kernel<<<static_cast<unsigned>(grid), kTcThreads, S::kSmemBytes, stream>>>(prm);
  *err = cudaGetLastError();
  return true;
}

template <int P>
constexpr int ws_stages() {
  constexpr int by_smem = (224 * 1024) / (P * kWsTileCells);
  return by_smem > 4 ? 4 : by_smem;
}

// The streamed kernel applies to contiguous destinations with the fractional
// path enabled, 16-byte aligned planes and at least one whole tile.
template <int P, bool kSigned>
bool launch_bounded_ws(const ExportArgs& a, cudaStream_t stream, cudaError_t* err) {
  constexpr int kStages = ws_stages<P>();
  const int64_t cells = a.m * a.n;
  if (kStages < 2 || !a.frac.enabled || a.ld != a.n || reinterpret_cast<uintptr_t>(a.dst) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(a.planes) % 16 != 0 || cells % 16 != 0 || cells < kWsTileCells)
    return false;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                               cudaSuccess || sms <= 0) {
    *err = cudaGetLastError();
    return true;
  }
  const int smem = kStages * P * kWsTileCells;
  auto kernel = export_bounded_ws_kernel<P, kSigned, kStages>;
  static std::atomic<uint64_t> configured{0};
  *err = raise_smem_limit_once(kernel, smem, configured);
  if (*err != cudaSuccess) return true;
  const int64_t tiles = cells / kWsTileCells;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  kernel<<<grid, kWsThreads, smem, stream>>>(a);
  *err = cudaGetLastError();
  return true;
}

template <int P, bool kSigned, int kCells>
cudaError_t launch_bounded(const ExportArgs& a, cudaStream_t stream) {
  const int64_t groups = a.m * a.n / kCells;
  int64_t blocks = (groups + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  const bool contig = a.ld == a.n && reinterpret_cast<uintptr_t>(a.dst) % 16 == 0;
  if (contig)
    export_bounded_kernel<P, kSigned, kCells, true><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
  else
    export_bounded_kernel<P, kSigned, kCells, false><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

#ifndef RNS8_EXPORT_CELLS
#define RNS8_EXPORT_CELLS 8
#endif

template <int P, Mode kMode>
cudaError_t launch_export(const ExportArgs& a, cudaStream_t stream) {
  const int64_t cells = a.m * a.n;
  if constexpr (kMode == Mode::I64 || kMode == Mode::U64) {
    constexpr bool kSigned = kMode == Mode::I64;
    cudaError_t ws_err = cudaSuccess;
    if (launch_bounded_ws<P, kSigned>(a, stream, &ws_err)) return ws_err;
    const uintptr_t base = reinterpret_cast<uintptr_t>(a.planes);
    constexpr int kWide = RNS8_EXPORT_CELLS;
    if (cells % kWide == 0 && base % kWide == 0) return launch_bounded<P, kSigned, kWide>(a, stream);
    if (cells % 4 == 0 && base % 4 == 0) return launch_bounded<P, kSigned, 4>(a, stream);
  }
  const bool vec = (cells % 4 == 0) && (reinterpret_cast<uintptr_t>(a.planes) % 4 == 0);
  const int64_t work = vec ? cells / 4 : cells;
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  if constexpr (kMode == Mode::LimbsSigned || kMode == Mode::LimbsUnsigned) {
    cudaError_t ws_err = cudaSuccess;
    if (launch_export_tc<P, kMode>(a, stream, &ws_err)) return ws_err;
    if (launch_limbs_ws<P, kMode>(a, stream, &ws_err)) return ws_err;
    if (vec && P >= 2) {
      export_limbs_frac_kernel<P, kMode><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
      return cudaGetLastError();
    }
  }
  if (vec)
    export_kernel<P, kMode, true><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
  else
    export_kernel<P, kMode, false><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

template <Mode kMode>
cudaError_t dispatch_export(const ExportArgs& a, uint32_t prefix, cudaStream_t stream) {
  switch (prefix) {
#define RNS8_EXPORT_CASE(P) \
  case P: return launch_export<P, kMode>(a, stream);
    RNS8_EXPORT_CASE(1) RNS8_EXPORT_CASE(2) RNS8_EXPORT_CASE(3) RNS8_EXPORT_CASE(4) RNS8_EXPORT_CASE(5)
    RNS8_EXPORT_CASE(6) RNS8_EXPORT_CASE(7) RNS8_EXPORT_CASE(8) RNS8_EXPORT_CASE(9) RNS8_EXPORT_CASE(10)
    RNS8_EXPORT_CASE(11) RNS8_EXPORT_CASE(12) RNS8_EXPORT_CASE(13) RNS8_EXPORT_CASE(14) RNS8_EXPORT_CASE(15)
    RNS8_EXPORT_CASE(16) RNS8_EXPORT_CASE(17) RNS8_EXPORT_CASE(18) RNS8_EXPORT_CASE(19) RNS8_EXPORT_CASE(20)
#undef RNS8_EXPORT_CASE
    default: return cudaErrorInvalidValue;
  }
}

int64_t frac_sum_f128(uint32_t prefix) {
  switch (prefix) {
#define RNS8_FRAC_CASE(P) \
  case P: return make_frac_table<P>().sumF128;
    RNS8_FRAC_CASE(1) RNS8_FRAC_CASE(2) RNS8_FRAC_CASE(3) RNS8_FRAC_CASE(4) RNS8_FRAC_CASE(5)
    RNS8_FRAC_CASE(6) RNS8_FRAC_CASE(7) RNS8_FRAC_CASE(8) RNS8_FRAC_CASE(9) RNS8_FRAC_CASE(10)
    RNS8_FRAC_CASE(11) RNS8_FRAC_CASE(12) RNS8_FRAC_CASE(13) RNS8_FRAC_CASE(14) RNS8_FRAC_CASE(15)
    RNS8_FRAC_CASE(16) RNS8_FRAC_CASE(17) RNS8_FRAC_CASE(18) RNS8_FRAC_CASE(19) RNS8_FRAC_CASE(20)
#undef RNS8_FRAC_CASE
    default: return 0;
  }
}

// Centered -> canonical: r < 0 ? r + m : r, on four packed bytes. The sign
// bit of each byte selects whether m is added; the per-byte add wraps modulo
// 256 (a negative residue is stored as 256 + r, and 256 + r + m = r + m mod
// 256), so no carry crosses into the next byte.
__device__ __forceinline__ uint32_t canonical4(uint32_t w, uint32_t m4) {
  const uint32_t neg = (w >> 7) & 0x01010101u;  // 1 in every byte holding a negative residue
  return __vadd4(w, neg * 0xFFu & m4);          // add m to exactly those bytes
}

// Contiguous rows (ld == n): 16 cells per thread, one 16-byte load and store.
__global__ void __launch_bounds__(256) export_u8_vec16_kernel(const uint4* __restrict__ res, int64_t groups,
                                                              uint32_t modulus, uint4* __restrict__ dst) {
  const uint32_t m4 = (modulus & 0xFFu) * 0x01010101u;  // m = 256 adds 0: the byte already is r mod 256
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < groups;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint4 v = __ldcs(res + i);
    v.x = canonical4(v.x, m4);
    v.y = canonical4(v.y, m4);
    v.z = canonical4(v.z, m4);
    v.w = canonical4(v.w, m4);
    __stcs(dst + i, v);
  }
}

// General layout: one thread per cell of a 2-D grid (x over columns, y over
// rows), so no division per cell.
__global__ void __launch_bounds__(256) export_u8_kernel(const int8_t* __restrict__ res, int64_t m, int64_t n,
                                                        uint32_t modulus, uint8_t* __restrict__ dst, int64_t ld) {
  for (int64_t row = blockIdx.y; row < m; row += gridDim.y) {
    for (int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; col < n;
         col += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int r = res[row * n + col];
      dst[row * ld + col] = static_cast<uint8_t>(r < 0 ? r + static_cast<int>(modulus) : r);
    }
  }
}

// ---- scheduled export: per-tile prefix and bound ----------------------------------
struct TileJob {
  int64_t row0, col0, rows, cols;
  BoundedLimits lim;
  FracLimits frac;
};

// One job (schedule tile) per block iteration; warps over rows, lanes over
// columns. Every cell: the fractional CRT with the tile's limits, the exact
// Garner path for undecided cells (or all cells when the fraction is off).
template <int P, bool kSigned>
__global__ void __launch_bounds__(256) export_tiles_kernel(const int8_t* __restrict__ planes, int64_t m, int64_t n,
                                                           const TileJob* __restrict__ jobs, uint32_t count,
                                                           uint64_t* __restrict__ dst, uint32_t* status) {
  const int64_t mn = m * n;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  bool bad = false;
  for (uint32_t j = blockIdx.x; j < count; j += gridDim.x) {
    const TileJob job = jobs[j];
    for (int64_t r = warp; r < job.rows; r += blockDim.x / 32) {
      const int64_t row = job.row0 + r;
      for (int64_t c = lane; c < job.cols; c += 32) {
        const int64_t cell = row * n + job.col0 + c;
        uint32_t u[P];
#pragma unroll
        for (int p = 0; p < P; ++p) u[p] = static_cast<uint32_t>(static_cast<int>(planes[p * mn + cell]) + 128);
        uint64_t v = 0;
        int verdict = job.frac.enabled ? frac_reconstruct<P>(u, job.frac, &v) : -1;
        if (verdict < 0) {
          int rr[P];
#pragma unroll
          for (int p = 0; p < P; ++p) rr[p] = static_cast<int>(u[p]) - 128;
          verdict = reconstruct_bounded<P, kSigned>(rr, job.lim, &v) ? 1 : 0;
        }
        bad |= verdict == 0;
        dst[cell] = v;
      }
    }
  }
  if (__any_sync(0xFFFFFFFFu, bad) && lane == 0) atomicOr(status, kDevRangeError);
}

__global__ void __launch_bounds__(256) zero_jobs_kernel(const TileJob* __restrict__ jobs, uint32_t count, int64_t n,
                                                        uint64_t* __restrict__ dst) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (uint32_t j = blockIdx.x; j < count; j += gridDim.x) {
    const TileJob job = jobs[j];
    for (int64_t r = warp; r < job.rows; r += blockDim.x / 32)
      for (int64_t c = lane; c < job.cols; c += 32) dst[(job.row0 + r) * n + job.col0 + c] = 0;
  }
}

template <bool kSigned>
cudaError_t launch_tiles(uint32_t prefix, const int8_t* planes, int64_t m, int64_t n, const TileJob* jobs,
                         uint32_t count, uint64_t* dst, uint32_t* status, cudaStream_t stream) {
  const unsigned blocks = count < 148u * 8u ? count : 148u * 8u;
  switch (prefix) {
#define RNS8_TILE_CASE(P)                                                                                   \
  case P:                                                                                                   \
    export_tiles_kernel<P, kSigned><<<blocks, 256, 0, stream>>>(planes, m, n, jobs, count, dst, status); \
    break;
    RNS8_TILE_CASE(1) RNS8_TILE_CASE(2) RNS8_TILE_CASE(3) RNS8_TILE_CASE(4) RNS8_TILE_CASE(5)
    RNS8_TILE_CASE(6) RNS8_TILE_CASE(7) RNS8_TILE_CASE(8) RNS8_TILE_CASE(9) RNS8_TILE_CASE(10)
    RNS8_TILE_CASE(11) RNS8_TILE_CASE(12) RNS8_TILE_CASE(13) RNS8_TILE_CASE(14) RNS8_TILE_CASE(15)
    RNS8_TILE_CASE(16) RNS8_TILE_CASE(17) RNS8_TILE_CASE(18) RNS8_TILE_CASE(19) RNS8_TILE_CASE(20)
#undef RNS8_TILE_CASE
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t export_i64(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, uint64_t bound, int64_t* dst,
                       int64_t ld, uint32_t* dev_status, cudaStream_t stream) {
  ExportArgs a{};
  a.planes = planes;
  a.m = m;
  a.n = n;
  a.ld = ld;
  a.lim = host_limits(prefix, bound);  // bound < M_P / 2 is guaranteed by plan validation
  a.frac = host_frac_limits(prefix, bound, true, frac_sum_f128(prefix));
  a.dst = dst;
  a.status = dev_status;
  return dispatch_export<Mode::I64>(a, prefix, stream);
}

cudaError_t export_u64(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, uint64_t bound, uint64_t* dst,
                       int64_t ld, uint32_t* dev_status, cudaStream_t stream) {
  ExportArgs a{};
  a.planes = planes;
  a.m = m;
  a.n = n;
  a.ld = ld;
  a.lim = host_limits(prefix, bound);
  a.frac = host_frac_limits(prefix, bound, false, frac_sum_f128(prefix));
  a.dst = dst;
  a.status = dev_status;
  return dispatch_export<Mode::U64>(a, prefix, stream);
}

cudaError_t export_limbs(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, bool is_signed,
                         uint32_t limb_count, uint64_t* dst, int64_t ld, uint32_t* dev_status, cudaStream_t stream) {
  if (limb_count == 0 || limb_count > 32) return cudaErrorInvalidValue;
  ExportArgs a{};
  a.planes = planes;
  a.m = m;
  a.n = n;
  a.ld = ld;
  a.limb_count = limb_count;
  a.dst = dst;
  a.status = dev_status;
  return is_signed ? dispatch_export<Mode::LimbsSigned>(a, prefix, stream)
                   : dispatch_export<Mode::LimbsUnsigned>(a, prefix, stream);
}

cudaError_t export_finite_u8(const int8_t* residues, int64_t m, int64_t n, uint32_t modulus, uint8_t* dst, int64_t ld,
                             cudaStream_t stream) {
  const int64_t cells = m * n;
  if (ld == n && cells % 16 == 0 && reinterpret_cast<uintptr_t>(residues) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(dst) % 16 == 0) {
    const int64_t groups = cells / 16;
    int64_t blocks = (groups + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (blocks < 1) blocks = 1;
    export_u8_vec16_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        reinterpret_cast<const uint4*>(residues), groups, modulus, reinterpret_cast<uint4*>(dst));
    return cudaGetLastError();
  }
  int64_t bx = (n + 255) / 256;
  if (bx > 64) bx = 64;
  const int64_t by = m < 65535 ? m : 65535;
  export_u8_kernel<<<dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by)), 256, 0, stream>>>(residues, m, n,
                                                                                                    modulus, dst, ld);
  return cudaGetLastError();
}

uint64_t export_scheduled_scratch_bytes(const PlaneSchedule& sched) {
  return (sched.tile_rows * sched.tile_cols * sizeof(TileJob) + 255) & ~uint64_t(255);
}

cudaError_t export_scheduled(const int8_t* planes, int64_t m, int64_t n, bool is_signed, const PlaneSchedule& sched,
                             const uint64_t* tile_bounds, void* dst, uint32_t* dev_status, void* scratch,
                             uint64_t scratch_bytes, cudaStream_t stream) {
  const uint64_t tiles = sched.tile_rows * sched.tile_cols;
  if (!scratch || scratch_bytes < export_scheduled_scratch_bytes(sched) || !tile_bounds) return cudaErrorInvalidValue;
  // Jobs ordered by prefix: proven-zero tiles first (prefix 0), then one run per prefix.
  std::vector<std::vector<TileJob>> by_prefix(21);
  for (uint64_t t = 0; t < tiles; ++t) {
    const uint8_t sel = sched.tile_sel[t];
    const uint32_t prefix = (sel & 0x80u) ? 0u : (sel & 0x7Fu);
    if (prefix > 20) return cudaErrorInvalidValue;
    TileJob job{};
    job.row0 = static_cast<int64_t>((t / sched.tile_cols) * sched.tile_m);
    job.col0 = static_cast<int64_t>((t % sched.tile_cols) * sched.tile_n);
    job.rows = std::min<int64_t>(sched.tile_m, m - job.row0);
    job.cols = std::min<int64_t>(sched.tile_n, n - job.col0);
    if (prefix > 0) {
      job.lim = host_limits(prefix, tile_bounds[t]);
      job.frac = host_frac_limits(prefix, tile_bounds[t], is_signed, frac_sum_f128(prefix));
    }
    by_prefix[prefix].push_back(job);
  }
  std::vector<TileJob> all;
  all.reserve(tiles);
  for (const auto& v : by_prefix) all.insert(all.end(), v.begin(), v.end());
  auto* jobs = static_cast<TileJob*>(scratch);
  cudaError_t e = cudaMemcpyAsync(jobs, all.data(), all.size() * sizeof(TileJob), cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  auto* out = static_cast<uint64_t*>(dst);
  uint64_t offset = 0;
  for (uint32_t prefix = 0; prefix <= 20; ++prefix) {
    const uint32_t count = static_cast<uint32_t>(by_prefix[prefix].size());
    if (count == 0) continue;
    if (prefix == 0) {
      zero_jobs_kernel<<<count < 148u * 8u ? count : 148u * 8u, 256, 0, stream>>>(jobs + offset, count, n, out);
      e = cudaGetLastError();
    } else if (is_signed) {
      e = launch_tiles<true>(prefix, planes, m, n, jobs + offset, count, out, dev_status, stream);
    } else {
      e = launch_tiles<false>(prefix, planes, m, n, jobs + offset, count, out, dev_status, stream);
    }
    if (e != cudaSuccess) return e;
    offset += count;
  }
  return cudaSuccess;
}

}  // namespace rns8cuda
