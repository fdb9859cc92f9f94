// Export kernels: centered residue planes -> bounded int64 / uint64, or
// fixed-width little-endian limbs (exact-wide), or canonical finite u8.
//
// Reference behaviour: src/reconstruct/crt.cpp:54-170 (Garner order,
// centering at ceil(P/2), fits checks, two's-complement limbs) and
// src/core/api_export.cpp:307-803 (a failing cell makes the whole export a
// RANGE_ERROR). The device status word replaces the reference's
// atomicCAS(status, 0, 5) (hip_direct_export_kernels.cuh:137-177).
//
// Mixed-radix digits: x = sum_i c_i * M_i with M_i = m_0 * ... * m_{i-1}.
// Digit i needs x_{<i} mod m_i = sum_{j<i} c_j * (M_j mod m_i); with every
// factor below 2^8 the sum stays under 2^21 and one mul-hi reduction gives
// it. c_i = (r_i - that) * (M_i mod m_i)^-1 mod m_i. All tables are
// compile-time constants of the prefix P, so they fold into immediates.
#include "device_common.cuh"
#include "kernels.hpp"

namespace rns8cuda {
namespace {

__host__ __device__ constexpr uint32_t ladder_at(int i) { return kLadder[i]; }

__host__ __device__ constexpr uint32_t inv_mod(uint32_t a, uint32_t m) {
  // a^-1 mod m by extended Euclid (compile time only).
  int64_t t = 0, nt = 1, r = m, nr = a % m;
  while (nr != 0) {
    const int64_t q = r / nr;
    const int64_t tt = t - q * nt;
    t = nt;
    nt = tt;
    const int64_t rr = r - q * nr;
    r = nr;
    nr = rr;
  }
  return static_cast<uint32_t>(t < 0 ? t + m : t);
}

struct Limbs3 {
  uint64_t w[3];
};
__host__ __device__ constexpr Limbs3 limbs_mul_small(Limbs3 a, uint32_t m) {
  Limbs3 r{{0, 0, 0}};
  uint64_t carry = 0;
  for (int i = 0; i < 3; ++i) {
    const uint64_t lo = a.w[i] & 0xFFFFFFFFull, hi = a.w[i] >> 32;
    const uint64_t plo = lo * m + (carry & 0xFFFFFFFFull);
    const uint64_t phi = hi * m + (carry >> 32) + (plo >> 32);
    r.w[i] = (plo & 0xFFFFFFFFull) | (phi << 32);
    carry = phi >> 32;
  }
  return r;
}

template <int P>
struct GarnerTable {
  uint32_t m[P];
  uint32_t magic[P];
  uint32_t inv[P];    // (M_i mod m_i)^-1 mod m_i
  uint32_t w[P][P];   // w[i][j] = M_j mod m_i, j < i
  uint32_t off[P];    // multiple of m_i above any digit sum, keeps differences non-negative
  Limbs3 product;     // M_P
  Limbs3 half;        // ceil(M_P / 2)
};

template <int P>
__host__ __device__ constexpr GarnerTable<P> make_table() {
  GarnerTable<P> t{};
  for (int i = 0; i < P; ++i) {
    t.m[i] = ladder_at(i);
    t.magic[i] = floor_magic(t.m[i]);
    uint32_t Mi = 1;  // M_i mod m_i, built incrementally
    for (int j = 0; j < i; ++j) {
      t.w[i][j] = Mi;
      Mi = (Mi * ladder_at(j)) % t.m[i];
    }
    t.inv[i] = inv_mod(Mi, t.m[i]);
    t.off[i] = t.m[i] * ((1u << 22) / t.m[i] + 1u);
  }
  Limbs3 prod{{1, 0, 0}};
  for (int i = 0; i < P; ++i) prod = limbs_mul_small(prod, ladder_at(i));
  t.product = prod;
  // half = (M + 1) / 2
  Limbs3 h = prod;
  uint64_t c = 1;
  for (int i = 0; i < 3; ++i) {
    const uint64_t s = h.w[i] + c;
    c = (s < h.w[i]) ? 1 : 0;
    h.w[i] = s;
  }
  for (int i = 0; i < 3; ++i) h.w[i] = (h.w[i] >> 1) | (i < 2 ? (h.w[i + 1] << 63) : 0);
  t.half = h;
  return t;
}

// Limb count needed for M_P: 1 for P <= 8 (M_8 < 2^64), 2 for P <= 16, else 3.
template <int P>
constexpr int limbs_for() { return P <= 8 ? 1 : (P <= 16 ? 2 : 3); }

template <int P>
__device__ __forceinline__ void garner_digits(const int (&r)[P], uint32_t (&c)[P]) {
  constexpr GarnerTable<P> T = make_table<P>();
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const uint32_t mi = T.m[i];
    const uint32_t ri = static_cast<uint32_t>(r[i] < 0 ? r[i] + static_cast<int>(mi) : r[i]);
    if (i == 0) {
      c[0] = ri;
      continue;
    }
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < i; ++j) s += c[j] * T.w[i][j];
    const uint32_t diff = umod_u32(ri + T.off[i] - s, mi, T.magic[i]);
    c[i] = umod_u32(diff * T.inv[i], mi, T.magic[i]);
  }
}

// x = sum c_i M_i by Horner from the top digit, L 64-bit limbs.
template <int P, int L>
__device__ __forceinline__ void horner(const uint32_t (&c)[P], uint64_t (&x)[L]) {
  constexpr GarnerTable<P> T = make_table<P>();
#pragma unroll
  for (int l = 0; l < L; ++l) x[l] = 0;
  x[0] = c[P - 1];
#pragma unroll
  for (int i = P - 2; i >= 0; --i) {
    uint64_t carry = c[i];
#pragma unroll
    for (int l = 0; l < L; ++l) {
      const uint64_t lo = x[l] * T.m[i];
      const uint64_t hi = __umul64hi(x[l], static_cast<uint64_t>(T.m[i]));
      const uint64_t s = lo + carry;
      carry = hi + (s < lo ? 1 : 0);
      x[l] = s;
    }
  }
}

template <int L>
__device__ __forceinline__ bool geq(const uint64_t (&x)[L], const uint64_t* y) {
#pragma unroll
  for (int l = L - 1; l >= 0; --l) {
    if (x[l] != y[l]) return x[l] > y[l];
  }
  return true;
}

enum class Mode : int { I64 = 0, U64 = 1, LimbsSigned = 2, LimbsUnsigned = 3 };

struct ExportArgs {
  const int8_t* planes;
  int64_t m, n;
  int64_t ld;
  uint64_t bound;         // I64/U64
  uint64_t low_limit;     // I64: min(bound, INT64_MAX)
  uint64_t high_limit[3]; // I64: M_P - bound (cells at or above it are negative values)
  uint32_t limb_count;    // limb modes
  void* dst;
  uint32_t* status;
};

template <int P, Mode kMode>
__device__ __forceinline__ bool export_cell(const ExportArgs& a, int64_t cell, const int (&r)[P]) {
  constexpr int L = limbs_for<P>();
  constexpr GarnerTable<P> T = make_table<P>();
  uint32_t c[P];
  garner_digits<P>(r, c);
  uint64_t x[L];
  horner<P, L>(c, x);
  const int64_t row = cell / a.n, col = cell - row * a.n;
  if (kMode == Mode::I64) {
    bool upper_zero = true;
#pragma unroll
    for (int l = 1; l < L; ++l) upper_zero = upper_zero && x[l] == 0;
    int64_t v;
    if (upper_zero && x[0] <= a.low_limit) {
      v = static_cast<int64_t>(x[0]);
    } else if (geq<L>(x, a.high_limit)) {
      v = static_cast<int64_t>(x[0] - T.product.w[0]);  // x - M_P, exact in 64 bits
    } else {
      return false;
    }
    static_cast<int64_t*>(a.dst)[row * a.ld + col] = v;
    return true;
  } else if (kMode == Mode::U64) {
    bool upper_zero = true;
#pragma unroll
    for (int l = 1; l < L; ++l) upper_zero = upper_zero && x[l] == 0;
    if (!upper_zero || x[0] > a.bound) return false;
    static_cast<uint64_t*>(a.dst)[row * a.ld + col] = x[0];
    return true;
  } else {
    // 192-bit two's complement working value.
    uint64_t v[3] = {0, 0, 0};
#pragma unroll
    for (int l = 0; l < L; ++l) v[l] = x[l];
    if (kMode == Mode::LimbsSigned && geq<L>(x, T.half.w)) {
      uint64_t borrow = 0;
#pragma unroll
      for (int l = 0; l < 3; ++l) {
        const uint64_t sub = T.product.w[l] + borrow;
        const uint64_t nb = (sub < borrow) || (v[l] < sub) ? 1 : 0;
        v[l] = v[l] - sub;
        borrow = nb;
      }
    }
    const uint32_t limbs = a.limb_count;
    const uint64_t sign_fill = (kMode == Mode::LimbsSigned && (v[2] >> 63)) ? ~0ull : 0ull;
    if (limbs < 3) {
      if (kMode == Mode::LimbsSigned) {
        // Value must equal the sign extension of its low `limbs` limbs.
        const uint64_t top = v[limbs - 1];
        const uint64_t ext = (top >> 63) ? ~0ull : 0ull;
        for (uint32_t l = limbs; l < 3; ++l)
          if (v[l] != ext) return false;
      } else {
        for (uint32_t l = limbs; l < 3; ++l)
          if (v[l] != 0) return false;
      }
    }
    uint64_t* out = static_cast<uint64_t*>(a.dst) + (row * a.ld + col) * static_cast<int64_t>(limbs);
    for (uint32_t l = 0; l < limbs; ++l) out[l] = l < 3 ? v[l] : sign_fill;
    return true;
  }
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
      int r[4][P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const uint32_t w = __ldcs(reinterpret_cast<const uint32_t*>(a.planes + static_cast<int64_t>(p) * cells) + g);
#pragma unroll
        for (int e = 0; e < 4; ++e) r[e][p] = static_cast<int8_t>((w >> (8 * e)) & 0xFFu);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) bad |= !export_cell<P, kMode>(a, 4 * g + e, r[e]);
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

template <int P, Mode kMode>
cudaError_t launch_export(const ExportArgs& a, cudaStream_t stream) {
  const int64_t cells = a.m * a.n;
  const bool vec = (cells % 4 == 0) && (reinterpret_cast<uintptr_t>(a.planes) % 4 == 0);
  const int64_t work = vec ? cells / 4 : cells;
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
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

// Host-side M_P as three limbs.
void host_product(uint32_t prefix, uint64_t out[3]) {
  Limbs3 p{{1, 0, 0}};
  for (uint32_t i = 0; i < prefix; ++i) p = limbs_mul_small(p, kLadder[i]);
  out[0] = p.w[0];
  out[1] = p.w[1];
  out[2] = p.w[2];
}

__global__ void __launch_bounds__(256) export_u8_kernel(const int8_t* __restrict__ res, int64_t m, int64_t n,
                                                        uint32_t modulus, uint8_t* __restrict__ dst, int64_t ld) {
  const int64_t cells = m * n;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < cells;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / n, col = i - row * n;
    const int r = res[i];
    dst[row * ld + col] = static_cast<uint8_t>(r < 0 ? r + static_cast<int>(modulus) : r);
  }
}

}  // namespace

cudaError_t export_i64(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, uint64_t bound, int64_t* dst,
                       int64_t ld, uint32_t* dev_status, cudaStream_t stream) {
  ExportArgs a{};
  a.planes = planes;
  a.m = m;
  a.n = n;
  a.ld = ld;
  a.bound = bound;
  a.low_limit = bound < 0x7FFFFFFFFFFFFFFFull ? bound : 0x7FFFFFFFFFFFFFFFull;
  uint64_t prod[3];
  host_product(prefix, prod);
  // high_limit = M_P - bound (bound < M_P / 2 is guaranteed by plan validation).
  uint64_t borrow = 0;
  const uint64_t b[3] = {bound, 0, 0};
  for (int l = 0; l < 3; ++l) {
    const uint64_t sub = b[l] + borrow;
    const uint64_t nb = (sub < borrow) || (prod[l] < sub) ? 1 : 0;
    a.high_limit[l] = prod[l] - sub;
    borrow = nb;
  }
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
  a.bound = bound;
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
  int64_t blocks = (m * n + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  export_u8_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(residues, m, n, modulus, dst, ld);
  return cudaGetLastError();
}

}  // namespace rns8cuda
