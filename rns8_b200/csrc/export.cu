// Export kernels: centered residue planes -> bounded int64 / uint64, or
// fixed-width little-endian limbs (exact-wide), or canonical finite u8.
//
// Reference behaviour: src/reconstruct/crt.cpp:54-170 (Garner order,
// centering at ceil(P/2), fits checks, two's-complement limbs) and
// src/core/api_export.cpp:307-803 (a failing cell makes the whole export a
// RANGE_ERROR). The device status word replaces the reference's
// atomicCAS(status, 0, 5) (hip_direct_export_kernels.cuh:137-177).
//
// Mixed-radix digits: x = sum_i c_i * M_i with M_i = m_0 * ... * m_{i-1}, so
//   c_i = (r_i - sum_{j<i} c_j * (M_j mod m_i)) * (M_i mod m_i)^-1  (mod m_i)
//       = (r_i * inv_i + sum_{j<i} c_j * w'_ij)                      (mod m_i)
// with w'_ij = -(M_j mod m_i) * inv_i mod m_i. Every digit and weight is a
// byte, so the sum is a chain of dp4a over digits packed four per word; it
// stays below 2^21, where q = mulhi(S, ceil(2^32/m)) is the exact quotient,
// so each digit costs one reduction. x is rebuilt by Horner in 32-bit limbs,
// each step touching only the limbs the partial product can occupy. All
// tables are compile-time constants of the prefix P.
#include "device_common.cuh"
#include "kernels.hpp"

namespace rns8cuda {
namespace {

__host__ __device__ constexpr uint32_t ladder_at(int i) { return kLadder[i]; }

__host__ __device__ constexpr uint32_t inv_mod(uint32_t a, uint32_t m) {
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

// ceil(2^32 / m): q = mulhi(S, it) is floor(S / m) exactly for S < 2^32 / m.
__host__ __device__ constexpr uint32_t ceil_magic(uint32_t m) {
  return static_cast<uint32_t>(((1ull << 32) + m - 1) / m);
}

constexpr int kLimbs32 = 5;  // M_20 < 2^155

template <int P>
struct GarnerTable {
  uint32_t m[P];
  uint32_t magic[P];
  uint32_t inv[P];                   // (M_i mod m_i)^-1 mod m_i
  uint32_t off[P];                   // multiple of m_i making r_i * inv_i + off_i >= 0
  uint32_t wpack[P][(P + 3) / 4];    // w'_ij packed four per word (zero for j >= i)
  uint32_t product[kLimbs32];        // M_P in 32-bit limbs
  uint32_t half[kLimbs32];           // ceil(M_P / 2)
};

template <int P>
__host__ __device__ constexpr GarnerTable<P> make_table() {
  GarnerTable<P> t{};
  for (int i = 0; i < P; ++i) {
    const uint32_t mi = ladder_at(i);
    t.m[i] = mi;
    t.magic[i] = ceil_magic(mi);
    uint32_t Mj = 1;  // M_j mod m_i
    uint32_t w[P] = {};
    for (int j = 0; j < i; ++j) {
      w[j] = Mj;
      Mj = (Mj * ladder_at(j)) % mi;
    }
    const uint32_t inv = inv_mod(Mj, mi);
    t.inv[i] = inv;
    t.off[i] = mi * ((32768u + mi - 1) / mi);
    for (int g = 0; g < (P + 3) / 4; ++g) t.wpack[i][g] = 0;
    for (int j = 0; j < i; ++j) {
      const uint32_t wp = ((mi - w[j]) % mi) * inv % mi;
      t.wpack[i][j / 4] |= wp << (8 * (j % 4));
    }
  }
  uint64_t prod[kLimbs32] = {1, 0, 0, 0, 0};
  for (int i = 0; i < P; ++i) {
    uint64_t carry = 0;
    for (int l = 0; l < kLimbs32; ++l) {
      const uint64_t v = prod[l] * ladder_at(i) + carry;
      prod[l] = v & 0xFFFFFFFFull;
      carry = v >> 32;
    }
  }
  for (int l = 0; l < kLimbs32; ++l) t.product[l] = static_cast<uint32_t>(prod[l]);
  // half = (M + 1) >> 1
  uint64_t c = 1;
  uint32_t h[kLimbs32] = {};
  for (int l = 0; l < kLimbs32; ++l) {
    const uint64_t v = prod[l] + c;
    h[l] = static_cast<uint32_t>(v);
    c = v >> 32;
  }
  for (int l = 0; l < kLimbs32; ++l) t.half[l] = (h[l] >> 1) | (l + 1 < kLimbs32 ? (h[l + 1] << 31) : 0u);
  return t;
}

// 32-bit limbs that M_P needs.
template <int P>
constexpr int limbs32_for() {
  constexpr GarnerTable<P> T = make_table<P>();
  int n = kLimbs32;
  while (n > 1 && T.product[n - 1] == 0) --n;
  return n;
}

// Digits of the mixed-radix representation, packed four per word.
template <int P>
__device__ __forceinline__ void garner_digits(const int (&r)[P], uint32_t (&cp)[(P + 3) / 4],
                                              uint32_t (&c)[P]) {
  constexpr GarnerTable<P> T = make_table<P>();
#pragma unroll
  for (int g = 0; g < (P + 3) / 4; ++g) cp[g] = 0;
  c[0] = static_cast<uint32_t>(r[0]) & 0xFFu;  // m_0 = 256: the low byte is the canonical residue
  cp[0] = c[0];
#pragma unroll
  for (int i = 1; i < P; ++i) {
    uint32_t s = static_cast<uint32_t>(r[i] * static_cast<int>(T.inv[i]) + static_cast<int>(T.off[i]));
#pragma unroll
    for (int g = 0; g < (i + 3) / 4; ++g) s = __dp4a(cp[g], T.wpack[i][g], s);
    const uint32_t q = __umulhi(s, T.magic[i]);
    c[i] = s - q * T.m[i];
    cp[i / 4] |= c[i] << (8 * (i % 4));
  }
}

// x = sum c_i M_i by Horner from the top digit, 32-bit limbs.
template <int P, int L>
__device__ __forceinline__ void horner32(const uint32_t (&c)[P], uint32_t (&x)[L]) {
  constexpr GarnerTable<P> T = make_table<P>();
#pragma unroll
  for (int l = 0; l < L; ++l) x[l] = 0;
  x[0] = c[P - 1];
#pragma unroll
  for (int i = P - 2; i >= 0; --i) {
    // Before this step x < 2^(8(P-1-i)); after it x < 2^(8(P-i)).
    constexpr int dummy = 0;
    (void)dummy;
    const int used = (8 * (P - i) + 31) / 32;
    uint64_t carry = c[i];
#pragma unroll
    for (int l = 0; l < L; ++l) {
      if (l < used) {
        const uint64_t t = static_cast<uint64_t>(x[l]) * T.m[i] + carry;
        x[l] = static_cast<uint32_t>(t);
        carry = t >> 32;
      }
    }
  }
}

template <int L>
__device__ __forceinline__ bool geq32(const uint32_t (&x)[L], const uint32_t* y) {
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
  uint64_t bound;                 // U64
  uint64_t low_limit;             // I64: min(bound, INT64_MAX)
  uint32_t high_limit[kLimbs32];  // I64: M_P - bound, 32-bit limbs
  uint32_t limb_count;            // limb modes
  void* dst;
  uint32_t* status;
};

__device__ __forceinline__ int64_t dst_index(const ExportArgs& a, int64_t cell) {
  if (a.ld == a.n) return cell;
  const int64_t row = cell / a.n;
  return row * a.ld + (cell - row * a.n);
}

// Reconstructs one cell into *out (one int64/uint64) or the limb array.
template <int P, Mode kMode>
__device__ __forceinline__ bool export_cell(const ExportArgs& a, int64_t cell, const int (&r)[P]) {
  constexpr int L = limbs32_for<P>();
  constexpr GarnerTable<P> T = make_table<P>();
  uint32_t c[P];
  uint32_t cp[(P + 3) / 4];
  garner_digits<P>(r, cp, c);
  uint32_t x[L];
  horner32<P, L>(c, x);
  const uint64_t lo64 = static_cast<uint64_t>(x[0]) | (L > 1 ? static_cast<uint64_t>(x[L > 1 ? 1 : 0]) << 32 : 0ull);
  bool upper_zero = true;
#pragma unroll
  for (int l = 2; l < L; ++l) upper_zero = upper_zero && x[l] == 0;
  if (kMode == Mode::I64) {
    int64_t v;
    if (upper_zero && lo64 <= a.low_limit) {
      v = static_cast<int64_t>(lo64);
    } else if (geq32<L>(x, a.high_limit)) {
      const uint64_t m64 = static_cast<uint64_t>(T.product[0]) | (static_cast<uint64_t>(T.product[1]) << 32);
      v = static_cast<int64_t>(lo64 - m64);  // x - M_P, exact in 64 bits
    } else {
      return false;
    }
    static_cast<int64_t*>(a.dst)[dst_index(a, cell)] = v;
    return true;
  } else if (kMode == Mode::U64) {
    if (!upper_zero || lo64 > a.bound) return false;
    static_cast<uint64_t*>(a.dst)[dst_index(a, cell)] = lo64;
    return true;
  } else {
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

// Host-side M_P as 32-bit limbs.
void host_product32(uint32_t prefix, uint32_t out[kLimbs32]) {
  uint64_t prod[kLimbs32] = {1, 0, 0, 0, 0};
  for (uint32_t i = 0; i < prefix; ++i) {
    uint64_t carry = 0;
    for (int l = 0; l < kLimbs32; ++l) {
      const uint64_t v = prod[l] * kLadder[i] + carry;
      prod[l] = v & 0xFFFFFFFFull;
      carry = v >> 32;
    }
  }
  for (int l = 0; l < kLimbs32; ++l) out[l] = static_cast<uint32_t>(prod[l]);
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
  uint32_t prod[kLimbs32];
  host_product32(prefix, prod);
  // high_limit = M_P - bound (bound < M_P / 2 is guaranteed by plan validation).
  const uint32_t b[kLimbs32] = {static_cast<uint32_t>(bound), static_cast<uint32_t>(bound >> 32), 0, 0, 0};
  uint64_t borrow = 0;
  for (int l = 0; l < kLimbs32; ++l) {
    const uint64_t sub = static_cast<uint64_t>(b[l]) + borrow;
    borrow = prod[l] < sub ? 1 : 0;
    a.high_limit[l] = static_cast<uint32_t>(static_cast<uint64_t>(prod[l]) - sub);
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
