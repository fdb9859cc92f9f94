// Residue-to-integer reconstruction used by the export kernels: the exact
// mixed-radix (Garner) path, and the fractional CRT for bounded values.
//
// x = sum_i c_i * M_i with M_i = m_0 * ... * m_{i-1}, so
//   c_i = (r_i - sum_{j<i} c_j * (M_j mod m_i)) * (M_i mod m_i)^-1  (mod m_i)
//       = (r_i * inv_i + sum_{j<i} c_j * w'_ij)                      (mod m_i)
// with w'_ij = -(M_j mod m_i) * inv_i mod m_i. Every digit and weight is a
// byte, so the sum is a chain of dp4a over digits packed four per word; it
// stays below 2^21, where q = mulhi(S, ceil(2^32/m)) is the exact quotient,
// so each digit costs one reduction. x is rebuilt by Horner in 32-bit limbs,
// each step touching only the limbs the partial product can occupy. All
// tables are compile-time constants of the prefix P. Reference order:
// src/reconstruct/crt.cpp:54-76 (the digits of a mixed-radix representation
// are unique, so any digit recurrence yields the same x).
#pragma once

#include "device_common.cuh"

namespace rns8cuda {
namespace garner {

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


// Bounded int64 / uint64 decision on the reconstructed value (crt.cpp:78-121):
// signed: x <= low_limit -> x; x >= M_P - bound -> x - M_P; otherwise a range
// error. Plans guarantee M_P > 2 * bound, which makes this identical to
// centering at ceil(M_P/2) followed by the |v| <= bound check.
struct BoundedLimits {
  uint64_t bound;                 // unsigned: x <= bound
  uint64_t low_limit;             // signed: min(bound, INT64_MAX)
  uint32_t high_limit[kLimbs32];  // signed: M_P - bound
};

template <int P, bool kSigned>
__device__ __forceinline__ bool reconstruct_bounded(const int (&r)[P], const BoundedLimits& lim, uint64_t* out) {
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
  if (kSigned) {
    if (upper_zero && lo64 <= lim.low_limit) {
      *out = lo64;
      return true;
    }
    if (geq32<L>(x, lim.high_limit)) {
      const uint64_t m64 = static_cast<uint64_t>(T.product[0]) | (static_cast<uint64_t>(T.product[1]) << 32);
      *out = lo64 - m64;  // x - M_P, exact in 64 bits
      return true;
    }
    return false;
  }
  if (!upper_zero || lo64 > lim.bound) return false;
  *out = lo64;
  return true;
}

// ---- fractional CRT for bounded values ---------------------------------------
// With E_i = M/m_i and inv_i = E_i^-1 mod m_i, every residue vector r
// satisfies sum_i r_i * E_i * inv_i = x + q*M for the value x it represents,
// and sum_i r_i * inv_i / m_i = x/M + q. When |x| is small against M (a
// bounded export), the fraction x/M is close to 0, so q is the nearest
// integer to that sum, which a fixed-point accumulation with 2^-31 resolution
// gives, and x = sum_i r_i * (E_i * inv_i) - q*M is then exact modulo 2^64.
// (Approximate-quotient CRT of Shenoy and Kumaresan; the same reconstruction
// is used by the Ozaki-II integer emulation of floating-point GEMM.) Cells
// whose fraction lies within the rounding error of the bound's edge are left
// to the exact Garner path.
constexpr int64_t kQuotientBias = 4096;  // > 128 * P + 1: keeps the biased quotient nonnegative

template <int P>
struct FracTable {
  uint32_t F[P];     // round(2^31 * inv_i / m_i)
  uint32_t Glo[P];   // (E_i * inv_i) mod 2^64, low and high words
  uint32_t Ghi[P];
  uint64_t C0;       // 128 * sum G_i - kQuotientBias * M  (mod 2^64)
  int64_t sumF128;   // 128 * sum F_i
  uint64_t M64;      // M mod 2^64
};

template <int P>
__host__ __device__ constexpr FracTable<P> make_frac_table() {
  FracTable<P> t{};
  uint64_t m64 = 1;
  for (int i = 0; i < P; ++i) m64 *= ladder_at(i);
  t.M64 = m64;
  uint64_t c0 = 0;
  int64_t sf = 0;
  for (int i = 0; i < P; ++i) {
    const uint32_t mi = ladder_at(i);
    uint64_t e64 = 1;      // E_i mod 2^64
    uint32_t emod = 1;     // E_i mod m_i
    for (int j = 0; j < P; ++j) {
      if (j == i) continue;
      e64 *= ladder_at(j);
      emod = (emod * ladder_at(j)) % mi;
    }
    const uint32_t inv = inv_mod(emod, mi);
    const uint64_t g = e64 * inv;
    t.F[i] = static_cast<uint32_t>(((static_cast<uint64_t>(inv) << 31) + mi / 2) / mi);
    t.Glo[i] = static_cast<uint32_t>(g);
    t.Ghi[i] = static_cast<uint32_t>(g >> 32);
    c0 += 128ull * g;
    sf += 128ll * t.F[i];
  }
  t.C0 = c0 - static_cast<uint64_t>(kQuotientBias) * m64;
  t.sumF128 = sf;
  return t;
}

// Per-call constants in units of 2^-31 of M. The device sum starts at s_init =
// 2^30 + kQuotientBias * 2^31 - (128 * sum F_i + center), so that s >> 31 is
// the rounded quotient plus the bias and the low 31 bits minus 2^30 are the
// signed fraction. Accepting |frac| <= t_in implies the quotient is right and
// the value is in range; |frac| >= t_out implies it is out of range; the band
// between goes to the exact path. A wrong quotient needs |frac| >= 2^30 - err,
// which exceeds t_in because the bound is below M/2 (signed) or M (unsigned).
struct FracLimits {
  int enabled;      // 0: use the exact path for every cell
  uint32_t t_in;
  uint32_t t_out;
  uint64_t s_init;
};

// ---- fractional CRT for exact-wide limbs ---------------------------------------
// The same approximate-quotient CRT at full width: v = sum_i r_i * G_i - q*M
// with G_i = E_i * inv_i (< M) is computed modulo 2^192, where the centered
// value |v| <= M/2 < 2^155 is exact in two's complement, and q is the nearest
// integer to sum_i r_i * inv_i / m_i (2^-31 fixed point). The quotient is
// only in doubt when |v| is within the rounding error of M/2, which no
// admitted exact-wide product reaches; such cells take the exact Garner path.
// Four planes' bytes of one cell form a word, so every byte-slice sum
// sum_i u_i * byte_b(G_i) over 4 planes is one dp4a.
template <int P>
constexpr int wide_bytes() {  // bytes of M_P
  uint64_t prod[kLimbs32] = {1, 0, 0, 0, 0};
  for (int i = 0; i < P; ++i) {
    uint64_t carry = 0;
    for (int l = 0; l < kLimbs32; ++l) {
      const uint64_t v = prod[l] * ladder_at(i) + carry;
      prod[l] = v & 0xFFFFFFFFull;
      carry = v >> 32;
    }
  }
  int bytes = 4 * kLimbs32;
  while (bytes > 1 && ((prod[(bytes - 1) / 4] >> (8 * ((bytes - 1) % 4))) & 0xFFu) == 0) --bytes;
  return bytes;
}

template <int P>
struct WideFracTable {
  static constexpr int kGroups = (P + 3) / 4;
  static constexpr int kBytes = wide_bytes<P>();
  uint32_t fpack[kGroups][4];       // byte b of F_i for planes 4g..4g+3
  uint32_t gpack[kGroups][kBytes];  // byte b of G_i for planes 4g..4g+3
  uint32_t c0[6];                   // 128 * sum G_i - kQuotientBias * M  (mod 2^192)
  uint32_t product[kLimbs32];       // M
  uint64_t s_init;                  // 2^30 + kQuotientBias * 2^31 - 128 * sum F_i
  uint32_t t_dec;                   // the quotient is certain when |frac| <= t_dec
};

template <int P>
__host__ __device__ constexpr WideFracTable<P> make_wide_frac_table() {
  WideFracTable<P> t{};
  constexpr int kG = WideFracTable<P>::kGroups;
  constexpr int kB = WideFracTable<P>::kBytes;
  uint64_t M[6] = {1, 0, 0, 0, 0, 0};  // 32-bit limbs in 64-bit words
  for (int i = 0; i < P; ++i) {
    uint64_t carry = 0;
    for (int l = 0; l < 6; ++l) {
      const uint64_t v = M[l] * ladder_at(i) + carry;
      M[l] = v & 0xFFFFFFFFull;
      carry = v >> 32;
    }
  }
  for (int l = 0; l < kLimbs32; ++l) t.product[l] = static_cast<uint32_t>(M[l]);
  uint64_t sumG[6] = {0, 0, 0, 0, 0, 0};
  int64_t sumF = 0;
  for (int g = 0; g < kG; ++g) {
    for (int b = 0; b < 4; ++b) t.fpack[g][b] = 0;
    for (int b = 0; b < kB; ++b) t.gpack[g][b] = 0;
  }
  for (int i = 0; i < P; ++i) {
    const uint32_t mi = ladder_at(i);
    uint64_t E[6] = {1, 0, 0, 0, 0, 0};  // M / m_i
    uint32_t emod = 1;
    for (int j = 0; j < P; ++j) {
      if (j == i) continue;
      uint64_t carry = 0;
      for (int l = 0; l < 6; ++l) {
        const uint64_t v = E[l] * ladder_at(j) + carry;
        E[l] = v & 0xFFFFFFFFull;
        carry = v >> 32;
      }
      emod = (emod * ladder_at(j)) % mi;
    }
    const uint32_t inv = inv_mod(emod, mi);
    uint64_t G[6] = {0, 0, 0, 0, 0, 0};  // E_i * inv_i < M
    uint64_t carry = 0;
    for (int l = 0; l < 6; ++l) {
      const uint64_t v = E[l] * inv + carry;
      G[l] = v & 0xFFFFFFFFull;
      carry = v >> 32;
    }
    const uint32_t F = static_cast<uint32_t>(((static_cast<uint64_t>(inv) << 31) + mi / 2) / mi);
    sumF += F;
    carry = 0;
    for (int l = 0; l < 6; ++l) {
      const uint64_t v = sumG[l] + G[l] + carry;
      sumG[l] = v & 0xFFFFFFFFull;
      carry = v >> 32;
    }
    const int g = i / 4, lane = i % 4;
    for (int b = 0; b < 4; ++b) t.fpack[g][b] |= ((F >> (8 * b)) & 0xFFu) << (8 * lane);
    for (int b = 0; b < kB; ++b) t.gpack[g][b] |= static_cast<uint32_t>((G[b / 4] >> (8 * (b % 4))) & 0xFFu) << (8 * lane);
  }
  // c0 = 128 * sumG - bias * M  (mod 2^192)
  uint64_t a[6] = {0, 0, 0, 0, 0, 0}, bm[6] = {0, 0, 0, 0, 0, 0};
  uint64_t carry = 0;
  for (int l = 0; l < 6; ++l) {
    const uint64_t v = sumG[l] * 128 + carry;
    a[l] = v & 0xFFFFFFFFull;
    carry = v >> 32;
  }
  carry = 0;
  for (int l = 0; l < 6; ++l) {
    const uint64_t v = M[l] * static_cast<uint64_t>(kQuotientBias) + carry;
    bm[l] = v & 0xFFFFFFFFull;
    carry = v >> 32;
  }
  uint64_t borrow = 0;
  for (int l = 0; l < 6; ++l) {
    const uint64_t sub = bm[l] + borrow;
    borrow = a[l] < sub ? 1 : 0;
    t.c0[l] = static_cast<uint32_t>((a[l] + (borrow << 32)) - sub);
  }
  t.s_init = (1ull << 30) + (static_cast<uint64_t>(kQuotientBias) << 31) - static_cast<uint64_t>(128 * sumF);
  t.t_dec = (1u << 30) - 2u * (64u * P + 2u);
  return t;
}

// v (192-bit two's complement, 32-bit limbs) of the cell whose four-plane
// words are cw[g] (u_i = r_i + 128 in byte i % 4 of word i / 4). Returns false
// when the quotient is in doubt.
template <int P>
__device__ __forceinline__ bool wide_frac_reconstruct(const uint32_t (&cw)[(P + 3) / 4], uint32_t (&v)[6]) {
  constexpr WideFracTable<P> T = make_wide_frac_table<P>();
  constexpr int kG = WideFracTable<P>::kGroups;
  constexpr int kB = WideFracTable<P>::kBytes;
  uint32_t tf[4] = {0, 0, 0, 0};
#pragma unroll
  for (int b = 0; b < 4; ++b)
#pragma unroll
    for (int g = 0; g < kG; ++g) tf[b] = __dp4a(cw[g], T.fpack[g][b], tf[b]);
  const uint64_t s = T.s_init + tf[0] + (static_cast<uint64_t>(tf[1]) << 8) + (static_cast<uint64_t>(tf[2]) << 16) +
                     (static_cast<uint64_t>(tf[3]) << 24);
  const int32_t frac = static_cast<int32_t>(static_cast<uint32_t>(s) & 0x7FFFFFFFu) - (1 << 30);
  if (static_cast<uint32_t>(frac < 0 ? -frac : frac) > T.t_dec) return false;
  const uint32_t q = static_cast<uint32_t>(s >> 31);
  // S = sum_i u_i * G_i (mod 2^192) from byte-slice sums (each < 2^21).
  uint64_t carry = 0;
#pragma unroll
  for (int l = 0; l < 6; ++l) {
    uint64_t acc = carry;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = 4 * l + j;
      if (b < kB) {
        uint32_t tb = 0;
#pragma unroll
        for (int g = 0; g < kG; ++g) tb = __dp4a(cw[g], T.gpack[g][b], tb);
        acc += static_cast<uint64_t>(tb) << (8 * j);
      }
    }
    v[l] = static_cast<uint32_t>(acc);
    carry = acc >> 32;
  }
  // v = S - c0 - q * M  (mod 2^192)
  uint64_t qm_carry = 0;
  int64_t borrow = 0;
#pragma unroll
  for (int l = 0; l < 6; ++l) {
    const uint64_t qm = static_cast<uint64_t>(q) * (l < kLimbs32 ? T.product[l] : 0u) + qm_carry;
    qm_carry = qm >> 32;
    const int64_t d = static_cast<int64_t>(v[l]) - T.c0[l] - static_cast<uint32_t>(qm) + borrow;
    v[l] = static_cast<uint32_t>(d);
    borrow = d >> 32;  // 0, -1 or -2
  }
  return true;
}

// 1 = value written to *out, 0 = out of range, -1 = undecided (use exact path).
// u_i = r_i + 128.
template <int P>
__device__ __forceinline__ int frac_reconstruct(const uint32_t (&u)[P], const FracLimits& fl, uint64_t* out) {
  constexpr FracTable<P> T = make_frac_table<P>();
  uint64_t s = fl.s_init;
  uint64_t vl = 0;
  uint32_t vh = 0;
#pragma unroll
  for (int i = 0; i < P; ++i) {
    s += static_cast<uint64_t>(u[i]) * T.F[i];
    vl += static_cast<uint64_t>(u[i]) * T.Glo[i];
    vh += u[i] * T.Ghi[i];
  }
  const uint32_t s_lo = static_cast<uint32_t>(s);
  const uint32_t q = __funnelshift_r(s_lo, static_cast<uint32_t>(s >> 32), 31);
  const int32_t frac = static_cast<int32_t>(s_lo & 0x7FFFFFFFu) - (1 << 30);
  const uint32_t afrac = static_cast<uint32_t>(frac < 0 ? -frac : frac);
  if (afrac >= fl.t_out) return 0;
  if (afrac > fl.t_in) return -1;
  *out = vl + (static_cast<uint64_t>(vh) << 32) - T.C0 - static_cast<uint64_t>(q) * T.M64;
  return 1;
}

// The same sums taken two planes at a time with dp2a (two 16-bit x 8-bit
// products plus a 32-bit addend): F_i and G_i mod 2^64 are written as signed
// 16-bit digits (F_i = d0 + d1 * 2^16, G_i = sum_b d_b * 2^(16b) mod 2^64),
// the digits of planes 2k and 2k+1 share a word, and one byte permute puts
// both planes' signed residues for two cells into the dp2a byte operand.
// Every digit sum stays below P * 128 * 2^15 < 2^27, so
//   sum_i r_i * F_i = f0 + f1 * 2^16   and   sum_i r_i * G_i = sum_b g_b * 2^(16b)  (mod 2^64)
// are the multiply-add form's integers exactly, with r_i in place of r_i + 128.
template <int P>
struct PairTable {
  static constexpr int kPairs = (P + 1) / 2;
  uint32_t f[kPairs][2];
  uint32_t g[kPairs][4];
  uint64_t m64;       // M mod 2^64
  uint64_t bias_m64;  // kQuotientBias * M mod 2^64
  uint64_t sumF128;   // 128 * sum F_i: turns FracLimits::s_init (for r + 128) into the start for r
};

__host__ __device__ constexpr uint32_t signed_digit16(uint64_t v, int b) {
  // digit b of the balanced base-2^16 expansion of v mod 2^64, as a 16-bit pattern
  for (int i = 0; i < b; ++i) {
    const uint32_t low = static_cast<uint32_t>(v & 0xFFFFu);
    v = (v >> 16) + (low >= 0x8000u ? 1u : 0u);
  }
  return static_cast<uint32_t>(v & 0xFFFFu);
}

template <int P>
__host__ __device__ constexpr PairTable<P> make_pair_table() {
  constexpr FracTable<P> T = make_frac_table<P>();
  PairTable<P> t{};
  for (int k = 0; k < PairTable<P>::kPairs; ++k) {
    for (int b = 0; b < 2; ++b) t.f[k][b] = 0;
    for (int b = 0; b < 4; ++b) t.g[k][b] = 0;
  }
  for (int i = 0; i < P; ++i) {
    const uint64_t g = static_cast<uint64_t>(T.Glo[i]) | (static_cast<uint64_t>(T.Ghi[i]) << 32);
    const int k = i / 2, sh = 16 * (i % 2);
    for (int b = 0; b < 2; ++b) t.f[k][b] |= signed_digit16(T.F[i], b) << sh;
    for (int b = 0; b < 4; ++b) t.g[k][b] |= signed_digit16(g, b) << sh;
  }
  t.m64 = T.M64;
  t.bias_m64 = static_cast<uint64_t>(kQuotientBias) * T.M64;
  t.sumF128 = static_cast<uint64_t>(T.sumF128);
  return t;
}

// Host: M_P as 32-bit limbs, and the limits for a bounded export.
inline void host_product32(uint32_t prefix, uint32_t out[kLimbs32]) {
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

// Thresholds of the fractional path for prefix P and bound. The accepted
// interval is [-bound, bound] (signed) or [0, bound] (unsigned), i.e. a
// half-width W = bound/M (or bound/2M) around center 0 (or bound/2M). The
// fixed-point sum errs by at most 64*P + 1 units (F_i rounding with |r_i| <=
// 128, plus the rounded center); the path is enabled only when the undecided
// band is small against W.
inline FracLimits host_frac_limits(uint32_t prefix, uint64_t bound, bool is_signed, int64_t sum_f128) {
  FracLimits fl{};
  uint32_t prod[kLimbs32];
  host_product32(prefix, prod);
  if (prod[4] != 0 || (prod[3] >> 31) != 0) return fl;  // M >= 2^127: fraction too fine for 2^-31 units
  unsigned __int128 M = 0;
  for (int l = 3; l >= 0; --l) M = (M << 32) | prod[l];
  const unsigned __int128 num = static_cast<unsigned __int128>(bound) << 31;
  const unsigned __int128 den = is_signed ? M : 2 * M;
  const int64_t w = static_cast<int64_t>(num / den);  // < 2^30: bound < M/2 (signed) or M (unsigned)
  const int64_t center = is_signed ? 0 : static_cast<int64_t>((num + M) / (2 * M));  // round(2^31 * bound / 2M)
  const int64_t err = 64 * static_cast<int64_t>(prefix) + 2;
  if (w - err - 1 <= 4 * err) return fl;
  // A signed bound of 2^63 admits -2^63 but not +2^63, an asymmetry the
  // fraction does not see: such calls take the exact path.
  if (is_signed && bound > 0x7FFFFFFFFFFFFFFFull) return fl;
  fl.enabled = 1;
  fl.t_in = static_cast<uint32_t>(w - err - 1);
  fl.t_out = static_cast<uint32_t>(w + err + 1);
  fl.s_init = (1ull << 30) + (static_cast<uint64_t>(kQuotientBias) << 31) - static_cast<uint64_t>(sum_f128 + center);
  return fl;
}

inline BoundedLimits host_limits(uint32_t prefix, uint64_t bound) {
  BoundedLimits lim{};
  lim.bound = bound;
  lim.low_limit = bound < 0x7FFFFFFFFFFFFFFFull ? bound : 0x7FFFFFFFFFFFFFFFull;
  uint32_t prod[kLimbs32];
  host_product32(prefix, prod);
  const uint32_t b[kLimbs32] = {static_cast<uint32_t>(bound), static_cast<uint32_t>(bound >> 32), 0, 0, 0};
  uint64_t borrow = 0;
  for (int l = 0; l < kLimbs32; ++l) {
    const uint64_t sub = static_cast<uint64_t>(b[l]) + borrow;
    borrow = prod[l] < sub ? 1 : 0;
    lim.high_limit[l] = static_cast<uint32_t>(static_cast<uint64_t>(prod[l]) - sub);
  }
  return lim;
}

}  // namespace garner
}  // namespace rns8cuda
