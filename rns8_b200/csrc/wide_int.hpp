// 256-bit two's-complement integer for host-side contract arithmetic:
// modulus products (<= 155 bits), K * 2^128 exact-wide ranges, and the
// exact-wide admission proofs (products of 64-bit magnitudes with K-long
// sums, < 2^193). It stands in for the reference's Boost cpp_int on these
// paths; every operation used there is exact within 256 bits.
#pragma once

#include <cstdint>

// Usable from device code too (the exact-wide admission kernels) when the
// including file is compiled as CUDA.
#ifdef __CUDACC__
#define RNS8_HD __host__ __device__ __forceinline__
#else
#define RNS8_HD inline
#endif

namespace rns8host {

struct i256 {
  uint64_t w[4] = {0, 0, 0, 0};

  RNS8_HD static i256 from_u64(uint64_t v) {
    i256 r;
    r.w[0] = v;
    return r;
  }
  RNS8_HD static i256 from_i64(int64_t v) {
    i256 r;
    const uint64_t s = v < 0 ? ~0ull : 0ull;
    r.w[0] = static_cast<uint64_t>(v);
    r.w[1] = r.w[2] = r.w[3] = s;
    return r;
  }
  RNS8_HD static i256 from_i128(__int128 v) {
    i256 r;
    const uint64_t s = v < 0 ? ~0ull : 0ull;
    r.w[0] = static_cast<uint64_t>(v);
    r.w[1] = static_cast<uint64_t>(static_cast<unsigned __int128>(v) >> 64);
    r.w[2] = r.w[3] = s;
    return r;
  }
  RNS8_HD static i256 from_u128(unsigned __int128 v) {
    i256 r;
    r.w[0] = static_cast<uint64_t>(v);
    r.w[1] = static_cast<uint64_t>(v >> 64);
    return r;
  }
  RNS8_HD bool neg() const { return (w[3] >> 63) != 0; }
  RNS8_HD bool zero() const { return (w[0] | w[1] | w[2] | w[3]) == 0; }
};

RNS8_HD i256 operator+(const i256& a, const i256& b) {
  i256 r;
  unsigned __int128 c = 0;
  for (int i = 0; i < 4; ++i) {
    c += static_cast<unsigned __int128>(a.w[i]) + b.w[i];
    r.w[i] = static_cast<uint64_t>(c);
    c >>= 64;
  }
  return r;
}
RNS8_HD i256 operator-(const i256& a) {
  i256 r;
  for (int i = 0; i < 4; ++i) r.w[i] = ~a.w[i];
  return r + i256::from_u64(1);
}
RNS8_HD i256 operator-(const i256& a, const i256& b) { return a + (-b); }
RNS8_HD int cmp(const i256& a, const i256& b) {
  if (a.neg() != b.neg()) return a.neg() ? -1 : 1;
  for (int i = 3; i >= 0; --i)
    if (a.w[i] != b.w[i]) return a.w[i] < b.w[i] ? -1 : 1;
  return 0;
}
RNS8_HD bool operator<(const i256& a, const i256& b) { return cmp(a, b) < 0; }
RNS8_HD bool operator>(const i256& a, const i256& b) { return cmp(a, b) > 0; }
RNS8_HD bool operator<=(const i256& a, const i256& b) { return cmp(a, b) <= 0; }
RNS8_HD bool operator>=(const i256& a, const i256& b) { return cmp(a, b) >= 0; }
RNS8_HD bool operator==(const i256& a, const i256& b) { return cmp(a, b) == 0; }
RNS8_HD i256 abs(const i256& a) { return a.neg() ? -a : a; }
RNS8_HD i256 max(const i256& a, const i256& b) { return a >= b ? a : b; }
RNS8_HD i256 min(const i256& a, const i256& b) { return a <= b ? a : b; }
// Truncating signed product.
RNS8_HD i256 operator*(const i256& a0, const i256& b0) {
  const bool n = a0.neg() != b0.neg();
  const i256 a = abs(a0), b = abs(b0);
  i256 r;
  for (int i = 0; i < 4; ++i) {
    if (a.w[i] == 0) continue;
    unsigned __int128 carry = 0;
    for (int j = 0; i + j < 4; ++j) {
      const unsigned __int128 cur = static_cast<unsigned __int128>(a.w[i]) * b.w[j] + r.w[i + j] + carry;
      r.w[i + j] = static_cast<uint64_t>(cur);
      carry = cur >> 64;
    }
  }
  return n ? -r : r;
}
RNS8_HD i256 shl(const i256& a, unsigned s) {
  i256 r;
  const unsigned limb = s / 64, bit = s % 64;
  for (int i = 3; i >= 0; --i) {
    const int src = i - static_cast<int>(limb);
    if (src < 0) continue;
    r.w[i] = a.w[src] << bit;
    if (bit && src >= 1) r.w[i] |= a.w[src - 1] >> (64 - bit);
  }
  return r;
}
// Signed division by two rounding toward zero (cpp_int semantics).
RNS8_HD i256 half_trunc(const i256& a) {
  const bool n = a.neg();
  i256 m = abs(a);
  for (int i = 0; i < 4; ++i) m.w[i] = (m.w[i] >> 1) | (i < 3 ? (m.w[i + 1] << 63) : 0);
  return n ? -m : m;
}
RNS8_HD uint32_t bit_length(const i256& a) {
  if (a.neg() || a.zero()) return 0;
  for (int i = 3; i >= 0; --i)
#ifdef __CUDA_ARCH__
    if (a.w[i]) return static_cast<uint32_t>(64 * i + 64 - __clzll(static_cast<long long>(a.w[i])));
#else
    if (a.w[i]) return static_cast<uint32_t>(64 * i + 64 - __builtin_clzll(a.w[i]));
#endif
  return 0;
}

}  // namespace rns8host
