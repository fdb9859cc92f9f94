// TEST INFRASTRUCTURE ONLY — the CPU oracle for the RNS8 hot path.
//
// This file restates, in plain C-style C++ without Boost, the reference's CPU
// algorithm for the path pack -> per-plane ring GEMM -> CRT/Garner export:
//   src/cpu/cpu_reference.cpp      (residue maps, pack/export loops, blocked GEMM)
//   src/cpu/cpu_parallel.cpp       (OpenMP partitioning and the 1<<20 threshold)
//   src/reconstruct/crt.cpp        (Garner order, centering, fits checks, limbs)
//   src/core/moduli.cpp            (ladder, prefix selection, descriptor validation)
//   src/core/api_plan_schedule.inc (global-bound prefix schedule)
//   src/core/api_oneshot.cpp       (oneshot orchestration and required ranges)
//   src/core/api_export.cpp        (stage-all-then-commit export semantics)
//   src/core/exact_range.hpp       (exact-wide admission proofs)
// Boost.Multiprecision cpp_int is replaced by a 256-bit two's-complement
// integer (wide256); every quantity on this path fits in 256 bits.
//
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
// this library, and only as the checker or the timed CPU baseline. The
// product library (rns8_b200) never links or calls it.

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <cmath>
#include <random>
#include <vector>
#include <new>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OX extern "C" __attribute__((visibility("default")))

namespace {

// ---- status / enum values (include/rns8/status.h, semantics.h, bounds.h) ----
enum {
  ST_SUCCESS = 0, ST_INVALID = 1, ST_UNSUPPORTED_BACKEND = 4, ST_RANGE = 5,
};
enum { SEM_I64 = 1, SEM_U64 = 2, SEM_EW_S = 3, SEM_EW_U = 4, SEM_WRAP = 5, SEM_RING = 6, SEM_FIELD = 7 };
enum { BK_NONE = 0, BK_ABS = 1, BK_UNS = 2, BK_TILE_ABS = 3, BK_TILE_UNS = 4, BK_INPUT = 5 };
constexpr uint32_t kMaxPrefix = 20;
constexpr uint32_t kDefaultBoundedPrefix = 9;
constexpr int64_t kSafeBlock = 65536;
constexpr uint32_t FLAG_FORCE = 1u, FLAG_ZERO_TILE = 2u, FLAG_ZERO_RC = 4u;

// src/core/internal.hpp:328-330 — the 28-entry ladder.
constexpr uint16_t kLadder[28] = {256, 255, 253, 251, 247, 239, 233, 229, 227, 223, 217, 211, 199, 197,
                                  193, 191, 181, 179, 173, 167, 163, 157, 151, 149, 139, 137, 131, 127};

// ---------------------------------------------------------------------------
// wide256: little-endian 4 x 64-bit two's-complement integer.
struct wide256 {
  uint64_t w[4];
};
wide256 w_zero() { return wide256{{0, 0, 0, 0}}; }
wide256 w_u64(uint64_t v) { return wide256{{v, 0, 0, 0}}; }
wide256 w_i64(int64_t v) {
  uint64_t s = v < 0 ? ~0ull : 0ull;
  return wide256{{static_cast<uint64_t>(v), s, s, s}};
}
bool w_neg(const wide256& a) { return (a.w[3] >> 63) != 0; }
bool w_is_zero(const wide256& a) { return (a.w[0] | a.w[1] | a.w[2] | a.w[3]) == 0; }
wide256 w_add(const wide256& a, const wide256& b) {
  wide256 r;
  unsigned __int128 c = 0;
  for (int i = 0; i < 4; ++i) {
    c += static_cast<unsigned __int128>(a.w[i]) + b.w[i];
    r.w[i] = static_cast<uint64_t>(c);
    c >>= 64;
  }
  return r;
}
wide256 w_not(const wide256& a) { return wide256{{~a.w[0], ~a.w[1], ~a.w[2], ~a.w[3]}}; }
wide256 w_negate(const wide256& a) { return w_add(w_not(a), w_u64(1)); }
wide256 w_sub(const wide256& a, const wide256& b) { return w_add(a, w_negate(b)); }
// Signed comparison.
int w_cmp(const wide256& a, const wide256& b) {
  const bool na = w_neg(a), nb = w_neg(b);
  if (na != nb) return na ? -1 : 1;
  for (int i = 3; i >= 0; --i) {
    if (a.w[i] != b.w[i]) return a.w[i] < b.w[i] ? -1 : 1;
  }
  return 0;
}
wide256 w_abs(const wide256& a) { return w_neg(a) ? w_negate(a) : a; }
// Truncating signed multiply (operands in this oracle never exceed 256 bits).
wide256 w_mul(const wide256& a0, const wide256& b0) {
  const bool neg = w_neg(a0) != w_neg(b0);
  const wide256 a = w_abs(a0), b = w_abs(b0);
  wide256 r = w_zero();
  for (int i = 0; i < 4; ++i) {
    unsigned __int128 carry = 0;
    for (int j = 0; i + j < 4; ++j) {
      unsigned __int128 cur = static_cast<unsigned __int128>(a.w[i]) * b.w[j] + r.w[i + j] + carry;
      r.w[i + j] = static_cast<uint64_t>(cur);
      carry = cur >> 64;
    }
  }
  return neg ? w_negate(r) : r;
}
wide256 w_mul_u32(const wide256& a, uint32_t m) { return w_mul(a, w_u64(m)); }
wide256 w_shl(const wide256& a, unsigned s) {
  wide256 r = w_zero();
  const unsigned limb = s / 64, bit = s % 64;
  for (int i = 3; i >= 0; --i) {
    const int src = i - static_cast<int>(limb);
    if (src < 0) continue;
    r.w[i] = a.w[src] << bit;
    if (bit && src - 1 >= 0) r.w[i] |= a.w[src - 1] >> (64 - bit);
  }
  return r;
}
// Non-negative value modulo a small modulus.
uint32_t w_umod_small(const wide256& a, uint32_t m) {
  unsigned __int128 rem = 0;
  for (int i = 3; i >= 0; --i) rem = ((rem << 64) | a.w[i]) % m;
  return static_cast<uint32_t>(rem);
}
// Signed truncating division by 2 (cpp_int semantics: rounds toward zero).
wide256 w_div2_trunc(const wide256& a) {
  const bool neg = w_neg(a);
  wide256 m = w_abs(a);
  for (int i = 0; i < 4; ++i) m.w[i] = (m.w[i] >> 1) | (i < 3 ? (m.w[i + 1] << 63) : 0);
  return neg ? w_negate(m) : m;
}
uint32_t w_bit_length(const wide256& a) {
  if (w_neg(a) || w_is_zero(a)) return 0;
  for (int i = 3; i >= 0; --i)
    if (a.w[i]) return static_cast<uint32_t>(64 * i + 64 - __builtin_clzll(a.w[i]));
  return 0;
}
wide256 w_max(const wide256& a, const wide256& b) { return w_cmp(a, b) >= 0 ? a : b; }
wide256 w_min(const wide256& a, const wide256& b) { return w_cmp(a, b) <= 0 ? a : b; }

// ---- src/core/moduli.cpp:164-190 ------------------------------------------------
wide256 modulus_product(uint32_t prefix) {
  wide256 p = w_u64(1);
  for (uint32_t i = 0; i < prefix; ++i) p = w_mul_u32(p, kLadder[i]);
  return p;
}
uint32_t required_prefix_for_range(const wide256& range) {
  wide256 product = w_u64(1);
  for (uint32_t prefix = 1; prefix <= kMaxPrefix; ++prefix) {
    product = w_mul_u32(product, kLadder[prefix - 1]);
    if (w_cmp(product, range) > 0) return prefix;
  }
  return 0;
}
// moduli.cpp:192-206
uint32_t default_prefix_for_semantics(uint32_t sem) {
  switch (sem) {
    case SEM_I64: case SEM_U64: return kDefaultBoundedPrefix;
    case SEM_EW_S: case SEM_EW_U: return kMaxPrefix;
    default: return 0;
  }
}
bool known_semantics(uint32_t s) { return s >= 1 && s <= 7; }
bool known_bound_kind(uint32_t b) { return b <= 5; }
bool valid_tile_size(uint32_t v) { return v == 0 || (v >= 64 && v <= 512 && (v & (v - 1u)) == 0); }
bool valid_finite_ring_modulus(uint32_t m) { return m >= 2 && m <= 256; }
bool valid_finite_field_modulus(uint32_t m) {
  if (m < 2 || m > 251) return false;
  for (uint32_t d = 2; d * d <= m; ++d)
    if (m % d == 0) return false;
  return true;
}
bool valid_finite_modulus_for_semantics(uint32_t sem, uint32_t m) {
  if (sem == SEM_FIELD) return valid_finite_field_modulus(m);
  if (sem == SEM_RING) return valid_finite_ring_modulus(m);
  return false;
}
// moduli.cpp:208-232 — k*lhs*rhs, bounded by the semantic's output range.
bool input_range_output_bound(uint32_t sem, uint32_t bound_kind, int64_t k, uint64_t lhs, uint64_t rhs,
                              uint64_t* out) {
  *out = 0;
  if (bound_kind != BK_INPUT || (sem != SEM_I64 && sem != SEM_U64) || k <= 0) return false;
  if (sem == SEM_I64) {
    const uint64_t max_mag = 1ull << 63;
    if (lhs > max_mag || rhs > max_mag) return false;
  }
  const wide256 product = w_mul(w_mul(w_i64(k), w_u64(lhs)), w_u64(rhs));
  const wide256 max_output = sem == SEM_I64 ? w_u64(1ull << 63) : w_u64(~0ull);
  if (w_neg(product) || w_cmp(product, max_output) > 0) return false;
  *out = product.w[0];
  return true;
}
// moduli.cpp:234-293
int validate_bound_contract(uint32_t sem, uint32_t bk, uint64_t bound, uint32_t prefix) {
  if (!known_semantics(sem) || !known_bound_kind(bk)) return ST_INVALID;
  if (prefix == 0 || prefix > kMaxPrefix) return ST_INVALID;
  const wide256 product = modulus_product(prefix);
  switch (sem) {
    case SEM_I64:
      if (bk == BK_INPUT) return ST_UNSUPPORTED_BACKEND;
      if (bk == BK_TILE_ABS) return bound == 0 ? ST_SUCCESS : ST_INVALID;
      if (bk == BK_NONE || bk == BK_UNS || bk == BK_TILE_UNS) return ST_INVALID;
      if (bk != BK_ABS) return ST_UNSUPPORTED_BACKEND;
      if (bound > (1ull << 63)) return ST_INVALID;
      return w_cmp(product, w_mul(w_u64(2), w_u64(bound))) > 0 ? ST_SUCCESS : ST_RANGE;
    case SEM_U64:
      if (bk == BK_INPUT) return ST_UNSUPPORTED_BACKEND;
      if (bk == BK_TILE_UNS) return bound == 0 ? ST_SUCCESS : ST_INVALID;
      if (bk == BK_NONE || bk == BK_ABS || bk == BK_TILE_ABS) return ST_INVALID;
      if (bk != BK_UNS) return ST_UNSUPPORTED_BACKEND;
      return w_cmp(product, w_u64(bound)) > 0 ? ST_SUCCESS : ST_RANGE;
    default:
      return ST_UNSUPPORTED_BACKEND;
  }
}

// The subset of rns8_gemm_desc the oracle's plan logic reads.
struct plan_desc {
  uint32_t semantics, bound_kind;
  int64_t m, n, k;
  uint64_t bound;
  uint32_t max_prefix, tile_m, tile_n, finite_modulus, flags;
  uint64_t lhs_bound, rhs_bound;
};

// moduli.cpp:295-387 (descriptor fields the oneshot contracts exercise;
// per-tile bounds and zero masks are not part of the oracle's path).
int validate_gemm_desc(const plan_desc& d, uint32_t prefix) {
  if (d.m <= 0 || d.n <= 0 || d.k <= 0) return ST_INVALID;
  if ((d.flags & ~(FLAG_FORCE | FLAG_ZERO_TILE | FLAG_ZERO_RC)) != 0) return ST_INVALID;
  const bool fixed = (d.flags & FLAG_FORCE) != 0;
  if (!valid_tile_size(d.tile_m) || !valid_tile_size(d.tile_n)) return ST_INVALID;
  const bool per_tile = d.bound_kind == BK_TILE_ABS || d.bound_kind == BK_TILE_UNS;
  if ((d.flags & FLAG_ZERO_RC) != 0) return ST_INVALID;  // masks never supplied here
  if ((d.flags & FLAG_ZERO_TILE) != 0 && !per_tile) return ST_INVALID;
  if (!known_semantics(d.semantics) || !known_bound_kind(d.bound_kind)) return ST_INVALID;
  if (d.semantics != SEM_RING && d.semantics != SEM_FIELD && d.finite_modulus != 0) return ST_INVALID;
  if (d.bound_kind != BK_INPUT && (d.lhs_bound != 0 || d.rhs_bound != 0)) return ST_INVALID;
  if (d.semantics == SEM_EW_S || d.semantics == SEM_EW_U) {
    if (d.bound_kind != BK_NONE || d.bound != 0) return ST_INVALID;
    if (prefix == 0 || prefix > kMaxPrefix) return ST_INVALID;
    const wide256 required = w_mul(w_i64(d.k), w_shl(w_u64(1), d.semantics == SEM_EW_S ? 127 : 128));
    return w_cmp(modulus_product(prefix), required) > 0 ? ST_SUCCESS : ST_RANGE;
  }
  if (d.semantics == SEM_WRAP) {
    if (d.bound_kind != BK_NONE || d.bound != 0 || prefix != 0 || fixed) return ST_INVALID;
    return ST_SUCCESS;
  }
  if (d.semantics == SEM_RING || d.semantics == SEM_FIELD) {
    if (d.bound_kind != BK_NONE || d.bound != 0 || d.max_prefix != 0 || prefix != 0 || fixed ||
        !valid_finite_modulus_for_semantics(d.semantics, d.finite_modulus))
      return ST_INVALID;
    return ST_SUCCESS;
  }
  if (d.bound_kind == BK_INPUT) {
    if (d.bound != 0) return ST_INVALID;
    uint64_t ob = 0;
    if (!input_range_output_bound(d.semantics, d.bound_kind, d.k, d.lhs_bound, d.rhs_bound, &ob)) return ST_RANGE;
    const wide256 required = d.semantics == SEM_I64 ? w_mul(w_u64(2), w_u64(ob)) : w_u64(ob);
    return w_cmp(modulus_product(prefix), required) > 0 ? ST_SUCCESS : ST_RANGE;
  }
  if (per_tile) return ST_UNSUPPORTED_BACKEND;  // per-tile schedules are outside the oracle
  return validate_bound_contract(d.semantics, d.bound_kind, d.bound, prefix);
}

// api_oneshot.cpp:473-504
wide256 schedule_required_range(const plan_desc& d) {
  switch (d.semantics) {
    case SEM_I64:
    case SEM_U64: {
      uint64_t b = d.bound;
      if (d.bound_kind == BK_INPUT) {
        if (!input_range_output_bound(d.semantics, d.bound_kind, d.k, d.lhs_bound, d.rhs_bound, &b)) return w_zero();
      }
      return d.semantics == SEM_I64 ? w_mul(w_u64(2), w_u64(b)) : w_u64(b);
    }
    case SEM_EW_S: return w_mul(w_i64(d.k), w_shl(w_u64(1), 127));
    case SEM_EW_U: return w_mul(w_i64(d.k), w_shl(w_u64(1), 128));
    default: return w_zero();
  }
}

// api_plan_public_api.inc:3-73 + api_plan_schedule.inc:263-278 for global bounds.
int plan_select_prefix(const plan_desc& d, uint32_t* selected, uint32_t* required, uint64_t* effective_bound) {
  const uint32_t prefix = d.max_prefix == 0 ? default_prefix_for_semantics(d.semantics) : d.max_prefix;
  const int v = validate_gemm_desc(d, prefix);
  if (v != ST_SUCCESS) return v;
  *effective_bound = d.bound;
  if (d.bound_kind == BK_INPUT &&
      !input_range_output_bound(d.semantics, d.bound_kind, d.k, d.lhs_bound, d.rhs_bound, effective_bound))
    return ST_RANGE;
  if (d.semantics == SEM_RING || d.semantics == SEM_FIELD || d.semantics == SEM_WRAP) {
    *selected = 0;
    *required = 0;
    return ST_SUCCESS;
  }
  const uint32_t req = required_prefix_for_range(schedule_required_range(d));
  if (req == 0 || req > prefix) return ST_RANGE;
  *required = req;
  *selected = (d.flags & FLAG_FORCE) ? prefix : req;
  return ST_SUCCESS;
}

// ---- src/cpu/cpu_parallel.cpp:15,89-102 ------------------------------------
uint64_t sat_mul(uint64_t a, uint64_t b) { return (a != 0 && b > UINT64_MAX / a) ? UINT64_MAX : a * b; }
uint64_t sat_mul3(uint64_t a, uint64_t b, uint64_t c) { return sat_mul(sat_mul(a, b), c); }
uint64_t g_threshold_ops = 1ull << 20;
bool parallel_should_use(uint64_t work) {
#ifdef _OPENMP
  return omp_get_max_threads() > 1 && work >= g_threshold_ops;
#else
  (void)work;
  return false;
#endif
}

// ---- src/cpu/cpu_reference.cpp:10-44 -----------------------------------------
uint32_t canonical_i64(int64_t v, uint16_t m) {
  __int128 r = static_cast<__int128>(v) % m;
  if (r < 0) r += m;
  return static_cast<uint32_t>(r);
}
uint32_t canonical_u64(uint64_t v, uint16_t m) { return static_cast<uint32_t>(v % m); }
int8_t center(uint32_t canonical, uint16_t m) {
  const uint32_t threshold = (static_cast<uint32_t>(m) + 1u) / 2u;
  return static_cast<int8_t>(canonical >= threshold ? static_cast<int>(canonical) - m : static_cast<int>(canonical));
}
uint32_t canonical_from_centered(int8_t r, uint16_t m) {
  return r < 0 ? static_cast<uint32_t>(r + static_cast<int>(m)) : static_cast<uint32_t>(r);
}
int8_t reduce_to_centered(int64_t value, uint16_t m) {
  int64_t r = value % static_cast<int64_t>(m);
  if (r < 0) r += m;
  if (r >= (static_cast<int64_t>(m) + 1) / 2) r -= m;
  return static_cast<int8_t>(r);
}

// cpu_reference.cpp:53-107 — modulus-major planes res[p*rows*cols + r*cols + c],
// OpenMP over plane rows.
template <typename T>
void pack_native(const T* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* out) {
  const int64_t plane_rows = static_cast<int64_t>(prefix) * rows;
  auto body = [&](int64_t pr) {
    const uint32_t p = static_cast<uint32_t>(pr / rows);
    const int64_t row = pr % rows;
    const uint16_t m = kLadder[p];
    int8_t* dst = out + (static_cast<size_t>(p) * rows + row) * cols;
    for (int64_t c = 0; c < cols; ++c) {
      const T v = src[row * ld + c];
      dst[c] = center(sizeof(T) == 8 && static_cast<T>(-1) < 0 ? canonical_i64(static_cast<int64_t>(v), m)
                                                              : canonical_u64(static_cast<uint64_t>(v), m),
                      m);
    }
  };
  if (parallel_should_use(sat_mul3(prefix, rows, cols))) {
#pragma omp parallel for schedule(static)
    for (int64_t pr = 0; pr < plane_rows; ++pr) body(pr);
    return;
  }
  for (int64_t pr = 0; pr < plane_rows; ++pr) body(pr);
}

// cpu_reference.cpp:156-206 — int32 row accumulator reset every 65536 K, each
// block folded into the previous centered residue: c = reduce(c + block_acc).
void ring_gemm_row(const int8_t* A, const int8_t* B, int8_t* C, int64_t n, int64_t k, int64_t lda, int64_t ldb,
                   int64_t ldc, uint16_t m, int64_t row, int32_t* acc) {
  int8_t* c_row = C + row * ldc;
  for (int64_t c = 0; c < n; ++c) c_row[c] = 0;
  for (int64_t off = 0; off < k;) {
    const int64_t block = (k - off) < kSafeBlock ? (k - off) : kSafeBlock;
    for (int64_t c = 0; c < n; ++c) acc[c] = 0;
    for (int64_t kk = 0; kk < block; ++kk) {
      const int av = A[row * lda + off + kk];
      const int8_t* b_row = B + (off + kk) * ldb;
      for (int64_t c = 0; c < n; ++c) acc[c] += av * static_cast<int>(b_row[c]);
    }
    for (int64_t c = 0; c < n; ++c) c_row[c] = reduce_to_centered(static_cast<int64_t>(c_row[c]) + acc[c], m);
    off += block;
  }
}
void ring_gemm_modulus(const int8_t* A, const int8_t* B, int8_t* C, int64_t m, int64_t n, int64_t k, int64_t lda,
                       int64_t ldb, int64_t ldc, uint16_t mod) {
  if (parallel_should_use(sat_mul3(m, n, k))) {
#pragma omp parallel
    {
      std::vector<int32_t> acc(static_cast<size_t>(n), 0);
#pragma omp for schedule(static)
      for (int64_t r = 0; r < m; ++r) ring_gemm_row(A, B, C, n, k, lda, ldb, ldc, mod, r, acc.data());
    }
    return;
  }
  std::vector<int32_t> acc(static_cast<size_t>(n), 0);
  for (int64_t r = 0; r < m; ++r) ring_gemm_row(A, B, C, n, k, lda, ldb, ldc, mod, r, acc.data());
}

// ---- src/reconstruct/crt.cpp:9-121 --------------------------------------------
uint32_t mod_inverse(uint32_t a, uint32_t m) {
  int64_t t = 0, nt = 1, r = m, nr = a % m;
  while (nr != 0) {
    const int64_t q = r / nr;
    int64_t tmp = t - q * nt;
    t = nt;
    nt = tmp;
    tmp = r - q * nr;
    r = nr;
    nr = tmp;
  }
  if (r != 1) return 0;
  if (t < 0) t += m;
  return static_cast<uint32_t>(t);
}
// crt.cpp:54-76 — mixed-radix Garner, x in [0, prod m_i).
wide256 reconstruct_canonical(const int8_t* residues, uint32_t prefix) {
  wide256 x = w_zero(), product = w_u64(1);
  for (uint32_t i = 0; i < prefix; ++i) {
    const uint32_t m = kLadder[i];
    const uint32_t target = canonical_from_centered(residues[i], static_cast<uint16_t>(m));
    const uint32_t x_mod = w_umod_small(x, m);
    const uint32_t inv = mod_inverse(w_umod_small(product, m), m);
    int64_t delta = (static_cast<int64_t>(target) - static_cast<int64_t>(x_mod)) % static_cast<int64_t>(m);
    if (delta < 0) delta += m;
    const uint32_t coeff = static_cast<uint32_t>((delta * inv) % m);
    x = w_add(x, w_mul_u32(product, coeff));
    product = w_mul_u32(product, m);
  }
  return x;
}
// crt.cpp:47-50
wide256 centered_from_canonical(const wide256& x, const wide256& product) {
  const wide256 threshold = w_div2_trunc(w_add(product, w_u64(1)));
  return w_cmp(x, threshold) >= 0 ? w_sub(x, product) : x;
}
// crt.cpp:78-98
int reconstruct_unsigned(const int8_t* residues, uint32_t prefix, uint64_t bound, uint64_t* out) {
  if (prefix == 0 || prefix > kMaxPrefix) return ST_INVALID;
  const int rs = validate_bound_contract(SEM_U64, BK_UNS, bound, prefix);
  if (rs != ST_SUCCESS) return rs;
  const wide256 v = reconstruct_canonical(residues, prefix);
  if (w_neg(v) || w_cmp(v, w_u64(~0ull)) > 0 || w_cmp(v, w_u64(bound)) > 0) return ST_RANGE;
  *out = v.w[0];
  return ST_SUCCESS;
}
// crt.cpp:100-121
int reconstruct_signed(const int8_t* residues, uint32_t prefix, uint64_t bound, int64_t* out) {
  if (prefix == 0 || prefix > kMaxPrefix) return ST_INVALID;
  const int rs = validate_bound_contract(SEM_I64, BK_ABS, bound, prefix);
  if (rs != ST_SUCCESS) return rs;
  const wide256 v = centered_from_canonical(reconstruct_canonical(residues, prefix), modulus_product(prefix));
  if (w_cmp(v, w_i64(INT64_MIN)) < 0 || w_cmp(v, w_i64(INT64_MAX)) > 0 || w_cmp(w_abs(v), w_u64(bound)) > 0)
    return ST_RANGE;
  *out = static_cast<int64_t>(v.w[0]);
  return ST_SUCCESS;
}
// crt.cpp:123-170 — fixed-width little-endian limbs.
int export_limbs(const int8_t* residues, uint32_t prefix, uint64_t* out, uint32_t limbs, bool is_signed) {
  if (!out || prefix == 0 || prefix > kMaxPrefix || limbs == 0 || limbs > 32) return ST_INVALID;
  const wide256 canon = reconstruct_canonical(residues, prefix);
  const uint32_t bits = 64u * limbs;
  if (!is_signed) {
    // value < 2^bits; canonical values are < 2^155, so >= 3 limbs always fit.
    if (bits < 256 && w_cmp(canon, w_shl(w_u64(1), bits)) >= 0) return ST_RANGE;
    for (uint32_t l = 0; l < limbs; ++l) out[l] = l < 4 ? canon.w[l] : 0;
    return ST_SUCCESS;
  }
  const wide256 v = centered_from_canonical(canon, modulus_product(prefix));
  if (bits < 256) {
    const wide256 hi = w_shl(w_u64(1), bits - 1);
    if (w_cmp(v, w_negate(hi)) < 0 || w_cmp(v, w_sub(hi, w_u64(1))) > 0) return ST_RANGE;
  }
  const uint64_t fill = w_neg(v) ? ~0ull : 0ull;  // two's complement sign extension
  for (uint32_t l = 0; l < limbs; ++l) out[l] = l < 4 ? v.w[l] : fill;
  return ST_SUCCESS;
}

void gather_cell(const int8_t* planes, int64_t cells, int64_t cell, uint32_t prefix, int8_t* r) {
  for (uint32_t p = 0; p < prefix; ++p) r[p] = planes[static_cast<size_t>(p) * cells + cell];
}

// ---- src/core/exact_range.hpp:12-154 -----------------------------------------
struct axis_range {
  wide256 max_magnitude, absolute_sum, sum, minimum, maximum, deviation_sum;
  bool sum_known;
};
void axis_init(axis_range& a) {
  a.max_magnitude = a.absolute_sum = a.sum = a.minimum = a.maximum = a.deviation_sum = w_zero();
  a.sum_known = false;
}
void add_native(axis_range& a, const wide256& v, bool first) {
  const wide256 mag = w_abs(v);
  a.max_magnitude = w_max(a.max_magnitude, mag);
  a.absolute_sum = w_add(a.absolute_sum, mag);
  a.sum = w_add(a.sum, v);
  if (first) {
    a.minimum = v;
    a.maximum = v;
  } else {
    a.minimum = w_min(a.minimum, v);
    a.maximum = w_max(a.maximum, v);
  }
  a.sum_known = true;
}
wide256 axis_center(const axis_range& a) { return w_div2_trunc(w_add(a.minimum, a.maximum)); }
wide256 axis_dev_max(const axis_range& a, const wide256& c) {
  return w_max(w_abs(w_sub(a.minimum, c)), w_abs(w_sub(a.maximum, c)));
}
template <typename T>
void native_exact_ranges(const T* src, int64_t rows, int64_t cols, int64_t ld, std::vector<axis_range>& rv,
                         std::vector<axis_range>& cv, wide256& maximum) {
  rv.resize(static_cast<size_t>(rows));
  cv.resize(static_cast<size_t>(cols));
  for (auto& a : rv) axis_init(a);
  for (auto& a : cv) axis_init(a);
  maximum = w_zero();
  auto val = [&](int64_t r, int64_t c) {
    return static_cast<T>(-1) < 0 ? w_i64(static_cast<int64_t>(src[r * ld + c]))
                                  : w_u64(static_cast<uint64_t>(src[r * ld + c]));
  };
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t c = 0; c < cols; ++c) {
      const wide256 v = val(r, c);
      add_native(rv[r], v, c == 0);
      add_native(cv[c], v, r == 0);
    }
    maximum = w_max(maximum, rv[r].max_magnitude);
  }
  for (int64_t r = 0; r < rows; ++r) {
    const wide256 rc = axis_center(rv[r]);
    for (int64_t c = 0; c < cols; ++c) {
      const wide256 v = val(r, c);
      rv[r].deviation_sum = w_add(rv[r].deviation_sum, w_abs(w_sub(v, rc)));
      cv[c].deviation_sum = w_add(cv[c].deviation_sum, w_abs(w_sub(v, axis_center(cv[c]))));
    }
  }
}
void tighten(wide256& bound, const wide256& cand) {
  if (w_cmp(cand, bound) < 0) bound = cand;
}
wide256 axis_product_bound(const axis_range& a, const axis_range& b, int64_t k) {
  wide256 bound = w_mul(w_mul(w_i64(k), a.max_magnitude), b.max_magnitude);
  tighten(bound, w_mul(a.absolute_sum, b.max_magnitude));
  tighten(bound, w_mul(a.max_magnitude, b.absolute_sum));
  if (a.sum_known && b.sum_known) {
    const wide256 ca = axis_center(a), cb = axis_center(b);
    const wide256 da = axis_dev_max(a, ca), db = axis_dev_max(b, cb);
    wide256 rem = w_mul(w_mul(w_i64(k), da), db);
    tighten(rem, w_mul(a.deviation_sum, db));
    tighten(rem, w_mul(da, b.deviation_sum));
    const wide256 center_term =
        w_sub(w_add(w_mul(ca, b.sum), w_mul(cb, a.sum)), w_mul(w_mul(w_i64(k), ca), cb));
    tighten(bound, w_add(w_abs(center_term), rem));
  }
  return bound;
}

void write_w(const wide256& v, uint64_t* out) {
  if (out) std::memcpy(out, v.w, sizeof(v.w));
}

std::vector<std::mt19937_64*> g_rngs;

}  // namespace

// =========================== exported oracle API ===========================

OX uint16_t oracle_modulus(uint32_t i) { return i < 28 ? kLadder[i] : 0; }
OX void oracle_modulus_product(uint32_t prefix, uint64_t* out4) { write_w(modulus_product(prefix), out4); }
OX uint32_t oracle_required_prefix_for_range(const uint64_t* range4) {
  wide256 r;
  std::memcpy(r.w, range4, sizeof(r.w));
  return required_prefix_for_range(r);
}
// moduli.cpp:21-30
OX double oracle_prefix_range_bits(uint32_t prefix) {
  if (prefix == 0 || prefix > 28) return 0.0;
  long double bits = 0.0L;
  for (uint32_t i = 0; i < prefix; ++i) bits += std::log2(static_cast<long double>(kLadder[i]));
  return static_cast<double>(bits);
}
OX int8_t oracle_centered_residue_i64(int64_t v, uint16_t m) { return center(canonical_i64(v, m), m); }
OX int8_t oracle_centered_residue_u64(uint64_t v, uint16_t m) { return center(canonical_u64(v, m), m); }
OX int8_t oracle_reduce_to_centered(int64_t v, uint16_t m) { return reduce_to_centered(v, m); }
OX void oracle_set_parallel_threshold(uint64_t ops) { g_threshold_ops = ops; }
OX int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
OX void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

OX void oracle_pack_i64(const int64_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* out) {
  pack_native<int64_t>(src, rows, cols, ld, prefix, out);
}
OX void oracle_pack_u64(const uint64_t* src, int64_t rows, int64_t cols, int64_t ld, uint32_t prefix, int8_t* out) {
  pack_native<uint64_t>(src, rows, cols, ld, prefix, out);
}
// cpu_reference.cpp:109-130
OX void oracle_pack_finite_u8(const uint8_t* src, int64_t rows, int64_t cols, int64_t ld, uint16_t m, int8_t* out) {
  auto body = [&](int64_t r) {
    for (int64_t c = 0; c < cols; ++c) out[r * cols + c] = center(canonical_u64(src[r * ld + c], m), m);
  };
  if (parallel_should_use(sat_mul(rows, cols))) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) body(r);
    return;
  }
  for (int64_t r = 0; r < rows; ++r) body(r);
}
// cpu_reference.cpp:132-153
OX void oracle_export_finite_u8(const int8_t* res, int64_t rows, int64_t cols, uint16_t m, uint8_t* dst, int64_t ld) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) dst[r * ld + c] = static_cast<uint8_t>(canonical_from_centered(res[r * cols + c], m));
}
OX void oracle_ring_gemm_modulus(const int8_t* A, const int8_t* B, int8_t* C, int64_t m, int64_t n, int64_t k,
                                 int64_t lda, int64_t ldb, int64_t ldc, uint16_t mod) {
  ring_gemm_modulus(A, B, C, m, n, k, lda, ldb, ldc, mod);
}
// cpu_reference.cpp:264-283 — one ring GEMM per plane, plane p uses kLadder[p].
OX void oracle_gemm_rns(const int8_t* A, const int8_t* B, int8_t* C, int64_t m, int64_t n, int64_t k,
                        uint32_t prefix) {
  for (uint32_t p = 0; p < prefix; ++p)
    ring_gemm_modulus(A + static_cast<size_t>(p) * m * k, B + static_cast<size_t>(p) * k * n,
                      C + static_cast<size_t>(p) * m * n, m, n, k, k, n, n, kLadder[p]);
}
// residue_dot.hpp:21-38 semantics: one cell, K blocked at 65536.
OX int8_t oracle_centered_residue_dot(const int8_t* a, const int8_t* b, int64_t k, int64_t b_stride, uint16_t m) {
  int8_t c = 0;
  for (int64_t off = 0; off < k; off += kSafeBlock) {
    const int64_t block = (k - off) < kSafeBlock ? (k - off) : kSafeBlock;
    int32_t acc = 0;
    for (int64_t i = 0; i < block; ++i) acc += static_cast<int32_t>(a[off + i]) * b[(off + i) * b_stride];
    c = reduce_to_centered(static_cast<int64_t>(c) + acc, m);
  }
  return c;
}

OX int oracle_reconstruct_signed(const int8_t* residues, uint32_t prefix, uint64_t bound, int64_t* out) {
  return reconstruct_signed(residues, prefix, bound, out);
}
OX int oracle_reconstruct_unsigned(const int8_t* residues, uint32_t prefix, uint64_t bound, uint64_t* out) {
  return reconstruct_unsigned(residues, prefix, bound, out);
}
OX void oracle_reconstruct_canonical(const int8_t* residues, uint32_t prefix, uint64_t* out4) {
  write_w(reconstruct_canonical(residues, prefix), out4);
}

// api_export.cpp:365-414 — stage every cell (OpenMP over cells), return the
// first failing status in cell order, and only then write dst.
OX int oracle_export_i64(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, uint64_t bound, int64_t* dst,
                         int64_t ld) {
  const int64_t cells = m * n;
  std::vector<int64_t> staged(static_cast<size_t>(cells), 0);
  std::vector<int> st(static_cast<size_t>(cells), ST_SUCCESS);
  auto body = [&](int64_t cell) {
    int8_t r[kMaxPrefix];
    gather_cell(planes, cells, cell, prefix, r);
    st[cell] = reconstruct_signed(r, prefix, bound, &staged[cell]);
  };
  if (parallel_should_use(sat_mul3(m, n, prefix))) {
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < cells; ++c) body(c);
  } else {
    for (int64_t c = 0; c < cells; ++c) body(c);
  }
  for (int s : st)
    if (s != ST_SUCCESS) return s;
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) dst[r * ld + c] = staged[r * n + c];
  return ST_SUCCESS;
}
// api_export.cpp:418-531
OX int oracle_export_u64(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, uint64_t bound, uint64_t* dst,
                         int64_t ld) {
  const int64_t cells = m * n;
  std::vector<uint64_t> staged(static_cast<size_t>(cells), 0);
  std::vector<int> st(static_cast<size_t>(cells), ST_SUCCESS);
  auto body = [&](int64_t cell) {
    int8_t r[kMaxPrefix];
    gather_cell(planes, cells, cell, prefix, r);
    st[cell] = reconstruct_unsigned(r, prefix, bound, &staged[cell]);
  };
  if (parallel_should_use(sat_mul3(m, n, prefix))) {
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < cells; ++c) body(c);
  } else {
    for (int64_t c = 0; c < cells; ++c) body(c);
  }
  for (int s : st)
    if (s != ST_SUCCESS) return s;
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) dst[r * ld + c] = staged[r * n + c];
  return ST_SUCCESS;
}
// api_export.cpp:617-803
OX int oracle_export_exact_wide_limbs(const int8_t* planes, int64_t m, int64_t n, uint32_t prefix, uint64_t* dst,
                                      int64_t ld, uint32_t limbs, int is_signed) {
  const int64_t cells = m * n;
  std::vector<uint64_t> staged(static_cast<size_t>(cells) * limbs, 0);
  std::vector<int> st(static_cast<size_t>(cells), ST_SUCCESS);
  auto body = [&](int64_t cell) {
    int8_t r[kMaxPrefix];
    gather_cell(planes, cells, cell, prefix, r);
    st[cell] = export_limbs(r, prefix, staged.data() + static_cast<size_t>(cell) * limbs, limbs, is_signed != 0);
  };
  if (parallel_should_use(sat_mul3(m, n, static_cast<uint64_t>(prefix) * limbs))) {
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < cells; ++c) body(c);
  } else {
    for (int64_t c = 0; c < cells; ++c) body(c);
  }
  for (int s : st)
    if (s != ST_SUCCESS) return s;
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c)
      std::memcpy(dst + (r * ld + c) * limbs, staged.data() + static_cast<size_t>(r * n + c) * limbs,
                  sizeof(uint64_t) * limbs);
  return ST_SUCCESS;
}

// Plan-time prefix choice for a descriptor given as scalars.
OX int oracle_plan_select_prefix(uint32_t semantics, uint32_t bound_kind, int64_t m, int64_t n, int64_t k,
                                 uint64_t bound, uint32_t max_prefix, uint32_t flags, uint32_t finite_modulus,
                                 uint64_t lhs_bound, uint64_t rhs_bound, uint32_t* selected, uint32_t* required,
                                 uint64_t* effective_bound) {
  plan_desc d{semantics, bound_kind, m, n, k, bound, max_prefix, 0, 0, finite_modulus, flags, lhs_bound, rhs_bound};
  uint32_t s = 0, r = 0;
  uint64_t eb = 0;
  const int st = plan_select_prefix(d, &s, &r, &eb);
  if (selected) *selected = s;
  if (required) *required = r;
  if (effective_bound) *effective_bound = eb;
  return st;
}

// api_oneshot.cpp:510-586 — validate, plan, pack A and B, one ring GEMM per
// plane, export. Bounded i64 (is_signed=1) or u64 (is_signed=0); global bounds.
OX int oracle_gemm_bounded_oneshot(int is_signed, uint32_t bound_kind, int64_t m, int64_t n, int64_t k,
                                   uint64_t bound, uint32_t max_prefix, uint32_t flags, uint64_t lhs_bound,
                                   uint64_t rhs_bound, const void* A, int64_t lda, const void* B, int64_t ldb,
                                   void* C, int64_t ldc, uint32_t* used_prefix) {
  plan_desc d{is_signed ? (uint32_t)SEM_I64 : (uint32_t)SEM_U64, bound_kind, m, n, k, bound, max_prefix, 0, 0, 0,
              flags, lhs_bound, rhs_bound};
  if (lda < k || ldb < n || ldc < n) return ST_INVALID;
  uint32_t prefix = 0, req = 0;
  uint64_t eb = 0;
  int st = plan_select_prefix(d, &prefix, &req, &eb);
  if (st != ST_SUCCESS) return st;
  if (used_prefix) *used_prefix = prefix;
  std::vector<int8_t> ra(static_cast<size_t>(prefix) * m * k), rb(static_cast<size_t>(prefix) * k * n),
      rc(static_cast<size_t>(prefix) * m * n);
  if (is_signed) {
    pack_native<int64_t>(static_cast<const int64_t*>(A), m, k, lda, prefix, ra.data());
    pack_native<int64_t>(static_cast<const int64_t*>(B), k, n, ldb, prefix, rb.data());
  } else {
    pack_native<uint64_t>(static_cast<const uint64_t*>(A), m, k, lda, prefix, ra.data());
    pack_native<uint64_t>(static_cast<const uint64_t*>(B), k, n, ldb, prefix, rb.data());
  }
  oracle_gemm_rns(ra.data(), rb.data(), rc.data(), m, n, k, prefix);
  return is_signed ? oracle_export_i64(rc.data(), m, n, prefix, eb, static_cast<int64_t*>(C), ldc)
                   : oracle_export_u64(rc.data(), m, n, prefix, eb, static_cast<uint64_t*>(C), ldc);
}

// api_oneshot.cpp:407-426 + cpu_reference.cpp:109-153,286-311 — finite u8 oneshot.
OX int oracle_gemm_finite_u8_oneshot(int field, uint16_t modulus, int64_t m, int64_t n, int64_t k, const uint8_t* A,
                                     int64_t lda, const uint8_t* B, int64_t ldb, uint8_t* C, int64_t ldc) {
  if (!valid_finite_modulus_for_semantics(field ? SEM_FIELD : SEM_RING, modulus)) return ST_INVALID;
  if (m <= 0 || n <= 0 || k <= 0 || lda < k || ldb < n || ldc < n) return ST_INVALID;
  std::vector<int8_t> ra(static_cast<size_t>(m) * k), rb(static_cast<size_t>(k) * n), rc(static_cast<size_t>(m) * n);
  oracle_pack_finite_u8(A, m, k, lda, modulus, ra.data());
  oracle_pack_finite_u8(B, k, n, ldb, modulus, rb.data());
  ring_gemm_modulus(ra.data(), rb.data(), rc.data(), m, n, k, k, n, n, modulus);
  oracle_export_finite_u8(rc.data(), m, n, modulus, C, ldc);
  return ST_SUCCESS;
}

// exact_range.hpp:51-154 for a pack(A), pack(B), gemm chain: the admission
// bound of the product and whether it fits the prefix (signed: 2*bound < P).
OX int oracle_exact_gemm_admission(int is_signed, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t m,
                                   int64_t n, int64_t k, uint32_t prefix, uint64_t* out_bound4,
                                   uint64_t* out_a_max4, uint64_t* out_b_max4) {
  std::vector<axis_range> ar, ac, br, bc;
  wide256 amax, bmax;
  if (is_signed) {
    native_exact_ranges<int64_t>(static_cast<const int64_t*>(A), m, k, lda, ar, ac, amax);
    native_exact_ranges<int64_t>(static_cast<const int64_t*>(B), k, n, ldb, br, bc, bmax);
  } else {
    native_exact_ranges<uint64_t>(static_cast<const uint64_t*>(A), m, k, lda, ar, ac, amax);
    native_exact_ranges<uint64_t>(static_cast<const uint64_t*>(B), k, n, ldb, br, bc, bmax);
  }
  const wide256 product = modulus_product(prefix);
  auto fits = [&](const wide256& b) {
    return !w_neg(b) && (is_signed ? w_cmp(w_mul(b, w_u64(2)), product) < 0 : w_cmp(b, product) < 0);
  };
  write_w(amax, out_a_max4);
  write_w(bmax, out_b_max4);
  // api_pack.cpp:61-64: each packed operand must itself fit the prefix.
  if (!fits(amax) || !fits(bmax)) return ST_RANGE;
  // exact_gemm_bound (exact_range.hpp:109-144) with both axis proofs present.
  wide256 bound = w_mul(w_mul(w_i64(k), amax), bmax);
  wide256 maximum = w_zero();
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) maximum = w_max(maximum, axis_product_bound(ar[r], bc[c], k));
  tighten(bound, maximum);
  write_w(bound, out_bound4);
  return fits(bound) ? ST_SUCCESS : ST_RANGE;
}

// The records an exact-wide GEMM keeps for its output (exact_range.hpp:108-143):
// per output row and column, the maximum and the sum of the cell bounds.
// row_stats[8*m], col_stats[8*n]: 4 limbs of the maximum, then 4 of the sum.
OX int oracle_exact_gemm_cell_stats(int is_signed, const void* A, int64_t lda, const void* B, int64_t ldb, int64_t m,
                                    int64_t n, int64_t k, uint64_t* row_stats, uint64_t* col_stats) {
  std::vector<axis_range> ar, ac, br, bc;
  wide256 amax, bmax;
  if (is_signed) {
    native_exact_ranges<int64_t>(static_cast<const int64_t*>(A), m, k, lda, ar, ac, amax);
    native_exact_ranges<int64_t>(static_cast<const int64_t*>(B), k, n, ldb, br, bc, bmax);
  } else {
    native_exact_ranges<uint64_t>(static_cast<const uint64_t*>(A), m, k, lda, ar, ac, amax);
    native_exact_ranges<uint64_t>(static_cast<const uint64_t*>(B), k, n, ldb, br, bc, bmax);
  }
  std::vector<wide256> rmax(static_cast<size_t>(m), w_zero()), rsum(static_cast<size_t>(m), w_zero());
  std::vector<wide256> cmax(static_cast<size_t>(n), w_zero()), csum(static_cast<size_t>(n), w_zero());
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) {
      const wide256 b = axis_product_bound(ar[r], bc[c], k);
      rmax[r] = w_max(rmax[r], b);
      rsum[r] = w_add(rsum[r], b);
      cmax[c] = w_max(cmax[c], b);
      csum[c] = w_add(csum[c], b);
    }
  for (int64_t r = 0; r < m; ++r) {
    write_w(rmax[r], row_stats + 8 * r);
    write_w(rsum[r], row_stats + 8 * r + 4);
  }
  for (int64_t c = 0; c < n; ++c) {
    write_w(cmax[c], col_stats + 8 * c);
    write_w(csum[c], col_stats + 8 * c + 4);
  }
  return ST_SUCCESS;
}

// ---- per-tile bound schedules ---------------------------------------------------
// configure_plan_schedule for per-tile bounds (api_plan_schedule.inc:178-261).
// out5[5*t..]: required, selected, group index, range bits, flags of tile t.
// summary[10]: min/max required, min/max selected, group count, max range
// bits, adaptive prefix, adaptive skip, schedule flags, collapsed (1 when the
// schedule is trivial and the reference clears it).
OX int oracle_plan_tile_schedule(uint32_t semantics, int64_t m, int64_t n, uint32_t tile_m, uint32_t tile_n,
                                 uint32_t max_prefix, uint32_t flags, const uint64_t* tile_bounds,
                                 const uint8_t* zero_a_rows, const uint8_t* zero_b_cols, uint32_t* out5,
                                 uint32_t* summary) {
  const uint32_t prefix = max_prefix ? max_prefix : default_prefix_for_semantics(semantics);
  const int64_t tile_rows = (m + tile_m - 1) / tile_m, tile_cols = (n + tile_n - 1) / tile_n;
  const bool fixed = (flags & FLAG_FORCE) != 0;
  const bool zero_tiles = (flags & 2u) != 0, zero_rc = (flags & 4u) != 0;
  uint32_t min_req = UINT32_MAX, max_req = 0, min_sel = UINT32_MAX, max_sel = 0, max_bits = 0, sched_flags = 0;
  std::vector<uint32_t> groups;
  const int64_t tiles = tile_rows * tile_cols;
  for (int64_t t = 0; t < tiles; ++t) {
    const uint64_t bound = tile_bounds[t];
    if (semantics == SEM_I64 && bound > (uint64_t{1} << 63)) return ST_INVALID;
    const wide256 range = semantics == SEM_I64 ? w_mul(w_u64(2), w_u64(bound)) : w_u64(bound);
    const uint32_t bits = w_bit_length(range);
    const uint32_t req = required_prefix_for_range(range);
    if (req == 0 || req > prefix) return ST_RANGE;
    const uint32_t sel = fixed ? prefix : req;
    min_req = std::min(min_req, req);
    max_req = std::max(max_req, req);
    min_sel = std::min(min_sel, sel);
    max_sel = std::max(max_sel, sel);
    max_bits = std::max(max_bits, bits);
    bool seen = false;
    for (uint32_t g : groups) seen = seen || g == sel;
    if (!seen) groups.push_back(sel);
    uint32_t f = (zero_tiles && bound == 0) ? 1u : 0u;
    if (zero_rc) {
      const int64_t r0 = (t / tile_cols) * tile_m, c0 = (t % tile_cols) * tile_n;
      const int64_t r1 = std::min<int64_t>(m, r0 + tile_m), c1 = std::min<int64_t>(n, c0 + tile_n);
      bool hit = false;
      for (int64_t r = r0; r < r1; ++r) hit = hit || zero_a_rows[r] != 0;
      for (int64_t c = c0; c < c1; ++c) hit = hit || zero_b_cols[c] != 0;
      if (hit) f |= 2u;
    }
    sched_flags |= f;
    out5[5 * t + 0] = req;
    out5[5 * t + 1] = sel;
    out5[5 * t + 3] = bits;
    out5[5 * t + 4] = f;
  }
  std::sort(groups.begin(), groups.end());
  for (int64_t t = 0; t < tiles; ++t)
    out5[5 * t + 2] = static_cast<uint32_t>(std::lower_bound(groups.begin(), groups.end(), out5[5 * t + 1]) -
                                            groups.begin());
  const uint32_t adaptive = groups.size() > 1 ? 1u : 0u, skip = max_sel < prefix ? 1u : 0u;
  const uint32_t collapsed = (groups.size() == 1 && min_req == prefix && max_req == prefix && min_sel == prefix &&
                              max_sel == prefix && adaptive == 0 && skip == 0 && sched_flags == 0) ? 1u : 0u;
  const uint32_t vals[10] = {min_req, max_req, min_sel, max_sel, static_cast<uint32_t>(groups.size()), max_bits,
                             adaptive, skip, sched_flags, collapsed};
  for (int i = 0; i < 10; ++i) summary[i] = vals[i];
  return ST_SUCCESS;
}

// cpu_gemm_rns under a tile schedule (cpu_reference.cpp:221-260): per tile,
// planes below its selected prefix; proven-zero tiles get zeros there.
// sel[t] = selected prefix | 0x80 for a proven-zero tile. C is updated in place.
OX void oracle_gemm_rns_scheduled(const int8_t* A, const int8_t* B, int8_t* C, int64_t m, int64_t n, int64_t k,
                                  uint32_t tile_m, uint32_t tile_n, const uint8_t* sel) {
  const int64_t tile_rows = (m + tile_m - 1) / tile_m, tile_cols = (n + tile_n - 1) / tile_n;
  for (int64_t t = 0; t < tile_rows * tile_cols; ++t) {
    const int64_t r0 = (t / tile_cols) * tile_m, c0 = (t % tile_cols) * tile_n;
    const int64_t rows = std::min<int64_t>(tile_m, m - r0), cols = std::min<int64_t>(tile_n, n - c0);
    for (uint32_t p = 0; p < (sel[t] & 0x7Fu); ++p) {
      int8_t* ct = C + p * m * n + r0 * n + c0;
      if (sel[t] & 0x80u) {
        for (int64_t r = 0; r < rows; ++r) std::memset(ct + r * n, 0, static_cast<size_t>(cols));
        continue;
      }
      ring_gemm_modulus(A + p * m * k + r0 * k, B + p * k * n + c0, ct, rows, cols, k, k, n, n, kLadder[p]);
    }
  }
}

// rns8_export_i64 / u64 under a per-tile plan (api_export.cpp:365-414): each
// cell with its tile's selected prefix and bound, staged, committed only when
// every cell passed (dst untouched otherwise).
OX int oracle_export_scheduled(const int8_t* planes, int64_t m, int64_t n, uint32_t tile_m, uint32_t tile_n,
                               const uint8_t* sel, const uint64_t* tile_bounds, int is_signed, void* dst, int64_t ld) {
  const int64_t tile_cols = (n + tile_n - 1) / tile_n;
  std::vector<uint64_t> staged(static_cast<size_t>(m * n), 0);
  for (int64_t row = 0; row < m; ++row)
    for (int64_t col = 0; col < n; ++col) {
      const int64_t t = (row / tile_m) * tile_cols + col / tile_n;
      if (sel[t] & 0x80u) continue;  // proven zero
      const uint32_t prefix = sel[t] & 0x7Fu;
      int8_t residues[32];
      for (uint32_t p = 0; p < prefix; ++p) residues[p] = planes[p * m * n + row * n + col];
      int st;
      if (is_signed) {
        int64_t v = 0;
        st = reconstruct_signed(residues, prefix, tile_bounds[t], &v);
        staged[row * n + col] = static_cast<uint64_t>(v);
      } else {
        uint64_t v = 0;
        st = reconstruct_unsigned(residues, prefix, tile_bounds[t], &v);
        staged[row * n + col] = v;
      }
      if (st != ST_SUCCESS) return st;
    }
  uint64_t* out = static_cast<uint64_t*>(dst);
  for (int64_t row = 0; row < m; ++row)
    for (int64_t col = 0; col < n; ++col) out[row * ld + col] = staged[row * n + col];
  return ST_SUCCESS;
}

// ---- WRAP_U64_MOD_2_64: src/backend_wrap64/wrap64_reference.cpp -------------
// cpu_gemm_wrap_u64 (:254-290): native uint64 multiply-accumulate, which wraps
// modulo 2^64, row by row (OpenMP over rows above the work threshold).
OX void oracle_wrap64_gemm(const uint64_t* A, int64_t lda, const uint64_t* B, int64_t ldb, uint64_t* C, int64_t ldc,
                           int64_t m, int64_t n, int64_t k) {
  auto row = [&](int64_t r) {
    std::vector<uint64_t> acc(static_cast<size_t>(n), 0);
    for (int64_t kk = 0; kk < k; ++kk) {
      const uint64_t a = A[r * lda + kk];
      const uint64_t* b = B + kk * ldb;
      for (int64_t c = 0; c < n; ++c) acc[c] += a * b[c];
    }
    for (int64_t c = 0; c < n; ++c) C[r * ldc + c] = acc[c];
  };
  if (parallel_should_use(sat_mul3(m, n, k))) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < m; ++r) row(r);
    return;
  }
  for (int64_t r = 0; r < m; ++r) row(r);
}

// wrap64_low_diagonal_byte_pair_gemm_cell (:166-190) with
// wrap64_low64_from_diagonals (:105-117): the 36 unsigned byte products of the
// low eight Comba diagonals, summed per diagonal (128-bit here; the reference
// uses cpp_int), then carried byte by byte into the low 64 bits.
OX void oracle_wrap64_gemm_diagonals(const uint64_t* A, int64_t lda, const uint64_t* B, int64_t ldb, uint64_t* C,
                                     int64_t ldc, int64_t m, int64_t n, int64_t k) {
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) {
      unsigned __int128 diag[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int64_t kk = 0; kk < k; ++kk) {
        const uint64_t a = A[r * lda + kk], b = B[kk * ldb + c];
        for (uint32_t i = 0; i < 8; ++i)
          for (uint32_t j = 0; i + j < 8; ++j)
            diag[i + j] += static_cast<uint32_t>((a >> (8 * i)) & 0xFFu) * static_cast<uint32_t>((b >> (8 * j)) & 0xFFu);
      }
      uint64_t out = 0;
      unsigned __int128 carry = 0;
      for (uint32_t d = 0; d < 8; ++d) {
        const unsigned __int128 column = diag[d] + carry;
        out |= static_cast<uint64_t>(column & 0xFFu) << (8 * d);
        carry = column >> 8;
      }
      C[r * ldc + c] = out;
    }
}

// Seeded inputs: std::mt19937_64 + std::uniform_int_distribution, as the
// reference's tests and benchmark generate them (rns8_bench_core_helpers.inc:
// 1150-1166, test_bounded_reference_sweeps.cpp:209-243).
OX int oracle_rng_new(uint64_t seed) {
  g_rngs.push_back(new std::mt19937_64(seed));
  return static_cast<int>(g_rngs.size() - 1);
}
OX void oracle_rng_free(int h) {
  if (h >= 0 && static_cast<size_t>(h) < g_rngs.size()) {
    delete g_rngs[h];
    g_rngs[h] = nullptr;
  }
}
OX uint64_t oracle_rng_next(int h) { return (*g_rngs[h])(); }
OX void oracle_rng_fill_i64(int h, int64_t lo, int64_t hi, int64_t* out, int64_t count) {
  std::uniform_int_distribution<int64_t> dist(lo, hi);
  for (int64_t i = 0; i < count; ++i) out[i] = dist(*g_rngs[h]);
}
OX void oracle_rng_fill_u64(int h, uint64_t lo, uint64_t hi, uint64_t* out, int64_t count) {
  std::uniform_int_distribution<uint64_t> dist(lo, hi);
  for (int64_t i = 0; i < count; ++i) out[i] = dist(*g_rngs[h]);
}

// Finite-u8 inputs: std::uniform_int_distribution<uint32_t>(0, hi) per byte, as
// the reference's finite lanes draw them (rns8_bench_finite_lanes.inc:28-31).
OX void oracle_rng_fill_u8(int h, uint32_t hi, uint8_t* out, int64_t count) {
  std::uniform_int_distribution<uint32_t> dist(0, hi);
  for (int64_t i = 0; i < count; ++i) out[i] = static_cast<uint8_t>(dist(*g_rngs[h]));
}
// Advances the engine past `count` draws of uniform_int_distribution<T>(lo, hi)
// (the values another rank's slab would take), storing nothing.
OX void oracle_rng_skip_i64(int h, int64_t lo, int64_t hi, int64_t count) {
  std::uniform_int_distribution<int64_t> dist(lo, hi);
  for (int64_t i = 0; i < count; ++i) (void)dist(*g_rngs[h]);
}
OX void oracle_rng_skip_u64(int h, uint64_t lo, uint64_t hi, int64_t count) {
  std::uniform_int_distribution<uint64_t> dist(lo, hi);
  for (int64_t i = 0; i < count; ++i) (void)dist(*g_rngs[h]);
}

// benchmarks/rns8_bench_event_phase_helpers.inc:544-552 + rns8_bench_support.cpp:96-99.
OX uint64_t oracle_checksum_u64(const uint64_t* v, int64_t rows, int64_t cols, int64_t ld) {
  uint64_t h = 1469598103934665603ull;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      h ^= v[r * ld + c];
      h *= 1099511628211ull;
    }
  return h;
}
// The same mix continued from a running hash `h` over `count` values (for
// outputs checksummed in chunks).
OX uint64_t oracle_checksum_u64_from(uint64_t h, const uint64_t* v, int64_t count) {
  for (int64_t i = 0; i < count; ++i) {
    h ^= v[i];
    h *= 1099511628211ull;
  }
  return h;
}
