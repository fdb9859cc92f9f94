// Contract arithmetic, descriptor validation and plan construction.
//
// Reference behaviour followed here:
//   src/core/moduli.cpp:10-448        ladder queries, prefix selection, validation
//   src/core/api_plan_public_api.inc:3-73, 80-117   plan creation and schedule info
//   src/core/api_plan_schedule.inc:109-279          global-bound prefix schedule
//   src/core/api_oneshot.cpp:473-504                required output range per semantic
//   src/core/status.cpp                             status text
// Per-tile bound schedules (RNS8_BOUND_PER_TILE_*) are validated like the
// reference but not executed by this backend: plan creation returns
// RNS8_UNSUPPORTED_BACKEND for them.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <limits>

#include "api_internal.hpp"

namespace rns8host {

bool valid_abi(uint64_t struct_size, uint32_t abi_version, size_t expected) {
  return abi_version == RNS8_ABI_VERSION && struct_size >= expected;
}

void set_text(char* dst, size_t cap, const std::string& s) {
  if (cap == 0) return;
  const size_t n = std::min(cap - 1, s.size());
  std::memcpy(dst, s.data(), n);
  dst[n] = '\0';
}

rns8_status cuda_status(cudaError_t e) { return e == cudaSuccess ? RNS8_SUCCESS : RNS8_BACKEND_FAILURE; }

int visible_device_count() {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return count;
}

i256 modulus_product(uint32_t prefix) {
  i256 p = i256::from_u64(1);
  for (uint32_t i = 0; i < prefix && i < static_cast<uint32_t>(rns8ladder::kCount); ++i)
    p = p * i256::from_u64(kLadder[i]);
  return p;
}

// Smallest prefix whose modulus product exceeds `range`; 0 if none <= 20.
uint32_t required_prefix_for_range(const i256& range) {
  i256 product = i256::from_u64(1);
  for (uint32_t prefix = 1; prefix <= RNS8_MAX_SUPPORTED_PREFIX; ++prefix) {
    product = product * i256::from_u64(kLadder[prefix - 1]);
    if (product > range) return prefix;
  }
  return 0;
}

uint32_t default_prefix_for_semantics(rns8_semantics s) {
  switch (s) {
    case RNS8_BOUNDED_I64:
    case RNS8_BOUNDED_U64:
      return RNS8_DEFAULT_BOUNDED_PREFIX;
    case RNS8_EXACT_WIDE_SIGNED:
    case RNS8_EXACT_WIDE_UNSIGNED:
      return RNS8_MAX_SUPPORTED_PREFIX;
    default:
      return 0;
  }
}

bool known_semantics(uint32_t s) { return s >= RNS8_BOUNDED_I64 && s <= RNS8_FINITE_FIELD_U8; }
bool known_bound_kind(uint32_t b) { return b <= RNS8_BOUND_INPUT_RANGE_AND_K; }
bool known_layout(uint32_t l) { return l == RNS8_LAYOUT_ROW_MAJOR || l == RNS8_LAYOUT_COLUMN_MAJOR; }
bool valid_tile_size(uint32_t v) { return v == 0 || (v >= 64 && v <= 512 && (v & (v - 1u)) == 0); }

bool valid_finite_modulus_for_semantics(rns8_semantics s, uint32_t m) {
  if (s == RNS8_FINITE_RING_U8) return m >= 2 && m <= 256;
  if (s == RNS8_FINITE_FIELD_U8) {
    if (m < 2 || m > 251) return false;
    for (uint32_t d = 2; d * d <= m; ++d)
      if (m % d == 0) return false;
    return true;
  }
  return false;
}

bool uses_rns_storage(rns8_semantics s) {
  return s == RNS8_BOUNDED_I64 || s == RNS8_BOUNDED_U64 || s == RNS8_EXACT_WIDE_SIGNED || s == RNS8_EXACT_WIDE_UNSIGNED;
}
bool uses_finite_storage(rns8_semantics s) { return s == RNS8_FINITE_RING_U8 || s == RNS8_FINITE_FIELD_U8; }
bool exact_wide(rns8_semantics s) { return s == RNS8_EXACT_WIDE_SIGNED || s == RNS8_EXACT_WIDE_UNSIGNED; }

bool valid_matrix_access(int64_t rows, int64_t cols, int64_t ld) {
  if (rows <= 0 || cols <= 0 || ld < cols) return false;
  return rows <= std::numeric_limits<int64_t>::max() / ld;
}

// k * lhs * rhs must fit the semantic's output range (moduli.cpp:208-232).
bool input_range_output_bound(const rns8_gemm_desc& d, uint64_t& out) {
  out = 0;
  if (d.bound_kind != RNS8_BOUND_INPUT_RANGE_AND_K ||
      (d.semantics != RNS8_BOUNDED_I64 && d.semantics != RNS8_BOUNDED_U64) || d.k <= 0)
    return false;
  constexpr uint64_t kSignedMax = 1ull << 63;
  if (d.semantics == RNS8_BOUNDED_I64 && (d.lhs_bound > kSignedMax || d.rhs_bound > kSignedMax)) return false;
  const i256 product = i256::from_i64(d.k) * i256::from_u64(d.lhs_bound) * i256::from_u64(d.rhs_bound);
  const i256 max_output = d.semantics == RNS8_BOUNDED_I64 ? i256::from_u64(kSignedMax) : i256::from_u64(~0ull);
  if (product.neg() || product > max_output) return false;
  out = product.w[0];
  return true;
}

// moduli.cpp:234-293
rns8_status validate_bound_contract(rns8_semantics s, rns8_bound_kind bk, uint64_t bound, uint32_t prefix) {
  if (!known_semantics(s) || !known_bound_kind(bk)) return RNS8_INVALID_ARGUMENT;
  if (prefix == 0 || prefix > RNS8_MAX_SUPPORTED_PREFIX) return RNS8_INVALID_ARGUMENT;
  const i256 product = modulus_product(prefix);
  switch (s) {
    case RNS8_BOUNDED_I64:
      if (bk == RNS8_BOUND_INPUT_RANGE_AND_K) return RNS8_UNSUPPORTED_BACKEND;
      if (bk == RNS8_BOUND_PER_TILE_MAX_ABS) return bound == 0 ? RNS8_SUCCESS : RNS8_INVALID_ARGUMENT;
      if (bk == RNS8_BOUND_NONE || bk == RNS8_BOUND_GLOBAL_MAX_UNSIGNED || bk == RNS8_BOUND_PER_TILE_MAX_UNSIGNED)
        return RNS8_INVALID_ARGUMENT;
      if (bk != RNS8_BOUND_GLOBAL_MAX_ABS) return RNS8_UNSUPPORTED_BACKEND;
      if (bound > (1ull << 63)) return RNS8_INVALID_ARGUMENT;
      return product > i256::from_u64(2) * i256::from_u64(bound) ? RNS8_SUCCESS : RNS8_RANGE_ERROR;
    case RNS8_BOUNDED_U64:
      if (bk == RNS8_BOUND_INPUT_RANGE_AND_K) return RNS8_UNSUPPORTED_BACKEND;
      if (bk == RNS8_BOUND_PER_TILE_MAX_UNSIGNED) return bound == 0 ? RNS8_SUCCESS : RNS8_INVALID_ARGUMENT;
      if (bk == RNS8_BOUND_NONE || bk == RNS8_BOUND_GLOBAL_MAX_ABS || bk == RNS8_BOUND_PER_TILE_MAX_ABS)
        return RNS8_INVALID_ARGUMENT;
      if (bk != RNS8_BOUND_GLOBAL_MAX_UNSIGNED) return RNS8_UNSUPPORTED_BACKEND;
      return product > i256::from_u64(bound) ? RNS8_SUCCESS : RNS8_RANGE_ERROR;
    default:
      return RNS8_UNSUPPORTED_BACKEND;
  }
}

static bool valid_zero_mask(const uint8_t* mask, uint64_t count, int64_t expected) {
  if (!mask || expected < 0 || count != static_cast<uint64_t>(expected)) return false;
  for (uint64_t i = 0; i < count; ++i)
    if (mask[i] > 1u) return false;
  return true;
}

// moduli.cpp:295-387
rns8_status validate_gemm_desc(const rns8_gemm_desc& d, uint32_t prefix) {
  if (!valid_abi(d.struct_size, d.abi_version, sizeof(d))) return RNS8_INVALID_ARGUMENT;
  if (d.m <= 0 || d.n <= 0 || d.k <= 0) return RNS8_INVALID_ARGUMENT;
  constexpr uint32_t kAllowed =
      RNS8_PLAN_FORCE_FIXED_PREFIX | RNS8_PLAN_ALLOW_PROVEN_ZERO_TILE_SKIPS | RNS8_PLAN_ALLOW_PROVEN_ZERO_ROW_COL_SKIPS;
  if ((d.flags & ~kAllowed) != 0) return RNS8_INVALID_ARGUMENT;
  const bool fixed = (d.flags & RNS8_PLAN_FORCE_FIXED_PREFIX) != 0;
  const bool zero_tiles = (d.flags & RNS8_PLAN_ALLOW_PROVEN_ZERO_TILE_SKIPS) != 0;
  const bool zero_rc = (d.flags & RNS8_PLAN_ALLOW_PROVEN_ZERO_ROW_COL_SKIPS) != 0;
  if (!valid_tile_size(d.tile_m) || !valid_tile_size(d.tile_n)) return RNS8_INVALID_ARGUMENT;
  const bool per_tile =
      d.bound_kind == RNS8_BOUND_PER_TILE_MAX_ABS || d.bound_kind == RNS8_BOUND_PER_TILE_MAX_UNSIGNED;
  if (!per_tile && (d.tile_bounds || d.tile_bounds_count != 0)) return RNS8_INVALID_ARGUMENT;
  if (!zero_rc && (d.zero_a_rows || d.zero_a_rows_count != 0 || d.zero_b_cols || d.zero_b_cols_count != 0))
    return RNS8_INVALID_ARGUMENT;
  if (zero_tiles && !per_tile) return RNS8_INVALID_ARGUMENT;
  if (zero_rc && (!per_tile || !valid_zero_mask(d.zero_a_rows, d.zero_a_rows_count, d.m) ||
                  !valid_zero_mask(d.zero_b_cols, d.zero_b_cols_count, d.n)))
    return RNS8_INVALID_ARGUMENT;
  if (!known_semantics(d.semantics) || !known_bound_kind(d.bound_kind)) return RNS8_INVALID_ARGUMENT;
  if (!uses_finite_storage(d.semantics) && d.finite_modulus != 0) return RNS8_INVALID_ARGUMENT;
  if (d.bound_kind != RNS8_BOUND_INPUT_RANGE_AND_K && (d.lhs_bound != 0 || d.rhs_bound != 0))
    return RNS8_INVALID_ARGUMENT;
  if (exact_wide(d.semantics)) {
    if (d.bound_kind != RNS8_BOUND_NONE || d.bound != 0) return RNS8_INVALID_ARGUMENT;
    if (prefix == 0 || prefix > RNS8_MAX_SUPPORTED_PREFIX) return RNS8_INVALID_ARGUMENT;
    const i256 required =
        i256::from_i64(d.k) * shl(i256::from_u64(1), d.semantics == RNS8_EXACT_WIDE_SIGNED ? 127u : 128u);
    return modulus_product(prefix) > required ? RNS8_SUCCESS : RNS8_RANGE_ERROR;
  }
  if (d.semantics == RNS8_WRAP_U64_MOD_2_64) {
    if (d.bound_kind != RNS8_BOUND_NONE || d.bound != 0 || prefix != 0 || fixed) return RNS8_INVALID_ARGUMENT;
    return RNS8_SUCCESS;
  }
  if (uses_finite_storage(d.semantics)) {
    if (d.bound_kind != RNS8_BOUND_NONE || d.bound != 0 || d.max_prefix != 0 || prefix != 0 || fixed ||
        !valid_finite_modulus_for_semantics(d.semantics, d.finite_modulus))
      return RNS8_INVALID_ARGUMENT;
    return RNS8_SUCCESS;
  }
  if (d.bound_kind == RNS8_BOUND_INPUT_RANGE_AND_K) {
    if (d.bound != 0 || d.tile_bounds || d.tile_bounds_count != 0) return RNS8_INVALID_ARGUMENT;
    uint64_t ob = 0;
    if (!input_range_output_bound(d, ob)) return RNS8_RANGE_ERROR;
    const i256 required =
        d.semantics == RNS8_BOUNDED_I64 ? i256::from_u64(2) * i256::from_u64(ob) : i256::from_u64(ob);
    return modulus_product(prefix) > required ? RNS8_SUCCESS : RNS8_RANGE_ERROR;
  }
  return validate_bound_contract(d.semantics, d.bound_kind, d.bound, prefix);
}

// moduli.cpp:389-448
rns8_status validate_matrix_desc(const rns8_matrix_desc& d, uint32_t prefix) {
  if (!valid_abi(d.struct_size, d.abi_version, sizeof(d))) return RNS8_INVALID_ARGUMENT;
  if (d.rows <= 0 || d.cols <= 0) return RNS8_INVALID_ARGUMENT;
  if (d.flags != 0) return RNS8_INVALID_ARGUMENT;
  if (!known_semantics(d.semantics) || !known_bound_kind(d.bound_kind) || !known_layout(d.logical_layout))
    return RNS8_INVALID_ARGUMENT;
  if (d.logical_ld != 0 && d.logical_ld < d.cols) return RNS8_INVALID_ARGUMENT;
  if (!valid_tile_size(d.tile_m) || !valid_tile_size(d.tile_n)) return RNS8_INVALID_ARGUMENT;
  const bool column_major = d.logical_layout == RNS8_LAYOUT_COLUMN_MAJOR;
  switch (d.semantics) {
    case RNS8_BOUNDED_I64:
      if (prefix == 0 || prefix > RNS8_MAX_SUPPORTED_PREFIX) return RNS8_INVALID_ARGUMENT;
      if (d.bound_kind != RNS8_BOUND_GLOBAL_MAX_ABS && d.bound_kind != RNS8_BOUND_PER_TILE_MAX_ABS)
        return RNS8_INVALID_ARGUMENT;
      return column_major ? RNS8_UNSUPPORTED_BACKEND : RNS8_SUCCESS;
    case RNS8_BOUNDED_U64:
      if (prefix == 0 || prefix > RNS8_MAX_SUPPORTED_PREFIX) return RNS8_INVALID_ARGUMENT;
      if (d.bound_kind != RNS8_BOUND_GLOBAL_MAX_UNSIGNED && d.bound_kind != RNS8_BOUND_PER_TILE_MAX_UNSIGNED)
        return RNS8_INVALID_ARGUMENT;
      return column_major ? RNS8_UNSUPPORTED_BACKEND : RNS8_SUCCESS;
    case RNS8_EXACT_WIDE_SIGNED:
    case RNS8_EXACT_WIDE_UNSIGNED:
      if (prefix == 0 || prefix > RNS8_MAX_SUPPORTED_PREFIX) return RNS8_INVALID_ARGUMENT;
      if (d.bound_kind != RNS8_BOUND_NONE) return RNS8_INVALID_ARGUMENT;
      return column_major ? RNS8_UNSUPPORTED_BACKEND : RNS8_SUCCESS;
    case RNS8_WRAP_U64_MOD_2_64:
      if (d.bound_kind != RNS8_BOUND_NONE || prefix != 0) return RNS8_INVALID_ARGUMENT;
      return column_major ? RNS8_UNSUPPORTED_BACKEND : RNS8_SUCCESS;
    case RNS8_FINITE_RING_U8:
    case RNS8_FINITE_FIELD_U8:
      if (prefix != 0 || d.max_prefix != 0 || d.bound_kind != RNS8_BOUND_NONE) return RNS8_INVALID_ARGUMENT;
      return column_major ? RNS8_UNSUPPORTED_BACKEND : RNS8_SUCCESS;
    default:
      return RNS8_INVALID_ARGUMENT;
  }
}

rns8_bound_kind storage_bound_kind(const rns8_plan& plan) {
  if (plan.desc.bound_kind != RNS8_BOUND_INPUT_RANGE_AND_K) return plan.desc.bound_kind;
  return plan.desc.semantics == RNS8_BOUNDED_I64 ? RNS8_BOUND_GLOBAL_MAX_ABS : RNS8_BOUND_GLOBAL_MAX_UNSIGNED;
}

bool backend_request_ok(rns8_backend_kind requested) {
  return requested == RNS8_BACKEND_AUTO || requested == RNS8_BACKEND_CUDA_SM100;
}

// Output range the prefix must exceed (api_oneshot.cpp:473-504).
static i256 schedule_required_range(const rns8_gemm_desc& d) {
  switch (d.semantics) {
    case RNS8_BOUNDED_I64:
    case RNS8_BOUNDED_U64: {
      uint64_t b = d.bound;
      if (d.bound_kind == RNS8_BOUND_INPUT_RANGE_AND_K && !input_range_output_bound(d, b)) return i256{};
      return d.semantics == RNS8_BOUNDED_I64 ? i256::from_u64(2) * i256::from_u64(b) : i256::from_u64(b);
    }
    case RNS8_EXACT_WIDE_SIGNED:
      return i256::from_i64(d.k) * shl(i256::from_u64(1), 127);
    case RNS8_EXACT_WIDE_UNSIGNED:
      return i256::from_i64(d.k) * shl(i256::from_u64(1), 128);
    default:
      return i256{};
  }
}

uint64_t plan_fingerprint(const rns8_plan& p) {
  uint64_t h = 1469598103934665603ull;
  auto mix = [&](uint64_t v) {
    h ^= v;
    h *= 1099511628211ull;
  };
  mix(p.desc.semantics);
  mix(p.desc.bound_kind);
  mix(static_cast<uint64_t>(p.desc.m));
  mix(static_cast<uint64_t>(p.desc.n));
  mix(static_cast<uint64_t>(p.desc.k));
  mix(p.desc.bound);
  mix(p.prefix);
  mix(p.desc.finite_modulus);
  mix(p.desc.lhs_bound);
  mix(p.desc.rhs_bound);
  mix(p.desc.flags);
  mix(p.desc.tile_m);
  mix(p.desc.tile_n);
  mix(static_cast<uint64_t>(p.device_id));
  // The schedule a workspace was sized for (plan_workspace_fingerprint,
  // api_plan_workspace_fingerprint.inc:29-90): same-shape plans with other
  // tile bounds, zero masks or selected prefixes do not share workspaces.
  for (uint64_t v : {p.tile_rows, p.tile_cols, p.tile_count}) mix(v);
  for (uint32_t v : {p.min_required, p.max_required, p.min_selected, p.max_selected, p.group_count,
                     p.range_bit_length, p.adaptive_prefix, p.adaptive_skip, p.schedule_flags})
    mix(v);
  mix(p.zero_a_row_count);
  mix(p.zero_b_col_count);
  mix(p.zero_row_col_product_count);
  mix(p.tile_bounds.size());
  for (uint64_t b : p.tile_bounds) mix(b);
  mix(p.zero_a_rows.size());
  for (uint8_t z : p.zero_a_rows) mix(z);
  mix(p.zero_b_cols.size());
  for (uint8_t z : p.zero_b_cols) mix(z);
  mix(p.tile_schedule.size());
  for (const rns8_plan_tile_schedule_entry& e : p.tile_schedule) {
    mix(e.required_prefix);
    mix(e.selected_prefix);
    mix(e.group_index);
    mix(e.range_bit_length);
    mix(e.flags);
  }
  return h;
}

static bool mask_range_has_set(const std::vector<uint8_t>& mask, int64_t begin, int64_t end) {
  for (int64_t i = begin; i < end; ++i)
    if (mask[static_cast<size_t>(i)]) return true;
  return false;
}

static rns8_plan_tile_schedule_entry make_tile_entry(const rns8_plan& plan, uint64_t index, uint32_t required,
                                                     uint32_t selected, uint32_t group, uint32_t range_bits,
                                                     uint32_t flags) {
  rns8_plan_tile_schedule_entry e{};
  e.struct_size = sizeof(e);
  e.abi_version = RNS8_ABI_VERSION;
  e.flags = flags;
  e.tile_row = index / plan.tile_cols;
  e.tile_col = index % plan.tile_cols;
  e.row_offset = static_cast<int64_t>(e.tile_row * plan.desc.tile_m);
  e.col_offset = static_cast<int64_t>(e.tile_col * plan.desc.tile_n);
  e.row_extent = std::min<int64_t>(plan.desc.tile_m, plan.desc.m - e.row_offset);
  e.col_extent = std::min<int64_t>(plan.desc.tile_n, plan.desc.n - e.col_offset);
  e.required_prefix = required;
  e.selected_prefix = selected;
  e.group_index = group;
  e.range_bit_length = range_bits;
  return e;
}

// configure_plan_schedule for per-tile bounds (api_plan_schedule.inc:109-261):
// each tile gets the smallest prefix its bound needs (or the plan prefix when
// forced), proven-zero tiles and zero row/column products are flagged, and a
// schedule where every tile runs the plan prefix unflagged collapses to none.
rns8_status build_tile_schedule(const rns8_gemm_desc& desc, rns8_plan& plan) {
  if (!desc.tile_bounds || desc.tile_bounds_count != plan.tile_count) return RNS8_INVALID_ARGUMENT;
  plan.tile_bounds.assign(desc.tile_bounds, desc.tile_bounds + desc.tile_bounds_count);
  plan.desc.tile_bounds_count = plan.tile_bounds.size();
  if ((desc.flags & RNS8_PLAN_ALLOW_PROVEN_ZERO_ROW_COL_SKIPS) != 0) {
    plan.zero_a_rows.assign(desc.zero_a_rows, desc.zero_a_rows + desc.zero_a_rows_count);
    plan.zero_b_cols.assign(desc.zero_b_cols, desc.zero_b_cols + desc.zero_b_cols_count);
    for (uint8_t v : plan.zero_a_rows) plan.zero_a_row_count += v;
    for (uint8_t v : plan.zero_b_cols) plan.zero_b_col_count += v;
    const uint64_t nonzero_rows = static_cast<uint64_t>(plan.desc.m) - plan.zero_a_row_count;
    plan.zero_row_col_product_count =
        plan.zero_a_row_count * static_cast<uint64_t>(plan.desc.n) + nonzero_rows * plan.zero_b_col_count;
  }
  plan.desc.zero_a_rows_count = plan.zero_a_rows.size();
  plan.desc.zero_b_cols_count = plan.zero_b_cols.size();
  const bool fixed = (plan.desc.flags & RNS8_PLAN_FORCE_FIXED_PREFIX) != 0;
  const bool zero_tiles = (plan.desc.flags & RNS8_PLAN_ALLOW_PROVEN_ZERO_TILE_SKIPS) != 0;
  const bool zero_rc = !plan.zero_a_rows.empty();
  uint32_t min_req = UINT32_MAX, max_req = 0, min_sel = UINT32_MAX, max_sel = 0, max_bits = 0;
  std::vector<uint32_t> groups;
  plan.tile_schedule.reserve(plan.tile_bounds.size());
  for (uint64_t index = 0; index < plan.tile_count; ++index) {
    const uint64_t bound = plan.tile_bounds[index];
    if (plan.desc.semantics == RNS8_BOUNDED_I64 && bound > (uint64_t{1} << 63)) return RNS8_INVALID_ARGUMENT;
    const i256 range = plan.desc.semantics == RNS8_BOUNDED_I64 ? i256::from_u64(2) * i256::from_u64(bound)
                                                                : i256::from_u64(bound);
    const uint32_t bits = bit_length(range);
    const uint32_t req = required_prefix_for_range(range);
    if (req == 0 || req > plan.prefix) return RNS8_RANGE_ERROR;
    const uint32_t sel = fixed ? plan.prefix : req;
    min_req = std::min(min_req, req);
    max_req = std::max(max_req, req);
    min_sel = std::min(min_sel, sel);
    max_sel = std::max(max_sel, sel);
    max_bits = std::max(max_bits, bits);
    if (std::find(groups.begin(), groups.end(), sel) == groups.end()) groups.push_back(sel);
    uint32_t flags = zero_tiles && bound == 0 ? RNS8_TILE_SCHEDULE_ZERO_OUTPUT : 0u;
    if (zero_rc) {
      const rns8_plan_tile_schedule_entry e = make_tile_entry(plan, index, 0, 0, 0, 0, 0);
      if (mask_range_has_set(plan.zero_a_rows, e.row_offset, e.row_offset + e.row_extent) ||
          mask_range_has_set(plan.zero_b_cols, e.col_offset, e.col_offset + e.col_extent))
        flags |= RNS8_TILE_SCHEDULE_ZERO_ROW_COL_PRODUCT;
    }
    plan.schedule_flags |= flags;
    plan.tile_schedule.push_back(make_tile_entry(plan, index, req, sel, 0, bits, flags));
  }
  std::sort(groups.begin(), groups.end());
  for (auto& e : plan.tile_schedule)
    e.group_index = static_cast<uint32_t>(std::lower_bound(groups.begin(), groups.end(), e.selected_prefix) -
                                          groups.begin());
  plan.min_required = min_req == UINT32_MAX ? 0 : min_req;
  plan.max_required = max_req;
  plan.min_selected = min_sel == UINT32_MAX ? 0 : min_sel;
  plan.max_selected = max_sel;
  plan.group_count = static_cast<uint32_t>(groups.size());
  plan.range_bit_length = max_bits;
  plan.adaptive_prefix = groups.size() > 1 ? 1u : 0u;
  plan.adaptive_skip = max_sel < plan.prefix ? 1u : 0u;
  if (plan.group_count == 1 && plan.min_required == plan.prefix && plan.max_required == plan.prefix &&
      plan.min_selected == plan.prefix && plan.max_selected == plan.prefix && plan.adaptive_prefix == 0 &&
      plan.adaptive_skip == 0 && plan.schedule_flags == 0)
    plan.tile_schedule.clear();
  plan.modulus_product = modulus_product(plan.prefix);
  plan.fingerprint = plan_fingerprint(plan);
  return RNS8_SUCCESS;
}

// rns8_get_plan_tile_schedule (api_plan_public_api.inc:119-167).
rns8_status plan_tile_schedule(const rns8_plan& plan, rns8_plan_tile_schedule_entry* entries, uint64_t capacity,
                               uint64_t* written) {
  *written = plan.tile_count;
  if (!entries || capacity == 0) return RNS8_SUCCESS;
  if (capacity < plan.tile_count) return RNS8_WORKSPACE_TOO_SMALL;
  if (!plan.tile_schedule.empty()) {
    std::copy(plan.tile_schedule.begin(), plan.tile_schedule.end(), entries);
    return RNS8_SUCCESS;
  }
  const bool per_tile = plan.desc.bound_kind == RNS8_BOUND_PER_TILE_MAX_ABS ||
                        plan.desc.bound_kind == RNS8_BOUND_PER_TILE_MAX_UNSIGNED;
  for (uint64_t index = 0; index < plan.tile_count; ++index) {
    if (per_tile && plan.tile_bounds.size() == plan.tile_count) {
      const uint64_t bound = plan.tile_bounds[index];
      const i256 range = plan.desc.semantics == RNS8_BOUNDED_I64 ? i256::from_u64(2) * i256::from_u64(bound)
                                                                  : i256::from_u64(bound);
      entries[index] = make_tile_entry(plan, index, required_prefix_for_range(range), plan.min_selected, 0,
                                       bit_length(range), 0);
      continue;
    }
    entries[index] = make_tile_entry(plan, index, plan.min_required, plan.min_selected, 0, plan.range_bit_length, 0);
  }
  return RNS8_SUCCESS;
}

// rns8_create_plan minus the context checks (api_plan_public_api.inc:3-73)
// and configure_plan_schedule for global bounds (api_plan_schedule.inc:109-279).
rns8_status build_plan(const rns8_gemm_desc& desc, rns8_plan& plan) {
  if (!valid_abi(desc.struct_size, desc.abi_version, sizeof(desc))) return RNS8_INVALID_ARGUMENT;
  const uint32_t prefix = desc.max_prefix == 0 ? default_prefix_for_semantics(desc.semantics) : desc.max_prefix;
  const rns8_status v = validate_gemm_desc(desc, prefix);
  if (v != RNS8_SUCCESS) return v;
  if (!backend_request_ok(desc.requested_backend)) return RNS8_UNSUPPORTED_BACKEND;
  plan.desc = desc;
  plan.desc.struct_size = sizeof(rns8_gemm_desc);
  plan.desc.max_prefix = prefix;
  if (plan.desc.tile_m == 0) plan.desc.tile_m = 128;
  if (plan.desc.tile_n == 0) plan.desc.tile_n = 128;
  plan.desc.tile_bounds = nullptr;
  plan.desc.zero_a_rows = nullptr;
  plan.desc.zero_b_cols = nullptr;
  if (plan.desc.bound_kind == RNS8_BOUND_INPUT_RANGE_AND_K && !input_range_output_bound(plan.desc, plan.desc.bound))
    return RNS8_RANGE_ERROR;
  plan.requested_max_prefix = prefix;
  plan.prefix = prefix;
  plan.tile_rows = (static_cast<uint64_t>(plan.desc.m) + plan.desc.tile_m - 1) / plan.desc.tile_m;
  plan.tile_cols = (static_cast<uint64_t>(plan.desc.n) + plan.desc.tile_n - 1) / plan.desc.tile_n;
  // A schedule whose tile count overflows is a range error (api_plan_schedule.inc:113-118).
  if (plan.tile_cols != 0 && plan.tile_rows > UINT64_MAX / plan.tile_cols) return RNS8_RANGE_ERROR;
  plan.tile_count = plan.tile_rows * plan.tile_cols;
  const i256 required_range = schedule_required_range(plan.desc);
  plan.range_bit_length = bit_length(required_range);
  if (uses_finite_storage(plan.desc.semantics) || plan.desc.semantics == RNS8_WRAP_U64_MOD_2_64) {
    plan.prefix = 0;  // finite: one residue plane; wrap64: eight byte planes, no CRT prefix
    plan.fingerprint = plan_fingerprint(plan);
    return RNS8_SUCCESS;
  }
  if (plan.desc.bound_kind == RNS8_BOUND_PER_TILE_MAX_ABS || plan.desc.bound_kind == RNS8_BOUND_PER_TILE_MAX_UNSIGNED)
    return build_tile_schedule(desc, plan);
  const uint32_t req = required_prefix_for_range(required_range);
  if (req == 0 || req > prefix) return RNS8_RANGE_ERROR;
  const bool fixed = (plan.desc.flags & RNS8_PLAN_FORCE_FIXED_PREFIX) != 0;
  const uint32_t sel = fixed ? prefix : req;
  plan.prefix = sel;
  plan.modulus_product = modulus_product(sel);
  plan.min_required = plan.max_required = req;
  plan.min_selected = plan.max_selected = sel;
  plan.group_count = 1;
  plan.adaptive_prefix = 0;
  plan.adaptive_skip = sel < prefix ? 1u : 0u;
  plan.fingerprint = plan_fingerprint(plan);
  return RNS8_SUCCESS;
}

uint64_t next_matrix_id() {
  static std::atomic<uint64_t> next{1};
  return next.fetch_add(1, std::memory_order_relaxed);
}

// The schedule info's bound-contract name (api_plan_contract_names.inc:39-52):
// how the plan's output bound was obtained, not the bound kind's own name.
static const char* bound_contract_name(const rns8_plan& plan) {
  switch (plan.desc.bound_kind) {
    case RNS8_BOUND_INPUT_RANGE_AND_K: return "input_range_and_k_derived_output_bound";
    case RNS8_BOUND_PER_TILE_MAX_ABS:
    case RNS8_BOUND_PER_TILE_MAX_UNSIGNED: return "per_tile_output_bounds";
    case RNS8_BOUND_GLOBAL_MAX_ABS:
    case RNS8_BOUND_GLOBAL_MAX_UNSIGNED: return "global_output_bound";
    case RNS8_BOUND_NONE: break;
  }
  return "not_applicable";
}

}  // namespace rns8host

using namespace rns8host;

// ---- status and ladder queries ------------------------------------------------
extern "C" const char* rns8_status_string(rns8_status status) {
  switch (status) {
    case RNS8_SUCCESS: return "success";
    case RNS8_INVALID_ARGUMENT: return "invalid argument";
    case RNS8_UNSUPPORTED_OS: return "unsupported operating system";
    case RNS8_UNSUPPORTED_ARCH: return "unsupported architecture";
    case RNS8_UNSUPPORTED_BACKEND: return "unsupported backend";
    case RNS8_RANGE_ERROR: return "range error";
    case RNS8_ACCUMULATION_OVERFLOW_RISK: return "accumulation overflow risk";
    case RNS8_WORKSPACE_TOO_SMALL: return "workspace too small";
    case RNS8_BACKEND_FAILURE: return "backend failure";
    case RNS8_VERIFICATION_FAILED: return "verification failed";
    case RNS8_INTERNAL_ERROR: return "internal error";
  }
  return "unknown status";
}

extern "C" uint32_t rns8_default_modulus_count(void) { return RNS8_DEFAULT_MODULUS_COUNT; }
extern "C" uint16_t rns8_default_modulus(uint32_t index) {
  return index < RNS8_DEFAULT_MODULUS_COUNT ? kLadder[index] : 0;
}
extern "C" double rns8_prefix_range_bits(uint32_t prefix) {
  if (prefix == 0 || prefix > RNS8_DEFAULT_MODULUS_COUNT) return 0.0;
  long double bits = 0.0L;
  for (uint32_t i = 0; i < prefix; ++i) bits += std::log2(static_cast<long double>(kLadder[i]));
  return static_cast<double>(bits);
}
extern "C" rns8_status rns8_validate_default_moduli(void) {
  for (int i = 0; i < rns8ladder::kCount; ++i)
    for (int j = i + 1; j < rns8ladder::kCount; ++j) {
      uint32_t a = kLadder[i], b = kLadder[j];
      while (b) {
        const uint32_t t = a % b;
        a = b;
        b = t;
      }
      if (a != 1) return RNS8_INTERNAL_ERROR;
    }
  return RNS8_SUCCESS;
}

// ---- plans ----------------------------------------------------------------------
extern "C" rns8_status rns8_create_plan(rns8_context* ctx, const rns8_gemm_desc* desc, rns8_plan** out) {
  return guard([&]() -> rns8_status {
    if (!ctx || !desc || !out) return RNS8_INVALID_ARGUMENT;
    *out = nullptr;
    auto* plan = new (std::nothrow) rns8_plan();
    if (!plan) return RNS8_INTERNAL_ERROR;
    plan->device_id = ctx->device_id;
    const rns8_status s = build_plan(*desc, *plan);
    if (s != RNS8_SUCCESS) {
      delete plan;
      return s;
    }
    plan->fingerprint = plan_fingerprint(*plan);
    *out = plan;
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_destroy_plan(rns8_plan* plan) {
  delete plan;
  return RNS8_SUCCESS;
}

extern "C" rns8_status rns8_get_plan_schedule_info(const rns8_plan* plan, rns8_plan_schedule_info* out) {
  return guard([&]() -> rns8_status {
    if (!plan || !out || !valid_abi(out->struct_size, out->abi_version, sizeof(*out))) return RNS8_INVALID_ARGUMENT;
    const uint64_t ss = out->struct_size;
    const uint32_t av = out->abi_version;
    *out = {};
    out->struct_size = ss;
    out->abi_version = av;
    out->tile_m = plan->desc.tile_m;
    out->tile_n = plan->desc.tile_n;
    out->tile_rows = plan->tile_rows;
    out->tile_cols = plan->tile_cols;
    out->tile_count = plan->tile_count;
    out->min_required_prefix = plan->min_required;
    out->max_required_prefix = plan->max_required;
    out->min_selected_prefix = plan->min_selected;
    out->max_selected_prefix = plan->max_selected;
    out->prefix_group_count = plan->group_count;
    out->adaptive_prefix_active = plan->adaptive_prefix;
    out->adaptive_skip_active = plan->adaptive_skip;
    out->range_bit_length = plan->range_bit_length;
    out->flags = plan->schedule_flags;
    out->bound_kind = plan->desc.bound_kind;
    out->effective_bound = plan->desc.bound;
    out->lhs_bound = plan->desc.lhs_bound;
    out->rhs_bound = plan->desc.rhs_bound;
    out->zero_a_row_count = plan->zero_a_row_count;
    out->zero_b_col_count = plan->zero_b_col_count;
    out->zero_row_col_product_count = plan->zero_row_col_product_count;
    set_text(out->bound_contract, sizeof(out->bound_contract), bound_contract_name(*plan));
    return RNS8_SUCCESS;
  });
}

// Global-bound plans have no per-tile schedule (the reference clears it for
// a uniform schedule, api_plan_schedule.inc:254-259), so zero entries exist.
extern "C" rns8_status rns8_get_plan_tile_schedule(const rns8_plan* plan, rns8_plan_tile_schedule_entry* entries,
                                                   uint64_t capacity, uint64_t* written) {
  return guard([&]() -> rns8_status {
    if (!plan || !written) return RNS8_INVALID_ARGUMENT;
    return plan_tile_schedule(*plan, entries, capacity, written);
  });
}

extern "C" rns8_status rns8_cuda_plan_tile_schedule_probe(const rns8_gemm_desc* desc,
                                                          rns8_plan_tile_schedule_entry* entries, uint64_t capacity,
                                                          uint64_t* written, rns8_plan_schedule_info* info) {
  return guard([&]() -> rns8_status {
    if (!desc || !written) return RNS8_INVALID_ARGUMENT;
    rns8_plan plan;
    const rns8_status s = build_plan(*desc, plan);
    if (s != RNS8_SUCCESS) return s;
    if (info) {
      const rns8_status i = rns8_get_plan_schedule_info(&plan, info);
      if (i != RNS8_SUCCESS) return i;
    }
    return plan_tile_schedule(plan, entries, capacity, written);
  });
}

static std::string selected_kernel_name(const rns8_plan& plan) {
  rns8cuda::PlaneGemmTask task{reinterpret_cast<const int8_t*>(256), reinterpret_cast<const int8_t*>(256),
                               reinterpret_cast<int8_t*>(256)};
  rns8cuda::PlaneGemmProblem prob{};
  prob.m = plan.desc.m;
  prob.n = plan.desc.n;
  prob.k = plan.desc.k;
  prob.planes = plan.prefix == 0 ? 1 : plan.prefix;
  prob.task_count = 1;
  prob.tasks = &task;
  const bool tc = prob.k % 16 == 0 && prob.n % 16 == 0;
  if (plan.desc.semantics == RNS8_WRAP_U64_MOD_2_64)
    return tc ? "sm100a_tcgen05_u8_byte_gemm36_128x256x128_wrap64" : "sm100a_simt_wrap64_u64_16x16";
  return tc ? "sm100a_tcgen05_i8_plane_gemm_128x256x128_modm_epilogue" : "sm100a_simt_plane_gemm_64x64_modm";
}

extern "C" rns8_status rns8_get_plan_backend_info(const rns8_plan* plan, rns8_plan_backend_info* out) {
  return guard([&]() -> rns8_status {
    if (!plan || !out || !valid_abi(out->struct_size, out->abi_version, sizeof(*out))) return RNS8_INVALID_ARGUMENT;
    const uint64_t ss = out->struct_size;
    const uint32_t av = out->abi_version;
    *out = {};
    out->struct_size = ss;
    out->abi_version = av;
    out->backend = plan->backend;
    out->is_accelerator = 1;
    out->is_correctness_backend = 0;
    out->is_matrix_engine_backend = 1;
    out->compiled_kernel_available = 1;
    out->exact_differential_validated = 1;
    out->performance_validated = 0;
    set_text(out->selected_kernel, sizeof(out->selected_kernel), selected_kernel_name(*plan));
    set_text(out->accelerator_library, sizeof(out->accelerator_library), "rns8_b200");
    set_text(out->accelerator_version, sizeof(out->accelerator_version), "sm_100a");
    set_text(out->capability_status, sizeof(out->capability_status), "available");
    set_text(out->epilogue_mode, sizeof(out->epilogue_mode), "int32_tmem_to_centered_residue_mulhi");
    set_text(out->workspace_mode, sizeof(out->workspace_mode), "split_k_int32_partial_sums_when_needed");
    set_text(out->isa_evidence, sizeof(out->isa_evidence), "tcgen05.mma.kind::i8 + cp.async.bulk.tensor");
    out->accumulator_k_block_size = RNS8_SAFE_INT32_K_BLOCK;
    out->accumulator_k_block_cap = RNS8_SAFE_INT32_K_BLOCK;
    out->accumulator_modulus = uses_finite_storage(plan->desc.semantics) ? plan->desc.finite_modulus : kLadder[0];
    out->accumulator_max_lhs_abs = 128;
    out->accumulator_max_rhs_abs = 128;
    out->accumulator_max_product = 16384;
    out->accumulator_uses_int32_inner_product = 1;
    out->accumulator_safe_for_k_block = 1;
    // Contract vocabulary of the accumulator fields (api_plan_contract_names.inc:462-530).
    const bool finite_plan = uses_finite_storage(plan->desc.semantics);
    set_text(out->accumulator_input_domain, sizeof(out->accumulator_input_domain),
             finite_plan ? "centered_i8_finite_u8_residues" : "centered_i8_rns_residue_planes");
    set_text(out->accumulator_signedness, sizeof(out->accumulator_signedness), "signed_i8x_signed_i8");
    set_text(out->accumulator_type, sizeof(out->accumulator_type), "int32");
    set_text(out->accumulator_modulus_policy, sizeof(out->accumulator_modulus_policy),
             finite_plan ? "finite_u8_modulus" : "selected_rns_modulus_ladder");
    set_text(out->accumulator_safety_status, sizeof(out->accumulator_safety_status), "safe_int32_k_block_split");
    if (plan->desc.semantics == RNS8_WRAP_U64_MOD_2_64) {
      // 36 unsigned byte-pair products on the low 8 diagonals; a 16384-product
      // K block keeps diagonals 0..3 exact in 32 bits, diagonals 4..7 only
      // matter modulo 2^32.
      set_text(out->epilogue_mode, sizeof(out->epilogue_mode), "u32_diagonal_shift_add_mod_2_64");
      set_text(out->workspace_mode, sizeof(out->workspace_mode), "uint64_result_accumulator");
      set_text(out->isa_evidence, sizeof(out->isa_evidence), "tcgen05.mma.kind::i8 (u8 x u8) + cp.async.bulk.tensor");
      out->accumulator_k_block_size = 16384;
      out->accumulator_k_block_cap = 16384;
      out->accumulator_modulus = 0;
      out->accumulator_max_lhs_abs = 255;
      out->accumulator_max_rhs_abs = 255;
      out->accumulator_max_product = 65025;
      set_text(out->accumulator_input_domain, sizeof(out->accumulator_input_domain), "uint8_byte_limb_pairs");
      set_text(out->accumulator_signedness, sizeof(out->accumulator_signedness), "unsigned_byte_limb");
      set_text(out->accumulator_type, sizeof(out->accumulator_type), "uint32_low_diagonal_then_uint64_carry");
      set_text(out->accumulator_modulus_policy, sizeof(out->accumulator_modulus_policy),
               "mod_2_64_wraparound_byte_limb");
      set_text(out->accumulator_safety_status, sizeof(out->accumulator_safety_status),
               "safe_uint32_byte_limb_gemm36_k_block");
    }
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_get_plan_packing_info(const rns8_plan* plan, rns8_plan_packing_info* out) {
  return guard([&]() -> rns8_status {
    if (!plan || !out || !valid_abi(out->struct_size, out->abi_version, sizeof(*out))) return RNS8_INVALID_ARGUMENT;
    const uint64_t ss = out->struct_size;
    const uint32_t av = out->abi_version;
    *out = {};
    out->struct_size = ss;
    out->abi_version = av;
    out->backend = plan->backend;
    out->semantics = plan->desc.semantics;
    out->uses_resident_matrix_inputs = 1;
    out->uses_transient_pack_workspace = 0;
    out->uses_matrix_engine_pack_layout = 0;
    out->flags = RNS8_PLAN_PACKING_SOURCE_VERSIONED_INPUTS | RNS8_PLAN_PACKING_SAME_SOURCE_VERSION_PACK_ELISION;
    const bool finite = uses_finite_storage(plan->desc.semantics);
    // Inputs and output live in the plan's storage domain (api_plan_contract_names.inc:277-302).
    out->input_domain = finite ? RNS8_OUTPUT_DOMAIN_FINITE_U8 : RNS8_OUTPUT_DOMAIN_RNS_RESIDUE;
    out->output_domain = out->input_domain;
    out->output_device_current = 1;
    out->next_op_flags = RNS8_NEXT_OP_FINAL_EXPORT | (finite ? 0u : static_cast<uint32_t>(RNS8_NEXT_OP_RNS_GEMM));
    rns8cuda::PlaneGemmTask task{reinterpret_cast<const int8_t*>(256), reinterpret_cast<const int8_t*>(256),
                                 reinterpret_cast<int8_t*>(256)};
    rns8cuda::PlaneGemmProblem prob{};
    prob.m = plan->desc.m;
    prob.n = plan->desc.n;
    prob.k = plan->desc.k;
    prob.planes = finite ? 1 : plan->prefix;
    prob.task_count = 1;
    prob.tasks = &task;
    out->accumulator_workspace_bytes = rns8cuda::plane_gemm_scratch_bytes(prob, 148);
    out->total_transient_workspace_bytes = out->accumulator_workspace_bytes;
    if (plan->desc.semantics == RNS8_WRAP_U64_MOD_2_64) {
      out->input_domain = RNS8_OUTPUT_DOMAIN_WRAP64_BYTE_LIMB;
      out->output_domain = RNS8_OUTPUT_DOMAIN_WRAP64_BYTE_LIMB;
      out->next_op_flags = RNS8_NEXT_OP_FINAL_EXPORT;
      out->accumulator_workspace_bytes = static_cast<uint64_t>(plan->desc.m) * plan->desc.n * 8;
      out->total_transient_workspace_bytes = out->accumulator_workspace_bytes;
      set_text(out->input_domain_name, sizeof(out->input_domain_name), "wrap64_byte_limb_current");
      set_text(out->output_domain_name, sizeof(out->output_domain_name), "wrap64_byte_limb_current");
      set_text(out->next_op_hint, sizeof(out->next_op_hint),
               "produces wrap64 byte-limb-current output; export reconstructs low 64-bit words");
      set_text(out->a_layout_version, sizeof(out->a_layout_version), "wrap64_byte_limb_v1");
      set_text(out->b_layout_version, sizeof(out->b_layout_version), "wrap64_byte_limb_v1");
      set_text(out->output_layout_version, sizeof(out->output_layout_version), "wrap64_byte_limb_v1");
      set_text(out->prepack_cache_scope, sizeof(out->prepack_cache_scope), "device_resident_no_prepack_cache");
      set_text(out->detail, sizeof(out->detail), "eight unsigned byte planes in HBM; 36 byte-pair tensor-core products");
      return RNS8_SUCCESS;
    }
    set_text(out->input_domain_name, sizeof(out->input_domain_name),
             finite ? "finite_u8_current" : "rns_residue_current");
    set_text(out->output_domain_name, sizeof(out->output_domain_name),
             finite ? "finite_u8_current" : "rns_residue_current");
    // Hint, layout and cache-scope identifiers are the reference's contract
    // names (api_plan_contract_names.inc:343-357, api_plan_workspace_packing.inc:227-235,
    // api_plan_public_api.inc:526-531 for device-resident storage).
    set_text(out->next_op_hint, sizeof(out->next_op_hint),
             finite ? "produces finite-current centered residues; export converts to canonical uint8 output"
                    : "produces residue-current RNS output; next same-contract RNS GEMM can consume it without "
                      "logical export");
    const char* layout = finite ? "finite_u8_centered_residue_v1" : "rns_centered_residue_planes_v1";
    set_text(out->a_layout_version, sizeof(out->a_layout_version), layout);
    set_text(out->b_layout_version, sizeof(out->b_layout_version), layout);
    set_text(out->output_layout_version, sizeof(out->output_layout_version), layout);
    set_text(out->prepack_cache_scope, sizeof(out->prepack_cache_scope), "device_resident_no_prepack_cache");
    set_text(out->detail, sizeof(out->detail), "resident planes in HBM; B read N-major by the tensor-core kernel");
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_get_grouped_dispatch_contract_info(const rns8_plan* plan, uint32_t task_count,
                                                               rns8_grouped_dispatch_contract_info* out) {
  return guard([&]() -> rns8_status {
    if (!plan || !out || !valid_abi(out->struct_size, out->abi_version, sizeof(*out))) return RNS8_INVALID_ARGUMENT;
    const uint64_t ss = out->struct_size;
    const uint32_t av = out->abi_version;
    *out = {};
    out->struct_size = ss;
    out->abi_version = av;
    out->backend = plan->backend;
    out->semantics = plan->desc.semantics;
    out->task_count = task_count;
    out->descriptor_contract_supported = 1;
    out->public_execution_available = task_count > 1 ? 1u : 0u;
    out->same_shape_required = 1;
    out->same_semantics_required = 1;
    out->compact_row_major_required = 1;
    out->unique_matrix_handles_required = 1;
    out->unique_workspace_handles_required = 0;
    out->same_plan_fingerprint_required = 1;
    out->same_device_required = 1;
    out->device_resident_inputs_required = 1;
    out->produces_device_current_output = 1;
    out->final_export_required_for_host_output = 1;
    out->flags = RNS8_GROUPED_DISPATCH_CONTRACT_SAME_SHAPE_REQUIRED |
                 RNS8_GROUPED_DISPATCH_CONTRACT_COMPACT_ROW_MAJOR_REQUIRED |
                 RNS8_GROUPED_DISPATCH_CONTRACT_UNIQUE_TASK_HANDLES_REQUIRED |
                 RNS8_GROUPED_DISPATCH_CONTRACT_SAME_DEVICE_REQUIRED |
                 RNS8_GROUPED_DISPATCH_CONTRACT_DEVICE_CURRENT_OUTPUT_REQUIRED |
                 RNS8_GROUPED_DISPATCH_CONTRACT_PUBLIC_PACK_EXPLICIT |
                 RNS8_GROUPED_DISPATCH_CONTRACT_PUBLIC_EXPORT_EXPLICIT;
    set_text(out->descriptor_layout, sizeof(out->descriptor_layout), "tensor_map_per_task_in_kernel_params");
    set_text(out->bucket_policy, sizeof(out->bucket_policy), "single_same_shape_bucket_32_tasks_per_launch");
    set_text(out->output_domain, sizeof(out->output_domain),
             uses_finite_storage(plan->desc.semantics) ? "finite_u8" : "rns_residue");
    return RNS8_SUCCESS;
  });
}

extern "C" rns8_status rns8_cuda_plan_probe(const rns8_gemm_desc* desc, uint32_t* selected_prefix,
                                            uint32_t* required_prefix, uint64_t* effective_bound) {
  return guard([&]() -> rns8_status {
    if (!desc) return RNS8_INVALID_ARGUMENT;
    rns8_plan plan;
    const rns8_status s = build_plan(*desc, plan);
    if (s != RNS8_SUCCESS) return s;
    if (selected_prefix) *selected_prefix = plan.prefix;
    if (required_prefix) *required_prefix = plan.min_required;
    if (effective_bound) *effective_bound = plan.desc.bound;
    return RNS8_SUCCESS;
  });
}
