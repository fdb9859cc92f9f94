// TEST INFRASTRUCTURE ONLY. Exposes the reference's own Boost-free epilogue
// arithmetic (src/backend_common/finite_u8_reducer.hpp:15-317 and
// src/backend_common/residue_dot.hpp:21-38) through a C ABI so the tests can
// pin the oracle's reduce/center/residue-dot against the reference itself.
// Built by oracle/Makefile against the headers where they lie in the reference
// tree; the output goes to oracle/_ref/ and is never part of the product.
#include <cstdint>

#include "backend_common/residue_dot.hpp"

#define RX extern "C" __attribute__((visibility("default")))

namespace f = rns8::detail::finite_u8;

RX int8_t ref_reduce_to_centered_i32(int32_t value, uint32_t modulus) {
  return f::reduce_to_centered_i32(value, modulus, f::modulus_reciprocal_u32(modulus));
}
RX int8_t ref_reduce_to_centered_accelerator_i32(int32_t value, uint32_t modulus) {
  return f::reduce_to_centered_accelerator_i32(value, modulus, f::modulus_reciprocal_u32(modulus));
}
RX int8_t ref_center_u8(uint8_t value, uint32_t modulus) { return f::center_u8(value, modulus); }
RX uint32_t ref_canonical_from_centered(int8_t residue, uint32_t modulus) {
  return f::canonical_from_centered(residue, modulus);
}
RX int8_t ref_centered_residue_dot(const int8_t* a, const int8_t* b, int64_t k, int64_t b_stride, uint32_t modulus) {
  return rns8::detail::centered_residue_dot(a, b, k, b_stride, modulus);
}
