// The fixed modulus ladder (reference src/core/internal.hpp:328-330), shared
// by host and device code. Plane p of an RNS matrix is reduced modulo
// kLadder[p]; a prefix P uses the first P entries. The entries are pairwise
// coprime and their product grows by about 7.7 bits per plane.
#pragma once

#include <cstdint>

namespace rns8ladder {
constexpr int kCount = 28;
constexpr uint16_t kLadder[kCount] = {256, 255, 253, 251, 247, 239, 233, 229, 227, 223, 217, 211, 199, 197,
                                      193, 191, 181, 179, 173, 167, 163, 157, 151, 149, 139, 137, 131, 127};
}  // namespace rns8ladder
