/* rns8 public ABI conventions.
 *
 * Every public enum is stored in 32 bits. C++ translation units give the
 * enums a fixed uint32_t underlying type so that any 32-bit value received
 * over the C ABI can be range-checked without undefined behaviour; C callers
 * rely on the platform's ordinary 32-bit enum ABI (never -fshort-enums).
 *
 * Interface source: include/rns8/abi.h of the RNS8 reference (same macro). */
#ifndef RNS8_ABI_H
#define RNS8_ABI_H

#include <stdint.h>

#ifdef __cplusplus
#define RNS8_ENUM_BASE : uint32_t
#else
#define RNS8_ENUM_BASE
#endif

#endif /* RNS8_ABI_H */
