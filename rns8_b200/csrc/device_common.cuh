// Device-side building blocks shared by the pack, plane-GEMM and Garner
// kernels: the modulus ladder, exact small-modulus reductions, and thin
// wrappers over the sm_100a PTX used by the tensor-core GEMM (mbarrier, TMA,
// tcgen05). Every spin-wait here is bounded by a cycle budget; a wait that
// runs out reports failure to its caller instead of hanging the GPU.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.hpp"
#include "ladder.hpp"

namespace rns8cuda {

using rns8ladder::kLadder;
constexpr int kMaxPrefix = 20;
constexpr int64_t kSafeKBlock = 65536;  // RNS8_SAFE_INT32_K_BLOCK


// ---- exact small-modulus arithmetic (host and device) -----------------------
// floor(2^32 / m) for 2 <= m <= 256.
__host__ __device__ constexpr uint32_t floor_magic(uint32_t m) {
  return static_cast<uint32_t>((1ull << 32) / m);
}

// u mod m for any 32-bit u. With magic = floor(2^32/m) the quotient estimate
// q = floor(u * magic / 2^32) satisfies Q-1 <= q <= Q (Q the true quotient),
// so one conditional subtraction finishes the reduction.
__device__ __forceinline__ uint32_t umod_u32(uint32_t u, uint32_t m, uint32_t magic) {
  const uint32_t q = __umulhi(u, magic);
  uint32_t r = u - q * m;
  return r >= m ? r - m : r;
}

// Centered representative of a canonical residue r in [0, m):
// r >= ceil(m/2) maps to r - m (m = 256 gives [-128, 127]).
__device__ __forceinline__ int center_residue(uint32_t r, uint32_t m) {
  return r >= ((m + 1u) >> 1) ? static_cast<int>(r) - static_cast<int>(m) : static_cast<int>(r);
}

// Per-modulus constants for reducing a signed int32 accumulator.
struct ModConst {
  uint32_t m;
  uint32_t magic;      // floor(2^32 / m)
  uint32_t off;        // 2^31 mod m
};
__host__ __device__ constexpr ModConst make_mod_const(uint32_t m) {
  return ModConst{m, floor_magic(m), static_cast<uint32_t>((1ull << 31) % m)};
}

// Any int32 v -> centered residue of v mod m. v + 2^31 is a non-negative
// 32-bit value; its residue minus (2^31 mod m) is v's residue.
__device__ __forceinline__ int reduce_i32_centered(int32_t v, const ModConst& c) {
  const uint32_t u = static_cast<uint32_t>(v) ^ 0x80000000u;
  uint32_t r = umod_u32(u, c.m, c.magic);
  r = r >= c.off ? r - c.off : r + c.m - c.off;
  return center_residue(r, c.m);
}

// ---- host: kernel attributes --------------------------------------------------
// Raises `kernel`'s dynamic shared-memory limit on the current device, once
// per process and device (`done` holds one bit per device id below 64).
// cudaFuncSetAttribute can wait for running instances of the kernel, so it is
// kept off the per-launch path: a second launch of the same kernel queued
// behind the first would otherwise leave the GPU idle while the host waits.
template <typename Kernel>
inline cudaError_t raise_smem_limit_once(Kernel kernel, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// ---- PTX wrappers ------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the barrier phase with the given parity completes, for at most
// `budget` SM cycles. Returns false when the budget ran out.
constexpr long long kWaitBudgetCycles = 4000000000ll;  // about two seconds
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, long long budget) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const long long start = clock64();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(addr, parity)) return true;
    if (clock64() - start > budget) return false;
  }
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  return mbar_wait_bounded(bar, parity, kWaitBudgetCycles);
}

// 3-D tiled TMA load global -> shared, completion signalled on an mbarrier.
// Coordinates are (innermost, middle, plane). No cluster multicast: every
// load in this library reads this GPU's own memory into this CTA only.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t c0, int32_t c1,
                                            int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// 1-D bulk copy global -> shared (no tensor map, no multicast), completion
// signalled on an mbarrier; both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// A shared-memory stage read with ordinary loads is refilled by bulk copies,
// which write through the async proxy: this orders the thread's reads of the
// stage before those writes. Each reader executes it before signalling that
// the stage is free.
__device__ __forceinline__ void release_stage_reads() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// tcgen05: tensor memory allocation, MMA, commit, loads, fences.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] x B[smem], int8 x int8 -> int32.
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier when every tcgen05 op issued so far by this
// thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same wait, naming the registers of the load it completes as read-write
// operands: the compiler sees them change here, so no use of them is
// scheduled before the wait (the load writes them asynchronously).
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (base_lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"): start
// address, leading/stride byte offsets (16-byte units), version 1 at bit 46,
// swizzle mode at bits 61-63 (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t make_smem_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for kind::i8: s32 accumulator, signed int8 A and B,
// A K-major, B MN-major, shape M x N.
__host__ __device__ constexpr uint32_t make_idesc_i8(uint32_t m, uint32_t n, bool b_mn_major) {
  return (2u << 4)                       // D format: s32
         | (1u << 7)                     // A format: signed int8
         | (1u << 10)                    // B format: signed int8
         | (0u << 15)                    // A K-major
         | ((b_mn_major ? 1u : 0u) << 16)  // B major
         | ((n >> 3) << 17)              // N / 8
         | ((m >> 4) << 24);             // M / 16
}

// Signed int8 A and B with A MN-major (its M elements contiguous, as in
// compact residue planes read cell-major) and B K-major.
__host__ __device__ constexpr uint32_t make_idesc_i8_mn_a(uint32_t m, uint32_t n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Same layout for unsigned 8-bit A and B (formats 0): u8 x u8 -> s32, the
// accumulator wrapping modulo 2^32 (saturation bit 3 left clear).
__host__ __device__ constexpr uint32_t make_idesc_u8(uint32_t m, uint32_t n, bool b_mn_major) {
  return (2u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

}  // namespace rns8cuda
