// Tensor-core plane GEMM for sm_100a: C_p = (A_p x B_p) mod m_p over every
// plane p of every task, in one persistent launch; and the wrap64 byte-plane
// GEMM (C = A x B mod 2^64) on the same pipeline.
//
// Roles (192 threads, one CTA per SM):
//   warp 0      one thread issues TMA loads of A (128 x 128, K-major) and B
//               (128 x 256, N-major, two 128-column boxes) into a 4-stage
//               shared-memory ring, completion tracked by mbarriers;
//   warp 1      one thread issues tcgen05.mma.kind::i8 (M=128, N=256, K=32)
//               into one of two 256-column int32 accumulators in tensor memory;
//   warps 2-5   epilogue: tcgen05.ld the accumulator, reduce every int32 to
//               the centered residue modulo the plane's modulus, store int8.
// Work unit = (task, plane, K split, 128 x 256 output tile). A unit never
// spans more than RNS8_SAFE_INT32_K_BLOCK products, so its int32 accumulator
// is exact (|sum| <= 65536 * 128 * 128 = 2^30). When K is longer, or when the
// output tiles alone cannot fill the GPU, K is split: each unit adds its
// centered partial residue into an int32 scratch plane and a finalize pass
// reduces the sum modulo m (reference: cpu_reference.cpp:171-174 folds each
// 65536 block into the running residue; the sum of per-block residues is
// congruent, so the results are identical).
//
// Every mbarrier wait is bounded; a wait that runs out sets the device status
// word and the CTA drains its own in-flight copies and MMAs, frees its tensor
// memory and exits.
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "device_common.cuh"
#include "gemm_internal.hpp"

namespace rns8cuda {
namespace {

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4, UMMA_K = 32;
constexpr int GROUP_M = 32;  // raster: 32 M-tiles per column sweep for L2 reuse
constexpr uint32_t A_BYTES = BM * BK;
constexpr uint32_t B_HALF_BYTES = BK * 128;
constexpr uint32_t B_BYTES = BK * BN;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t ACC_COLS = BN;
constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;
constexpr int THREADS = 192;
constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
constexpr int kMaxKbPerUnit = static_cast<int>(kSafeKBlock / BK);  // 512

// Division of a 32-bit n by a fixed d as a multiply-high and a shift
// (Granlund-Montgomery, round-up multiplier; the 33-bit sum in 64 bits), so
// that decoding a work unit costs a few dozen cycles instead of a chain of
// division subroutines.
struct FastDiv {
  uint32_t d, mul, shift;
};
inline FastDiv make_fast_div(uint32_t d) {
  uint32_t l = 0;
  while (l < 32 && (1ull << l) < d) ++l;
  return FastDiv{d, static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - d)) / d + 1), l};
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
  return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, f.mul)) + n) >> f.shift);
}

struct __align__(64) TcParams {
  CUtensorMap tmA[kMaxGroupTasks];
  CUtensorMap tmB[kMaxGroupTasks];
  int8_t* C[kMaxGroupTasks];
  int32_t* scratch;  // split-K partial sums, [task][plane][m][n]
  int64_t m, n, k;
  uint32_t planes, tasks;
  uint32_t m_tiles, n_tiles, total_kb, splits, kb_per_split;
  uint64_t units;
  uint32_t* status;
  uint16_t moduli[20];
  // Per plane, the constants of centered_byte() (EpilogueReduce, host-made).
  uint32_t red_bias[20], red_magic[20];
  uint8_t red_shift[20];
  // Scheduled plans: the units to run (plane | split << 8 | mt << 24 | nt << 44)
  // and, per schedule tile, its selected prefix (| 0x80 for a proven-zero
  // output, which is filled elsewhere); the epilogue stores a cell only when
  // the cell's tile needs the plane.
  const uint64_t* unit_list;
  const uint8_t* tile_sel;
  uint32_t sched_shift_m, sched_shift_n, sched_cols;
  // Row-slab exchange (slab_count > 0, one task, no split-K): output row r
  // belongs to slab s = r / slab_rows and its plane p is stored at
  // slab_dst[s] + dst_plane[p] * slab_stride[s] + (r - s * slab_rows) * n,
  // in this GPU's memory or a peer's over NVLink.
  int8_t* slab_dst[kMaxSlabs];
  int64_t slab_stride[kMaxSlabs];
  int64_t slab_rows;
  uint32_t slab_count;
  uint8_t dst_plane[20];
  FastDiv div_tiles, div_splits, div_planes, div_span;  // m_tiles*n_tiles, splits, planes, GROUP_M*n_tiles
};

struct Unit {
  uint32_t t, p, mt, nt, kb0, kb1;
};

// Centered residue of an accumulator v modulo m (2 <= m <= 256) in five
// integer operations: with h = floor(m/2) and u = v + h + m*ceil(2^30/m),
// u mod m = (v + h) mod m and u - floor(u/m)*m - h is v's residue in
// [-h, m-1-h]. A unit sums at most 65536 products of int8 values, so
// |v| <= 2^30 and 0 <= u < 2^31 + 384. For such u, q = mulhi(u, magic) >> shift
// is floor(u/m) exactly: with 2^shift <= m < 2^(shift+1) and the round-up
// multiplier magic = ceil(2^(32+shift)/m) (Granlund-Montgomery), the excess
// e = magic*m - 2^(32+shift) < m makes u*e < 2^(32+shift); powers of two use
// mulhi(u, 2^31) >> (shift-1) = u >> shift, exact for every 32-bit u.
struct EpilogueReduce {
  uint32_t bias, magic, shift;
};
inline EpilogueReduce make_epilogue_reduce(uint32_t m) {
  uint32_t s = 0;
  while ((2u << s) <= m) ++s;  // 2^s <= m < 2^(s+1)
  EpilogueReduce r;
  if ((m & (m - 1)) == 0) {  // powers of two: mulhi(u, 2^31) >> (s-1) = u >> s
    r.magic = 0x80000000u;
    r.shift = s ? s - 1 : 0;
  } else {
    r.magic = static_cast<uint32_t>(((1ull << (32 + s)) + m - 1) / m);
    r.shift = s;
  }
  r.bias = (m >> 1) + m * static_cast<uint32_t>(((1ull << 30) + m - 1) / m);
  return r;
}
__device__ __forceinline__ uint32_t centered_byte(uint32_t v, uint32_t bias, uint32_t magic, uint32_t shift,
                                                  uint32_t m, uint32_t h) {
  const uint32_t u = v + bias;
  const uint32_t q = __umulhi(u, magic) >> shift;
  return u - (q * m + h);  // the low byte is the centered residue's
}

// 32-bit arithmetic with precomputed divisors (the host keeps the unit count
// below 2^32): the producer and the MMA thread decode every unit at its start,
// and a chain of division subroutines there would idle the tensor pipe.
__device__ __forceinline__ Unit decode_unit(const TcParams& prm, uint32_t u) {
  if (prm.unit_list) {
    const uint64_t e = prm.unit_list[u];
    Unit w;
    w.t = 0;
    w.p = static_cast<uint32_t>(e & 0xFFu);
    const uint32_t s = static_cast<uint32_t>((e >> 8) & 0xFFFFu);
    w.mt = static_cast<uint32_t>((e >> 24) & 0xFFFFFu);
    w.nt = static_cast<uint32_t>((e >> 44) & 0xFFFFFu);
    w.kb0 = s * prm.kb_per_split;
    w.kb1 = min(prm.total_kb, w.kb0 + prm.kb_per_split);
    return w;
  }
  const uint32_t rest = fast_div(u, prm.div_tiles);
  const uint32_t tile = u - rest * prm.div_tiles.d;
  const uint32_t tp = fast_div(rest, prm.div_splits);
  const uint32_t s = rest - tp * prm.div_splits.d;
  Unit w;
  w.t = fast_div(tp, prm.div_planes);
  w.p = tp - w.t * prm.planes;
  const uint32_t group = fast_div(tile, prm.div_span);
  const uint32_t first_m = group * GROUP_M;
  const uint32_t in_group = tile - group * prm.div_span.d;
  if (prm.m_tiles - first_m >= static_cast<uint32_t>(GROUP_M)) {
    w.mt = first_m + in_group % GROUP_M;
    w.nt = in_group / GROUP_M;
  } else {  // the last, narrower group
    const uint32_t gsize = prm.m_tiles - first_m;
    w.mt = first_m + in_group % gsize;
    w.nt = in_group / gsize;
  }
  w.kb0 = s * prm.kb_per_split;
  w.kb1 = min(prm.total_kb, w.kb0 + prm.kb_per_split);
  return w;
}

__device__ __forceinline__ void report_timeout(const TcParams& prm, volatile int* abort_flag) {
  *abort_flag = 1;
  atomicOr(prm.status, kDevWaitTimeout);
}

__global__ void __launch_bounds__(THREADS, 1) tc_plane_gemm_kernel(const __grid_constant__ TcParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    for (uint32_t t = 0; t < prm.tasks; ++t) {
      tma_prefetch_desc(&prm.tmA[t]);
      tma_prefetch_desc(&prm.tmB[t]);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      uint32_t stage = 0, phase = 0;
      uint32_t pending = 0, pending_parity = 0;
      bool ok = true;
      for (uint64_t u = blockIdx.x; ok && u < prm.units; u += gridDim.x) {
        const Unit w = decode_unit(prm, static_cast<uint32_t>(u));
        for (uint32_t kb = w.kb0; kb < w.kb1; ++kb) {
          if (*abort_flag || !mbar_wait_bounded(&empty[stage], phase ^ 1u)) {
            if (!*abort_flag) report_timeout(prm, abort_flag);
            ok = false;
            break;
          }
          pending &= ~(1u << stage);
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          const int32_t kc = static_cast<int32_t>(kb * BK);
          tma_load_3d(sa, &prm.tmA[w.t], &full[stage], kc, static_cast<int32_t>(w.mt * BM), static_cast<int32_t>(w.p));
          tma_load_3d(sb, &prm.tmB[w.t], &full[stage], static_cast<int32_t>(w.nt * BN), kc, static_cast<int32_t>(w.p));
          tma_load_3d(sb + B_HALF_BYTES, &prm.tmB[w.t], &full[stage], static_cast<int32_t>(w.nt * BN + 128), kc,
                      static_cast<int32_t>(w.p));
          pending |= 1u << stage;
          pending_parity = (pending_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Loads issued but never consumed (abort path) must land before exit.
      for (int s = 0; s < STAGES; ++s)
        if (pending & (1u << s)) (void)mbar_wait_bounded(&full[s], (pending_parity >> s) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = make_idesc_i8(BM, BN, /*b_mn_major=*/true);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (uint64_t u = blockIdx.x; ok && u < prm.units; u += gridDim.x) {
        const Unit w = decode_unit(prm, static_cast<uint32_t>(u));
        if (*abort_flag || !mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u)) {
          if (!*abort_flag) report_timeout(prm, abort_flag);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (uint32_t kb = w.kb0; kb < w.kb1; ++kb) {
          if (*abort_flag || !mbar_wait_bounded(&full[stage], phase)) {
            if (!*abort_flag) report_timeout(prm, abort_flag);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // A: K-major rows of 128 B, 8-row swizzle atoms 1 KiB apart.
            const uint64_t adesc = make_smem_desc_sw128(sa + kk * UMMA_K, 16, 1024);
            // B: N-major, two 128-column chunks 16 KiB apart, 8 K-rows per 1 KiB atom.
            const uint64_t bdesc = make_smem_desc_sw128(sb + kk * UMMA_K * 128, B_HALF_BYTES, 1024);
            tc_mma_i8(d_tmem, adesc, bdesc, idesc, (kb > w.kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA this thread issued completes before tensor memory is freed.
      tc_commit(drain);
      (void)mbar_wait_bounded(drain, 0);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const uint32_t quarter = static_cast<uint32_t>(warp & 3);  // TMEM lanes this warp may read
    uint32_t acc = 0, acc_phase = 0;
    for (uint64_t u = blockIdx.x; u < prm.units; u += gridDim.x) {
      const Unit w = decode_unit(prm, static_cast<uint32_t>(u));
      if (*abort_flag || !mbar_wait_bounded(&acc_full[acc], acc_phase)) {
        if (!*abort_flag) report_timeout(prm, abort_flag);
        break;
      }
      tc_fence_after();
      const uint32_t m_p = prm.moduli[w.p];
      const ModConst mc = prm.scratch ? make_mod_const(m_p) : ModConst{};
      const uint32_t rb = prm.red_bias[w.p], rm = prm.red_magic[w.p], rs = prm.red_shift[w.p], rh = m_p >> 1;
      const int64_t row = static_cast<int64_t>(w.mt) * BM + quarter * 32 + lane;
      const bool row_ok = row < prm.m;
      const int64_t plane_elems = prm.m * prm.n;
      int8_t* crow;
      if (prm.slab_count) {
        const int64_t s = row_ok ? row / prm.slab_rows : 0;
        crow = prm.slab_dst[s] + prm.dst_plane[w.p] * prm.slab_stride[s] + (row - s * prm.slab_rows) * prm.n;
      } else {
        crow = prm.C[w.t] + static_cast<int64_t>(w.p) * plane_elems + row * prm.n;
      }
      int32_t* srow = prm.scratch
                          ? prm.scratch + (static_cast<int64_t>(w.t) * prm.planes + w.p) * plane_elems + row * prm.n
                          : nullptr;
      // One 32-column chunk of this thread's accumulator row: reduce, pack,
      // store (or add into the split-K sums).
      auto store_chunk = [&](int c, const uint32_t (&v)[32]) {
        const int64_t col = static_cast<int64_t>(w.nt) * BN + c * 32;
        if (!row_ok || col >= prm.n) return;
        if (prm.tile_sel) {  // schedule tiles are >= 64 wide: a 32-column chunk lies in one
          const uint8_t sel = prm.tile_sel[(row >> prm.sched_shift_m) * prm.sched_cols + (col >> prm.sched_shift_n)];
          if ((sel & 0x80u) || w.p >= (sel & 0x7Fu)) return;
        }
        if (srow) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col + j < prm.n) atomicAdd(srow + col + j, reduce_i32_centered(static_cast<int32_t>(v[j]), mc));
        } else {
          uint32_t packed[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint32_t r0 = centered_byte(v[4 * q + 0], rb, rm, rs, m_p, rh);
            const uint32_t r1 = centered_byte(v[4 * q + 1], rb, rm, rs, m_p, rh);
            const uint32_t r2 = centered_byte(v[4 * q + 2], rb, rm, rs, m_p, rh);
            const uint32_t r3 = centered_byte(v[4 * q + 3], rb, rm, rs, m_p, rh);
            packed[q] = __byte_perm(__byte_perm(r0, r1, 0x0040), __byte_perm(r2, r3, 0x0040), 0x5410);
          }
          // n is a multiple of 16, so a 32-column chunk is whole, half, or absent.
          uint4* dst = reinterpret_cast<uint4*>(crow + col);
          dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          if (col + 32 <= prm.n) dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
      };
      // The next chunk's tensor-memory load is in flight while this one is
      // reduced and stored (tcgen05.wait::ld waits for all of a thread's loads,
      // so each load is issued right after the previous wait).
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + acc * ACC_COLS;
      uint32_t va[32], vb[32];
      tmem_ld_32x32b_x32(taddr, va);
#pragma unroll 1
      for (int c = 0; c < BN / 32; c += 2) {
        tmem_wait_ld(va);
        tmem_ld_32x32b_x32(taddr + (c + 1) * 32, vb);
        store_chunk(c, va);
        tmem_wait_ld(vb);
        if (c + 2 < BN / 32) tmem_ld_32x32b_x32(taddr + (c + 2) * 32, va);
        store_chunk(c + 1, vb);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Slab stores may target a peer GPU: make them visible system-wide before
    // this kernel counts as complete to the host-side exchange barrier.
    if (prm.slab_count) __threadfence_system();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Split-K finalize: C = centered(sum of partial residues mod m). With a
// schedule, only the cells whose tile needs the plane are written.
struct SchedMask {
  const uint8_t* tile_sel;
  uint32_t shift_m, shift_n, cols;
  int64_t n;
};

__global__ void __launch_bounds__(256) split_finalize_kernel(const int32_t* __restrict__ scratch, int64_t plane_elems,
                                                             uint32_t planes, PlaneModuli moduli,
                                                             int8_t* __restrict__ c, SchedMask mask) {
  const int64_t total = plane_elems * planes;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t p = static_cast<uint32_t>(i / plane_elems);
    if (mask.tile_sel) {
      const int64_t e = i - static_cast<int64_t>(p) * plane_elems;
      const int64_t row = e / mask.n, col = e - row * mask.n;
      const uint8_t sel = mask.tile_sel[(row >> mask.shift_m) * mask.cols + (col >> mask.shift_n)];
      if ((sel & 0x80u) || p >= (sel & 0x7Fu)) continue;
    }
    c[i] = static_cast<int8_t>(reduce_i32_centered(scratch[i], make_mod_const(moduli.m[p])));
  }
}

// Proven-zero tiles (RNS8_TILE_SCHEDULE_ZERO_OUTPUT): planes below the tile's
// selected prefix are zero (cpu_reference.cpp:236-238). One block per tile.
__global__ void __launch_bounds__(256) zero_tiles_kernel(const ZeroTile* __restrict__ tiles, uint32_t count,
                                                         int8_t* __restrict__ c, int64_t m, int64_t n) {
  for (uint32_t t = blockIdx.x; t < count; t += gridDim.x) {
    const ZeroTile z = tiles[t];
    for (uint32_t p = 0; p < z.planes; ++p)
      for (int64_t r = threadIdx.x / 32; r < z.rows; r += blockDim.x / 32)
        for (int64_t col = threadIdx.x % 32; col < z.cols; col += 32)
          c[static_cast<int64_t>(p) * m * n + (z.row0 + r) * n + z.col0 + col] = 0;
  }
}

// ---- wrap64: C = A x B mod 2^64 from unsigned byte planes ---------------------
// With A = sum_i 2^(8i) A_i and B = sum_j 2^(8j) B_j (byte planes), the low 64
// bits of A x B are sum_{d<8} 2^(8d) S_d with S_d = sum_{i+j=d} A_i x B_j: the
// 36 byte-pair products of the low eight Comba diagonals (reference
// src/backend_wrap64/wrap64_reference.cpp:105-117). A work unit is one output
// tile over one K range; it runs the diagonals in order, each as one u8 x u8
// MMA chain over (K block, byte pair) into a 32-bit TMEM accumulator, and the
// epilogue adds S_d * 2^(8d) into the 64-bit output with wrapping atomic adds
// (the output is zeroed first). Only S_d mod 2^(64-8d) matters: for d >= 4 that
// is S_d mod 2^32, which the accumulator keeps whatever K is; for d <= 3 a unit
// spans at most 16384 products, so S_d <= 4 * 16384 * 255^2 < 2^32 is exact.
// Longer K is split into several units whose sums the atomics add up.
constexpr int kWrapMaxKbPerUnit = 16384 / BK;  // 128

struct __align__(64) WrapParams {
  CUtensorMap tmA;  // (k, m, 8) byte planes of A
  CUtensorMap tmB;  // (n, k, 8) byte planes of B
  unsigned long long* C;
  int64_t m, n;
  uint32_t m_tiles, n_tiles, total_kb, splits, kb_per_split;
  uint64_t units;
  uint32_t* status;
};

struct WrapUnit {
  uint32_t mt, nt, kb0, kb1;
};

__device__ __forceinline__ WrapUnit decode_wrap_unit(const WrapParams& prm, uint64_t u) {
  const uint64_t tiles = static_cast<uint64_t>(prm.m_tiles) * prm.n_tiles;
  const uint64_t tile = u % tiles;
  const uint32_t s = static_cast<uint32_t>(u / tiles);
  WrapUnit w;
  const uint32_t span = GROUP_M * prm.n_tiles;
  const uint32_t group = static_cast<uint32_t>(tile / span);
  const uint32_t first_m = group * GROUP_M;
  const uint32_t gsize = min(prm.m_tiles - first_m, static_cast<uint32_t>(GROUP_M));
  const uint32_t in_group = static_cast<uint32_t>(tile % span);
  w.mt = first_m + in_group % gsize;
  w.nt = in_group / gsize;
  w.kb0 = s * prm.kb_per_split;
  w.kb1 = min(prm.total_kb, w.kb0 + prm.kb_per_split);
  return w;
}

__device__ __forceinline__ void report_wrap_timeout(uint32_t* status, volatile int* abort_flag) {
  *abort_flag = 1;
  atomicOr(status, kDevWaitTimeout);
}

__global__ void __launch_bounds__(THREADS, 1) tc_wrap64_kernel(const __grid_constant__ WrapParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&prm.tmA);
    tma_prefetch_desc(&prm.tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: (diagonal, K block, byte pair) ----------------
      uint32_t stage = 0, phase = 0;
      uint32_t pending = 0, pending_parity = 0;
      bool ok = true;
      for (uint64_t u = blockIdx.x; ok && u < prm.units; u += gridDim.x) {
        const WrapUnit w = decode_wrap_unit(prm, u);
        for (int d = 0; ok && d < 8; ++d) {
          for (uint32_t kb = w.kb0; ok && kb < w.kb1; ++kb) {
            for (int i = 0; i <= d; ++i) {
              if (*abort_flag || !mbar_wait_bounded(&empty[stage], phase ^ 1u)) {
                if (!*abort_flag) report_wrap_timeout(prm.status, abort_flag);
                ok = false;
                break;
              }
              pending &= ~(1u << stage);
              mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
              uint8_t* sa = smem + stage * STAGE_BYTES;
              uint8_t* sb = sa + A_BYTES;
              const int32_t kc = static_cast<int32_t>(kb * BK);
              tma_load_3d(sa, &prm.tmA, &full[stage], kc, static_cast<int32_t>(w.mt * BM), i);
              tma_load_3d(sb, &prm.tmB, &full[stage], static_cast<int32_t>(w.nt * BN), kc, d - i);
              tma_load_3d(sb + B_HALF_BYTES, &prm.tmB, &full[stage], static_cast<int32_t>(w.nt * BN + 128), kc, d - i);
              pending |= 1u << stage;
              pending_parity = (pending_parity & ~(1u << stage)) | (phase << stage);
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
            }
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (pending & (1u << s)) (void)mbar_wait_bounded(&full[s], (pending_parity >> s) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: one accumulator per diagonal ----------------
      constexpr uint32_t idesc = make_idesc_u8(BM, BN, /*b_mn_major=*/true);
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      for (uint64_t u = blockIdx.x; ok && u < prm.units; u += gridDim.x) {
        const WrapUnit w = decode_wrap_unit(prm, u);
        for (int d = 0; ok && d < 8; ++d) {
          if (*abort_flag || !mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u)) {
            if (!*abort_flag) report_wrap_timeout(prm.status, abort_flag);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
          bool first = true;
          for (uint32_t kb = w.kb0; ok && kb < w.kb1; ++kb) {
            for (int i = 0; i <= d; ++i) {
              if (*abort_flag || !mbar_wait_bounded(&full[stage], phase)) {
                if (!*abort_flag) report_wrap_timeout(prm.status, abort_flag);
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
              const uint32_t sb = sa + A_BYTES;
#pragma unroll
              for (int kk = 0; kk < BK / UMMA_K; ++kk) {
                const uint64_t adesc = make_smem_desc_sw128(sa + kk * UMMA_K, 16, 1024);
                const uint64_t bdesc = make_smem_desc_sw128(sb + kk * UMMA_K * 128, B_HALF_BYTES, 1024);
                tc_mma_i8(d_tmem, adesc, bdesc, idesc, (first && kk == 0) ? 0u : 1u);
              }
              first = false;
              tc_commit(&empty[stage]);
              if (++stage == STAGES) {
                stage = 0;
                phase ^= 1u;
              }
            }
          }
          if (!ok) break;
          tc_commit(&acc_full[acc]);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
      }
      tc_commit(drain);
      (void)mbar_wait_bounded(drain, 0);
    }
  } else {
    // ---------------- epilogue: C += S_d * 2^(8d) ----------------
    const uint32_t quarter = static_cast<uint32_t>(warp & 3);
    uint32_t acc = 0, acc_phase = 0;
    bool ok = true;
    for (uint64_t u = blockIdx.x; ok && u < prm.units; u += gridDim.x) {
      const WrapUnit w = decode_wrap_unit(prm, u);
      const int64_t row = static_cast<int64_t>(w.mt) * BM + quarter * 32 + lane;
      const bool row_ok = row < prm.m;
      unsigned long long* crow = prm.C + row * prm.n;
      for (int d = 0; d < 8; ++d) {
        if (*abort_flag || !mbar_wait_bounded(&acc_full[acc], acc_phase)) {
          if (!*abort_flag) report_wrap_timeout(prm.status, abort_flag);
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem_base + ((quarter * 32u) << 16) + acc * ACC_COLS + c * 32, v);
          tmem_wait_ld(v);
          const int64_t col = static_cast<int64_t>(w.nt) * BN + c * 32;
          if (!row_ok || col >= prm.n) continue;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col + j < prm.n) atomicAdd(crow + col + j, static_cast<unsigned long long>(v[j]) << (8 * d));
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---- host side ---------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D int8 tensor (inner, outer, plane) with a 128 x 128 box, 128-byte swizzle.
bool encode_planes(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t planes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {inner, outer, planes};
  const cuuint64_t strides[2] = {inner, inner * outer};  // bytes, dims 1 and 2
  const cuuint32_t box[3] = {128, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

TcSchedule tc_schedule(const PlaneGemmProblem& prob, int sm_count) {
  TcSchedule s{};
  s.m_tiles = static_cast<uint32_t>((prob.m + BM - 1) / BM);
  s.n_tiles = static_cast<uint32_t>((prob.n + BN - 1) / BN);
  s.total_kb = static_cast<uint32_t>((prob.k + BK - 1) / BK);
  const uint64_t tiles = static_cast<uint64_t>(prob.task_count) * prob.planes * s.m_tiles * s.n_tiles;
  uint32_t splits = (s.total_kb + kMaxKbPerUnit - 1) / kMaxKbPerUnit;
  if (tiles * splits < static_cast<uint64_t>(sm_count) && s.total_kb >= 8) {
    // Too few output tiles to occupy every SM: split K. The kernel's time is
    // about (waves of units) x (K blocks per unit + ~2 for the unit's fill and
    // epilogue); take the smallest split count that minimises it, keeping at
    // least four K blocks per unit. (Rounding the unit count up to just past
    // one wave would leave most SMs idle in a second wave.)
    const uint32_t cap = std::max(splits, s.total_kb / 4);
    const uint32_t limit = std::min<uint64_t>(cap, 4 * (static_cast<uint64_t>(sm_count) / tiles + 1));
    uint64_t best_cost = ~0ull;
    uint32_t best = splits;
    for (uint32_t c = splits; c <= limit; ++c) {
      const uint64_t waves = (tiles * c + sm_count - 1) / static_cast<uint64_t>(sm_count);
      const uint64_t cost = waves * ((s.total_kb + c - 1) / c + 2);
      if (cost < best_cost) {
        best_cost = cost;
        best = c;
      }
    }
    splits = best;
  }
  s.kb_per_split = (s.total_kb + splits - 1) / splits;
  s.splits = (s.total_kb + s.kb_per_split - 1) / s.kb_per_split;
  s.units = tiles * s.splits;
  return s;
}

cudaError_t tc_plane_gemm(const PlaneGemmProblem& prob, int sm_count, void* scratch, uint64_t scratch_bytes,
                          uint32_t* dev_status, cudaStream_t stream, const TcScheduleUnits* sched,
                          const SlabScatter* scatter) {
  if (prob.task_count == 0 || prob.task_count > kMaxGroupTasks || prob.planes == 0 || prob.planes > 20)
    return cudaErrorInvalidValue;
  static std::atomic<uint64_t> configured{0};
  const cudaError_t attr_err = raise_smem_limit_once(tc_plane_gemm_kernel, static_cast<int>(SMEM_BYTES), configured);
  if (attr_err != cudaSuccess) return attr_err;

  const TcSchedule s = tc_schedule(prob, sm_count);
  if (s.units >= (1ull << 32) || static_cast<uint64_t>(s.m_tiles) * s.n_tiles >= (1ull << 32) ||
      (sched && sched->unit_count >= (1ull << 32)))
    return cudaErrorInvalidValue;  // the kernel decodes units in 32-bit arithmetic
  const bool split = s.splits > 1;
  const uint64_t plane_elems = static_cast<uint64_t>(prob.m) * prob.n;
  const uint64_t need = split ? plane_elems * prob.planes * prob.task_count * sizeof(int32_t) : 0;
  if (split && (scratch == nullptr || scratch_bytes < need)) return cudaErrorInvalidValue;
  if (scatter && (split || sched || prob.task_count != 1 || scatter->slab_count == 0 ||
                  scatter->slab_count > static_cast<uint32_t>(kMaxSlabs) || scatter->slab_rows <= 0))
    return cudaErrorInvalidValue;

  static thread_local TcParams prm;  // 8+ KiB: keep it off the stack
  std::memset(&prm, 0, sizeof(prm));
  for (uint32_t t = 0; t < prob.task_count; ++t) {
    if (!encode_planes(&prm.tmA[t], prob.tasks[t].a, prob.k, prob.m, prob.planes) ||
        !encode_planes(&prm.tmB[t], prob.tasks[t].b, prob.n, prob.k, prob.planes))
      return cudaErrorInvalidValue;
    prm.C[t] = prob.tasks[t].c;
  }
  prm.scratch = split ? static_cast<int32_t*>(scratch) : nullptr;
  prm.m = prob.m;
  prm.n = prob.n;
  prm.k = prob.k;
  prm.planes = prob.planes;
  prm.tasks = prob.task_count;
  prm.m_tiles = s.m_tiles;
  prm.n_tiles = s.n_tiles;
  prm.total_kb = s.total_kb;
  prm.splits = s.splits;
  prm.kb_per_split = s.kb_per_split;
  prm.units = s.units;
  prm.status = dev_status;
  prm.div_tiles = make_fast_div(s.m_tiles * s.n_tiles);
  prm.div_splits = make_fast_div(s.splits);
  prm.div_planes = make_fast_div(prob.planes);
  prm.div_span = make_fast_div(static_cast<uint32_t>(GROUP_M) * s.n_tiles);
  for (uint32_t p = 0; p < prob.planes; ++p) {
    prm.moduli[p] = prob.moduli[p];
    const EpilogueReduce r = make_epilogue_reduce(prob.moduli[p]);
    prm.red_bias[p] = r.bias;
    prm.red_magic[p] = r.magic;
    prm.red_shift[p] = static_cast<uint8_t>(r.shift);
  }
  if (sched) {
    if (prob.task_count != 1) return cudaErrorInvalidValue;
    prm.unit_list = sched->units_dev;
    prm.units = sched->unit_count;
    prm.tile_sel = sched->tile_sel_dev;
    prm.sched_shift_m = sched->shift_m;
    prm.sched_shift_n = sched->shift_n;
    prm.sched_cols = sched->cols;
  }

  if (scatter) {
    prm.slab_rows = scatter->slab_rows;
    prm.slab_count = scatter->slab_count;
    for (uint32_t sl = 0; sl < scatter->slab_count; ++sl) {
      const int64_t rows = std::min<int64_t>(scatter->slab_rows, prob.m - static_cast<int64_t>(sl) * scatter->slab_rows);
      if (rows <= 0 || scatter->slab_dst[sl] == nullptr || reinterpret_cast<uintptr_t>(scatter->slab_dst[sl]) % 16)
        return cudaErrorInvalidValue;
      prm.slab_dst[sl] = scatter->slab_dst[sl];
      prm.slab_stride[sl] = rows * prob.n;
    }
    for (uint32_t p = 0; p < prob.planes; ++p) {
      if (scatter->dst_plane[p] >= 20) return cudaErrorInvalidValue;
      prm.dst_plane[p] = static_cast<uint8_t>(scatter->dst_plane[p]);
    }
  }
  if (split) {
    const cudaError_t e = cudaMemsetAsync(scratch, 0, need, stream);
    if (e != cudaSuccess) return e;
  }
  const uint64_t grid = prm.units < static_cast<uint64_t>(sm_count) ? prm.units : static_cast<uint64_t>(sm_count);
  if (grid > 0) tc_plane_gemm_kernel<<<static_cast<unsigned>(grid), THREADS, SMEM_BYTES, stream>>>(prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !split) return e;
  PlaneModuli pm{};
  for (uint32_t p = 0; p < prob.planes; ++p) pm.m[p] = prob.moduli[p];
  for (uint32_t t = 0; t < prob.task_count; ++t) {
    int64_t blocks = static_cast<int64_t>((plane_elems * prob.planes + 255) / 256);
    if (blocks > sm_count * 8) blocks = sm_count * 8;
    SchedMask mask{sched ? sched->tile_sel_dev : nullptr, sched ? sched->shift_m : 0u, sched ? sched->shift_n : 0u,
                   sched ? sched->cols : 0u, prob.n};
    split_finalize_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const int32_t*>(scratch) + static_cast<uint64_t>(t) * prob.planes * plane_elems,
        static_cast<int64_t>(plane_elems), prob.planes, pm, prob.tasks[t].c, mask);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// ---- wrap64 host side -----------------------------------------------------------
bool tma_encode_available() { return encode_fn() != nullptr; }

bool encode_plane_cells(CUtensorMap* map, const void* planes, uint64_t cells, uint32_t plane_count,
                        uint32_t box_rows, uint32_t box_chunks) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || reinterpret_cast<uintptr_t>(planes) % 16 != 0 || cells % 128 != 0) return false;
  if (box_rows == 0 || box_rows > 32 || box_rows % 8 != 0 || box_chunks == 0 || box_chunks > 16) return false;
  // (cell within a 128-cell chunk, plane, chunk): the chunk stride (128 bytes)
  // is below the plane stride, so one box is box_chunks consecutive chunks,
  // each box_rows planes of 128 cells, chunk-major in shared memory.
  const cuuint64_t dims[3] = {128, plane_count, cells / 128};
  const cuuint64_t strides[2] = {cells, 128};  // bytes, dims 1 and 2
  const cuuint32_t box[3] = {128, box_rows, box_chunks};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(planes), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t tc_wrap64_gemm(const uint8_t* a_limbs, const uint8_t* b_limbs, uint64_t* c, int64_t m, int64_t n,
                           int64_t k, int sm_count, uint32_t* dev_status, cudaStream_t stream) {
  static std::atomic<uint64_t> configured{0};
  const cudaError_t attr_err = raise_smem_limit_once(tc_wrap64_kernel, static_cast<int>(SMEM_BYTES), configured);
  if (attr_err != cudaSuccess) return attr_err;
  WrapParams prm;
  std::memset(&prm, 0, sizeof(prm));
  if (!encode_planes(&prm.tmA, a_limbs, static_cast<uint64_t>(k), static_cast<uint64_t>(m), 8) ||
      !encode_planes(&prm.tmB, b_limbs, static_cast<uint64_t>(n), static_cast<uint64_t>(k), 8))
    return cudaErrorInvalidValue;
  prm.m_tiles = static_cast<uint32_t>((m + BM - 1) / BM);
  prm.n_tiles = static_cast<uint32_t>((n + BN - 1) / BN);
  prm.total_kb = static_cast<uint32_t>((k + BK - 1) / BK);
  const uint64_t tiles = static_cast<uint64_t>(prm.m_tiles) * prm.n_tiles;
  uint32_t splits = (prm.total_kb + kWrapMaxKbPerUnit - 1) / kWrapMaxKbPerUnit;
  if (tiles * splits < static_cast<uint64_t>(sm_count) && prm.total_kb >= 8) {
    const uint64_t want = (static_cast<uint64_t>(sm_count) + tiles - 1) / tiles;
    const uint32_t cap = prm.total_kb / 4;
    const uint32_t target = static_cast<uint32_t>(want < cap ? want : cap);
    if (target > splits) splits = target;
  }
  prm.kb_per_split = (prm.total_kb + splits - 1) / splits;
  prm.splits = (prm.total_kb + prm.kb_per_split - 1) / prm.kb_per_split;
  prm.units = tiles * prm.splits;
  prm.C = reinterpret_cast<unsigned long long*>(c);
  prm.m = m;
  prm.n = n;
  prm.status = dev_status;
  cudaError_t e = cudaMemsetAsync(c, 0, static_cast<size_t>(m) * n * sizeof(uint64_t), stream);
  if (e != cudaSuccess) return e;
  const uint64_t grid = prm.units < static_cast<uint64_t>(sm_count) ? prm.units : static_cast<uint64_t>(sm_count);
  tc_wrap64_kernel<<<static_cast<unsigned>(grid), THREADS, SMEM_BYTES, stream>>>(prm);
  return cudaGetLastError();
}

// ---- dispatch --------------------------------------------------------------
bool tensor_core_path_supported(const PlaneGemmProblem& prob) {
  if (prob.m <= 0 || prob.n <= 0 || prob.k <= 0) return false;
  if (prob.k % 16 != 0 || prob.n % 16 != 0) return false;  // TMA row strides must be 16-byte multiples
  if (prob.task_count == 0 || prob.planes == 0 || prob.planes > 20) return false;
  if (prob.m > (int64_t(1) << 31) || prob.n > (int64_t(1) << 31) || prob.k > (int64_t(1) << 31)) return false;
  for (uint32_t t = 0; t < prob.task_count; ++t) {
    if (reinterpret_cast<uintptr_t>(prob.tasks[t].a) % 16 || reinterpret_cast<uintptr_t>(prob.tasks[t].b) % 16 ||
        reinterpret_cast<uintptr_t>(prob.tasks[t].c) % 16)
      return false;
  }
  return encode_fn() != nullptr;
}

// ---- unaligned shapes on the tensor cores ---------------------------------------
// TMA needs every row pitch to be a multiple of 16 bytes. When K or N is not
// (or a plane pointer is not 16-byte aligned), the planes are copied into
// zero-padded ones (K and N rounded up to 16) in scratch, the padded problem
// runs on the tensor cores, and C's first n columns are copied out. Zero
// columns of A and zero rows of B add nothing to any sum, so the residues are
// those of the unpadded product.
namespace {

int64_t round16(int64_t v) { return (v + 15) / 16 * 16; }
uint64_t round256_u(uint64_t v) { return (v + 255) / 256 * 256; }
bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// dst (planes x drows x dcols, dcols % 16 == 0, 16-byte aligned) = src
// (planes x rows x cols, any pitch and alignment) inside, zero outside. One
// 16-byte dst chunk per thread step: when the chunk's 20-byte aligned source
// window lies inside the source row, five aligned word loads and funnel
// shifts assemble it; otherwise (row ends, misaligned row starts) bytes.
__global__ void __launch_bounds__(256) pad_planes_kernel(const int8_t* __restrict__ src, int64_t rows, int64_t cols,
                                                         uint32_t planes, int8_t* __restrict__ dst, int64_t drows,
                                                         int64_t dcols) {
  const int64_t chunks = dcols / 16;
  const int64_t total = static_cast<int64_t>(planes) * drows * chunks;
  // (row, chunk) pairs flattened, so narrow rows (a few chunks each) still
  // give every thread work.
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t pr = idx / chunks, ch = idx - pr * chunks;
    const int64_t p = pr / drows, r = pr - p * drows;
    uint4* out = reinterpret_cast<uint4*>(dst + pr * dcols);
    const uint8_t* row = reinterpret_cast<const uint8_t*>(src) + (p * rows + r) * cols;
    {
      const int64_t c0 = ch * 16;
      uint32_t w[4] = {0, 0, 0, 0};
      if (r < rows && c0 < cols) {
        const uintptr_t addr = reinterpret_cast<uintptr_t>(row + c0);
        const uintptr_t base = addr & ~uintptr_t(3);
        if (base >= reinterpret_cast<uintptr_t>(row) && base + 20 <= reinterpret_cast<uintptr_t>(row + cols)) {
          const uint32_t* wp = reinterpret_cast<const uint32_t*>(base);
          const uint32_t sh = static_cast<uint32_t>(addr - base) * 8;
          uint32_t v[5];
#pragma unroll
          for (int j = 0; j < 5; ++j) v[j] = wp[j];
#pragma unroll
          for (int j = 0; j < 4; ++j) w[j] = __funnelshift_r(v[j], v[j + 1], sh);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < cols) w[j / 4] |= static_cast<uint32_t>(row[c0 + j]) << (8 * (j % 4));
        }
      }
      out[ch] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// dst (planes x rows x cols, compact, 16-byte aligned) = the first cols
// columns of src (planes x rows x scols, scols % 16 == 0, 16-byte aligned).
// One aligned 16-byte chunk of the flattened dst per thread step; a chunk
// inside one row reads its 16 source bytes as five aligned words (when they
// lie inside the source row) shifted into place, a chunk that crosses rows
// gathers bytes.
__global__ void __launch_bounds__(256) crop_planes_kernel(const int8_t* __restrict__ src, int64_t rows, int64_t scols,
                                                          uint32_t planes, int8_t* __restrict__ dst, int64_t cols) {
  const int64_t total = static_cast<int64_t>(planes) * rows * cols;
  const int64_t chunks = (total + 15) / 16;
  const uint8_t* s8 = reinterpret_cast<const uint8_t*>(src);
  for (int64_t ch = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; ch < chunks;
       ch += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i0 = ch * 16;
    const int64_t pr = i0 / cols, c0 = i0 - pr * cols;
    uint32_t w[4] = {0, 0, 0, 0};
    const uintptr_t row = reinterpret_cast<uintptr_t>(s8 + pr * scols);
    const uintptr_t addr = row + static_cast<uintptr_t>(c0);
    const uintptr_t base = addr & ~uintptr_t(3);
    if (c0 + 16 <= cols && i0 + 16 <= total && base + 20 <= row + static_cast<uintptr_t>(scols)) {
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(base);
      const uint32_t sh = static_cast<uint32_t>(addr - base) * 8;
      uint32_t v[5];
#pragma unroll
      for (int j = 0; j < 5; ++j) v[j] = wp[j];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = __funnelshift_r(v[j], v[j + 1], sh);
      reinterpret_cast<uint4*>(dst)[ch] = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      for (int j = 0; j < 16 && i0 + j < total; ++j) {
        const int64_t i = i0 + j;
        const int64_t r = i / cols;
        dst[i] = static_cast<int8_t>(s8[r * scols + (i - r * cols)]);
      }
    }
  }
}

// The same for a destination that is not 16-byte aligned: one byte per step.
__global__ void __launch_bounds__(256) crop_planes_bytes_kernel(const int8_t* __restrict__ src, int64_t rows,
                                                                int64_t scols, uint32_t planes,
                                                                int8_t* __restrict__ dst, int64_t cols) {
  const int64_t total = static_cast<int64_t>(planes) * rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols;
    dst[i] = src[r * scols + (i - r * cols)];
  }
}

unsigned flat_grid(int64_t work, int sm_count) {
  const int64_t blocks = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count) * 16;
  return static_cast<unsigned>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}



struct PadPlan {
  int64_t kp, np;
  bool pad_a, pad_b, pad_c;
  uint64_t a_bytes, b_bytes, c_bytes;  // per task, 256-rounded (0 when not padded)
  uint64_t per_task() const { return a_bytes + b_bytes + c_bytes; }
};

PadPlan pad_plan(const PlaneGemmProblem& prob, const PlaneGemmTask* tasks, uint32_t count) {
  PadPlan pp{};
  pp.kp = round16(prob.k);
  pp.np = round16(prob.n);
  bool a_mis = false, b_mis = false, c_mis = false;
  for (uint32_t t = 0; t < count; ++t) {
    a_mis |= !aligned16(tasks[t].a);
    b_mis |= !aligned16(tasks[t].b);
    c_mis |= !aligned16(tasks[t].c);
  }
  pp.pad_a = pp.kp != prob.k || a_mis;
  pp.pad_b = pp.kp != prob.k || pp.np != prob.n || b_mis;
  pp.pad_c = pp.np != prob.n || c_mis;
  const uint64_t P = prob.planes;
  pp.a_bytes = pp.pad_a ? round256_u(P * prob.m * pp.kp) : 0;
  pp.b_bytes = pp.pad_b ? round256_u(P * pp.kp * pp.np) : 0;
  pp.c_bytes = pp.pad_c ? round256_u(P * prob.m * pp.np) : 0;
  return pp;
}

uint64_t tc_split_bytes(const PlaneGemmProblem& prob, int sm_count);

bool padded_path_possible(const PlaneGemmProblem& prob) {
  return prob.m > 0 && prob.n >= 16 && prob.k > 0 && prob.task_count > 0 && prob.planes > 0 && prob.planes <= 20 &&
         round16(prob.m) <= (int64_t(1) << 31) && round16(prob.n) <= (int64_t(1) << 31) &&
         round16(prob.k) <= (int64_t(1) << 31) && encode_fn() != nullptr;
}

// Scratch of the padded run: padded planes for one chunk of tasks and the
// split-K sums of the padded chunk.
uint64_t padded_scratch_bytes(const PlaneGemmProblem& prob, int sm_count) {
  const uint32_t chunk = prob.task_count < kMaxGroupTasks ? prob.task_count : kMaxGroupTasks;
  const PadPlan pp = pad_plan(prob, prob.tasks, chunk);
  PlaneGemmProblem padded = prob;
  padded.k = pp.kp;
  padded.n = pp.np;
  padded.task_count = chunk;
  return chunk * pp.per_task() + tc_split_bytes(padded, sm_count);
}

}  // namespace

namespace {
uint64_t tc_split_bytes(const PlaneGemmProblem& prob, int sm_count) {
  const uint32_t chunk = prob.task_count < kMaxGroupTasks ? prob.task_count : kMaxGroupTasks;
  PlaneGemmProblem one = prob;
  one.task_count = chunk;
  const TcSchedule s = tc_schedule(one, sm_count);
  if (s.splits <= 1) return 0;
  return static_cast<uint64_t>(prob.m) * prob.n * prob.planes * chunk * sizeof(int32_t);
}

cudaError_t padded_plane_gemm(const PlaneGemmProblem& prob, int sm_count, void* scratch, uint64_t scratch_bytes,
                              uint32_t* dev_status, cudaStream_t stream) {
  for (uint32_t t0 = 0; t0 < prob.task_count; t0 += kMaxGroupTasks) {
    const uint32_t count = prob.task_count - t0 < static_cast<uint32_t>(kMaxGroupTasks)
                               ? prob.task_count - t0
                               : static_cast<uint32_t>(kMaxGroupTasks);
    const PlaneGemmTask* tasks = prob.tasks + t0;
    const PadPlan pp = pad_plan(prob, tasks, count);
    uint8_t* base = static_cast<uint8_t*>(scratch);
    const uint64_t pads = count * pp.per_task();
    if (pads > scratch_bytes) return cudaErrorInvalidValue;
    PlaneGemmTask padded_tasks[kMaxGroupTasks];
    for (uint32_t t = 0; t < count; ++t) {
      uint8_t* slot = base + t * pp.per_task();
      int8_t* a = pp.pad_a ? reinterpret_cast<int8_t*>(slot) : const_cast<int8_t*>(tasks[t].a);
      int8_t* b = pp.pad_b ? reinterpret_cast<int8_t*>(slot + pp.a_bytes) : const_cast<int8_t*>(tasks[t].b);
      int8_t* c = pp.pad_c ? reinterpret_cast<int8_t*>(slot + pp.a_bytes + pp.b_bytes) : tasks[t].c;
      if (pp.pad_a)
        pad_planes_kernel<<<flat_grid(prob.planes * prob.m * (pp.kp / 16), sm_count), 256, 0, stream>>>(
            tasks[t].a, prob.m, prob.k, prob.planes, a, prob.m, pp.kp);
      if (pp.pad_b)
        pad_planes_kernel<<<flat_grid(prob.planes * pp.kp * (pp.np / 16), sm_count), 256, 0, stream>>>(
            tasks[t].b, prob.k, prob.n, prob.planes, b, pp.kp, pp.np);
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return e;
      padded_tasks[t] = {a, b, c};
    }
    PlaneGemmProblem padded = prob;
    padded.k = pp.kp;
    padded.n = pp.np;
    padded.tasks = padded_tasks;
    padded.task_count = count;
    if (!tensor_core_path_supported(padded)) return cudaErrorInvalidValue;
    cudaError_t e = tc_plane_gemm(padded, sm_count, base + pads, scratch_bytes - pads, dev_status, stream);
    if (e != cudaSuccess) return e;
    if (pp.pad_c) {
      for (uint32_t t = 0; t < count; ++t) {
        const int64_t total = static_cast<int64_t>(prob.planes) * prob.m * prob.n;
        if (aligned16(tasks[t].c))
          crop_planes_kernel<<<flat_grid((total + 15) / 16, sm_count), 256, 0, stream>>>(
              padded_tasks[t].c, prob.m, pp.np, prob.planes, tasks[t].c, prob.n);
        else
          crop_planes_bytes_kernel<<<flat_grid(total, sm_count), 256, 0, stream>>>(padded_tasks[t].c, prob.m, pp.np,
                                                                                   prob.planes, tasks[t].c, prob.n);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
      }
    }
  }
  return cudaSuccess;
}
}  // namespace

uint64_t plane_gemm_scratch_bytes(const PlaneGemmProblem& prob, int sm_count) {
  if (!tensor_core_path_supported(prob)) {
    if (skinny_path_supported(prob)) return skinny_scratch_bytes(prob);
    return padded_path_possible(prob) ? padded_scratch_bytes(prob, sm_count) : 0;
  }
  const uint32_t chunk = prob.task_count < kMaxGroupTasks ? prob.task_count : kMaxGroupTasks;
  PlaneGemmProblem one = prob;
  one.task_count = chunk;
  const TcSchedule s = tc_schedule(one, sm_count);
  if (s.splits <= 1) return 0;
  return static_cast<uint64_t>(prob.m) * prob.n * prob.planes * chunk * sizeof(int32_t);
}

cudaError_t plane_gemm(const PlaneGemmProblem& prob, GemmPath path, int sm_count, void* scratch,
                       uint64_t scratch_bytes, uint32_t* dev_status, cudaStream_t stream, GemmPath* used) {
  const bool tc_ok = tensor_core_path_supported(prob);
  if (path == GemmPath::TensorCore && !tc_ok) return cudaErrorInvalidValue;
  if (path == GemmPath::Auto && !tc_ok && skinny_path_supported(prob) && scratch &&
      scratch_bytes >= skinny_scratch_bytes(prob)) {
    if (used) *used = GemmPath::Simt;  // the narrow-output kernel (CUDA cores)
    return skinny_plane_gemm(prob, scratch, scratch_bytes, stream, sm_count);
  }
  if (path == GemmPath::Auto && !tc_ok && padded_path_possible(prob) && scratch &&
      scratch_bytes >= padded_scratch_bytes(prob, sm_count)) {
    if (used) *used = GemmPath::TensorCore;  // zero-padded copies on the tensor cores
    return padded_plane_gemm(prob, sm_count, scratch, scratch_bytes, dev_status, stream);
  }
  if (path == GemmPath::Simt || !tc_ok) {
    if (used) *used = GemmPath::Simt;
    return simt_plane_gemm(prob, stream);
  }
  if (used) *used = GemmPath::TensorCore;
  for (uint32_t t0 = 0; t0 < prob.task_count; t0 += kMaxGroupTasks) {
    PlaneGemmProblem chunk = prob;
    chunk.tasks = prob.tasks + t0;
    chunk.task_count = prob.task_count - t0 < static_cast<uint32_t>(kMaxGroupTasks) ? prob.task_count - t0
                                                                                   : static_cast<uint32_t>(kMaxGroupTasks);
    const cudaError_t e = tc_plane_gemm(chunk, sm_count, scratch, scratch_bytes, dev_status, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// ---- row-slab exchange (plane sharding) ------------------------------------------
bool plane_gemm_scatter_fusable(const PlaneGemmProblem& prob, int sm_count) {
  if (prob.task_count != 1 || !tensor_core_path_supported(prob)) return false;
  return tc_schedule(prob, sm_count).splits <= 1;
}

namespace {
uint64_t local_planes_bytes(const PlaneGemmProblem& prob) {
  return (static_cast<uint64_t>(prob.m) * prob.n * prob.planes + 255) / 256 * 256;
}
}  // namespace

uint64_t plane_gemm_scatter_scratch_bytes(const PlaneGemmProblem& prob, int sm_count, bool copy_exchange) {
  if (!copy_exchange && plane_gemm_scatter_fusable(prob, sm_count)) return 0;
  return local_planes_bytes(prob) + plane_gemm_scratch_bytes(prob, sm_count);
}

cudaError_t plane_gemm_scatter(const PlaneGemmProblem& prob, const SlabScatter& sc, bool copy_exchange,
                               int sm_count, void* scratch, uint64_t scratch_bytes, uint32_t* dev_status,
                               cudaStream_t stream, bool* fused_used) {
  if (prob.task_count != 1 || prob.planes == 0 || prob.planes > 20 || !sc.slab_dst || !sc.dst_plane ||
      sc.slab_count == 0 || sc.slab_count > static_cast<uint32_t>(kMaxSlabs) || sc.slab_rows <= 0)
    return cudaErrorInvalidValue;
  // Every slab holds at least one row and together they cover exactly m rows.
  if (static_cast<int64_t>(sc.slab_count - 1) * sc.slab_rows >= prob.m ||
      static_cast<int64_t>(sc.slab_count) * sc.slab_rows < prob.m)
    return cudaErrorInvalidValue;
  for (uint32_t sl = 0; sl < sc.slab_count; ++sl)
    if (sc.slab_dst[sl] == nullptr) return cudaErrorInvalidValue;
  for (uint32_t p = 0; p < prob.planes; ++p)
    if (sc.dst_plane[p] >= 20) return cudaErrorInvalidValue;
  PlaneGemmTask task = prob.tasks[0];
  task.c = sc.slab_dst[0];  // stands in for C in the alignment check of the fused form
  PlaneGemmProblem one = prob;
  one.tasks = &task;
  bool aligned = true;
  for (uint32_t sl = 0; sl < sc.slab_count; ++sl) aligned &= reinterpret_cast<uintptr_t>(sc.slab_dst[sl]) % 16 == 0;
  if (!copy_exchange && aligned && plane_gemm_scatter_fusable(one, sm_count)) {
    if (fused_used) *fused_used = true;
    return tc_plane_gemm(one, sm_count, nullptr, 0, dev_status, stream, nullptr, &sc);
  }
  if (fused_used) *fused_used = false;
  const uint64_t local = local_planes_bytes(prob);
  if (!scratch || scratch_bytes < local) return cudaErrorInvalidValue;
  task.c = static_cast<int8_t*>(scratch);
  cudaError_t e = plane_gemm(one, GemmPath::Auto, sm_count, static_cast<uint8_t*>(scratch) + local,
                             scratch_bytes - local, dev_status, stream);
  if (e != cudaSuccess) return e;
  const uint64_t plane_elems = static_cast<uint64_t>(prob.m) * prob.n;
  for (uint32_t p = 0; p < prob.planes; ++p) {
    for (uint32_t sl = 0; sl < sc.slab_count; ++sl) {
      const int64_t row0 = static_cast<int64_t>(sl) * sc.slab_rows;
      const int64_t rows = std::min<int64_t>(sc.slab_rows, prob.m - row0);
      const uint64_t bytes = static_cast<uint64_t>(rows) * prob.n;
      e = cudaMemcpyAsync(sc.slab_dst[sl] + static_cast<uint64_t>(sc.dst_plane[p]) * bytes,
                          task.c + p * plane_elems + static_cast<uint64_t>(row0) * prob.n, bytes, cudaMemcpyDefault,
                          stream);
      if (e != cudaSuccess) return e;
    }
  }
  return cudaSuccess;
}

// ---- scheduled (per-tile prefix) plane GEMM --------------------------------------
namespace {

uint32_t log2_u32(uint32_t v) {
  uint32_t s = 0;
  while ((1u << s) < v) ++s;
  return s;
}

// Host-side work lists of a scheduled run.
struct ScheduledWork {
  std::vector<uint64_t> units;  // tensor-core units, plane-outer
  std::vector<ZeroTile> zeros;  // proven-zero schedule tiles
  TcSchedule s{};
  bool tc = false;
};

ScheduledWork scheduled_work(const PlaneGemmProblem& prob, const PlaneSchedule& sched, int sm_count) {
  ScheduledWork w;
  const uint64_t tiles = sched.tile_rows * sched.tile_cols;
  for (uint64_t t = 0; t < tiles; ++t) {
    const uint8_t sel = sched.tile_sel[t];
    if (!(sel & 0x80u) || (sel & 0x7Fu) == 0) continue;
    const uint64_t tr = t / sched.tile_cols, tc = t % sched.tile_cols;
    ZeroTile z{};
    z.row0 = static_cast<int64_t>(tr * sched.tile_m);
    z.col0 = static_cast<int64_t>(tc * sched.tile_n);
    z.rows = std::min<int64_t>(sched.tile_m, prob.m - z.row0);
    z.cols = std::min<int64_t>(sched.tile_n, prob.n - z.col0);
    z.planes = sel & 0x7Fu;
    w.zeros.push_back(z);
  }
  w.tc = tensor_core_path_supported(prob);
  if (!w.tc) return w;
  w.s = tc_schedule(prob, sm_count);
  // Planes each 128 x 256 kernel tile must compute: the largest selected
  // prefix among the schedule tiles it covers that are not proven zero.
  std::vector<uint8_t> need(static_cast<size_t>(w.s.m_tiles) * w.s.n_tiles, 0);
  for (uint32_t mt = 0; mt < w.s.m_tiles; ++mt)
    for (uint32_t nt = 0; nt < w.s.n_tiles; ++nt) {
      const uint64_t r0 = static_cast<uint64_t>(mt) * BM / sched.tile_m;
      const uint64_t r1 = std::min<uint64_t>((static_cast<uint64_t>(mt) * BM + BM - 1) / sched.tile_m,
                                             sched.tile_rows - 1);
      const uint64_t c0 = static_cast<uint64_t>(nt) * BN / sched.tile_n;
      const uint64_t c1 = std::min<uint64_t>((static_cast<uint64_t>(nt) * BN + BN - 1) / sched.tile_n,
                                             sched.tile_cols - 1);
      uint8_t v = 0;
      for (uint64_t r = r0; r <= r1; ++r)
        for (uint64_t c = c0; c <= c1; ++c) {
          const uint8_t sel = sched.tile_sel[r * sched.tile_cols + c];
          if (!(sel & 0x80u)) v = std::max<uint8_t>(v, sel & 0x7Fu);
        }
      need[static_cast<size_t>(mt) * w.s.n_tiles + nt] = v;
    }
  const uint64_t raster = static_cast<uint64_t>(w.s.m_tiles) * w.s.n_tiles;
  for (uint32_t p = 0; p < prob.planes; ++p)
    for (uint32_t sp = 0; sp < w.s.splits; ++sp)
      for (uint64_t tile = 0; tile < raster; ++tile) {
        // the grouped raster order of decode_unit
        const uint32_t span = GROUP_M * w.s.n_tiles;
        const uint32_t group = static_cast<uint32_t>(tile / span);
        const uint32_t first_m = group * GROUP_M;
        const uint32_t gsize = std::min<uint32_t>(w.s.m_tiles - first_m, GROUP_M);
        const uint32_t in_group = static_cast<uint32_t>(tile % span);
        const uint32_t mt = first_m + in_group % gsize, nt = in_group / gsize;
        if (p >= need[static_cast<size_t>(mt) * w.s.n_tiles + nt]) continue;
        w.units.push_back(static_cast<uint64_t>(p) | (static_cast<uint64_t>(sp) << 8) |
                          (static_cast<uint64_t>(mt) << 24) | (static_cast<uint64_t>(nt) << 44));
      }
  return w;
}

uint64_t r256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

// Cells whose tile needs plane p take the value computed into `src`.
__global__ void __launch_bounds__(256) masked_copy_kernel(const int8_t* __restrict__ src, int8_t* __restrict__ dst,
                                                          int64_t m, int64_t n, uint32_t planes,
                                                          const uint8_t* __restrict__ tile_sel, uint32_t shift_m,
                                                          uint32_t shift_n, uint32_t cols) {
  for (int64_t row = blockIdx.y; row < m; row += gridDim.y)
    for (int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; col < n;
         col += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const uint8_t sel = tile_sel[(row >> shift_m) * cols + (col >> shift_n)];
      if (sel & 0x80u) continue;
      for (uint32_t p = 0; p < (sel & 0x7Fu) && p < planes; ++p)
        dst[static_cast<int64_t>(p) * m * n + row * n + col] = src[static_cast<int64_t>(p) * m * n + row * n + col];
    }
}

}  // namespace

uint64_t plane_gemm_scheduled_scratch_bytes(const PlaneGemmProblem& prob, const PlaneSchedule& sched, int sm_count) {
  const ScheduledWork w = scheduled_work(prob, sched, sm_count);
  const uint64_t tiles = sched.tile_rows * sched.tile_cols;
  uint64_t bytes = r256(tiles) + r256(w.zeros.size() * sizeof(ZeroTile));
  if (w.tc)
    bytes += r256(w.units.size() * sizeof(uint64_t)) + r256(plane_gemm_scratch_bytes(prob, sm_count));
  else
    bytes += r256(static_cast<uint64_t>(prob.planes) * prob.m * prob.n);  // SIMT result before the masked copy
  return bytes;
}

cudaError_t plane_gemm_scheduled(const PlaneGemmProblem& prob, const PlaneSchedule& sched, int sm_count,
                                 void* scratch, uint64_t scratch_bytes, uint32_t* dev_status, cudaStream_t stream) {
  if (prob.task_count != 1 || sched.tile_m < 64 || sched.tile_n < 64) return cudaErrorInvalidValue;
  const ScheduledWork w = scheduled_work(prob, sched, sm_count);
  if (scratch_bytes < plane_gemm_scheduled_scratch_bytes(prob, sched, sm_count) || !scratch)
    return cudaErrorInvalidValue;
  const uint64_t tiles = sched.tile_rows * sched.tile_cols;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  uint8_t* sel_dev = base;
  base += r256(tiles);
  auto* zeros_dev = reinterpret_cast<ZeroTile*>(base);
  base += r256(w.zeros.size() * sizeof(ZeroTile));
  cudaError_t e = cudaMemcpyAsync(sel_dev, sched.tile_sel, tiles, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  int8_t* c = prob.tasks[0].c;
  const uint32_t shift_m = log2_u32(sched.tile_m), shift_n = log2_u32(sched.tile_n);
  const uint32_t cols = static_cast<uint32_t>(sched.tile_cols);
  if (!w.zeros.empty()) {
    e = cudaMemcpyAsync(zeros_dev, w.zeros.data(), w.zeros.size() * sizeof(ZeroTile), cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    const unsigned blocks = static_cast<unsigned>(std::min<size_t>(w.zeros.size(), 148 * 8));
    zero_tiles_kernel<<<blocks, 256, 0, stream>>>(zeros_dev, static_cast<uint32_t>(w.zeros.size()), c, prob.m, prob.n);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  if (!w.tc) {
    // Unaligned shapes: every plane into scratch with the SIMT kernel, then the
    // cells each tile needs into C.
    int8_t* tmp = reinterpret_cast<int8_t*>(base);
    PlaneGemmTask task = prob.tasks[0];
    task.c = tmp;
    PlaneGemmProblem p2 = prob;
    p2.tasks = &task;
    if ((e = simt_plane_gemm(p2, stream)) != cudaSuccess) return e;
    const int64_t by = prob.m < 65535 ? prob.m : 65535;
    const int64_t bx = std::min<int64_t>((prob.n + 255) / 256, 64);
    masked_copy_kernel<<<dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by)), 256, 0, stream>>>(
        tmp, c, prob.m, prob.n, prob.planes, sel_dev, shift_m, shift_n, cols);
    return cudaGetLastError();
  }
  if (w.units.empty()) return cudaSuccess;
  auto* units_dev = reinterpret_cast<uint64_t*>(base);
  base += r256(w.units.size() * sizeof(uint64_t));
  e = cudaMemcpyAsync(units_dev, w.units.data(), w.units.size() * sizeof(uint64_t), cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  TcScheduleUnits su{units_dev, w.units.size(), sel_dev, shift_m, shift_n, cols};
  const uint64_t rest = scratch_bytes - static_cast<uint64_t>(base - static_cast<uint8_t*>(scratch));
  return tc_plane_gemm(prob, sm_count, base, rest, dev_status, stream, &su);
}

// ---- GEMM followed by the bounded export --------------------------------------
// Scratch: C planes (planes * m * n bytes, 256-byte aligned), then the split-K
// sums of plane_gemm.
uint64_t gemm_export_bounded_scratch_bytes(const PlaneGemmProblem& prob, int sm_count) {
  const uint64_t planes = (static_cast<uint64_t>(prob.planes) * prob.m * prob.n + 255) & ~uint64_t(255);
  return planes + plane_gemm_scratch_bytes(prob, sm_count);
}

cudaError_t gemm_export_bounded(const PlaneGemmProblem& prob, bool is_signed, uint64_t bound, void* out, int64_t ld,
                                int sm_count, void* scratch, uint64_t scratch_bytes, uint32_t* dev_status,
                                cudaStream_t stream) {
  if (prob.task_count != 1) return cudaErrorInvalidValue;
  const uint64_t need = gemm_export_bounded_scratch_bytes(prob, sm_count);
  if (!scratch || scratch_bytes < need) return cudaErrorInvalidValue;
  const uint64_t planes = (static_cast<uint64_t>(prob.planes) * prob.m * prob.n + 255) & ~uint64_t(255);
  int8_t* c = static_cast<int8_t*>(scratch);
  PlaneGemmTask task = prob.tasks[0];
  task.c = c;
  PlaneGemmProblem p2 = prob;
  p2.tasks = &task;
  const cudaError_t e = plane_gemm(p2, GemmPath::Auto, sm_count, static_cast<uint8_t*>(scratch) + planes,
                                   scratch_bytes - planes, dev_status, stream);
  if (e != cudaSuccess) return e;
  return is_signed ? export_i64(c, prob.m, prob.n, prob.planes, bound, static_cast<int64_t*>(out), ld, dev_status, stream)
                   : export_u64(c, prob.m, prob.n, prob.planes, bound, static_cast<uint64_t*>(out), ld, dev_status,
                                stream);
}

}  // namespace rns8cuda
