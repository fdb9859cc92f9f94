/* Device-pointer seam of the sm_100a backend.
 *
 * These entry points take raw device pointers and a CUDA stream (passed as
 * void*, NULL = the legacy default stream) and only enqueue work: they do not
 * synchronise, allocate, or copy to or from the host. They are the CUDA
 * counterparts of the reference's internal backend seam
 * (src/backend_hip_direct/hip_backend.hpp:246 hip_direct_pack_i64_device,
 * :346 hip_direct_gemm_rns_device, :758 hip_direct_gemm_finite_u8_resident_device,
 * :835 hip_direct_export_i64_device, :933 hip_direct_export_exact_wide_*),
 * exported with plain C types so a caller that already holds residue planes
 * in HBM can drive the pipeline without host round trips.
 *
 * Layout: residue planes are modulus-major and compact; plane p of an
 * R x C matrix is the int8 array base[p*R*C .. (p+1)*R*C) in row-major order.
 * Plane p uses modulus rns8_default_modulus(p).
 *
 * Device status words: export and GEMM calls OR an error code into *d_status
 * (5 = a value violated its range contract, 0x100 = a bounded device wait ran
 * out). The caller zeroes the word before the call and reads it after
 * synchronising. On a non-zero status the destination contents are
 * unspecified.
 *
 * Return value: RNS8_SUCCESS when the work was enqueued, RNS8_INVALID_ARGUMENT
 * for malformed arguments, RNS8_BACKEND_FAILURE for a CUDA launch error. */
#ifndef RNS8_RNS8_CUDA_H
#define RNS8_RNS8_CUDA_H

#include <stdint.h>

#include "rns8/rns8.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Kernel selection for the plane GEMM. AUTO uses the tcgen05 tensor-core
 * kernel whenever K and N are multiples of 16 and the SIMT kernel otherwise. */
#define RNS8_CUDA_GEMM_AUTO 0u
#define RNS8_CUDA_GEMM_TENSOR_CORE 1u
#define RNS8_CUDA_GEMM_SIMT 2u

/* Native int64/uint64 (row-major, leading dimension ld >= cols) -> prefix
 * centered residue planes. Replaces hip_backend.hpp:246 / :296. */
RNS8_API rns8_status rns8_cuda_pack_i64_device(int device_id, const int64_t* d_src, int64_t rows, int64_t cols,
                                               int64_t ld, uint32_t prefix, int8_t* d_planes, void* stream);
RNS8_API rns8_status rns8_cuda_pack_u64_device(int device_id, const uint64_t* d_src, int64_t rows, int64_t cols,
                                               int64_t ld, uint32_t prefix, int8_t* d_planes, void* stream);
/* uint8 -> centered residues modulo `modulus` in [2, 256]. Replaces
 * hip_backend.hpp pack_finite_u8. */
RNS8_API rns8_status rns8_cuda_pack_finite_u8_device(int device_id, const uint8_t* d_src, int64_t rows, int64_t cols,
                                                     int64_t ld, uint16_t modulus, int8_t* d_residues, void* stream);

/* Scratch bytes the plane GEMM needs on this shape (0 = none): split-K sums,
 * and, when K or N is not a multiple of 16, the zero-padded plane copies that
 * let such shapes run on the tensor cores (given less, they run on the CUDA
 * cores). */
RNS8_API uint64_t rns8_cuda_gemm_rns_scratch_bytes(int device_id, int64_t m, int64_t n, int64_t k, uint32_t prefix);

/* Per plane p < prefix: C_p = (A_p x B_p) mod m_p, centered. A is m x k, B is
 * k x n, C is m x n, all compact planes. Replaces hip_backend.hpp:346. */
RNS8_API rns8_status rns8_cuda_gemm_rns_device(int device_id, const int8_t* d_a, const int8_t* d_b, int8_t* d_c,
                                               int64_t m, int64_t n, int64_t k, uint32_t prefix, uint32_t gemm_path,
                                               void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status,
                                               void* stream);

/* Plane GEMM followed by the bounded Garner export, in one call: per plane
 * p < prefix, C_p = A_p x B_p mod m_p into planes held in d_scratch, then
 * every cell is reconstructed and written to d_out[row * ld + col] as int64
 * (is_signed) or uint64, with the bound contract of
 * rns8_cuda_export_i64_device. d_scratch must hold
 * rns8_cuda_gemm_export_bounded_scratch_bytes() bytes. This is
 * hip_backend.hpp:346 followed by :835 for callers that do not keep the
 * residue planes of C. */
RNS8_API uint64_t rns8_cuda_gemm_export_bounded_scratch_bytes(int device_id, int64_t m, int64_t n, int64_t k,
                                                              uint32_t prefix);
RNS8_API rns8_status rns8_cuda_gemm_export_bounded_device(int device_id, const int8_t* d_a, const int8_t* d_b,
                                                          int64_t m, int64_t n, int64_t k, uint32_t prefix,
                                                          uint32_t is_signed, uint64_t bound, void* d_out, int64_t ld,
                                                          void* d_scratch, uint64_t scratch_bytes,
                                                          uint32_t* d_status, void* stream);

/* The plane GEMM above for callers that cannot allocate device memory (a
 * host whose device memory belongs to a fixed-budget allocator, a foreign-
 * language caller holding only its input and output buffers, or a loop where
 * cudaMalloc/cudaFree would synchronise the device). It has no counterpart in
 * the reference. Scratch and the status word come from a file-scope device
 * array of 8 MiB (+256 B) that every GPU loading the library holds until
 * exit; the call allocates nothing. Shapes whose split-K sums need more than
 * 8 MiB (prefix * m * n * 4 bytes when K is split) return
 * RNS8_WORKSPACE_TOO_SMALL. The first call on a device looks up the array's
 * device address (make it before any stream capture) and keeps it for the
 * life of the process: do not call this across a cudaDeviceReset, which
 * reloads the array elsewhere. All calls share the array: each clears what
 * must start at zero, and calls that overlap on the GPU race. A device_id
 * that is negative or not below the visible device count returns
 * RNS8_INVALID_ARGUMENT; the caller's current device is unchanged on return.
 * The call enqueues on `stream`, then synchronises that stream and returns
 * RNS8_BACKEND_FAILURE if a bounded device wait ran out. */
RNS8_API rns8_status rns8_cuda_gemm_rns_device_no_alloc(int device_id, const int8_t* d_a, const int8_t* d_b,
                                                        int8_t* d_c, int64_t m, int64_t n, int64_t k,
                                                        uint32_t prefix, void* stream);

/* Same-shape batch of single-plane GEMMs modulo `modulus` (finite u8 ring or
 * field). d_a/d_b/d_c are host arrays of task_count device pointers.
 * Replaces hip_backend.hpp:758 and the grouped finite dispatch. */
RNS8_API uint64_t rns8_cuda_gemm_finite_u8_scratch_bytes(int device_id, int64_t m, int64_t n, int64_t k,
                                                         uint32_t task_count);
RNS8_API rns8_status rns8_cuda_gemm_finite_u8_grouped_device(int device_id, const int8_t* const* d_a,
                                                             const int8_t* const* d_b, int8_t* const* d_c,
                                                             uint32_t task_count, int64_t m, int64_t n, int64_t k,
                                                             uint16_t modulus, uint32_t gemm_path, void* d_scratch,
                                                             uint64_t scratch_bytes, uint32_t* d_status,
                                                             void* stream);

/* Garner reconstruction + bounded export. The bound must satisfy the plan
 * contract for the prefix (product > 2*bound signed, > bound unsigned).
 * Replaces hip_backend.hpp:835 and the u64 variant. */
RNS8_API rns8_status rns8_cuda_export_i64_device(int device_id, const int8_t* d_planes, int64_t m, int64_t n,
                                                 uint32_t prefix, uint64_t bound, int64_t* d_dst, int64_t ld,
                                                 uint32_t* d_status, void* stream);
RNS8_API rns8_status rns8_cuda_export_u64_device(int device_id, const int8_t* d_planes, int64_t m, int64_t n,
                                                 uint32_t prefix, uint64_t bound, uint64_t* d_dst, int64_t ld,
                                                 uint32_t* d_status, void* stream);
/* Exact-wide limbs: dst[(row*ld + col)*limb_count + limb]. Replaces
 * hip_backend.hpp:933 and the unsigned variant. */
RNS8_API rns8_status rns8_cuda_export_limbs_device(int device_id, const int8_t* d_planes, int64_t m, int64_t n,
                                                   uint32_t prefix, uint32_t is_signed, uint32_t limb_count,
                                                   uint64_t* d_dst, int64_t ld, uint32_t* d_status, void* stream);
RNS8_API rns8_status rns8_cuda_export_finite_u8_device(int device_id, const int8_t* d_residues, int64_t m, int64_t n,
                                                       uint16_t modulus, uint8_t* d_dst, int64_t ld, void* stream);

/* WRAP_U64_MOD_2_64 byte-limb path (reference src/backend_wrap64/wrap64_hip.hpp:
 * 12 pack, :22 GEMM, :31 export). A wrap64 matrix is eight unsigned byte
 * planes, limb-major: byte l of cell (r, c) of an R x C matrix is
 * d_limbs[l*R*C + r*C + c].
 * pack:   uint64 d_src (row-major, ld >= cols) -> d_limbs (8*rows*cols bytes).
 * gemm:   d_c (m x n uint64, compact row-major) = A x B mod 2^64 from byte
 *         planes; the tensor-core path (K and N multiples of 16) ORs 0x100
 *         into *d_status if a bounded wait ran out (d_status may be NULL only
 *         for RNS8_CUDA_GEMM_SIMT).
 * export: d_limbs -> uint64 d_dst[row*ld + col]. */
RNS8_API rns8_status rns8_cuda_pack_wrap_u64_device(int device_id, const uint64_t* d_src, int64_t rows, int64_t cols,
                                                    int64_t ld, uint8_t* d_limbs, void* stream);
RNS8_API rns8_status rns8_cuda_gemm_wrap_u64_device(int device_id, const uint8_t* d_a_limbs, const uint8_t* d_b_limbs,
                                                    uint64_t* d_c, int64_t m, int64_t n, int64_t k,
                                                    uint32_t gemm_path, uint32_t* d_status, void* stream);
RNS8_API rns8_status rns8_cuda_export_wrap_u64_device(int device_id, const uint8_t* d_limbs, int64_t rows,
                                                      int64_t cols, uint64_t* d_dst, int64_t ld, void* stream);

/* Exact-wide admission proof (reference src/core/exact_range.hpp:51-154 and
 * api_pack.cpp:61-64) of A x B for native matrices already in device memory:
 * A is m x k, B is k x n, both compact (ld = cols) int64 (is_signed = 1) or
 * uint64 (0). Writes the admission bound (the smallest valid bound on every
 * |C[r][c]|, maximised over the cells) to out_bound[4] and the largest |a|
 * and |b| to out_a_max[4] / out_b_max[4], all 256-bit little-endian.
 * out_row_stats[8*m] / out_col_stats[8*n], when not NULL, receive per output
 * row / column the maximum and the sum of the cell bounds (4 + 4 limbs): the
 * records an exact-wide GEMM keeps for its output. A GEMM is admitted when
 * 2*bound < M_P (signed) or bound < M_P (unsigned). The reference computes
 * this on the host inside pack and GEMM; here it runs on the device. Unlike
 * the other calls in this header it allocates device scratch, synchronises
 * `stream` and writes host memory. */
RNS8_API rns8_status rns8_cuda_exact_gemm_bound_device(int device_id, const void* d_a, const void* d_b, int64_t m,
                                                       int64_t n, int64_t k, uint32_t is_signed, uint64_t* out_bound,
                                                       uint64_t* out_a_max, uint64_t* out_b_max,
                                                       uint64_t* out_row_stats, uint64_t* out_col_stats,
                                                       void* stream);

/* Host-only: run the plan validation and prefix schedule of rns8_create_plan
 * for a descriptor without a context (no device needed). Writes the selected
 * and required prefix and the effective output bound on success. */
RNS8_API rns8_status rns8_cuda_plan_probe(const rns8_gemm_desc* desc, uint32_t* selected_prefix,
                                          uint32_t* required_prefix, uint64_t* effective_bound);

/* Host-only: the tile schedule rns8_create_plan would build for a descriptor
 * (per-tile bound plans: required and selected prefix, group and flags per
 * tile), with the rns8_get_plan_tile_schedule contract (written = tile count;
 * RNS8_WORKSPACE_TOO_SMALL when capacity is short). info may be NULL. */
RNS8_API rns8_status rns8_cuda_plan_tile_schedule_probe(const rns8_gemm_desc* desc,
                                                        rns8_plan_tile_schedule_entry* entries, uint64_t capacity,
                                                        uint64_t* written, rns8_plan_schedule_info* info);

/* ---- Plane sharding across GPUs (no counterpart in the reference, which runs
 * on one device; its research spec describes splitting by modulus). Every GPU
 * packs and multiplies a subset of the residue planes for all of C, and every
 * GPU then needs all planes of its own row slab of C to reconstruct it. The
 * exchange is a row-slab scatter: the plane GEMM's epilogue stores each output
 * row straight into the slab owner's buffer, over NVLink when the owner is a
 * peer GPU whose buffer is mapped into this process (rns8_cuda_ipc_*). */

/* Pack only the planes plane_index[0..plane_count) (ladder indices < 20):
 * plane j of d_planes holds the centered residues modulo ladder entry
 * plane_index[j], compact (rows x cols). */
RNS8_API rns8_status rns8_cuda_pack_i64_planes_device(int device_id, const int64_t* d_src, int64_t rows, int64_t cols,
                                                      int64_t ld, const uint32_t* plane_index, uint32_t plane_count,
                                                      int8_t* d_planes, void* stream);
RNS8_API rns8_status rns8_cuda_pack_u64_planes_device(int device_id, const uint64_t* d_src, int64_t rows,
                                                      int64_t cols, int64_t ld, const uint32_t* plane_index,
                                                      uint32_t plane_count, int8_t* d_planes, void* stream);

#define RNS8_CUDA_EXCHANGE_FUSED 0u /* epilogue stores into the slab buffers (copy form when it cannot) */
#define RNS8_CUDA_EXCHANGE_COPY 1u  /* local planes in scratch, then one device copy per (plane, slab) */

/* Scratch for rns8_cuda_gemm_rns_slabs_device (0 when the fused form runs). */
RNS8_API uint64_t rns8_cuda_gemm_rns_slabs_scratch_bytes(int device_id, int64_t m, int64_t n, int64_t k,
                                                         uint32_t plane_count, uint32_t exchange);
/* Per local plane j: C_j = (A_j x B_j) mod ladder[plane_index[j]], A (m x k)
 * and B (k x n) compact planes as packed above. Output rows are split into
 * slab_count (<= 8) slabs of slab_rows rows (the last may be shorter, none
 * empty); slab s's rows go to slab_dst[s] (a host array of device pointers,
 * this GPU's or a mapped peer's), which holds planes at stride rows_s * n:
 * local plane j lands in plane slot plane_index[j], row r at (r - s *
 * slab_rows) * n. The call only enqueues; the caller orders it against the
 * slab owners' readers (a barrier across GPUs before the owners export).
 * *out_fused (may be NULL) tells whether the fused form ran. */
RNS8_API rns8_status rns8_cuda_gemm_rns_slabs_device(int device_id, const int8_t* d_a, const int8_t* d_b, int64_t m,
                                                     int64_t n, int64_t k, const uint32_t* plane_index,
                                                     uint32_t plane_count, int8_t* const* slab_dst,
                                                     uint32_t slab_count, int64_t slab_rows, uint32_t exchange,
                                                     void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status,
                                                     uint32_t* out_fused, void* stream);

/* Device buffers shared between processes (one process per GPU): allocate a
 * buffer and its 64-byte IPC handle, open a peer's handle in this process
 * (peer access enabled), close an opened mapping, free an allocation. */
#define RNS8_CUDA_IPC_HANDLE_BYTES 64
RNS8_API rns8_status rns8_cuda_ipc_alloc(int device_id, uint64_t bytes, void** d_ptr, uint8_t* handle);
RNS8_API rns8_status rns8_cuda_ipc_free(int device_id, void* d_ptr);
RNS8_API rns8_status rns8_cuda_ipc_open(int device_id, const uint8_t* handle, void** d_ptr);
RNS8_API rns8_status rns8_cuda_ipc_close(int device_id, void* d_ptr);

/* Failure detection without a fault: launches one CTA that waits on an
 * mbarrier with the bounded wait the GEMM kernels use. arrive = 1: a thread
 * arrives first and the call returns RNS8_SUCCESS. arrive = 0: nothing arrives,
 * the wait gives up after budget_cycles SM cycles (1 .. 4e9), the kernel sets
 * the timeout bit in *d_status and the call returns RNS8_BACKEND_FAILURE, as
 * any call whose kernel wait ran out does; the context stays usable.
 * Synchronises `stream`. */
RNS8_API rns8_status rns8_cuda_wait_probe(int device_id, uint32_t arrive, uint64_t budget_cycles,
                                          uint32_t* d_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RNS8_RNS8_CUDA_H */
