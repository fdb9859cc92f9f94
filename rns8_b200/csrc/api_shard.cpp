// Plane-sharding seam (include/rns8/rns8_cuda.h): pack of selected planes, the
// row-slab scatter plane GEMM, and the IPC helpers that map one process's
// device buffer into another's. Enqueue-only like the rest of the seam, except
// the IPC calls, which allocate, map and free.
#include <cstring>

#include "api_internal.hpp"

namespace {

using rns8host::cuda_status;


int sm_count_of(int device_id) {
  int count = 0;
  if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device_id) != cudaSuccess || count <= 0) return 148;
  return count;
}

rns8_status launch_result(cudaError_t e) {
  if (e == cudaErrorInvalidValue) return RNS8_INVALID_ARGUMENT;
  return cuda_status(e);
}

bool valid_planes(const uint32_t* plane_index, uint32_t count) {
  if (!plane_index || count == 0 || count > RNS8_MAX_SUPPORTED_PREFIX) return false;
  for (uint32_t j = 0; j < count; ++j)
    if (plane_index[j] >= RNS8_MAX_SUPPORTED_PREFIX) return false;
  return true;
}

rns8cuda::PlaneGemmProblem subset_problem(int64_t m, int64_t n, int64_t k, const uint32_t* plane_index,
                                          uint32_t count, const rns8cuda::PlaneGemmTask* task) {
  rns8cuda::PlaneGemmProblem prob{};
  prob.m = m;
  prob.n = n;
  prob.k = k;
  prob.planes = count;
  for (uint32_t j = 0; j < count; ++j) prob.moduli[j] = rns8ladder::kLadder[plane_index[j]];
  prob.task_count = 1;
  prob.tasks = task;
  return prob;
}

}  // namespace

extern "C" rns8_status rns8_cuda_pack_i64_planes_device(int device_id, const int64_t* d_src, int64_t rows,
                                                        int64_t cols, int64_t ld, const uint32_t* plane_index,
                                                        uint32_t plane_count, int8_t* d_planes, void* stream) {
  if (!d_src || !d_planes || !rns8host::valid_matrix_access(rows, cols, ld) || !valid_planes(plane_index, plane_count))
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::pack_planes_i64(d_src, rows, cols, ld, plane_index, plane_count, d_planes,
                                                 static_cast<cudaStream_t>(stream)));
}

extern "C" rns8_status rns8_cuda_pack_u64_planes_device(int device_id, const uint64_t* d_src, int64_t rows,
                                                        int64_t cols, int64_t ld, const uint32_t* plane_index,
                                                        uint32_t plane_count, int8_t* d_planes, void* stream) {
  if (!d_src || !d_planes || !rns8host::valid_matrix_access(rows, cols, ld) || !valid_planes(plane_index, plane_count))
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::pack_planes_u64(d_src, rows, cols, ld, plane_index, plane_count, d_planes,
                                                 static_cast<cudaStream_t>(stream)));
}

extern "C" uint64_t rns8_cuda_gemm_rns_slabs_scratch_bytes(int device_id, int64_t m, int64_t n, int64_t k,
                                                           uint32_t plane_count, uint32_t exchange) {
  if (m <= 0 || n <= 0 || k <= 0 || plane_count == 0 || plane_count > RNS8_MAX_SUPPORTED_PREFIX ||
      exchange > RNS8_CUDA_EXCHANGE_COPY)
    return 0;
  uint32_t index[RNS8_MAX_SUPPORTED_PREFIX];
  for (uint32_t j = 0; j < plane_count; ++j) index[j] = j;  // moduli do not change the size
  const rns8cuda::PlaneGemmTask task{reinterpret_cast<const int8_t*>(256), reinterpret_cast<const int8_t*>(256),
                                     reinterpret_cast<int8_t*>(256)};
  return rns8cuda::plane_gemm_scatter_scratch_bytes(subset_problem(m, n, k, index, plane_count, &task),
                                                    sm_count_of(device_id), exchange == RNS8_CUDA_EXCHANGE_COPY);
}

extern "C" rns8_status rns8_cuda_gemm_rns_slabs_device(int device_id, const int8_t* d_a, const int8_t* d_b, int64_t m,
                                                       int64_t n, int64_t k, const uint32_t* plane_index,
                                                       uint32_t plane_count, int8_t* const* slab_dst,
                                                       uint32_t slab_count, int64_t slab_rows, uint32_t exchange,
                                                       void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status,
                                                       uint32_t* out_fused, void* stream) {
  if (!d_a || !d_b || !slab_dst || !d_status || m <= 0 || n <= 0 || k <= 0 || !valid_planes(plane_index, plane_count) ||
      slab_count == 0 || slab_count > static_cast<uint32_t>(rns8cuda::kMaxSlabs) || slab_rows <= 0 ||
      exchange > RNS8_CUDA_EXCHANGE_COPY)
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  const rns8cuda::PlaneGemmTask task{d_a, d_b, nullptr};
  const rns8cuda::PlaneGemmProblem prob = subset_problem(m, n, k, plane_index, plane_count, &task);
  const rns8cuda::SlabScatter sc{slab_dst, slab_rows, slab_count, plane_index};
  bool fused = false;
  const cudaError_t e =
      rns8cuda::plane_gemm_scatter(prob, sc, exchange == RNS8_CUDA_EXCHANGE_COPY, sm_count_of(device_id), d_scratch,
                                   scratch_bytes, d_status, static_cast<cudaStream_t>(stream), &fused);
  if (out_fused) *out_fused = fused ? 1u : 0u;
  return launch_result(e);
}

extern "C" rns8_status rns8_cuda_ipc_alloc(int device_id, uint64_t bytes, void** d_ptr, uint8_t* handle) {
  if (!d_ptr || !handle || bytes == 0) return RNS8_INVALID_ARGUMENT;
  *d_ptr = nullptr;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return RNS8_INTERNAL_ERROR;
  cudaIpcMemHandle_t h{};
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return RNS8_BACKEND_FAILURE;
  }
  static_assert(sizeof(h) == RNS8_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *d_ptr = p;
  return RNS8_SUCCESS;
}

extern "C" rns8_status rns8_cuda_ipc_free(int device_id, void* d_ptr) {
  if (!d_ptr) return RNS8_SUCCESS;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return cudaFree(d_ptr) == cudaSuccess ? RNS8_SUCCESS : RNS8_BACKEND_FAILURE;
}

extern "C" rns8_status rns8_cuda_ipc_open(int device_id, const uint8_t* handle, void** d_ptr) {
  if (!handle || !d_ptr) return RNS8_INVALID_ARGUMENT;
  *d_ptr = nullptr;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  cudaIpcMemHandle_t h{};
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return RNS8_BACKEND_FAILURE;
  *d_ptr = p;
  return RNS8_SUCCESS;
}

extern "C" rns8_status rns8_cuda_ipc_close(int device_id, void* d_ptr) {
  if (!d_ptr) return RNS8_SUCCESS;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return cudaIpcCloseMemHandle(d_ptr) == cudaSuccess ? RNS8_SUCCESS : RNS8_BACKEND_FAILURE;
}
