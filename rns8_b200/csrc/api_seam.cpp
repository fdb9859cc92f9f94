// Device-pointer seam (include/rns8/rns8_cuda.h): enqueue-only wrappers over
// the sm_100a kernels for callers that hold their data in HBM. Each call sets
// the device, launches on the caller's stream and returns; nothing here
// synchronises, allocates or touches host memory.
#include "api_internal.hpp"

namespace {

using rns8host::cuda_status;

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }


int sm_count_of(int device_id) {
  int count = 0;
  if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device_id) != cudaSuccess || count <= 0) return 148;
  return count;
}

bool valid_prefix(uint32_t p) { return p >= 1 && p <= RNS8_MAX_SUPPORTED_PREFIX; }

rns8cuda::GemmPath path_of(uint32_t v, bool* ok) {
  *ok = v <= RNS8_CUDA_GEMM_SIMT;
  return v == RNS8_CUDA_GEMM_TENSOR_CORE ? rns8cuda::GemmPath::TensorCore
                                         : (v == RNS8_CUDA_GEMM_SIMT ? rns8cuda::GemmPath::Simt : rns8cuda::GemmPath::Auto);
}

rns8_status launch_result(cudaError_t e) {
  if (e == cudaErrorInvalidValue) return RNS8_INVALID_ARGUMENT;
  return cuda_status(e);
}

}  // namespace

extern "C" rns8_status rns8_cuda_pack_i64_device(int device_id, const int64_t* d_src, int64_t rows, int64_t cols,
                                                 int64_t ld, uint32_t prefix, int8_t* d_planes, void* stream) {
  if (!d_src || !d_planes || !rns8host::valid_matrix_access(rows, cols, ld) || !valid_prefix(prefix))
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::pack_i64(d_src, rows, cols, ld, prefix, d_planes, as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_pack_u64_device(int device_id, const uint64_t* d_src, int64_t rows, int64_t cols,
                                                 int64_t ld, uint32_t prefix, int8_t* d_planes, void* stream) {
  if (!d_src || !d_planes || !rns8host::valid_matrix_access(rows, cols, ld) || !valid_prefix(prefix))
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::pack_u64(d_src, rows, cols, ld, prefix, d_planes, as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_pack_finite_u8_device(int device_id, const uint8_t* d_src, int64_t rows, int64_t cols,
                                                       int64_t ld, uint16_t modulus, int8_t* d_residues, void* stream) {
  if (!d_src || !d_residues || !rns8host::valid_matrix_access(rows, cols, ld) || modulus < 2 || modulus > 256)
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::pack_finite_u8(d_src, rows, cols, ld, modulus, d_residues, as_stream(stream)));
}

static rns8cuda::PlaneGemmProblem seam_problem(int64_t m, int64_t n, int64_t k, uint32_t planes, uint16_t finite,
                                               const rns8cuda::PlaneGemmTask* tasks, uint32_t count) {
  rns8cuda::PlaneGemmProblem prob{};
  prob.m = m;
  prob.n = n;
  prob.k = k;
  prob.planes = planes;
  for (uint32_t p = 0; p < planes; ++p) prob.moduli[p] = finite ? finite : rns8ladder::kLadder[p];
  prob.task_count = count;
  prob.tasks = tasks;
  return prob;
}

extern "C" uint64_t rns8_cuda_gemm_rns_scratch_bytes(int device_id, int64_t m, int64_t n, int64_t k, uint32_t prefix) {
  if (m <= 0 || n <= 0 || k <= 0 || !valid_prefix(prefix)) return 0;
  const rns8cuda::PlaneGemmTask task{reinterpret_cast<const int8_t*>(256), reinterpret_cast<const int8_t*>(256),
                                     reinterpret_cast<int8_t*>(256)};
  return rns8cuda::plane_gemm_scratch_bytes(seam_problem(m, n, k, prefix, 0, &task, 1), sm_count_of(device_id));
}

extern "C" rns8_status rns8_cuda_gemm_rns_device(int device_id, const int8_t* d_a, const int8_t* d_b, int8_t* d_c,
                                                 int64_t m, int64_t n, int64_t k, uint32_t prefix, uint32_t gemm_path,
                                                 void* d_scratch, uint64_t scratch_bytes, uint32_t* d_status,
                                                 void* stream) {
  bool path_ok = false;
  const rns8cuda::GemmPath path = path_of(gemm_path, &path_ok);
  if (!d_a || !d_b || !d_c || !d_status || m <= 0 || n <= 0 || k <= 0 || !valid_prefix(prefix) || !path_ok)
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  const rns8cuda::PlaneGemmTask task{d_a, d_b, d_c};
  const auto prob = seam_problem(m, n, k, prefix, 0, &task, 1);
  return launch_result(rns8cuda::plane_gemm(prob, path, sm_count_of(device_id), d_scratch, scratch_bytes, d_status,
                                            as_stream(stream)));
}

extern "C" uint64_t rns8_cuda_gemm_export_bounded_scratch_bytes(int device_id, int64_t m, int64_t n, int64_t k,
                                                                uint32_t prefix) {
  if (m <= 0 || n <= 0 || k <= 0 || !valid_prefix(prefix)) return 0;
  const rns8cuda::PlaneGemmTask task{reinterpret_cast<const int8_t*>(256), reinterpret_cast<const int8_t*>(256),
                                     reinterpret_cast<int8_t*>(256)};
  return rns8cuda::gemm_export_bounded_scratch_bytes(seam_problem(m, n, k, prefix, 0, &task, 1),
                                                     sm_count_of(device_id));
}

extern "C" rns8_status rns8_cuda_gemm_export_bounded_device(int device_id, const int8_t* d_a, const int8_t* d_b,
                                                            int64_t m, int64_t n, int64_t k, uint32_t prefix,
                                                            uint32_t is_signed, uint64_t bound, void* d_out,
                                                            int64_t ld, void* d_scratch, uint64_t scratch_bytes,
                                                            uint32_t* d_status, void* stream) {
  if (!d_a || !d_b || !d_out || !d_status || m <= 0 || n <= 0 || k <= 0 || !valid_prefix(prefix) || ld < n)
    return RNS8_INVALID_ARGUMENT;
  const rns8_status c = is_signed ? rns8host::validate_bound_contract(RNS8_BOUNDED_I64, RNS8_BOUND_GLOBAL_MAX_ABS,
                                                                      bound, prefix)
                                  : rns8host::validate_bound_contract(RNS8_BOUNDED_U64,
                                                                      RNS8_BOUND_GLOBAL_MAX_UNSIGNED, bound, prefix);
  if (c != RNS8_SUCCESS) return c;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  const rns8cuda::PlaneGemmTask task{d_a, d_b, nullptr};
  const auto prob = seam_problem(m, n, k, prefix, 0, &task, 1);
  return launch_result(rns8cuda::gemm_export_bounded(prob, is_signed != 0, bound, d_out, ld, sm_count_of(device_id),
                                                     d_scratch, scratch_bytes, d_status, as_stream(stream)));
}

extern "C" uint64_t rns8_cuda_gemm_finite_u8_scratch_bytes(int device_id, int64_t m, int64_t n, int64_t k,
                                                           uint32_t task_count) {
  if (m <= 0 || n <= 0 || k <= 0 || task_count == 0) return 0;
  std::vector<rns8cuda::PlaneGemmTask> tasks(task_count, rns8cuda::PlaneGemmTask{reinterpret_cast<const int8_t*>(256),
                                                                                  reinterpret_cast<const int8_t*>(256),
                                                                                  reinterpret_cast<int8_t*>(256)});
  return rns8cuda::plane_gemm_scratch_bytes(seam_problem(m, n, k, 1, 251, tasks.data(), task_count),
                                            sm_count_of(device_id));
}

extern "C" rns8_status rns8_cuda_gemm_finite_u8_grouped_device(int device_id, const int8_t* const* d_a,
                                                               const int8_t* const* d_b, int8_t* const* d_c,
                                                               uint32_t task_count, int64_t m, int64_t n, int64_t k,
                                                               uint16_t modulus, uint32_t gemm_path, void* d_scratch,
                                                               uint64_t scratch_bytes, uint32_t* d_status,
                                                               void* stream) {
  bool path_ok = false;
  const rns8cuda::GemmPath path = path_of(gemm_path, &path_ok);
  if (!d_a || !d_b || !d_c || !d_status || task_count == 0 || m <= 0 || n <= 0 || k <= 0 || modulus < 2 ||
      modulus > 256 || !path_ok)
    return RNS8_INVALID_ARGUMENT;
  std::vector<rns8cuda::PlaneGemmTask> tasks(task_count);
  for (uint32_t t = 0; t < task_count; ++t) {
    if (!d_a[t] || !d_b[t] || !d_c[t]) return RNS8_INVALID_ARGUMENT;
    tasks[t] = {d_a[t], d_b[t], d_c[t]};
  }
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  const auto prob = seam_problem(m, n, k, 1, modulus, tasks.data(), task_count);
  return launch_result(rns8cuda::plane_gemm(prob, path, sm_count_of(device_id), d_scratch, scratch_bytes, d_status,
                                            as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_export_i64_device(int device_id, const int8_t* d_planes, int64_t m, int64_t n,
                                                   uint32_t prefix, uint64_t bound, int64_t* d_dst, int64_t ld,
                                                   uint32_t* d_status, void* stream) {
  if (!d_planes || !d_dst || !d_status || !rns8host::valid_matrix_access(m, n, ld) || !valid_prefix(prefix))
    return RNS8_INVALID_ARGUMENT;
  const rns8_status c = rns8host::validate_bound_contract(RNS8_BOUNDED_I64, RNS8_BOUND_GLOBAL_MAX_ABS, bound, prefix);
  if (c != RNS8_SUCCESS) return c;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::export_i64(d_planes, m, n, prefix, bound, d_dst, ld, d_status, as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_export_u64_device(int device_id, const int8_t* d_planes, int64_t m, int64_t n,
                                                   uint32_t prefix, uint64_t bound, uint64_t* d_dst, int64_t ld,
                                                   uint32_t* d_status, void* stream) {
  if (!d_planes || !d_dst || !d_status || !rns8host::valid_matrix_access(m, n, ld) || !valid_prefix(prefix))
    return RNS8_INVALID_ARGUMENT;
  const rns8_status c =
      rns8host::validate_bound_contract(RNS8_BOUNDED_U64, RNS8_BOUND_GLOBAL_MAX_UNSIGNED, bound, prefix);
  if (c != RNS8_SUCCESS) return c;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::export_u64(d_planes, m, n, prefix, bound, d_dst, ld, d_status, as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_export_limbs_device(int device_id, const int8_t* d_planes, int64_t m, int64_t n,
                                                     uint32_t prefix, uint32_t is_signed, uint32_t limb_count,
                                                     uint64_t* d_dst, int64_t ld, uint32_t* d_status, void* stream) {
  if (!d_planes || !d_dst || !d_status || !rns8host::valid_matrix_access(m, n, ld) || !valid_prefix(prefix) ||
      limb_count == 0 || limb_count > 32)
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::export_limbs(d_planes, m, n, prefix, is_signed != 0, limb_count, d_dst, ld, d_status,
                                              as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_export_finite_u8_device(int device_id, const int8_t* d_residues, int64_t m, int64_t n,
                                                         uint16_t modulus, uint8_t* d_dst, int64_t ld, void* stream) {
  if (!d_residues || !d_dst || !rns8host::valid_matrix_access(m, n, ld) || modulus < 2 || modulus > 256)
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::export_finite_u8(d_residues, m, n, modulus, d_dst, ld, as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_pack_wrap_u64_device(int device_id, const uint64_t* d_src, int64_t rows, int64_t cols,
                                                    int64_t ld, uint8_t* d_limbs, void* stream) {
  if (!d_src || !d_limbs || !rns8host::valid_matrix_access(rows, cols, ld)) return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::wrap_pack_u64(d_src, rows, cols, ld, d_limbs, as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_gemm_wrap_u64_device(int device_id, const uint8_t* d_a_limbs, const uint8_t* d_b_limbs,
                                                    uint64_t* d_c, int64_t m, int64_t n, int64_t k,
                                                    uint32_t gemm_path, uint32_t* d_status, void* stream) {
  bool ok = false;
  const rns8cuda::GemmPath path = path_of(gemm_path, &ok);
  if (!ok || !d_a_limbs || !d_b_limbs || !d_c || m <= 0 || n <= 0 || k <= 0) return RNS8_INVALID_ARGUMENT;
  if (!rns8host::valid_matrix_access(m, k, k) || !rns8host::valid_matrix_access(k, n, n)) return RNS8_INVALID_ARGUMENT;
  if (!d_status && path != rns8cuda::GemmPath::Simt) return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::wrap_gemm(d_a_limbs, d_b_limbs, d_c, m, n, k, path, sm_count_of(device_id), d_status,
                                           as_stream(stream)));
}

extern "C" rns8_status rns8_cuda_export_wrap_u64_device(int device_id, const uint8_t* d_limbs, int64_t rows,
                                                      int64_t cols, uint64_t* d_dst, int64_t ld, void* stream) {
  if (!d_limbs || !d_dst || !rns8host::valid_matrix_access(rows, cols, ld)) return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  return launch_result(rns8cuda::wrap_export_u64(d_limbs, rows, cols, d_dst, ld, as_stream(stream)));
}
