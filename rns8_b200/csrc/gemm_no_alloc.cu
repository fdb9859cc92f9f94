// Plane GEMM for callers that cannot allocate device memory.
//
// rns8_cuda_gemm_rns_device takes its split-K scratch and status word from
// the caller. Some callers have no way to provide them: a host whose device
// memory is owned by a fixed-budget allocator it may not call into, a
// foreign-language caller that holds only the input and output buffers, or a
// latency-critical loop where cudaMalloc/cudaFree would synchronise the whole
// device and stall every other stream. This entry point serves them with
// scratch that lives in a file-scope device array instead: every GPU that
// loads the library holds kNoAllocScratchBytes (8 MiB) plus a 256-byte status
// area for the life of the process, and nothing is allocated per call.
//
// The array's name is only a host-side stand-in in host code, so the device
// address is looked up once per device (with that device current) through
// cudaGetSymbolAddress and passed to the kernels. The first call on a device
// performs that look-up; make it before any stream capture. The address is
// kept for the life of the process, so the entry point must not be used
// across a cudaDeviceReset (or a release and re-creation of the primary
// context), which loads the array at a new address. Every call shares the
// array and it keeps the last call's contents, so each call clears the status
// word and the split-K sums before use; calls that overlap on the GPU (other
// streams, other host threads on the same device) race on it.
#include <mutex>

#include "api_internal.hpp"
#include "device_common.cuh"

namespace {

constexpr uint64_t kStatusAreaBytes = 256;
constexpr uint64_t kNoAllocScratchBytes = 8ull << 20;  // split-K sums, largest supported problem
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_no_alloc_scratch[kStatusAreaBytes + kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_device_address[kMaxDevices] = {};

// Device address of g_no_alloc_scratch on the current device `dev`.
cudaError_t scratch_address(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_device_address[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_no_alloc_scratch);
    if (e != cudaSuccess) return e;
    g_device_address[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_device_address[dev]);
  return cudaSuccess;
}

}  // namespace

extern "C" rns8_status rns8_cuda_gemm_rns_device_no_alloc(int device_id, const int8_t* d_a, const int8_t* d_b,
                                                          int8_t* d_c, int64_t m, int64_t n, int64_t k,
                                                          uint32_t prefix, void* stream) {
  if (!d_a || !d_b || !d_c || m <= 0 || n <= 0 || k <= 0 || prefix == 0 || prefix > RNS8_MAX_SUPPORTED_PREFIX ||
      device_id < 0 || device_id >= kMaxDevices || device_id >= rns8host::visible_device_count())
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);  // the caller's current device is restored on return
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* base = nullptr;
  if (scratch_address(device_id, &base) != cudaSuccess) {
    (void)cudaGetLastError();
    return RNS8_BACKEND_FAILURE;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_id) != cudaSuccess || sms <= 0)
    return RNS8_BACKEND_FAILURE;

  const rns8cuda::PlaneGemmTask task{d_a, d_b, d_c};
  rns8cuda::PlaneGemmProblem prob{};
  prob.m = m;
  prob.n = n;
  prob.k = k;
  prob.planes = prefix;
  for (uint32_t p = 0; p < prefix; ++p) prob.moduli[p] = rns8ladder::kLadder[p];
  prob.task_count = 1;
  prob.tasks = &task;
  uint64_t need = rns8cuda::plane_gemm_scratch_bytes(prob, sms);
  if (need > kNoAllocScratchBytes) {
    // Tensor-core shapes whose split-K sums do not fit are refused. Shapes
    // the tensor cores cannot address directly offer the whole array: the
    // GEMM pads them onto the tensor cores when the padded copies fit, and
    // otherwise runs the CUDA-core kernels, which need no more.
    if (rns8cuda::tensor_core_path_supported(prob)) return RNS8_WORKSPACE_TOO_SMALL;
    need = kNoAllocScratchBytes;
  }

  uint32_t* status = reinterpret_cast<uint32_t*>(base);
  void* scratch = need ? base + kStatusAreaBytes : nullptr;
  if (cudaMemsetAsync(status, 0, sizeof(uint32_t), s) != cudaSuccess) return RNS8_BACKEND_FAILURE;
  // plane_gemm zeroes the split-K sums itself before its kernel runs.
  const cudaError_t e =
      rns8cuda::plane_gemm(prob, rns8cuda::GemmPath::Auto, sms, scratch, need, status, s);
  if (e != cudaSuccess) return e == cudaErrorInvalidValue ? RNS8_INVALID_ARGUMENT : RNS8_BACKEND_FAILURE;
  uint32_t word = 0;
  if (cudaMemcpyAsync(&word, status, sizeof(word), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  return word == 0 ? RNS8_SUCCESS : RNS8_BACKEND_FAILURE;
}
