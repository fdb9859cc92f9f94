// The bounded mbarrier wait of the persistent kernels, in isolation, so that
// the failure path can be exercised without a GPU fault. One CTA initialises
// a barrier that expects one arrival. With `arrive` set, a thread arrives and
// the wait completes; otherwise nothing ever arrives, the wait gives up after
// `budget` SM cycles and the kernel ORs kDevWaitTimeout into the status word,
// exactly as a GEMM whose producer or MMA thread stalled would. No trap, no bad
// address, no unbounded loop: the kernel returns and the context stays usable.
#include "api_internal.hpp"
#include "device_common.cuh"

namespace {

__global__ void wait_probe_kernel(uint32_t* status, uint32_t arrive, long long budget) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    rns8cuda::mbar_init(&bar, 1);
    rns8cuda::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && arrive) rns8cuda::mbar_arrive(&bar);
  __syncthreads();
  if (threadIdx.x == 0 && !rns8cuda::mbar_wait_bounded(&bar, 0, budget)) atomicOr(status, rns8cuda::kDevWaitTimeout);
}

}  // namespace

extern "C" rns8_status rns8_cuda_wait_probe(int device_id, uint32_t arrive, uint64_t budget_cycles,
                                            uint32_t* d_status, void* stream) {
  if (!d_status || arrive > 1 || budget_cycles == 0 ||
      budget_cycles > static_cast<uint64_t>(rns8cuda::kWaitBudgetCycles))
    return RNS8_INVALID_ARGUMENT;
  rns8host::DeviceScope scope(device_id);
  if (!scope.ok) return RNS8_BACKEND_FAILURE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(d_status, 0, sizeof(uint32_t), s) != cudaSuccess) return RNS8_BACKEND_FAILURE;
  wait_probe_kernel<<<1, 32, 0, s>>>(d_status, arrive, static_cast<long long>(budget_cycles));
  uint32_t word = 0;
  if (cudaGetLastError() != cudaSuccess ||
      cudaMemcpyAsync(&word, d_status, sizeof(word), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return RNS8_BACKEND_FAILURE;
  return (word & rns8cuda::kDevWaitTimeout) ? RNS8_BACKEND_FAILURE : RNS8_SUCCESS;
}
