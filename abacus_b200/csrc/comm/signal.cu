// Device-side signalling with bounded waits.
//
// wait_flag_kernel spins (with %globaltimer) until *flag >= expected or the
// deadline passes; on timeout it records kStatusTimeoutPeer in the device
// status word and returns, leaving the context usable. The same primitive
// (ld.acquire.sys + deadline) is what the cross-GPU kernels use to wait for a
// peer's flag, so a peer that never signals turns into an error status the
// host can read instead of a hung GPU.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "../api.h"
#include "../common/host.h"
#include "../common/sm100.cuh"

namespace abacus {
namespace comm {

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Returns true when *flag >= expected before `timeout_ns`; otherwise records
// kStatusTimeoutPeer and returns false.
__device__ __forceinline__ bool wait_flag_bounded(const int* flag, int expected, unsigned long long timeout_ns,
                                                  int* status) {
  const unsigned long long start = globaltimer_ns();
  unsigned it = 0;
  while (ld_acquire_sys(flag) < expected) {
    if ((++it & 63u) == 0) {
      if (*reinterpret_cast<volatile int*>(status) != kStatusOk) return false;
      if (globaltimer_ns() - start > timeout_ns) {
        atomicCAS(status, kStatusOk, kStatusTimeoutPeer);
        return false;
      }
    }
    __nanosleep(64);
  }
  return true;
}

namespace {

__global__ void wait_flag_kernel(const int* flag, int expected, unsigned long long timeout_ns, int* status,
                                 int* result) {
  if (threadIdx.x == 0) *result = wait_flag_bounded(flag, expected, timeout_ns, status) ? 1 : 0;
}

__global__ void set_flag_kernel(int* flag, int value) {
  if (threadIdx.x == 0) st_release_sys(flag, value);
}

}  // namespace

void wait_flag(torch::Tensor flag, int64_t expected, double timeout_ms, torch::Tensor result) {
  const c10::cuda::CUDAGuard guard(flag.device());
  TORCH_CHECK(flag.is_cuda() && flag.scalar_type() == torch::kInt32 && flag.numel() >= 1, "flag must be int32 CUDA");
  TORCH_CHECK(result.is_cuda() && result.scalar_type() == torch::kInt32, "result must be int32 CUDA");
  TORCH_CHECK(timeout_ms > 0 && timeout_ms <= 10000, "timeout must be in (0, 10000] ms");
  wait_flag_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      flag.data_ptr<int>(), static_cast<int>(expected), static_cast<unsigned long long>(timeout_ms * 1e6),
      host::status_ptr(flag.device().index()), result.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

void set_flag(torch::Tensor flag, int64_t value) {
  const c10::cuda::CUDAGuard guard(flag.device());
  set_flag_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(flag.data_ptr<int>(), static_cast<int>(value));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

}  // namespace comm
}  // namespace abacus
