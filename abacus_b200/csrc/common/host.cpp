#include "host.h"
#include <c10/util/Exception.h>
#include <c10/cuda/CUDAException.h>

namespace abacus {
namespace host {

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  thread_local int bound_device = -1;
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (bound_device != dev) {
    C10_CUDA_CHECK(cudaSetDevice(dev));  // makes the primary context current on this thread
    bound_device = dev;
  }
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr != nullptr, "cuTensorMapEncodeTiled is unavailable");
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

namespace {
std::atomic<long long> g_launches{0};
std::mutex g_mu;
int* g_status[64] = {nullptr};
}  // namespace

int* status_ptr(int device) {
  TORCH_CHECK(device >= 0 && device < 64, "bad device index");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_status[device] == nullptr) {
    int prev = 0;
    C10_CUDA_CHECK(cudaGetDevice(&prev));
    C10_CUDA_CHECK(cudaSetDevice(device));
    C10_CUDA_CHECK(cudaMalloc(&g_status[device], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(g_status[device], 0, sizeof(int)));
    C10_CUDA_CHECK(cudaSetDevice(prev));
  }
  return g_status[device];
}

void note_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

int read_status(int device) {
  int v = 0;
  C10_CUDA_CHECK(cudaMemcpy(&v, status_ptr(device), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

void reset_status(int device) { C10_CUDA_CHECK(cudaMemset(status_ptr(device), 0, sizeof(int))); }

}  // namespace host
}  // namespace abacus
