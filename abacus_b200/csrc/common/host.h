// Host-side helpers shared by every abacus_b200 CUDA op: the driver entry
// point for tensor-map encoding, the per-device status word that bounded
// device waits report into, and a per-device "run once" guard.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <atomic>
#include <cstdint>
#include <mutex>

namespace abacus {
namespace host {

// cuTensorMapEncodeTiled, fetched through the runtime so the extension does not
// link libcuda directly. Also binds the current device's primary context to
// the calling thread (driver-API calls need a current context, which threads
// such as the autograd engine's workers may not have yet).
PFN_cuTensorMapEncodeTiled_v12000 encode_tiled();

// Device pointer to this device's status word (zero = healthy). Kernels record
// the first timeout / bad-argument code here instead of trapping.
int* status_ptr(int device);
int read_status(int device);
void reset_status(int device);

// Number of abacus kernels launched by this process (every launch site calls
// note_launch right after its <<<>>>), so benchmarks can report how many of
// the timed region's kernels are this library's own.
void note_launch(int n = 1);
long long launch_count();

// Runs `fn` once per CUDA device (the current one).
class PerDeviceOnce {
 public:
  template <class F>
  void run(F&& fn) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (done_.load(std::memory_order_acquire) & bit) return;
    std::lock_guard<std::mutex> lock(mu_);
    if (done_.load(std::memory_order_relaxed) & bit) return;
    fn();
    done_.fetch_or(bit, std::memory_order_release);
  }

 private:
  std::atomic<uint64_t> done_{0};
  std::mutex mu_;
};

}  // namespace host
}  // namespace abacus
