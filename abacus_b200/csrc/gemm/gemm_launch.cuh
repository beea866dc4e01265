// Kernel launchers for the tcgen05 GEMM. Each instantiation family lives in
// its own translation unit (gemm_inst_*.cu) so the build compiles them in
// parallel; gemm.cu only sees these declarations.
#pragma once
#include <c10/cuda/CUDAException.h>
#include "gemm_tcgen05.cuh"
#include "../common/host.h"

namespace abacus {
namespace gemm {

template <int BN, bool A_MN, bool B_MN, int PASSES, int EPI>
void launch_t(const Params& p, dim3 grid, cudaStream_t stream) {
  constexpr int STAGES = PASSES == 3 ? 4 : (BN == 256 ? 4 : 6);
  using Cfg = Config<BN, A_MN, B_MN, PASSES, STAGES>;
  auto kern = gemm_kernel<BN, A_MN, B_MN, PASSES, EPI, STAGES>;
  static host::PerDeviceOnce once;
  once.run([&] {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  });
  kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

template <int BN, int EPI>
void dispatch_layout(const Params& p, dim3 grid, bool a_mn, bool b_mn, int passes, cudaStream_t s) {
#define ABACUS_GEMM_CASE(AM, BMJ, PS) \
  if (a_mn == AM && b_mn == BMJ && passes == PS) return launch_t<BN, AM, BMJ, PS, EPI>(p, grid, s);
  ABACUS_GEMM_CASE(false, false, 1)
  ABACUS_GEMM_CASE(false, true, 1)
  ABACUS_GEMM_CASE(true, false, 1)
  ABACUS_GEMM_CASE(true, true, 1)
  // 3xTF32 keeps its K-chunk accumulator in registers: 128-column tiles only.
  if constexpr (BN == 128) {
    ABACUS_GEMM_CASE(false, false, 3)
    ABACUS_GEMM_CASE(false, true, 3)
    ABACUS_GEMM_CASE(true, false, 3)
    ABACUS_GEMM_CASE(true, true, 3)
  }
#undef ABACUS_GEMM_CASE
  TORCH_CHECK(false, "unsupported GEMM configuration");
}

// N-tile width for a GEMM of output width n in the given precision mode.
inline int pick_bn(long long n, int passes) {
  if (passes == 3) return 128;
  return (n >= 2048 || (n % 256 == 0 && n >= 512)) ? 256 : 128;
}

// Defined in gemm_inst_*.cu.
void launch_store(const Params& p, dim3 grid, int bn, bool a_mn, bool b_mn, int passes, cudaStream_t s);
void launch_swiglu(const Params& p, dim3 grid, int bn, int passes, cudaStream_t s);
void launch_swiglu_bwd(const Params& p, dim3 grid, int bn, int passes, cudaStream_t s);

}  // namespace gemm
}  // namespace abacus
