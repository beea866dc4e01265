// Kernel launchers for the tcgen05 GEMM. Each instantiation family lives in
// its own translation unit (gemm_inst_*.cu) so the build compiles them in
// parallel; gemm.cu only sees these declarations.
#pragma once
#include <c10/cuda/CUDAException.h>
#include <algorithm>
#include "gemm_tcgen05.cuh"
#include "../common/host.h"

namespace abacus {
namespace gemm {

// Phase-trace buffer for the next launches (diagnostics; null: off).
inline long long*& gemm_trace_buffer() {
  static long long* t = nullptr;
  return t;
}

// Number of CTA pairs of the last pair launch (diagnostics).
inline int& last_pair_clusters() {
  static int n = 0;
  return n;
}

template <int BN, bool A_MN, bool B_MN, int PASSES, int EPI, bool PAIR = false>
void launch_t(const Params& params, dim3 grid, cudaStream_t stream) {
  Params p = params;
  p.trace = gemm_trace_buffer();
  // 3xTF32 stages hold A (16 KB), B and B lo: 48 KB per stage on one CTA,
  // 32 KB on a CTA pair (half of B). Pairs keep 4 stages too: 6 (with the TMEM
  // A stages recycled separately) measured slower (gemm3 0.621 vs 0.594 ms).
  constexpr int STAGES = PASSES == 3 ? 4 : (BN == 256 ? 4 : 6);
  using Cfg = Config<BN, A_MN, B_MN, PASSES, STAGES, PAIR>;
  auto kern = gemm_kernel<BN, A_MN, B_MN, PASSES, EPI, STAGES, PAIR>;
  static host::PerDeviceOnce once;
  once.run([&] {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
  });
  if constexpr (PAIR) {
    // CTA pairs: (2, 1, 1) clusters; the grid is a whole number of pairs.
    TORCH_CHECK(grid.x % 2 == 0 && p.persistent && p.wait_flags == nullptr && !p.batched && p.causal == 0,
                "CTA-pair GEMM launch");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // A persistent grid must not hold more pairs than can be resident at once
    // (pairs need two free SMs of one GPC): the rest would run as a second wave.
    static int max_pairs[64] = {0};
    int dev = 0;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    if (dev < 64 && max_pairs[dev] == 0) {
      int n = 0;
      C10_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      max_pairs[dev] = n > 0 ? n : 1;
    }
    if (dev < 64) cfg.gridDim.x = std::min<unsigned>(grid.x, 2u * static_cast<unsigned>(max_pairs[dev]));
    last_pair_clusters() = static_cast<int>(cfg.gridDim.x / 2);
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, p));
  } else {
    kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, stream>>>(p);
  }
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

// Defined in gemm_inst_*.cu. `pair`: 3xTF32 on CTA pairs (gemm_inst_pair.cu).
void launch_store(const Params& p, dim3 grid, int bn, bool a_mn, bool b_mn, int passes, cudaStream_t s,
                  bool pair = false);
void launch_swiglu(const Params& p, dim3 grid, int bn, int passes, cudaStream_t s, bool pair = false);
void launch_swiglu_bwd(const Params& p, dim3 grid, int bn, int passes, cudaStream_t s, bool pair = false);
void launch_store_pair(const Params& p, dim3 grid, bool a_mn, bool b_mn, cudaStream_t s);
void launch_swiglu_pair(const Params& p, dim3 grid, cudaStream_t s);
void launch_swiglu_bwd_pair(const Params& p, dim3 grid, cudaStream_t s);

}  // namespace gemm
}  // namespace abacus
