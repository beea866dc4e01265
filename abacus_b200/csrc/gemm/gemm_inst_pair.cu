// 3xTF32 GEMM instantiations on CTA pairs (cta_group::2, 256 x 128 tiles).
#include "gemm_launch.cuh"

namespace abacus {
namespace gemm {

void launch_store_pair(const Params& p, dim3 grid, bool a_mn, bool b_mn, cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_t<128, false, false, 3, kEpiStore, true>(p, grid, s);
  if (!a_mn && b_mn) return launch_t<128, false, true, 3, kEpiStore, true>(p, grid, s);
  if (a_mn && !b_mn) return launch_t<128, true, false, 3, kEpiStore, true>(p, grid, s);
  return launch_t<128, true, true, 3, kEpiStore, true>(p, grid, s);
}

void launch_swiglu_pair(const Params& p, dim3 grid, cudaStream_t s) {
  launch_t<128, false, true, 3, kEpiSwiGLU, true>(p, grid, s);
}

void launch_swiglu_bwd_pair(const Params& p, dim3 grid, cudaStream_t s) {
  launch_t<128, false, false, 3, kEpiSwiGLUBwd, true>(p, grid, s);
}

}  // namespace gemm
}  // namespace abacus
