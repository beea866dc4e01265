// Store-epilogue GEMM instantiations with a 128-column N tile.
#include "gemm_launch.cuh"

namespace abacus {
namespace gemm {

void launch_store_128(const Params& p, dim3 grid, bool a_mn, bool b_mn, int passes, cudaStream_t s) {
  dispatch_layout<128, kEpiStore>(p, grid, a_mn, b_mn, passes, s);
}

}  // namespace gemm
}  // namespace abacus
