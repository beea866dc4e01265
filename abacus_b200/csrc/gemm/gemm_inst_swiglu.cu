// SwiGLU forward / backward epilogue GEMM instantiations.
#include "gemm_launch.cuh"

namespace abacus {
namespace gemm {

void launch_store_128(const Params& p, dim3 grid, bool a_mn, bool b_mn, int passes, cudaStream_t s);
void launch_store_256(const Params& p, dim3 grid, bool a_mn, bool b_mn, int passes, cudaStream_t s);

void launch_store(const Params& p, dim3 grid, int bn, bool a_mn, bool b_mn, int passes, cudaStream_t s, bool pair) {
  if (pair) {
    TORCH_CHECK(bn == 128 && passes == 3, "CTA pairs run 3xTF32 with 128-column tiles");
    launch_store_pair(p, grid, a_mn, b_mn, s);
  } else if (bn == 256) {
    launch_store_256(p, grid, a_mn, b_mn, passes, s);
  } else {
    launch_store_128(p, grid, a_mn, b_mn, passes, s);
  }
}

void launch_swiglu(const Params& p, dim3 grid, int bn, int passes, cudaStream_t s, bool pair) {
  TORCH_CHECK(bn == (passes == 3 ? 128 : 256), "SwiGLU tile width");
  if (pair) {
    TORCH_CHECK(passes == 3, "CTA pairs run 3xTF32");
    launch_swiglu_pair(p, grid, s);
  } else if (passes == 3) launch_t<128, false, true, 3, kEpiSwiGLU>(p, grid, s);
  else launch_t<256, false, true, 1, kEpiSwiGLU>(p, grid, s);
}

void launch_swiglu_bwd(const Params& p, dim3 grid, int bn, int passes, cudaStream_t s, bool pair) {
  if (pair) {
    TORCH_CHECK(bn == 128 && passes == 3, "CTA pairs run 3xTF32 with 128-column tiles");
    launch_swiglu_bwd_pair(p, grid, s);
  } else if (bn == 256) {
    TORCH_CHECK(passes == 1, "3xTF32 uses 128-column tiles");
    launch_t<256, false, false, 1, kEpiSwiGLUBwd>(p, grid, s);
  } else {
    if (passes == 3) launch_t<128, false, false, 3, kEpiSwiGLUBwd>(p, grid, s);
    else launch_t<128, false, false, 1, kEpiSwiGLUBwd>(p, grid, s);
  }
}

}  // namespace gemm
}  // namespace abacus
