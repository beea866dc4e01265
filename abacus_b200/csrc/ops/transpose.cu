// out = in^T for fp32 matrices. One CTA moves a 64 x 64 tile: 256 threads read
// it as 16-byte row segments (coalesced), stage it in shared memory with a
// padded row so the column reads are conflict-free, and write the transposed
// tile as 16-byte row segments of the output. HBM-bound: one read and one
// write of the matrix.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cstdint>
#include "transpose.h"
#include "../common/host.h"

namespace abacus {
namespace ops {
namespace {

constexpr int kTile = 64;

__global__ void __launch_bounds__(256) transpose_kernel(const float* __restrict__ in, long long ld_in,
                                                        float* __restrict__ out, long long ld_out, int rows,
                                                        int cols) {
  __shared__ float tile[kTile][kTile + 1];
  const int r0 = blockIdx.y * kTile, c0 = blockIdx.x * kTile;
  const int t = threadIdx.x;
  const int seg = t % 16, row = t / 16;  // 16 float4 segments per 64-wide row, 16 rows per pass
  const bool vec_in = (ld_in % 4 == 0) && (reinterpret_cast<uintptr_t>(in) % 16 == 0);
#pragma unroll
  for (int pass = 0; pass < kTile / 16; ++pass) {
    const int r = r0 + pass * 16 + row, c = c0 + seg * 4;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < rows) {
      const float* src = in + static_cast<long long>(r) * ld_in + c;
      if (vec_in && c + 3 < cols) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(src));
        v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (c + k < cols) v[k] = src[k];
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) tile[pass * 16 + row][seg * 4 + k] = v[k];
  }
  __syncthreads();
  const bool vec_out = (ld_out % 4 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0);
#pragma unroll
  for (int pass = 0; pass < kTile / 16; ++pass) {
    // Output row = input column c0 + j; output columns = input rows r0 + 4*seg ...
    const int j = pass * 16 + row;
    const int oc = c0 + j, orr = r0 + seg * 4;
    if (oc >= cols) continue;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = tile[seg * 4 + k][j];
    float* dst = out + static_cast<long long>(oc) * ld_out + orr;
    if (vec_out && orr + 3 < rows) {
      *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (orr + k < rows) dst[k] = v[k];
    }
  }
}

}  // namespace

void transpose2d(torch::Tensor in, torch::Tensor out) {
  const c10::cuda::CUDAGuard guard(in.device());
  TORCH_CHECK(in.is_cuda() && in.scalar_type() == torch::kFloat32 && in.dim() == 2 && in.stride(1) == 1,
              "in: 2-D fp32 CUDA tensor with unit column stride");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kFloat32 && out.dim() == 2 && out.stride(1) == 1 &&
                  out.size(0) == in.size(1) && out.size(1) == in.size(0),
              "out: (N, M) fp32 with unit column stride");
  const int rows = static_cast<int>(in.size(0)), cols = static_cast<int>(in.size(1));
  if (rows == 0 || cols == 0) return;
  dim3 grid(static_cast<unsigned>((cols + kTile - 1) / kTile), static_cast<unsigned>((rows + kTile - 1) / kTile));
  TORCH_CHECK(grid.y <= 65535u, "too many rows for one transpose launch");
  transpose_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      in.data_ptr<float>(), in.stride(0), out.data_ptr<float>(), out.stride(0), rows, cols);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

}  // namespace ops
}  // namespace abacus
