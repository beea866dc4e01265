// Row kernels of the materialised causal attention used where the flash
// kernels have no fp32-accurate tile shape (head_dim 128 in 3xTF32 mode):
// S = scale * Q K^T and O = P V run on the batched tcgen05 GEMM, these
// kernels turn S into P (forward) and dP into dS (backward) in place.
//
// Layout: (Z, L, L) rows with row stride `ld` and matrix stride `zs`
// (elements). Row i attends to columns [0, i]. Both kernels also write zeros
// in the masked columns (i, round_up(i + 1, 128)) so the next GEMM, which
// reads whole 128-wide diagonal tiles, sees exact zeros there; columns past
// that are never read (the GEMMs skip those tiles).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "../api.h"
#include "../common/host.h"

namespace abacus {
namespace attn {
namespace {

constexpr int kDiag = 128;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row. Pass 1: running max / sum over the valid columns with
// rescaling (one read). Pass 2: write exp(s - max) / sum and the zero pad.
__global__ void __launch_bounds__(256) causal_softmax_fwd_kernel(float* __restrict__ s, long long rows, int L,
                                                                 long long ld, long long zs) {
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= rows) return;
  const long long z = gw / L;
  const int i = static_cast<int>(gw % L);
  float* row = s + z * zs + i * ld;
  const int valid = i + 1;
  const int pad_end = min(L, (i / kDiag + 1) * kDiag);
  float m = -INFINITY, l = 0.f;
  for (int j = lane * 4; j < valid; j += 128) {
    const float4 v = *reinterpret_cast<const float4*>(row + j);
    const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (j + e < valid) {
        const float x = xs[e];
        if (x > m) {
          l = l * expf(m - x) + 1.f;
          m = x;
        } else {
          l += expf(x - m);
        }
      }
    }
  }
  const float gm = warp_max(m);
  l = (m == -INFINITY) ? 0.f : l * expf(m - gm);
  const float inv = 1.f / warp_sum(l);
  for (int j = lane * 4; j < pad_end; j += 128) {
    float4 v = *reinterpret_cast<const float4*>(row + j);
    float* xs = reinterpret_cast<float*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) xs[e] = (j + e < valid) ? expf(xs[e] - gm) * inv : 0.f;
    *reinterpret_cast<float4*>(row + j) = v;
  }
}

// dS = scale * P * (dP - sum_j P_j dP_j), in place of dP.
__global__ void __launch_bounds__(256) causal_softmax_bwd_kernel(const float* __restrict__ p, float* __restrict__ dp,
                                                                 long long rows, int L, long long ld, long long zs,
                                                                 long long ld_dp, long long zs_dp, float scale) {
  const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (gw >= rows) return;
  const long long z = gw / L;
  const int i = static_cast<int>(gw % L);
  const float* prow = p + z * zs + i * ld;
  float* drow = dp + z * zs_dp + i * ld_dp;
  const int valid = i + 1;
  const int pad_end = min(L, (i / kDiag + 1) * kDiag);
  float acc = 0.f;
  for (int j = lane * 4; j < valid; j += 128) {
    const float4 a = *reinterpret_cast<const float4*>(prow + j);
    const float4 b = *reinterpret_cast<const float4*>(drow + j);
    const float pa[4] = {a.x, a.y, a.z, a.w}, pb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (j + e < valid) acc += pa[e] * pb[e];
  }
  const float delta = warp_sum(acc);
  for (int j = lane * 4; j < pad_end; j += 128) {
    const float4 a = *reinterpret_cast<const float4*>(prow + j);
    float4 b = *reinterpret_cast<const float4*>(drow + j);
    const float pa[4] = {a.x, a.y, a.z, a.w};
    float* pb = reinterpret_cast<float*>(&b);
#pragma unroll
    for (int e = 0; e < 4; ++e) pb[e] = (j + e < valid) ? scale * pa[e] * (pb[e] - delta) : 0.f;
    *reinterpret_cast<float4*>(drow + j) = b;
  }
}

void check_square(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.dim() == 4 && t.size(2) == t.size(3), name,
              " must be a (B, H, L, L) CUDA fp32 view");
  TORCH_CHECK(t.stride(3) == 1 && t.stride(2) % 4 == 0 && t.size(3) % 4 == 0 &&
                  reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              name, " rows must be 16-byte aligned with unit inner stride");
  TORCH_CHECK(t.stride(0) == t.size(1) * t.stride(1), name, " must be contiguous over (B, H)");
}

}  // namespace

void causal_softmax_fwd(torch::Tensor s) {
  check_square(s, "S");
  const c10::cuda::CUDAGuard guard(s.device());
  const int L = static_cast<int>(s.size(2));
  const long long rows = s.size(0) * s.size(1) * static_cast<long long>(L);
  if (rows == 0) return;
  const long long threads = rows * 32;
  causal_softmax_fwd_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0,
                              at::cuda::getCurrentCUDAStream()>>>(s.data_ptr<float>(), rows, L, s.stride(2),
                                                                  s.stride(1));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

void causal_softmax_bwd(torch::Tensor p, torch::Tensor dp, double scale) {
  check_square(p, "P");
  check_square(dp, "dP");
  TORCH_CHECK(p.sizes() == dp.sizes(), "P and dP shapes differ");
  const c10::cuda::CUDAGuard guard(p.device());
  const int L = static_cast<int>(p.size(2));
  const long long rows = p.size(0) * p.size(1) * static_cast<long long>(L);
  if (rows == 0) return;
  const long long threads = rows * 32;
  causal_softmax_bwd_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0,
                              at::cuda::getCurrentCUDAStream()>>>(p.data_ptr<float>(), dp.data_ptr<float>(), rows, L,
                                                                  p.stride(2), p.stride(1), dp.stride(2), dp.stride(1),
                                                                  static_cast<float>(scale));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

}  // namespace attn
}  // namespace abacus
