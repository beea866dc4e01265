// MoE router scores (reference: abacus/moe/router.py:40-54, logits = x @ w_DE)
// and their gradients, as memory-bound kernels: the expert count E is small
// (8 in the benchmark), so the product is a handful of dot products per token
// and is bound by one read of x.
//
// * forward: one warp per token; lane l accumulates x[t, d] * w[d, e] over
//   d = l, l + 32, ... for every e (w staged transposed in shared memory),
//   then a fixed xor-shuffle tree sums the lanes: deterministic.
// * backward dx[t, d] = sum_e dlogits[t, e] * w[d, e]: one warp per token.
// * backward dw[d, e] = sum_t x[t, d] * dlogits[t, e]: each block sums its
//   token range into a partial (D, E) slab, then a second kernel adds the
//   slabs in block order: deterministic, no atomics.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <algorithm>
#include "router.h"
#include "../common/host.h"

namespace abacus {
namespace ops {
namespace {

constexpr int kMaxExperts = 64;
constexpr int kWarps = 8;

template <int E>
__global__ void __launch_bounds__(kWarps * 32) router_fwd_kernel(const float* __restrict__ x, long long ld_x,
                                                                  const float* __restrict__ w, float* __restrict__ out,
                                                                  int tokens, int dim) {
  extern __shared__ float sw[];  // (E, dim): lanes of a warp read consecutive d, no bank conflicts
  for (int i = threadIdx.x; i < dim * E; i += blockDim.x) sw[(i % E) * dim + i / E] = w[i];
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (long long t = static_cast<long long>(blockIdx.x) * kWarps + warp; t < tokens;
       t += static_cast<long long>(gridDim.x) * kWarps) {
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    const float* row = x + t * ld_x;
    for (int d = lane; d < dim; d += 32) {
      const float xv = row[d];
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] = fmaf(xv, sw[e * dim + d], acc[e]);
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int e = 0; e < E; ++e) out[t * E + e] = acc[e];
    }
  }
}

template <int E>
__global__ void __launch_bounds__(kWarps * 32) router_dx_kernel(const float* __restrict__ dl, const float* __restrict__ w,
                                                                 float* __restrict__ dx, long long ld_dx, int tokens,
                                                                 int dim) {
  extern __shared__ float sw[];  // (E, dim): lanes of a warp read consecutive d, no bank conflicts
  for (int i = threadIdx.x; i < dim * E; i += blockDim.x) sw[(i % E) * dim + i / E] = w[i];
  __syncthreads();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (long long t = static_cast<long long>(blockIdx.x) * kWarps + warp; t < tokens;
       t += static_cast<long long>(gridDim.x) * kWarps) {
    float g[E];
#pragma unroll
    for (int e = 0; e < E; ++e) g[e] = dl[t * E + e];
    float* row = dx + t * ld_dx;
    for (int d = lane; d < dim; d += 32) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) s = fmaf(g[e], sw[e * dim + d], s);
      row[d] = s;
    }
  }
}

// Block b sums tokens [b * per, (b + 1) * per) into partial[b] (dim x E).
// Thread i owns columns d = i, i + blockDim, ... with E accumulators each: the
// x loads of a warp are coalesced and dlogits[t, :] is one broadcast read.
template <int E>
__global__ void __launch_bounds__(256) router_dw_partial_kernel(const float* __restrict__ x, long long ld_x,
                                                                 const float* __restrict__ dl,
                                                                 float* __restrict__ partial, int tokens, int dim,
                                                                 int per) {
  const int t0 = blockIdx.x * per, t1 = min(tokens, t0 + per);
  float* slab = partial + static_cast<long long>(blockIdx.x) * dim * E;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    for (int t = t0; t < t1; ++t) {
      const float xv = x[static_cast<long long>(t) * ld_x + d];
      const float* g = dl + static_cast<long long>(t) * E;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] = fmaf(xv, g[e], acc[e]);
    }
#pragma unroll
    for (int e = 0; e < E; ++e) slab[d * E + e] = acc[e];
  }
}

__global__ void router_dw_reduce_kernel(const float* __restrict__ partial, float* __restrict__ dw, int slabs, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int b = 0; b < slabs; ++b) s += partial[static_cast<long long>(b) * n + i];
  dw[i] = s;
}

void check_inputs(const torch::Tensor& x, const torch::Tensor& w) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.dim() == 2 && x.stride(1) == 1,
              "x: (tokens, D) fp32 with unit column stride");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.dim() == 2 &&
                  w.size(0) == x.size(1),
              "w: contiguous (D, E) fp32");
  TORCH_CHECK(w.size(1) >= 1 && w.size(1) <= kMaxExperts, "1 to 64 experts");
  TORCH_CHECK(w.numel() * 4 <= 200 * 1024, "router weight must fit in shared memory");
}

int grid_for(long long tokens, const torch::Device& dev) {
  const int sms = at::cuda::getDeviceProperties(dev.index())->multiProcessorCount;
  return static_cast<int>(std::max<long long>(1, std::min<long long>((tokens + kWarps - 1) / kWarps, 8LL * sms)));
}

#define ABACUS_ROUTER_DISPATCH(E, ...)                                   \
  switch (E) {                                                           \
    case 1: { constexpr int kE = 1; __VA_ARGS__; break; }                \
    case 2: { constexpr int kE = 2; __VA_ARGS__; break; }                \
    case 4: { constexpr int kE = 4; __VA_ARGS__; break; }                \
    case 8: { constexpr int kE = 8; __VA_ARGS__; break; }                \
    case 16: { constexpr int kE = 16; __VA_ARGS__; break; }              \
    case 32: { constexpr int kE = 32; __VA_ARGS__; break; }              \
    case 64: { constexpr int kE = 64; __VA_ARGS__; break; }              \
    default: TORCH_CHECK(false, "router kernels support 1, 2, 4, 8, 16, 32 or 64 experts"); \
  }

}  // namespace

void router_logits(torch::Tensor x, torch::Tensor w, torch::Tensor logits) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_inputs(x, w);
  const int tokens = static_cast<int>(x.size(0)), dim = static_cast<int>(x.size(1));
  const int experts = static_cast<int>(w.size(1));
  TORCH_CHECK(logits.is_cuda() && logits.is_contiguous() && logits.scalar_type() == torch::kFloat32 &&
                  logits.numel() == static_cast<int64_t>(tokens) * experts,
              "logits: contiguous (tokens, E) fp32");
  if (tokens == 0) return;
  const int grid = grid_for(tokens, x.device());
  const size_t smem = static_cast<size_t>(dim) * experts * sizeof(float);
  auto s = at::cuda::getCurrentCUDAStream();
  ABACUS_ROUTER_DISPATCH(experts, {
    if (smem > 48 * 1024) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(router_fwd_kernel<kE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)));
    }
    router_fwd_kernel<kE><<<grid, kWarps * 32, smem, s>>>(x.data_ptr<float>(), x.stride(0), w.data_ptr<float>(),
                                                          logits.data_ptr<float>(), tokens, dim);
  })
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

void router_logits_bwd(torch::Tensor dlogits, torch::Tensor x, torch::Tensor w, torch::Tensor dx, torch::Tensor dw) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_inputs(x, w);
  const int tokens = static_cast<int>(x.size(0)), dim = static_cast<int>(x.size(1));
  const int experts = static_cast<int>(w.size(1));
  TORCH_CHECK(dlogits.is_contiguous() && dlogits.numel() == static_cast<int64_t>(tokens) * experts, "dlogits");
  TORCH_CHECK(dx.is_cuda() && dx.stride(1) == 1 && dx.size(0) == tokens && dx.size(1) == dim, "dx: (tokens, D)");
  TORCH_CHECK(dw.is_contiguous() && dw.numel() == w.numel(), "dw: (D, E)");
  if (tokens == 0) {
    dw.zero_();
    return;
  }
  auto s = at::cuda::getCurrentCUDAStream();
  const size_t smem = static_cast<size_t>(dim) * experts * sizeof(float);
  const int grid = grid_for(tokens, x.device());
  const int sms = at::cuda::getDeviceProperties(x.device().index())->multiProcessorCount;
  const int slabs = std::max(1, std::min(4 * sms, (tokens + 15) / 16));
  const int per = (tokens + slabs - 1) / slabs;
  auto partial = torch::empty({slabs, dim * experts}, x.options());
  ABACUS_ROUTER_DISPATCH(experts, {
    if (smem > 48 * 1024) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(router_dx_kernel<kE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)));
    }
    router_dx_kernel<kE><<<grid, kWarps * 32, smem, s>>>(dlogits.data_ptr<float>(), w.data_ptr<float>(),
                                                         dx.data_ptr<float>(), dx.stride(0), tokens, dim);
    router_dw_partial_kernel<kE><<<slabs, 256, 0, s>>>(x.data_ptr<float>(), x.stride(0), dlogits.data_ptr<float>(),
                                                       partial.data_ptr<float>(), tokens, dim, per);
  })
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int n = dim * experts;
  router_dw_reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(partial.data_ptr<float>(), dw.data_ptr<float>(), slabs, n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch(3);
}

}  // namespace ops
}  // namespace abacus
