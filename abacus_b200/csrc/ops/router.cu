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

// ---------------------------------------------------------------- routing
// One thread per token (E <= 64 logits in registers). Probabilities are the
// softmax over the experts (mode 0) or the per-expert sigmoid (mode 1); the
// top_k experts are chosen by probability (softmax) or by probability +
// selection bias (sigmoid; the bias only steers selection), ties going to the
// lower expert index; their probabilities, renormalised to sum 1 and scaled
// by route_scale, are the routing weights.
template <int E>
__global__ void __launch_bounds__(256) route_topk_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                                                         int mode, int top_k, float route_scale, int tokens,
                                                         float* __restrict__ probs, float* __restrict__ weights,
                                                         int64_t* __restrict__ indices) {
  const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= tokens) return;
  float pr[E];
  const float* row = logits + t * E;
  if (mode == 0) {
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      pr[e] = row[e];
      m = fmaxf(m, pr[e]);
    }
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      pr[e] = __expf(pr[e] - m);
      sum += pr[e];
    }
    const float inv = 1.f / sum;
#pragma unroll
    for (int e = 0; e < E; ++e) pr[e] *= inv;
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) pr[e] = 1.f / (1.f + __expf(-row[e]));
  }
#pragma unroll
  for (int e = 0; e < E; ++e) probs[t * E + e] = pr[e];
  // Selection: top_k passes of an argmax over the not yet chosen experts.
  unsigned long long chosen = 0ull;
  float picked_sum = 0.f;
  for (int k = 0; k < top_k; ++k) {
    int best = -1;
    float best_v = -INFINITY;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float v = pr[e] + (mode == 1 && bias != nullptr ? bias[e] : 0.f);
      if (!((chosen >> e) & 1ull) && (best < 0 || v > best_v)) {
        best = e;
        best_v = v;
      }
    }
    chosen |= 1ull << best;
    indices[t * top_k + k] = best;
    float pb = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) pb = e == best ? pr[e] : pb;
    weights[t * top_k + k] = pb;
    picked_sum += pb;
  }
  const float scale = route_scale / picked_sum;
  for (int k = 0; k < top_k; ++k) weights[t * top_k + k] *= scale;
}

// dlogits from the gradients of the routing weights (and of the probabilities,
// for the auxiliary loss): with S the chosen experts' probability sum,
// d p_i = route_scale * (dw_i / S - sum_j dw_j p_j / S^2) for chosen i, plus
// dprobs; then through the softmax (p_e (g_e - sum_f g_f p_f)) or the sigmoid
// (g_e p_e (1 - p_e)).
template <int E>
__global__ void __launch_bounds__(256) route_topk_bwd_kernel(const float* __restrict__ probs,
                                                             const int64_t* __restrict__ indices,
                                                             const float* __restrict__ dweights,
                                                             const float* __restrict__ dprobs, int mode, int top_k,
                                                             float route_scale, int tokens,
                                                             float* __restrict__ dlogits) {
  const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= tokens) return;
  float pr[E], g[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    pr[e] = probs[t * E + e];
    g[e] = dprobs ? dprobs[t * E + e] : 0.f;
  }
  float s = 0.f, dot = 0.f;
  for (int k = 0; k < top_k; ++k) {
    const int i = static_cast<int>(indices[t * top_k + k]);
    float pi = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) pi = e == i ? pr[e] : pi;
    s += pi;
    dot += dweights[t * top_k + k] * pi;
  }
  for (int k = 0; k < top_k; ++k) {
    const int i = static_cast<int>(indices[t * top_k + k]);
    const float add = route_scale * (dweights[t * top_k + k] / s - dot / (s * s));
#pragma unroll
    for (int e = 0; e < E; ++e) g[e] += e == i ? add : 0.f;
  }
  if (mode == 0) {
    float gp = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) gp += g[e] * pr[e];
#pragma unroll
    for (int e = 0; e < E; ++e) dlogits[t * E + e] = pr[e] * (g[e] - gp);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) dlogits[t * E + e] = g[e] * pr[e] * (1.f - pr[e]);
  }
}

// Rank of every assignment among the assignments to the same expert, in
// assignment order (the capacity slot of static expert slabs): one block per
// expert walks the assignments in chunks of blockDim, a block-wide exclusive
// scan of the match flags giving each match its rank. Deterministic.
__global__ void __launch_bounds__(1024) expert_rank_kernel(const int64_t* __restrict__ experts, long long n,
                                                           int64_t* __restrict__ rank) {
  __shared__ int warp_sums[32];
  __shared__ long long carry;
  const int e = blockIdx.x;
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, warps = blockDim.x / 32;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (long long base = 0; base < n; base += blockDim.x) {
    const long long a = base + threadIdx.x;
    const int hit = (a < n && experts[a] == e) ? 1 : 0;
    const unsigned ballot = __ballot_sync(0xffffffffu, hit);
    const int before_in_warp = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) warp_sums[warp] = __popc(ballot);
    __syncthreads();
    int before_warps = 0, total = 0;
    for (int w = 0; w < warps; ++w) {
      const int c = warp_sums[w];
      before_warps += w < warp ? c : 0;
      total += c;
    }
    if (hit) rank[a] = carry + before_warps + before_in_warp;
    __syncthreads();
    if (threadIdx.x == 0) carry += total;
    __syncthreads();
  }
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

namespace abacus {
namespace ops {

void route_topk(torch::Tensor logits, c10::optional<torch::Tensor> bias, int64_t mode, int64_t top_k,
                double route_scale, torch::Tensor probs, torch::Tensor weights, torch::Tensor indices) {
  const c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kFloat32 && logits.is_contiguous() && logits.dim() == 2,
              "logits: contiguous (tokens, E) fp32");
  const int tokens = static_cast<int>(logits.size(0)), experts = static_cast<int>(logits.size(1));
  TORCH_CHECK(mode == 0 || mode == 1, "mode: 0 softmax, 1 sigmoid");
  TORCH_CHECK(top_k >= 1 && top_k <= experts, "top_k in [1, E]");
  TORCH_CHECK(probs.is_contiguous() && probs.sizes() == logits.sizes(), "probs: (tokens, E)");
  TORCH_CHECK(weights.is_contiguous() && weights.scalar_type() == torch::kFloat32 && weights.numel() == tokens * top_k,
              "weights: (tokens, top_k) fp32");
  TORCH_CHECK(indices.is_contiguous() && indices.scalar_type() == torch::kInt64 && indices.numel() == tokens * top_k,
              "indices: (tokens, top_k) int64");
  const float* b = nullptr;
  if (bias) {
    TORCH_CHECK(bias->is_cuda() && bias->scalar_type() == torch::kFloat32 && bias->is_contiguous() &&
                    bias->numel() == experts,
                "bias: (E,) fp32");
    b = bias->data_ptr<float>();
  }
  if (tokens == 0) return;
  auto s = at::cuda::getCurrentCUDAStream();
  const int grid = (tokens + 255) / 256;
  ABACUS_ROUTER_DISPATCH(experts, {
    route_topk_kernel<kE><<<grid, 256, 0, s>>>(logits.data_ptr<float>(), b, static_cast<int>(mode),
                                               static_cast<int>(top_k), static_cast<float>(route_scale), tokens,
                                               probs.data_ptr<float>(), weights.data_ptr<float>(),
                                               indices.data_ptr<int64_t>());
  })
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

void route_topk_bwd(torch::Tensor probs, torch::Tensor indices, torch::Tensor dweights,
                    c10::optional<torch::Tensor> dprobs, int64_t mode, int64_t top_k, double route_scale,
                    torch::Tensor dlogits) {
  const c10::cuda::CUDAGuard guard(probs.device());
  TORCH_CHECK(probs.is_contiguous() && probs.dim() == 2 && probs.scalar_type() == torch::kFloat32, "probs");
  const int tokens = static_cast<int>(probs.size(0)), experts = static_cast<int>(probs.size(1));
  TORCH_CHECK(indices.is_contiguous() && indices.numel() == tokens * top_k && indices.scalar_type() == torch::kInt64,
              "indices");
  TORCH_CHECK(dweights.is_contiguous() && dweights.numel() == tokens * top_k, "dweights");
  TORCH_CHECK(dlogits.is_contiguous() && dlogits.sizes() == probs.sizes(), "dlogits");
  const float* dp = nullptr;
  if (dprobs) {
    TORCH_CHECK(dprobs->is_contiguous() && dprobs->sizes() == probs.sizes(), "dprobs");
    dp = dprobs->data_ptr<float>();
  }
  if (tokens == 0) return;
  auto s = at::cuda::getCurrentCUDAStream();
  const int grid = (tokens + 255) / 256;
  ABACUS_ROUTER_DISPATCH(experts, {
    route_topk_bwd_kernel<kE><<<grid, 256, 0, s>>>(probs.data_ptr<float>(), indices.data_ptr<int64_t>(),
                                                   dweights.data_ptr<float>(), dp, static_cast<int>(mode),
                                                   static_cast<int>(top_k), static_cast<float>(route_scale), tokens,
                                                   dlogits.data_ptr<float>());
  })
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

}  // namespace ops
}  // namespace abacus

namespace abacus {
namespace ops {

void expert_rank(torch::Tensor experts, int64_t n_experts, torch::Tensor rank) {
  const c10::cuda::CUDAGuard guard(experts.device());
  TORCH_CHECK(experts.is_cuda() && experts.scalar_type() == torch::kInt64 && experts.is_contiguous(),
              "experts: contiguous int64 assignment list");
  TORCH_CHECK(rank.is_cuda() && rank.scalar_type() == torch::kInt64 && rank.is_contiguous() &&
                  rank.numel() == experts.numel(),
              "rank: int64, one per assignment");
  TORCH_CHECK(n_experts >= 1 && n_experts <= 65535, "1..65535 experts");
  if (experts.numel() == 0) return;
  expert_rank_kernel<<<static_cast<unsigned>(n_experts), 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      experts.data_ptr<int64_t>(), experts.numel(), rank.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

}  // namespace ops
}  // namespace abacus
