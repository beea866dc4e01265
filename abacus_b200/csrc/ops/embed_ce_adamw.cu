// Embedding gather / deterministic scatter-add (abacus/embedding.py:19-23),
// cross entropy with the gradient written in the same pass
// (abacus/trainer.py:81-85, F.cross_entropy semantics with ignore_index),
// and multi-tensor AdamW (abacus/optimizers/adamw.py:84-119).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cfloat>
#include "../api.h"
#include "../common/host.h"

namespace abacus {
namespace ops {
namespace {

// ---------------------------------------------------------------- embedding
// out[t, :] = w[tok[t], :]; one warp per token, float4 traffic.
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ tok, const float* __restrict__ w, float* __restrict__ out,
                                     long long tokens, int dim, long long vocab) {
  const long long t = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  if (t >= tokens) return;
  const int lane = threadIdx.x % 32;
  long long v = tok[t];
  v = v < 0 ? 0 : (v >= vocab ? vocab - 1 : v);
  const float4* src = reinterpret_cast<const float4*>(w + v * dim);
  float4* dst = reinterpret_cast<float4*>(out + t * dim);
  for (int i = lane; i < dim / 4; i += 32) dst[i] = src[i];
}

// dw[v, :] = sum over the sorted run of tokens equal to v (fixed order).
// sorted_tok / perm come from a stable sort, so the sum order is the token
// order: deterministic run to run.
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ sorted_tok, const int64_t* __restrict__ perm,
                                     const float* __restrict__ dy, float* __restrict__ dw, long long tokens, int dim) {
  const long long i = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  if (i >= tokens) return;
  const long long v = sorted_tok[i];
  if (i > 0 && sorted_tok[i - 1] == v) return;  // not the start of a run
  const int lane = threadIdx.x % 32;
  float4* dst = reinterpret_cast<float4*>(dw + v * dim);
  for (int c = lane; c < dim / 4; c += 32) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (long long j = i; j < tokens && sorted_tok[j] == v; ++j) {
      const float4 g = reinterpret_cast<const float4*>(dy + perm[j] * dim)[c];
      acc.x += g.x; acc.y += g.y; acc.z += g.z; acc.w += g.w;
    }
    dst[c] = acc;
  }
}

// ---------------------------------------------------------------- cross entropy
// One block per row. Pass 1: online max / sum-of-exp. Pass 2: overwrite the
// logits row with d(loss)/d(logits) * grad_scale. loss[row] = lse - z[target]
// (0 for ignored rows).
constexpr int kCeThreads = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  s = (m == -FLT_MAX ? 0.f : s * __expf(m - mx)) + (m2 == -FLT_MAX ? 0.f : s2 * __expf(m2 - mx));
  m = mx;
}

__global__ void __launch_bounds__(kCeThreads) ce_fwd_bwd_kernel(float* __restrict__ logits, long long ld,
                                                                const int64_t* __restrict__ target, float* __restrict__ loss,
                                                                float* __restrict__ lse_out, int vocab, long long ignore_index,
                                                                const float* __restrict__ grad_scale, int write_grad) {
  const long long row = blockIdx.x;
  float* z = logits + row * ld;
  const long long t = target[row];
  const bool ignored = (t == ignore_index);
  float m = -FLT_MAX, s = 0.f;
  const int n4 = vocab / 4;
  const float4* z4 = reinterpret_cast<const float4*>(z);
  for (int i = threadIdx.x; i < n4; i += kCeThreads) {
    const float4 v = z4[i];
    const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
    if (mx > m) {
      s = (m == -FLT_MAX ? 0.f : s * __expf(m - mx));
      m = mx;
    }
    s += __expf(v.x - m) + __expf(v.y - m) + __expf(v.z - m) + __expf(v.w - m);
  }
  for (int i = n4 * 4 + threadIdx.x; i < vocab; i += kCeThreads) {
    const float v = z[i];
    if (v > m) {
      s = (m == -FLT_MAX ? 0.f : s * __expf(m - v));
      m = v;
    }
    s += __expf(v - m);
  }
  // Block reduction of (m, s).
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[kCeThreads / 32], ss[kCeThreads / 32];
  __shared__ float lse_sh;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < kCeThreads / 32 ? sm[lane] : -FLT_MAX;
    s = lane < kCeThreads / 32 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      lse_sh = m + logf(s);
      const float zt = (ignored || t < 0 || t >= vocab) ? 0.f : z[t];
      loss[row] = ignored ? 0.f : lse_sh - zt;
      if (lse_out) lse_out[row] = lse_sh;
    }
  }
  __syncthreads();
  if (!write_grad) return;
  const float lse = lse_sh;
  const float scale = ignored ? 0.f : *grad_scale;
  float4* w4 = reinterpret_cast<float4*>(z);
  for (int i = threadIdx.x; i < n4; i += kCeThreads) {
    float4 v = z4[i];
    v.x = __expf(v.x - lse) * scale;
    v.y = __expf(v.y - lse) * scale;
    v.z = __expf(v.z - lse) * scale;
    v.w = __expf(v.w - lse) * scale;
    w4[i] = v;
  }
  for (int i = n4 * 4 + threadIdx.x; i < vocab; i += kCeThreads) z[i] = __expf(z[i] - lse) * scale;
  __syncthreads();
  if (threadIdx.x == 0 && !ignored && t >= 0 && t < vocab) z[t] -= scale;
}

// Gradient only, from a saved log-sum-exp: grad = (softmax - onehot) * scale.
// `grad` may alias `logits`.
__global__ void __launch_bounds__(kCeThreads) ce_grad_kernel(const float* __restrict__ logits, long long ld,
                                                             float* __restrict__ grad, long long ldg,
                                                             const int64_t* __restrict__ target,
                                                             const float* __restrict__ lse_in, int vocab,
                                                             long long ignore_index, const float* __restrict__ grad_scale) {
  const long long row = blockIdx.x;
  const float* z = logits + row * ld;
  float* gz = grad + row * ldg;
  const long long t = target[row];
  const bool ignored = (t == ignore_index);
  const float lse = lse_in[row];
  const float scale = ignored ? 0.f : *grad_scale;
  const int n4 = vocab / 4;
  for (int i = threadIdx.x; i < n4; i += kCeThreads) {
    float4 v = reinterpret_cast<const float4*>(z)[i];
    v.x = __expf(v.x - lse) * scale;
    v.y = __expf(v.y - lse) * scale;
    v.z = __expf(v.z - lse) * scale;
    v.w = __expf(v.w - lse) * scale;
    reinterpret_cast<float4*>(gz)[i] = v;
  }
  for (int i = n4 * 4 + threadIdx.x; i < vocab; i += kCeThreads) gz[i] = __expf(z[i] - lse) * scale;
  __syncthreads();
  if (threadIdx.x == 0 && !ignored && t >= 0 && t < vocab) gz[t] -= scale;
}

// ---------------------------------------------------------------- AdamW
// Reference update order (abacus/optimizers/adamw.py:107-119):
//   w *= 1 - lr*wd; m = lerp(m, g, 1-b1); v = b2*v + (1-b2)*g*g
//   w -= (lr/bc1) * m / (sqrt(v)/sqrt(bc2) + eps)
constexpr int kMaxTensors = 36;

struct AdamWBatch {
  float* w[kMaxTensors];
  const float* g[kMaxTensors];
  float* m[kMaxTensors];
  float* v[kMaxTensors];
  long long numel[kMaxTensors];
  int block_start[kMaxTensors + 1];
  int count;
};

constexpr int kAdamChunk = 4096;

__global__ void __launch_bounds__(256) adamw_kernel(const __grid_constant__ AdamWBatch b, float lr, float beta1, float beta2,
                                                    float eps, float wd, float bc1, float bc2_sqrt) {
  int ti = 0;
  while (ti + 1 < b.count && b.block_start[ti + 1] <= static_cast<int>(blockIdx.x)) ++ti;
  const long long base = static_cast<long long>(blockIdx.x - b.block_start[ti]) * kAdamChunk;
  const long long n = b.numel[ti];
  float* w = b.w[ti];
  const float* g = b.g[ti];
  float* m = b.m[ti];
  float* v = b.v[ti];
  const float decay = 1.f - lr * wd;
  const float step_size = lr / bc1;
  const float w1 = 1.f - beta1, w2 = 1.f - beta2;
  for (long long i = base + threadIdx.x; i < min(n, base + kAdamChunk); i += blockDim.x) {
    float wi = w[i];
    if (wd != 0.f) wi *= decay;
    const float gi = g[i];
    float mi = m[i];
    // torch.lerp for weight < 0.5: start + weight * (end - start)
    mi = w1 < 0.5f ? mi + w1 * (gi - mi) : gi - (gi - mi) * (1.f - w1);
    float vi = v[i] * beta2;
    vi = vi + gi * gi * w2;
    const float denom = sqrtf(vi) / bc2_sqrt + eps;
    wi = wi - step_size * (mi / denom);
    w[i] = wi;
    m[i] = mi;
    v[i] = vi;
  }
}

}  // namespace

void embedding_fwd(torch::Tensor tokens, torch::Tensor weight, torch::Tensor out) {
  const c10::cuda::CUDAGuard guard(weight.device());
  TORCH_CHECK(tokens.scalar_type() == torch::kInt64 && tokens.is_contiguous(), "tokens must be contiguous int64");
  TORCH_CHECK(weight.is_contiguous() && out.is_contiguous() && weight.size(1) % 4 == 0, "embedding layout");
  const long long n = tokens.numel();
  if (n == 0) return;
  const int warps = 8;
  embedding_fwd_kernel<<<static_cast<int>((n + warps - 1) / warps), warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      tokens.data_ptr<int64_t>(), weight.data_ptr<float>(), out.data_ptr<float>(), n, static_cast<int>(weight.size(1)),
      weight.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

void embedding_bwd(torch::Tensor sorted_tokens, torch::Tensor perm, torch::Tensor dy, torch::Tensor dw) {
  const c10::cuda::CUDAGuard guard(dy.device());
  TORCH_CHECK(dy.is_contiguous() && dw.is_contiguous() && dw.size(1) % 4 == 0, "embedding grad layout");
  const long long n = sorted_tokens.numel();
  if (n == 0) return;
  const int warps = 8;
  embedding_bwd_kernel<<<static_cast<int>((n + warps - 1) / warps), warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      sorted_tokens.data_ptr<int64_t>(), perm.data_ptr<int64_t>(), dy.data_ptr<float>(), dw.data_ptr<float>(), n,
      static_cast<int>(dw.size(1)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

void cross_entropy_fwd_bwd(torch::Tensor logits, torch::Tensor target, torch::Tensor loss, c10::optional<torch::Tensor> lse,
                           int64_t ignore_index, torch::Tensor grad_scale, bool write_grad) {
  const c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == torch::kFloat32, "logits layout");
  TORCH_CHECK(logits.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0, "logits alignment");
  TORCH_CHECK(target.scalar_type() == torch::kInt64 && target.is_contiguous(), "target must be contiguous int64");
  const long long rows = logits.size(0);
  if (rows == 0) return;
  TORCH_CHECK(rows < (1LL << 31), "too many rows");
  ce_fwd_bwd_kernel<<<static_cast<int>(rows), kCeThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.stride(0), target.data_ptr<int64_t>(), loss.data_ptr<float>(),
      lse ? lse->data_ptr<float>() : nullptr, static_cast<int>(logits.size(1)), ignore_index,
      grad_scale.data_ptr<float>(), write_grad ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

void cross_entropy_grad(torch::Tensor logits, torch::Tensor grad, torch::Tensor target, torch::Tensor lse,
                        int64_t ignore_index, torch::Tensor grad_scale) {
  const c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.stride(1) == 1 && grad.stride(1) == 1 && logits.stride(0) % 4 == 0 && grad.stride(0) % 4 == 0,
              "cross entropy layouts");
  const long long rows = logits.size(0);
  if (rows == 0) return;
  ce_grad_kernel<<<static_cast<int>(rows), kCeThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), logits.stride(0), grad.data_ptr<float>(), grad.stride(0), target.data_ptr<int64_t>(),
      lse.data_ptr<float>(), static_cast<int>(logits.size(1)), ignore_index, grad_scale.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

void adamw_step(std::vector<torch::Tensor> params, std::vector<torch::Tensor> grads, std::vector<torch::Tensor> exp_avgs,
                std::vector<torch::Tensor> exp_avg_sqs, double lr, double beta1, double beta2, double eps,
                double weight_decay, int64_t step) {
  TORCH_CHECK(params.size() == grads.size() && params.size() == exp_avgs.size() && params.size() == exp_avg_sqs.size());
  if (params.empty()) return;
  const c10::cuda::CUDAGuard guard(params[0].device());
  const float bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  const float bc2_sqrt = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  auto stream = at::cuda::getCurrentCUDAStream();
  size_t i = 0;
  while (i < params.size()) {
    AdamWBatch b;
    memset(&b, 0, sizeof(b));
    int blocks = 0;
    int c = 0;
    for (; i < params.size() && c < kMaxTensors; ++i) {
      auto& p = params[i];
      TORCH_CHECK(p.is_contiguous() && grads[i].is_contiguous() && exp_avgs[i].is_contiguous() &&
                      exp_avg_sqs[i].is_contiguous(),
                  "AdamW tensors must be contiguous");
      TORCH_CHECK(p.numel() == grads[i].numel() && p.numel() == exp_avgs[i].numel(), "AdamW size mismatch");
      if (p.numel() == 0) continue;
      b.w[c] = p.data_ptr<float>();
      b.g[c] = grads[i].data_ptr<float>();
      b.m[c] = exp_avgs[i].data_ptr<float>();
      b.v[c] = exp_avg_sqs[i].data_ptr<float>();
      b.numel[c] = p.numel();
      b.block_start[c] = blocks;
      blocks += static_cast<int>((p.numel() + kAdamChunk - 1) / kAdamChunk);
      ++c;
    }
    b.count = c;
    b.block_start[c] = blocks;
    if (c == 0) continue;
    adamw_kernel<<<blocks, 256, 0, stream>>>(b, static_cast<float>(lr), static_cast<float>(beta1), static_cast<float>(beta2),
                                             static_cast<float>(eps), static_cast<float>(weight_decay), bc1, bc2_sqrt);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
  }
}

}  // namespace ops
}  // namespace abacus
