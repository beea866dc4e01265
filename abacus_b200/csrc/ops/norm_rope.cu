// RMSNorm (abacus/norm.py:23-31) and the attention prologue QK-RMSNorm + RoPE
// (abacus/attention.py:196-213, abacus/rope.py:31-47), forward and backward.
//
// These are HBM-bound: one warp owns one row (a token for RMSNorm, a
// (token, head) pair for the QK prologue), keeps it in registers, and reads
// and writes it exactly once. gamma gradients are reduced deterministically:
// each block writes a partial row, a second kernel sums the partials.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "../api.h"
#include "rmsnorm_noalloc.h"
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>
#include "../common/host.h"

namespace abacus {
namespace ops {
namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------- RMSNorm
template <int VPL>  // float4 vectors per lane
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                                 float* __restrict__ y, float* __restrict__ rstd, int rows,
                                                                 int dim, float eps) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row = blockIdx.x * kWarps + warp;
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(row) * dim);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  float4 v[VPL];
  float ss = 0.f;
  const int n4 = dim / 4;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int idx = lane + 32 * i;
    v[i] = idx < n4 ? xr[idx] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / dim + eps);
  if (lane == 0) rstd[row] = r;
  float4* yr = reinterpret_cast<float4*>(y + static_cast<long long>(row) * dim);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int idx = lane + 32 * i;
    if (idx < n4) {
      const float4 g = g4[idx];
      yr[idx] = make_float4(g.x * v[i].x * r, g.y * v[i].y * r, g.z * v[i].z * r, g.w * v[i].w * r);
    }
  }
}

// dx = r * (g*dy) - x * r^3 * mean(g*dy*x); partial dgamma += dy * x * r
template <int VPL>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                                 const float* __restrict__ gamma, const float* __restrict__ rstd,
                                                                 float* __restrict__ dx, float* __restrict__ partial, int rows,
                                                                 int dim, int rows_per_block) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n4 = dim / 4;
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  float4 acc[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  const int row_begin = blockIdx.x * rows_per_block;
  const int row_end = min(rows, row_begin + rows_per_block);
  for (int row = row_begin + warp; row < row_end; row += kWarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<long long>(row) * dim);
    const float4* dr = reinterpret_cast<const float4*>(dy + static_cast<long long>(row) * dim);
    const float r = rstd[row];
    float4 xv[VPL], gd[VPL];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int idx = lane + 32 * i;
      if (idx < n4) {
        xv[i] = xr[idx];
        const float4 d = dr[idx];
        const float4 g = g4[idx];
        gd[i] = make_float4(g.x * d.x, g.y * d.y, g.z * d.z, g.w * d.w);
        dot += gd[i].x * xv[i].x + gd[i].y * xv[i].y + gd[i].z * xv[i].z + gd[i].w * xv[i].w;
        acc[i].x += d.x * xv[i].x * r;
        acc[i].y += d.y * xv[i].y * r;
        acc[i].z += d.z * xv[i].z * r;
        acc[i].w += d.w * xv[i].w * r;
      }
    }
    dot = warp_sum(dot);
    const float c = dot * r * r * r / dim;
    float4* dxr = reinterpret_cast<float4*>(dx + static_cast<long long>(row) * dim);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int idx = lane + 32 * i;
      if (idx < n4)
        dxr[idx] = make_float4(r * gd[i].x - xv[i].x * c, r * gd[i].y - xv[i].y * c, r * gd[i].z - xv[i].z * c,
                               r * gd[i].w - xv[i].w * c);
    }
  }
  // Per-warp partial rows of dgamma (reduced by reduce_partials_kernel).
  float4* prow = reinterpret_cast<float4*>(partial + (static_cast<long long>(blockIdx.x) * kWarps + warp) * dim);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int idx = lane + 32 * i;
    if (idx < n4) prow[idx] = acc[i];
  }
}

// out[j] = sum_b partial[b][j] (fixed order -> deterministic)
__global__ void reduce_partials_kernel(const float* __restrict__ partial, float* __restrict__ out, int nblocks, int dim) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= dim) return;
  float s = 0.f;
  for (int b = 0; b < nblocks; ++b) s += partial[static_cast<long long>(b) * dim + j];
  out[j] = s;
}

// Column sums of a (rows, dim) partial matrix in two deterministic passes:
// block (column tile of 32, row split) sums its rows with 8 row lanes in a
// fixed order and combines the lanes in order; then reduce_partials_kernel
// adds the splits in order. Enough CTAs to keep HBM busy for tall inputs.
__global__ void __launch_bounds__(256) colsum_split_kernel(const float* __restrict__ in, float* __restrict__ out,
                                                           long long rows, int dim, long long rows_per_split) {
  const int lane = threadIdx.x % 32, r0 = threadIdx.x / 32;
  const int c = blockIdx.x * 32 + lane;
  const long long begin = static_cast<long long>(blockIdx.y) * rows_per_split;
  const long long end = min(rows, begin + rows_per_split);
  float acc = 0.f;
  if (c < dim) {
    for (long long r = begin + r0; r < end; r += 8) acc += in[r * dim + c];
  }
  __shared__ float sh[8][32];
  sh[r0][lane] = acc;
  __syncthreads();
  if (r0 == 0 && c < dim) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += sh[k][lane];
    out[static_cast<long long>(blockIdx.y) * dim + c] = t;
  }
}

void column_sums(const float* partial, long long rows, int dim, float* out, const torch::TensorOptions& opts,
                 cudaStream_t s) {
  const long long splits = std::max<long long>(1, std::min<long long>(1024, (rows + 63) / 64));
  const long long per = (rows + splits - 1) / splits;
  auto mid = torch::empty({splits, dim}, opts);
  dim3 grid(static_cast<unsigned>((dim + 31) / 32), static_cast<unsigned>(splits));
  colsum_split_kernel<<<grid, 256, 0, s>>>(partial, mid.data_ptr<float>(), rows, dim, per);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
  reduce_partials_kernel<<<(dim + 255) / 256, 256, 0, s>>>(mid.data_ptr<float>(), out, static_cast<int>(splits), dim);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

// ---------------------------------------------------------------- QK prologue
// One warp per (token, head). Lane i handles the rotate-half pairs (i, i+K/2),
// (i+32, i+32+K/2), ... so normalisation and rotation stay in registers.
// qkv: (T, 3*H*K) raw projections; positions: (T,) int64 (global positions);
// cos/sin: (P, K/2) tables indexed by position.
template <int PPL>  // pairs per lane = K / 64
__global__ void __launch_bounds__(kWarps * 32) qk_prologue_fwd_kernel(
    const float* __restrict__ qkv, long long ld_qkv, const float* __restrict__ gq, const float* __restrict__ gk,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, const int64_t* __restrict__ positions,
    int seq_len, float* __restrict__ q_out, float* __restrict__ k_out, float* __restrict__ rstd, int tokens, int heads,
    int head_dim, float eps) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const long long item = static_cast<long long>(blockIdx.x) * kWarps + warp;  // (token, which, head)
  const long long total = static_cast<long long>(tokens) * 2 * heads;
  if (item >= total) return;
  const int head = static_cast<int>(item % heads);
  const int which = static_cast<int>((item / heads) % 2);  // 0 = q, 1 = k
  const long long t = item / (2 * heads);
  const int half = head_dim / 2;
  const float* src = qkv + t * ld_qkv + static_cast<long long>(which) * heads * head_dim + head * head_dim;
  const float* gamma = which == 0 ? gq : gk;
  const long long pos = positions ? positions[t] : (t % seq_len);
  float a[PPL], b[PPL];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < PPL; ++p) {
    const int i = lane + 32 * p;
    a[p] = i < half ? src[i] : 0.f;
    b[p] = i < half ? src[i + half] : 0.f;
    ss += a[p] * a[p] + b[p] * b[p];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / head_dim + eps);
  if (lane == 0) rstd[item] = r;
  float* dst = (which == 0 ? q_out : k_out) + t * static_cast<long long>(heads) * head_dim + head * head_dim;
#pragma unroll
  for (int p = 0; p < PPL; ++p) {
    const int i = lane + 32 * p;
    if (i < half) {
      const float n1 = gamma[i] * a[p] * r;
      const float n2 = gamma[i + half] * b[p] * r;
      const float c = cos_t[pos * half + i];
      const float s = sin_t[pos * half + i];
      dst[i] = n1 * c - n2 * s;
      dst[i + half] = n2 * c + n1 * s;
    }
  }
}

// Backward: inverse-rotate dq/dk, then RMSNorm backward over head_dim.
// dqkv receives dq, dk in its first two thirds; partial dgamma rows:
// partial[(block, which)][K].
template <int PPL>
__global__ void __launch_bounds__(kWarps * 32) qk_prologue_bwd_kernel(
    const float* __restrict__ qkv, long long ld_qkv, const float* __restrict__ gq, const float* __restrict__ gk,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, const int64_t* __restrict__ positions,
    int seq_len, const float* __restrict__ dq, const float* __restrict__ dk, const float* __restrict__ rstd,
    float* __restrict__ dqkv, long long ld_dqkv, float* __restrict__ partial, int tokens, int heads, int head_dim,
    int items_per_block) {
  extern __shared__ float sh[];  // [2][kWarps][head_dim]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int half = head_dim / 2;
  float acc_a[2][PPL], acc_b[2][PPL];
#pragma unroll
  for (int w = 0; w < 2; ++w)
#pragma unroll
    for (int p = 0; p < PPL; ++p) acc_a[w][p] = acc_b[w][p] = 0.f;
  const long long total = static_cast<long long>(tokens) * 2 * heads;
  const long long begin = static_cast<long long>(blockIdx.x) * items_per_block;
  const long long end = min(total, begin + items_per_block);
  for (long long item = begin + warp; item < end; item += kWarps) {
    const int head = static_cast<int>(item % heads);
    const int which = static_cast<int>((item / heads) % 2);
    const long long t = item / (2 * heads);
    const float* src = qkv + t * ld_qkv + static_cast<long long>(which) * heads * head_dim + head * head_dim;
    const float* grad = (which == 0 ? dq : dk) + t * static_cast<long long>(heads) * head_dim + head * head_dim;
    const float* gamma = which == 0 ? gq : gk;
    const long long pos = positions ? positions[t] : (t % seq_len);
    const float r = rstd[item];
    float xa[PPL], xb[PPL], gna[PPL], gnb[PPL];
    float dot = 0.f;
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane + 32 * p;
      if (i < half) {
        const float c = cos_t[pos * half + i];
        const float s = sin_t[pos * half + i];
        const float d1 = grad[i], d2 = grad[i + half];
        // d(normed) = R^T d(rotated)
        const float dn1 = d1 * c + d2 * s;
        const float dn2 = -d1 * s + d2 * c;
        xa[p] = src[i];
        xb[p] = src[i + half];
        gna[p] = gamma[i] * dn1;
        gnb[p] = gamma[i + half] * dn2;
        dot += gna[p] * xa[p] + gnb[p] * xb[p];
        if (which == 0) {
          acc_a[0][p] += dn1 * xa[p] * r;
          acc_b[0][p] += dn2 * xb[p] * r;
        } else {
          acc_a[1][p] += dn1 * xa[p] * r;
          acc_b[1][p] += dn2 * xb[p] * r;
        }
      } else {
        xa[p] = xb[p] = gna[p] = gnb[p] = 0.f;
      }
    }
    dot = warp_sum(dot);
    const float cc = dot * r * r * r / head_dim;
    float* out = dqkv + t * ld_dqkv + static_cast<long long>(which) * heads * head_dim + head * head_dim;
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane + 32 * p;
      if (i < half) {
        out[i] = r * gna[p] - xa[p] * cc;
        out[i + half] = r * gnb[p] - xb[p] * cc;
      }
    }
  }
#pragma unroll
  for (int w = 0; w < 2; ++w)
#pragma unroll
    for (int p = 0; p < PPL; ++p) {
      const int i = lane + 32 * p;
      if (i < half) {
        sh[(w * kWarps + warp) * head_dim + i] = acc_a[w][p];
        sh[(w * kWarps + warp) * head_dim + i + half] = acc_b[w][p];
      }
    }
  __syncthreads();
  for (int j = threadIdx.x; j < 2 * head_dim; j += blockDim.x) {
    const int w = j / head_dim, i = j % head_dim;
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < kWarps; ++q) s += sh[(w * kWarps + q) * head_dim + i];
    partial[(static_cast<long long>(blockIdx.x) * 2 + w) * head_dim + i] = s;
  }
}

void check_f32_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32, name, " must be a CUDA fp32 tensor");
}

int partial_blocks(const torch::Device& dev, long long items) {
  const int sms = at::cuda::getDeviceProperties(dev.index())->multiProcessorCount;
  return static_cast<int>(std::max<long long>(1, std::min<long long>(items, 4LL * sms)));
}

}  // namespace

void rmsnorm_fwd(torch::Tensor x, torch::Tensor gamma, torch::Tensor y, torch::Tensor rstd, double eps) {
  check_f32_cuda(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = static_cast<int>(x.size(0)), dim = static_cast<int>(x.size(1));
  TORCH_CHECK(dim % 4 == 0 && dim <= 4096, "RMSNorm kernel supports dim % 4 == 0 and dim <= 4096");
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && gamma.is_contiguous(), "contiguous tensors required");
  if (rows == 0) return;
  const int grid = (rows + kWarps - 1) / kWarps;
  auto s = at::cuda::getCurrentCUDAStream();
  const int vpl = (dim / 4 + 31) / 32;
#define LAUNCH(V)                                                                                                    \
  rmsnorm_fwd_kernel<V><<<grid, kWarps * 32, 0, s>>>(x.data_ptr<float>(), gamma.data_ptr<float>(), y.data_ptr<float>(), \
                                                    rstd.data_ptr<float>(), rows, dim, static_cast<float>(eps))
  if (vpl <= 2) LAUNCH(2);
  else if (vpl <= 4) LAUNCH(4);
  else if (vpl <= 8) LAUNCH(8);
  else if (vpl <= 16) LAUNCH(16);
  else LAUNCH(32);
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor gamma, torch::Tensor rstd, torch::Tensor dx,
                 torch::Tensor dgamma) {
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = static_cast<int>(x.size(0)), dim = static_cast<int>(x.size(1));
  TORCH_CHECK(dim % 4 == 0 && dim <= 4096, "RMSNorm kernel supports dim % 4 == 0 and dim <= 4096");
  if (rows == 0) {
    dgamma.zero_();
    return;
  }
  const int nblocks = partial_blocks(x.device(), (rows + kWarps - 1) / kWarps);
  const int rows_per_block = (rows + nblocks - 1) / nblocks;
  auto partial = torch::empty({nblocks * kWarps, dim}, x.options());
  auto s = at::cuda::getCurrentCUDAStream();
  const int vpl = (dim / 4 + 31) / 32;
  const size_t smem = 0;
#define LAUNCH(V)                                                                                                   \
  rmsnorm_bwd_kernel<V><<<nblocks, kWarps * 32, smem, s>>>(dy.data_ptr<float>(), x.data_ptr<float>(),                \
                                                          gamma.data_ptr<float>(), rstd.data_ptr<float>(),         \
                                                          dx.data_ptr<float>(), partial.data_ptr<float>(), rows, dim, \
                                                          rows_per_block)
  if (vpl <= 2) LAUNCH(2);
  else if (vpl <= 4) LAUNCH(4);
  else if (vpl <= 8) LAUNCH(8);
  else if (vpl <= 16) LAUNCH(16);
  else LAUNCH(32);
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
  column_sums(partial.data_ptr<float>(), static_cast<long long>(nblocks) * kWarps, dim, dgamma.data_ptr<float>(),
              x.options(), s);
}

void qk_prologue_fwd(torch::Tensor qkv, torch::Tensor gq, torch::Tensor gk, torch::Tensor cos_t, torch::Tensor sin_t,
                     c10::optional<torch::Tensor> positions, int64_t seq_len, torch::Tensor q_out, torch::Tensor k_out,
                     torch::Tensor rstd, int64_t heads, int64_t head_dim, double eps) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int tokens = static_cast<int>(qkv.size(0));
  TORCH_CHECK(head_dim % 2 == 0 && head_dim <= 256, "head_dim must be even and <= 256");
  TORCH_CHECK(qkv.stride(1) == 1 && qkv.size(1) >= 2 * heads * head_dim, "qkv layout");
  TORCH_CHECK(q_out.is_contiguous() && k_out.is_contiguous(), "q/k outputs must be contiguous");
  if (tokens == 0) return;
  const long long items = static_cast<long long>(tokens) * 2 * heads;
  const int grid = static_cast<int>((items + kWarps - 1) / kWarps);
  const int64_t* pos = positions ? positions->data_ptr<int64_t>() : nullptr;
  auto s = at::cuda::getCurrentCUDAStream();
#define LAUNCH(P)                                                                                                      \
  qk_prologue_fwd_kernel<P><<<grid, kWarps * 32, 0, s>>>(                                                              \
      qkv.data_ptr<float>(), qkv.stride(0), gq.data_ptr<float>(), gk.data_ptr<float>(), cos_t.data_ptr<float>(),      \
      sin_t.data_ptr<float>(), pos, static_cast<int>(seq_len), q_out.data_ptr<float>(), k_out.data_ptr<float>(),      \
      rstd.data_ptr<float>(), tokens, static_cast<int>(heads), static_cast<int>(head_dim), static_cast<float>(eps))
  if (head_dim <= 64) LAUNCH(1);
  else if (head_dim <= 128) LAUNCH(2);
  else LAUNCH(4);
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

void qk_prologue_bwd(torch::Tensor qkv, torch::Tensor gq, torch::Tensor gk, torch::Tensor cos_t, torch::Tensor sin_t,
                     c10::optional<torch::Tensor> positions, int64_t seq_len, torch::Tensor dq, torch::Tensor dk,
                     torch::Tensor rstd, torch::Tensor dqkv, torch::Tensor dgq, torch::Tensor dgk, int64_t heads,
                     int64_t head_dim) {
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int tokens = static_cast<int>(qkv.size(0));
  const long long items = static_cast<long long>(tokens) * 2 * heads;
  if (tokens == 0) {
    dgq.zero_();
    dgk.zero_();
    return;
  }
  TORCH_CHECK(dq.is_contiguous() && dk.is_contiguous() && dqkv.stride(1) == 1, "layouts");
  const int nblocks = partial_blocks(qkv.device(), (items + kWarps - 1) / kWarps);
  const int per_block = static_cast<int>((items + nblocks - 1) / nblocks);
  auto partial = torch::empty({nblocks, 2, head_dim}, qkv.options());
  const int64_t* pos = positions ? positions->data_ptr<int64_t>() : nullptr;
  auto s = at::cuda::getCurrentCUDAStream();
  const size_t smem = 2 * kWarps * head_dim * sizeof(float);
#define LAUNCH(P)                                                                                                   \
  qk_prologue_bwd_kernel<P><<<nblocks, kWarps * 32, smem, s>>>(                                                     \
      qkv.data_ptr<float>(), qkv.stride(0), gq.data_ptr<float>(), gk.data_ptr<float>(), cos_t.data_ptr<float>(),   \
      sin_t.data_ptr<float>(), pos, static_cast<int>(seq_len), dq.data_ptr<float>(), dk.data_ptr<float>(),         \
      rstd.data_ptr<float>(), dqkv.data_ptr<float>(), dqkv.stride(0), partial.data_ptr<float>(), tokens,            \
      static_cast<int>(heads), static_cast<int>(head_dim), per_block)
  if (head_dim <= 64) LAUNCH(1);
  else if (head_dim <= 128) LAUNCH(2);
  else LAUNCH(4);
#undef LAUNCH
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
  auto sums = torch::empty({2 * head_dim}, qkv.options());
  column_sums(partial.data_ptr<float>(), nblocks, static_cast<int>(2 * head_dim), sums.data_ptr<float>(), qkv.options(),
              s);
  dgq.copy_(sums.narrow(0, 0, head_dim));
  dgk.copy_(sums.narrow(0, head_dim, head_dim));
}

}  // namespace ops
}  // namespace abacus

// ============================================================================
// Allocation-free RMSNorm backward (C ABI). Declared in rmsnorm_noalloc.h.
//
// The backward above reduces dgamma through a scratch buffer of per-warp
// partial rows that it allocates on every call. This variant runs the same two
// kernels but keeps that scratch in a fixed file-scope device array, so the
// call performs no device allocation at all.
// ============================================================================
namespace abacus {
namespace ops {
namespace {

// Scratch for the dgamma reduction, split in two regions: per-warp partial
// rows ((blocks * kWarps) rows of `dim` floats) and the per-split column sums
// of those rows (`splits` rows of `dim` floats).
constexpr long long kNoAllocScratchFloats = 1LL << 20;  // 4 MiB per GPU
constexpr long long kNoAllocMidFloats = 1LL << 18;      // last 1 MiB: split sums
constexpr long long kNoAllocPartialFloats = kNoAllocScratchFloats - kNoAllocMidFloats;
static __device__ __align__(256) float g_rmsnorm_noalloc_scratch[kNoAllocScratchFloats];

// Per device: SM count, then the scratch array's device address. The address
// is published last with release order, so a reader that sees it (acquire)
// also sees the SM count.
std::atomic<float*> g_scratch_addr[64] = {};
std::atomic<int> g_sm_count[64] = {};
std::mutex g_noalloc_mu;

int noalloc_setup(int device) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_scratch_addr[device].load(std::memory_order_acquire) != nullptr) return 0;
  // Host code cannot use the array's name as a device address: ask the
  // runtime for it, with `device` current.
  void* ptr = nullptr;
  cudaError_t err = cudaGetSymbolAddress(&ptr, g_rmsnorm_noalloc_scratch);
  if (err != cudaSuccess) return static_cast<int>(err);
  int sms = 0;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (err != cudaSuccess) return static_cast<int>(err);
  g_sm_count[device].store(sms, std::memory_order_relaxed);
  g_scratch_addr[device].store(static_cast<float*>(ptr), std::memory_order_release);
  return 0;
}

bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

}  // namespace
}  // namespace ops
}  // namespace abacus

extern "C" __attribute__((visibility("default"))) int abacus_rmsnorm_bwd_noalloc(
    const float* dy, const float* x, const float* gamma, const float* rstd, float* dx, float* dgamma, int rows,
    int dim, void* stream) {
  using namespace abacus::ops;
  if (rows < 0 || dim <= 0 || dim % 4 != 0 || dim > 4096) return ABACUS_NOALLOC_EBADSIZE;
  if (dy == nullptr || x == nullptr || gamma == nullptr || rstd == nullptr || dx == nullptr || dgamma == nullptr)
    return ABACUS_NOALLOC_EBADSIZE;
  // The kernels move dy / x / dx / gamma / dgamma / scratch rows as float4.
  if (misaligned16(dy) || misaligned16(x) || misaligned16(gamma) || misaligned16(rstd) || misaligned16(dx) ||
      misaligned16(dgamma))
    return ABACUS_NOALLOC_EBADSIZE;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return static_cast<int>(err);
  if (device < 0 || device >= 64) return ABACUS_NOALLOC_EBADSIZE;
  float* scratch = g_scratch_addr[device].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    const int rc = noalloc_setup(device);
    if (rc != 0) return rc;
    scratch = g_scratch_addr[device].load(std::memory_order_acquire);
  }
  const int sms = g_sm_count[device].load(std::memory_order_relaxed);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* partial = scratch;
  float* mid = scratch + kNoAllocPartialFloats;
  // Partial rows that fit in their region; at least one block.
  const long long max_blocks = kNoAllocPartialFloats / (static_cast<long long>(kWarps) * dim);
  if (max_blocks < 1) return ABACUS_NOALLOC_EBADSIZE;
  const long long want = std::max<long long>(1, std::min<long long>((rows + kWarps - 1) / kWarps, 4LL * sms));
  const int nblocks = static_cast<int>(std::min(want, max_blocks));
  const int rows_per_block = rows == 0 ? 0 : (rows + nblocks - 1) / nblocks;
  const int vpl = (dim / 4 + 31) / 32;
  // Every partial row read below is written by this call (idle warps write
  // zeros), and every split sum is written before it is read, so the scratch
  // needs no clearing between calls.
#define ABACUS_NOALLOC_LAUNCH(V)                                                                                  \
  rmsnorm_bwd_kernel<V><<<nblocks, kWarps * 32, 0, s>>>(dy, x, gamma, rstd, dx, partial, rows, dim, rows_per_block)
  if (vpl <= 2) ABACUS_NOALLOC_LAUNCH(2);
  else if (vpl <= 4) ABACUS_NOALLOC_LAUNCH(4);
  else if (vpl <= 8) ABACUS_NOALLOC_LAUNCH(8);
  else if (vpl <= 16) ABACUS_NOALLOC_LAUNCH(16);
  else ABACUS_NOALLOC_LAUNCH(32);
#undef ABACUS_NOALLOC_LAUNCH
  err = cudaGetLastError();
  if (err != cudaSuccess) return static_cast<int>(err);
  // Two-pass deterministic column sums of the partial rows (the regular
  // backward's schedule), with the split sums in the second region.
  const long long prow = static_cast<long long>(nblocks) * kWarps;
  const long long max_splits = std::max<long long>(1, kNoAllocMidFloats / dim);
  const long long splits = std::max<long long>(1, std::min<long long>({max_splits, 1024LL, (prow + 63) / 64}));
  const long long per = (prow + splits - 1) / splits;
  dim3 grid(static_cast<unsigned>((dim + 31) / 32), static_cast<unsigned>(splits));
  colsum_split_kernel<<<grid, 256, 0, s>>>(partial, mid, prow, dim, per);
  err = cudaGetLastError();
  if (err != cudaSuccess) return static_cast<int>(err);
  reduce_partials_kernel<<<(dim + 255) / 256, 256, 0, s>>>(mid, dgamma, static_cast<int>(splits), dim);
  err = cudaGetLastError();
  if (err != cudaSuccess) return static_cast<int>(err);
  abacus::host::note_launch(3);
  return 0;
}
