// Sequence-parallel <-> tensor-parallel boundary kernels over NVLink peer
// memory (Megatron SP, reference: abacus/distributed/tensor_parallel.py:24-99,
// which runs them as NCCL all-gather / reduce-scatter calls).
//
// Layout. Activations in the SP region are (B, l, D) shards: rank r holds
// positions [r*l, (r+1)*l) of every sequence. The gathered (B*L, D) matrix
// (L = P*l) lives in a symmetric buffer on every rank; rank r's rows are
// b*L + r*l + i.
//
// * tp_push_rows (all-gather, push side): each rank writes its shard rows into
//   every rank's gathered buffer (P2P stores, coalesced 16-byte per lane) and
//   the last CTA to finish publishes `epoch` in every rank's flag slot for
//   this rank (fence + release, system scope). The consuming GEMM waits on
//   those flags per CTA (gemm_tcgen05.cuh, wait_*), so the gather is fused
//   into its first consumer instead of being a separate collective.
// * tp_reduce_rows (reduce-scatter, owner side): the producing GEMM's epilogue
//   already stored every partial tile into its owner's staging slot over
//   NVLink while the other tiles were still computing (scatter_*). This kernel
//   waits for all arrival counters, then sums the P slots in rank order (fixed
//   order: deterministic) and adds the residual in the same pass.
//
// All waits are bounded (ABACUS_PEER_WAIT_NS) and record kStatusTimeoutPeer.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "../api.h"
#include "../common/host.h"
#include "../common/sm100.cuh"

namespace abacus {
namespace comm {
namespace {

constexpr int kMaxRanks = 8;

struct PushArgs {
  float* dst[kMaxRanks];  // gathered buffer base on each rank
  int* flag[kMaxRanks];   // this rank's flag slot on each rank
};

__global__ void __launch_bounds__(256) tp_push_kernel(const __grid_constant__ PushArgs a, const float* __restrict__ x,
                                                      long long rows, int dim, int chunk, int seq, int world, int self,
                                                      int epoch, int* done, int* status) {
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int d4 = dim / 4;
  const bool healthy = *reinterpret_cast<volatile int*>(status) == kStatusOk;
  if (healthy) {
    for (long long r = static_cast<long long>(blockIdx.x) * warps + warp; r < rows;
         r += static_cast<long long>(gridDim.x) * warps) {
      const long long b = r / chunk, i = r % chunk;
      const long long g = b * seq + static_cast<long long>(self) * chunk + i;
      const float4* src = reinterpret_cast<const float4*>(x + r * dim);
      // Four 16-byte loads in flight per lane before the stores.
      for (int c0 = lane; c0 < d4; c0 += 128) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (c0 + 32 * u < d4) v[u] = __ldg(src + c0 + 32 * u);
        }
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p) {
          if (p < world) {
            float4* out = reinterpret_cast<float4*>(a.dst[p] + g * dim);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              if (c0 + 32 * u < d4) out[c0 + 32 * u] = v[u];
            }
          }
        }
      }
    }
  }
  // Last CTA out publishes the epoch (every CTA's stores are fenced first).
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(done, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      __threadfence_system();
      if (healthy) {
        for (int p = 0; p < world; ++p) st_release_sys(a.flag[p], epoch);
      }
      atomicExch(done, 0);
    }
  }
}

__global__ void __launch_bounds__(256) tp_reduce_kernel(const float* __restrict__ staging, long long slot, int world,
                                                        const unsigned* counters, unsigned target,
                                                        const float* __restrict__ residual, float* __restrict__ out,
                                                        long long n4, int* status) {
  __shared__ int ok;
  if (threadIdx.x < 32) {
    bool good = *reinterpret_cast<volatile int*>(status) == kStatusOk;
    if (good && threadIdx.x < world) {
      good = wait_flag_geq(reinterpret_cast<const int*>(counters) + threadIdx.x, static_cast<int>(target), status);
    }
    good = __all_sync(0xffffffffu, good);
    if (threadIdx.x == 0) ok = good ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  const float4* s4 = reinterpret_cast<const float4*>(staging);
  const long long slot4 = slot / 4;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 acc = residual ? reinterpret_cast<const float4*>(residual)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < world; ++q) {
      const float4 v = s4[q * slot4 + i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
}

}  // namespace

void tp_push_rows(torch::Tensor x, std::vector<int64_t> dst_ptrs, std::vector<int64_t> flag_ptrs, int64_t chunk,
                  int64_t seq, int64_t self, int64_t epoch, torch::Tensor done) {
  const c10::cuda::CUDAGuard guard(x.device());
  const size_t world = dst_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && flag_ptrs.size() == world, "1..8 ranks");
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.dim() == 2, "x (rows, D)");
  TORCH_CHECK(x.size(1) % 4 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "rows must be float4 aligned");
  TORCH_CHECK(chunk > 0 && seq == chunk * static_cast<int64_t>(world) && x.size(0) % chunk == 0, "bad SP chunking");
  TORCH_CHECK(self >= 0 && self < static_cast<int64_t>(world), "rank out of range");
  TORCH_CHECK(done.is_cuda() && done.scalar_type() == torch::kInt32 && done.numel() >= 1, "done counter");
  PushArgs a;
  memset(&a, 0, sizeof(a));
  for (size_t p = 0; p < world; ++p) {
    TORCH_CHECK(dst_ptrs[p] % 16 == 0, "gathered buffers must be 16-byte aligned");
    a.dst[p] = reinterpret_cast<float*>(dst_ptrs[p]);
    a.flag[p] = reinterpret_cast<int*>(flag_ptrs[p]);
  }
  const long long rows = x.size(0);
  const int sms = at::cuda::getDeviceProperties(x.device().index())->multiProcessorCount;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((rows + 7) / 8, 4LL * sms)));
  tp_push_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, x.data_ptr<float>(), rows, static_cast<int>(x.size(1)), static_cast<int>(chunk), static_cast<int>(seq),
      static_cast<int>(world), static_cast<int>(self), static_cast<int>(epoch), done.data_ptr<int>(),
      host::status_ptr(x.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

void tp_reduce_rows(torch::Tensor staging, int64_t world, torch::Tensor counters, int64_t target,
                    c10::optional<torch::Tensor> residual, torch::Tensor out) {
  const c10::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "1..8 ranks");
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.scalar_type() == torch::kFloat32, "out");
  TORCH_CHECK(out.numel() % 4 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out float4 aligned");
  TORCH_CHECK(staging.is_contiguous() && staging.numel() == world * out.numel(), "staging holds one slot per rank");
  TORCH_CHECK(counters.scalar_type() == torch::kInt32 && counters.numel() >= world, "counters");
  if (residual) {
    TORCH_CHECK(residual->is_contiguous() && residual->numel() == out.numel(), "residual shape");
  }
  const long long n4 = out.numel() / 4;
  const int sms = at::cuda::getDeviceProperties(out.device().index())->multiProcessorCount;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((n4 + 255) / 256, 4LL * sms)));
  tp_reduce_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      staging.data_ptr<float>(), out.numel(), static_cast<int>(world),
      reinterpret_cast<const unsigned*>(counters.data_ptr<int>()), static_cast<unsigned>(target),
      residual ? residual->data_ptr<float>() : nullptr, out.data_ptr<float>(), n4, host::status_ptr(out.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

}  // namespace comm
}  // namespace abacus
