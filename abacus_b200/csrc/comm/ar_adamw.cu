// Data-parallel gradient all-reduce fused with the AdamW update, over NVLink
// peer memory (one process per GPU, buffers mapped into every peer).
//
// Every rank keeps its gradients (flat, fp32) and its replica of the
// parameters (flat) in symmetric buffers. One step:
//
//   1. symm_barrier: every rank's gradients are complete (bounded wait on the
//      peers' signal-pad flags, release / acquire at system scope).
//   2. ar_adamw_kernel: rank r owns the flat slice [lo_r, hi_r). For each
//      element of its slice it loads the P peers' gradients over NVLink,
//      forms the token-weighted mean sum_p w_p * g_p (w_p = count_p / total),
//      applies AdamW with the moments of the owned slice (the moments exist
//      only there), and stores the new parameter value into every peer's
//      replica. Reduce-scatter, optimizer and all-gather are one pass:
//      2 N (P-1) / P bytes cross NVLink per rank, the all-reduce minimum, and
//      no separate optimizer pass over the parameters.
//   3. symm_barrier: every peer's stores into this replica, and every peer's
//      reads of this rank's gradients, are done before the next step.
//
// All waits are bounded: a peer that never arrives turns into
// kStatusTimeoutPeer in the device status word and the kernels return.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "../api.h"
#include "../common/host.h"
#include "../common/sm100.cuh"

namespace abacus {
namespace comm {
namespace {

constexpr int kMaxPeers = 8;

struct PeerTable {
  float* grad[kMaxPeers];
  float* param[kMaxPeers];
  int* signal[kMaxPeers];
  float* exch[kMaxPeers];  // per-rank exchange rows carried by the barrier
  const float* counts;     // device: per-rank target-token counts
  long long counts_stride;
};

__device__ __forceinline__ int ld_acquire_sys_i32(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_i32(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread p < world copies `payload` (n floats) into row [rank] of peer p's
// exchange buffer, publishes `epoch` into peer p's slot [rank] (the release
// orders the row before the flag), then waits until its own slot [p] reaches
// `epoch`. Epochs only grow, so one set of slots serves every barrier: a rank
// can reach epoch e+1 only after every rank arrived at e.
__global__ void symm_barrier_kernel(const __grid_constant__ PeerTable t, int rank, int world, int slot_base, int epoch,
                                    unsigned long long timeout_ns, int* status, const float* payload, int n) {
  const int p = threadIdx.x;
  __threadfence_system();
  if (p < world && n > 0) {
    for (int j = 0; j < n; ++j) t.exch[p][rank * n + j] = payload[j];
  }
  if (p < world) st_release_sys_i32(t.signal[p] + slot_base + rank, epoch);
  if (p < world) {
    const int* mine = t.signal[rank] + slot_base + p;
    const unsigned long long start = globaltimer_ns();
    unsigned it = 0;
    while (ld_acquire_sys_i32(mine) < epoch) {
      if ((++it & 63u) == 0 && globaltimer_ns() - start > timeout_ns) {
        atomicCAS(status, kStatusOk, kStatusTimeoutPeer);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  __threadfence_system();
}

// With `local` set (ZeRO-3: this rank stores only its own slice of the
// parameters), the slice is read from and written to local[i - lo4] and no
// replica is updated on the peers: a reduce-scatter fused with the
// partitioned AdamW update.
__global__ void __launch_bounds__(256) ar_adamw_kernel(const __grid_constant__ PeerTable t, int rank, int world,
                                                        long long lo4, long long hi4, float* __restrict__ m,
                                                        float* __restrict__ v, float lr, float beta1, float beta2,
                                                        float eps, float wd, float bc1, float bc2_sqrt, int normalize,
                                                        float* __restrict__ local, int* status) {
  if (*reinterpret_cast<volatile int*>(status) != kStatusOk) return;
  const float decay = 1.f - lr * wd;
  const float step_size = lr / bc1;
  const float w1 = 1.f - beta1, w2 = 1.f - beta2;
  // Token-weighted mean: w_p = count_p / sum_q count_q (reference semantics,
  // abacus/distributed/data_parallel.py:141-161); plain sum when !normalize.
  float weight[kMaxPeers];
  float total = 0.f;
#pragma unroll
  for (int p = 0; p < kMaxPeers; ++p) {
    weight[p] = p < world ? t.counts[p * t.counts_stride] : 0.f;
    total += weight[p];
  }
  const float inv_total = !normalize ? 1.f : (total > 0.f ? 1.f / total : 0.f);
#pragma unroll
  for (int p = 0; p < kMaxPeers; ++p) weight[p] *= inv_total;
  const float4* params = local ? reinterpret_cast<const float4*>(local) - lo4
                                : reinterpret_cast<const float4*>(t.param[rank]);
  float4* m4 = reinterpret_cast<float4*>(m);
  float4* v4 = reinterpret_cast<float4*>(v);
  for (long long i = lo4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < hi4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < kMaxPeers; ++p) {
      if (p < world) {
        const float4 x = reinterpret_cast<const float4*>(t.grad[p])[i];
        const float w = weight[p];
        g.x += w * x.x;
        g.y += w * x.y;
        g.z += w * x.z;
        g.w += w * x.w;
      }
    }
    float4 wv = params[i];
    float4 mv = m4[i - lo4];
    float4 vv = v4[i - lo4];
    auto upd = [&](float& wi, float& mi, float& vi, float gi) {
      if (wd != 0.f) wi *= decay;
      mi = w1 < 0.5f ? mi + w1 * (gi - mi) : gi - (gi - mi) * (1.f - w1);
      vi = vi * beta2 + gi * gi * w2;
      wi = wi - step_size * (mi / (sqrtf(vi) / bc2_sqrt + eps));
    };
    upd(wv.x, mv.x, vv.x, g.x);
    upd(wv.y, mv.y, vv.y, g.y);
    upd(wv.z, mv.z, vv.z, g.z);
    upd(wv.w, mv.w, vv.w, g.w);
    m4[i - lo4] = mv;
    v4[i - lo4] = vv;
    if (local) {
      reinterpret_cast<float4*>(local)[i - lo4] = wv;
    } else {
#pragma unroll
      for (int p = 0; p < kMaxPeers; ++p) {
        if (p < world) reinterpret_cast<float4*>(t.param[p])[i] = wv;
      }
    }
  }
  __threadfence_system();
}

PeerTable make_table(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& param_ptrs,
                     const std::vector<int64_t>& signal_ptrs, const std::vector<int64_t>& exch_ptrs) {
  const size_t world = grad_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxPeers, "1 to 8 ranks");
  TORCH_CHECK(param_ptrs.size() == world && signal_ptrs.size() == world, "pointer tables differ in size");
  PeerTable t;
  memset(&t, 0, sizeof(t));
  for (size_t p = 0; p < world; ++p) {
    TORCH_CHECK(grad_ptrs[p] % 16 == 0 && param_ptrs[p] % 16 == 0, "peer buffers must be 16-byte aligned");
    t.grad[p] = reinterpret_cast<float*>(grad_ptrs[p]);
    t.param[p] = reinterpret_cast<float*>(param_ptrs[p]);
    t.signal[p] = reinterpret_cast<int*>(signal_ptrs[p]);
    t.exch[p] = exch_ptrs.empty() ? nullptr : reinterpret_cast<float*>(exch_ptrs[p]);
  }
  return t;
}

}  // namespace

void symm_barrier(std::vector<int64_t> signal_ptrs, int64_t rank, int64_t slot_base, int64_t epoch, double timeout_ms,
                  std::vector<int64_t> exch_ptrs, c10::optional<torch::Tensor> payload) {
  const size_t world = signal_ptrs.size();
  TORCH_CHECK(rank >= 0 && rank < static_cast<int64_t>(world), "rank out of range");
  TORCH_CHECK(epoch > 0 && epoch < (1LL << 31), "epoch must be a positive int32");
  std::vector<int64_t> dummy(world, 0);
  int n = 0;
  const float* pay = nullptr;
  if (payload.has_value()) {
    TORCH_CHECK(exch_ptrs.size() == world, "one exchange buffer per rank");
    TORCH_CHECK(payload->is_cuda() && payload->scalar_type() == torch::kFloat32 && payload->is_contiguous(),
                "payload must be contiguous float32 on the device");
    n = static_cast<int>(payload->numel());
    pay = payload->data_ptr<float>();
  } else {
    exch_ptrs.clear();
  }
  PeerTable t = make_table(dummy, dummy, signal_ptrs, exch_ptrs);
  auto s = at::cuda::getCurrentCUDAStream();
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  symm_barrier_kernel<<<1, 32, 0, s>>>(t, static_cast<int>(rank), static_cast<int>(world), static_cast<int>(slot_base),
                                       static_cast<int>(epoch), static_cast<unsigned long long>(timeout_ms * 1e6),
                                       host::status_ptr(dev), pay, n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

void ar_adamw(std::vector<int64_t> grad_ptrs, std::vector<int64_t> param_ptrs, torch::Tensor counts,
              bool normalize, int64_t rank, int64_t lo, int64_t hi, torch::Tensor exp_avg, torch::Tensor exp_avg_sq,
              double lr, double beta1, double beta2, double eps, double weight_decay, int64_t step, int64_t max_ctas,
              c10::optional<torch::Tensor> local_param) {
  const c10::cuda::CUDAGuard guard(exp_avg.device());
  TORCH_CHECK(lo % 4 == 0 && hi % 4 == 0 && hi >= lo, "owned range must be float4 aligned");
  TORCH_CHECK(exp_avg.is_contiguous() && exp_avg_sq.is_contiguous() && exp_avg.numel() == hi - lo &&
                  exp_avg_sq.numel() == hi - lo,
              "moments must cover the owned range");
  TORCH_CHECK(counts.is_cuda() && counts.scalar_type() == torch::kFloat32 && counts.dim() == 1 &&
                  counts.numel() == static_cast<int64_t>(grad_ptrs.size()),
              "counts must be a 1-D float32 CUDA tensor with one entry per rank");
  TORCH_CHECK(rank >= 0 && rank < static_cast<int64_t>(grad_ptrs.size()), "rank out of range");
  float* local = nullptr;
  if (local_param) {
    TORCH_CHECK(local_param->is_cuda() && local_param->scalar_type() == torch::kFloat32 &&
                    local_param->is_contiguous() && local_param->numel() == hi - lo &&
                    reinterpret_cast<uintptr_t>(local_param->data_ptr()) % 16 == 0,
                "local_param: the owned slice, contiguous fp32, 16-byte aligned");
    local = local_param->data_ptr<float>();
    param_ptrs.assign(grad_ptrs.size(), 0);  // no replica to update
  }
  std::vector<int64_t> dummy(grad_ptrs.size(), 0);
  PeerTable t = make_table(grad_ptrs, param_ptrs, dummy, {});
  t.counts = counts.data_ptr<float>();
  t.counts_stride = counts.stride(0);
  if (hi == lo) return;
  const float bc1 = static_cast<float>(1.0 - std::pow(beta1, static_cast<double>(step)));
  const float bc2s = static_cast<float>(std::sqrt(1.0 - std::pow(beta2, static_cast<double>(step))));
  const long long n4 = (hi - lo) / 4;
  const int sms = at::cuda::getDeviceProperties(exp_avg.device().index())->multiProcessorCount;
  // max_ctas > 0 caps the grid, so a reduction that runs beside other
  // kernels (under backward) leaves them most of the SMs.
  const long long cap = max_ctas > 0 ? max_ctas : 8LL * sms;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((n4 + 255) / 256, cap)));
  ar_adamw_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      t, static_cast<int>(rank), static_cast<int>(grad_ptrs.size()), lo / 4, hi / 4, exp_avg.data_ptr<float>(),
      exp_avg_sq.data_ptr<float>(), static_cast<float>(lr), static_cast<float>(beta1), static_cast<float>(beta2),
      static_cast<float>(eps), static_cast<float>(weight_decay), bc1, bc2s, normalize ? 1 : 0, local,
      host::status_ptr(exp_avg.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

}  // namespace comm
}  // namespace abacus
