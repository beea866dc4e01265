// Expert-parallel dispatch / combine over NVLink peer memory (reference:
// abacus/distributed/expert_parallel.py:29-59 and abacus/moe/moe.py, which
// permute rows by expert, exchange them with an NCCL all-to-all, run the
// experts, exchange back and un-permute).
//
// * ep_push_rows (dispatch, fused with the router's permutation): assignment
//   a = (token t, slot j) is written straight into its expert's slab on the
//   owning rank, at the row the host precomputed from the exchanged counts
//   (slab of local expert, then source rank, then (t, j) order), optionally
//   scaled (backward: the router weight). A side array records, per received
//   row, where its result must go back: meta = a * 8 + source rank. The last
//   CTA publishes `epoch` in every rank's flag slot for this rank; the expert
//   GEMMs wait for all ranks' flags before reading (gemm wait operand 2).
// * The expert down-projection GEMM then stores each output row straight back
//   into its source rank's return buffer at row a (gemm row-map scatter) and
//   counts the rows per destination.
// * ep_combine (source side): waits until every row came back, then
//   out[t] = sum_j w[t, j] * ret[t*k + j] in slot order (or the plain sum).
//
// With a capacity (static slabs: every source owns a fixed-size region of
// each expert's slab, so no counts exchange and no host sync is needed), an
// assignment over its expert's capacity has dest_rank -1 and is not sent;
// its source credits the missing rows to its own return counter (ep_credit)
// and gives the slot weight 0 in the combine.
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

struct EpPeers {
  float* rows[kMaxRanks];  // destination row buffer on each rank
  int* meta[kMaxRanks];    // destination meta array on each rank
  int* flag[kMaxRanks];    // this rank's flag slot on each rank
};

__global__ void __launch_bounds__(256) ep_push_kernel(const __grid_constant__ EpPeers peers, const float* __restrict__ src,
                                                      int top_k, const int* __restrict__ dest_rank,
                                                      const int* __restrict__ dest_row, const float* __restrict__ scale,
                                                      long long assignments, int dim, int world, int self, int epoch,
                                                      int* done, int* status) {
  const int warps = blockDim.x / 32;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int d4 = dim / 4;
  const bool healthy = *reinterpret_cast<volatile int*>(status) == kStatusOk;
  if (healthy) {
    for (long long a = static_cast<long long>(blockIdx.x) * warps + warp; a < assignments;
         a += static_cast<long long>(gridDim.x) * warps) {
      const int r = dest_rank[a];
      if (r < 0) continue;  // dropped (over its expert's capacity): not sent
      const long long row = dest_row[a];
      const float s = scale ? scale[a] : 1.f;
      const float4* in = reinterpret_cast<const float4*>(src + (a / top_k) * dim);
      float4* out = reinterpret_cast<float4*>(peers.rows[r] + row * dim);
      for (int c = lane; c < d4; c += 32) {
        float4 v = in[c];
        v.x *= s;
        v.y *= s;
        v.z *= s;
        v.w *= s;
        out[c] = v;
      }
      if (lane == 0) peers.meta[r][row] = static_cast<int>(a) * 8 + self;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(done, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      __threadfence_system();
      if (healthy) {
        for (int p = 0; p < world; ++p) st_release_sys(peers.flag[p], epoch);
      }
      atomicExch(done, 0);
    }
  }
}

__global__ void __launch_bounds__(256) ep_combine_kernel(const float* __restrict__ ret, const float* __restrict__ weights,
                                                         int top_k, long long tokens, int dim, const int* counter,
                                                         int target, float* __restrict__ out, int* status) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const bool good = *reinterpret_cast<volatile int*>(status) == kStatusOk && wait_flag_geq(counter, target, status);
    ok = good ? 1 : 0;
  }
  __syncthreads();
  if (!ok) return;
  const int d4 = dim / 4;
  const long long n4 = tokens * d4;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long t = i / d4, c = i % d4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < top_k; ++j) {
      const float w = weights ? weights[t * top_k + j] : 1.f;
      // A zero weight marks a slot with nothing to add (an assignment dropped
      // over capacity has no returned row; its buffer row is stale).
      if (w == 0.f) continue;
      const float4 v = reinterpret_cast<const float4*>(ret + (t * top_k + j) * dim)[c];
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
}

// Adds amount[0] * multiplier to a return counter on this GPU. Rows that were
// never sent (dropped over capacity) never come back; crediting them keeps the
// counter target a host-side constant. Atomic against the peers' concurrent
// system-scope adds to the same counter.
__global__ void ep_credit_kernel(int* counter, const int* amount, int multiplier) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const int add = amount[0] * multiplier;
    if (add != 0) atomicAdd(counter, add);
  }
}

}  // namespace

void ep_credit(torch::Tensor counter, torch::Tensor amount, int64_t multiplier) {
  const c10::cuda::CUDAGuard guard(counter.device());
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == torch::kInt32 && counter.numel() >= 1, "counter");
  TORCH_CHECK(amount.is_cuda() && amount.scalar_type() == torch::kInt32 && amount.numel() >= 1, "amount: int32");
  ep_credit_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(counter.data_ptr<int>(), amount.data_ptr<int>(),
                                                                    static_cast<int>(multiplier));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

void ep_push_rows(torch::Tensor src, int64_t top_k, torch::Tensor dest_rank, torch::Tensor dest_row,
                  c10::optional<torch::Tensor> scale, std::vector<int64_t> row_ptrs, std::vector<int64_t> meta_ptrs,
                  std::vector<int64_t> flag_ptrs, int64_t self, int64_t epoch, torch::Tensor done) {
  const c10::cuda::CUDAGuard guard(src.device());
  const size_t world = row_ptrs.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && meta_ptrs.size() == world && flag_ptrs.size() == world,
              "1..8 ranks");
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kFloat32 && src.is_contiguous() && src.dim() == 2,
              "src (tokens, D) contiguous fp32");
  TORCH_CHECK(src.size(1) % 4 == 0 && reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0, "rows float4 aligned");
  const long long assignments = src.size(0) * top_k;
  TORCH_CHECK(assignments < (1LL << 28), "too many assignments for the row meta encoding");
  TORCH_CHECK(dest_rank.scalar_type() == torch::kInt32 && dest_row.scalar_type() == torch::kInt32 &&
                  dest_rank.numel() == assignments && dest_row.numel() == assignments && dest_rank.is_contiguous() &&
                  dest_row.is_contiguous(),
              "dest_rank / dest_row: int32, one per assignment");
  if (scale) TORCH_CHECK(scale->scalar_type() == torch::kFloat32 && scale->numel() == assignments && scale->is_contiguous(),
                         "scale: fp32, one per assignment");
  TORCH_CHECK(self >= 0 && self < static_cast<int64_t>(world), "rank out of range");
  EpPeers peers;
  memset(&peers, 0, sizeof(peers));
  for (size_t p = 0; p < world; ++p) {
    TORCH_CHECK(row_ptrs[p] % 16 == 0 && meta_ptrs[p] % 4 == 0, "peer buffers misaligned");
    peers.rows[p] = reinterpret_cast<float*>(row_ptrs[p]);
    peers.meta[p] = reinterpret_cast<int*>(meta_ptrs[p]);
    peers.flag[p] = reinterpret_cast<int*>(flag_ptrs[p]);
  }
  const int sms = at::cuda::getDeviceProperties(src.device().index())->multiProcessorCount;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((assignments + 7) / 8, 2LL * sms)));
  ep_push_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      peers, src.data_ptr<float>(), static_cast<int>(top_k), dest_rank.data_ptr<int>(), dest_row.data_ptr<int>(),
      scale ? scale->data_ptr<float>() : nullptr, assignments, static_cast<int>(src.size(1)), static_cast<int>(world),
      static_cast<int>(self), static_cast<int>(epoch), done.data_ptr<int>(), host::status_ptr(src.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

void ep_combine(torch::Tensor ret, c10::optional<torch::Tensor> weights, int64_t top_k, torch::Tensor counter,
                int64_t target, torch::Tensor out) {
  const c10::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(out.is_contiguous() && out.dim() == 2 && out.size(1) % 4 == 0, "out (tokens, D)");
  TORCH_CHECK(ret.is_contiguous() && ret.numel() >= out.numel() * top_k, "return buffer (tokens*k, D)");
  if (weights) TORCH_CHECK(weights->is_contiguous() && weights->numel() == out.size(0) * top_k, "weights (tokens, k)");
  TORCH_CHECK(counter.scalar_type() == torch::kInt32 && counter.numel() >= 1, "counter");
  const long long n4 = out.numel() / 4;
  const int sms = at::cuda::getDeviceProperties(out.device().index())->multiProcessorCount;
  const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((n4 + 255) / 256, 4LL * sms)));
  ep_combine_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ret.data_ptr<float>(), weights ? weights->data_ptr<float>() : nullptr, static_cast<int>(top_k), out.size(0),
      static_cast<int>(out.size(1)), counter.data_ptr<int>(), static_cast<int>(target), out.data_ptr<float>(),
      host::status_ptr(out.device().index()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  host::note_launch();
}

}  // namespace comm
}  // namespace abacus
