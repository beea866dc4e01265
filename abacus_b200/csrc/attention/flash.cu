// Host side of the tcgen05 flash attention: tensor maps over token-major
// (B*L, ld) q / k / v matrices (head h occupies columns [h*D, (h+1)*D)),
// launch configuration and argument checks.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cmath>
#include "flash_fwd.cuh"
#include "flash_bwd.cuh"
#include "../common/host.h"
#include "../api.h"

namespace abacus {
namespace attn {
namespace {

CUtensorMap map2d(const torch::Tensor& t, int box_rows, bool mn_major) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.dim() == 2 && t.stride(1) == 1,
              "attention operands must be 2-D fp32 CUDA tensors with unit inner stride");
  TORCH_CHECK(t.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "attention operand rows must be 16-byte aligned");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(t.size(1)), static_cast<cuuint64_t>(t.size(0))};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(t.stride(0) * 4)};
  cuuint32_t box[2] = {32, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = host::encode_tiled()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, t.data_ptr(), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", static_cast<int>(r), ")");
  return m;
}

template <int D, int PASSES>
void launch_fwd(const FwdParams& p, dim3 grid, cudaStream_t s) {
  using Cfg = FwdCfg<D, PASSES>;
  static host::PerDeviceOnce once;
  once.run([&] {
    C10_CUDA_CHECK(cudaFuncSetAttribute(flash_fwd_kernel<D, PASSES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Cfg::kSmemBytes));
  });
  flash_fwd_kernel<D, PASSES><<<grid, Cfg::kThreads, Cfg::kSmemBytes, s>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

// Optional phase trace of the forward kernel (debugging / profiling aid).
long long* g_fwd_trace = nullptr;
long long* g_bwd_trace = nullptr;

const int64_t* positions_ptr(const c10::optional<torch::Tensor>& pos, int64_t len, const char* name) {
  if (!pos) return nullptr;
  TORCH_CHECK(pos->is_cuda() && pos->scalar_type() == torch::kInt64 && pos->is_contiguous() && pos->numel() == len,
              name, " must be a contiguous int64 CUDA tensor of the sequence length");
  return pos->data_ptr<int64_t>();
}

}  // namespace

namespace {
void flash_fwd_impl(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                    int64_t batch, int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes,
                    const std::vector<int64_t>& wait);
void flash_bwd_impl(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor dout,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, int64_t batch,
                    int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes,
                    const std::vector<int64_t>& scatter);
}  // namespace

// Point the forward kernel's phase trace at `buf` (>= 9 * 64 int64 on the
// device), or switch it off with None.
void flash_fwd_trace(c10::optional<torch::Tensor> buf) {
  if (!buf) {
    g_fwd_trace = nullptr;
    g_bwd_trace = nullptr;
    return;
  }
  TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == torch::kInt64 && buf->is_contiguous() && buf->numel() >= 18 * 64,
              "trace buffer: contiguous int64 CUDA tensor of >= 1152 entries");
  g_fwd_trace = reinterpret_cast<long long*>(buf->data_ptr<int64_t>());
  g_bwd_trace = g_fwd_trace + 9 * 64;  // the dK/dV kernel's stamps follow
}

void flash_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                    int64_t batch, int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes) {
  flash_fwd_impl(q, k, v, out, lse, batch, heads, head_dim, lq, lk, scale, q_pos, k_pos, passes, {});
}

// Context-parallel forward: K / V are the gathered buffers every rank pushes
// its shard into; wait = [flags_ptr, epoch, ranks, self].
void flash_attn_fwd_cp(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                       int64_t batch, int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                       c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes,
                       std::vector<int64_t> wait) {
  TORCH_CHECK(wait.size() == 4, "wait = [flags, epoch, ranks, self]");
  flash_fwd_impl(q, k, v, out, lse, batch, heads, head_dim, lq, lk, scale, q_pos, k_pos, passes, wait);
}

namespace {
void flash_fwd_impl(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                    int64_t batch, int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes,
                    const std::vector<int64_t>& wait) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(passes == 1 || passes == 3, "passes must be 1 or 3");
  TORCH_CHECK(head_dim == 64 || (head_dim == 128 && passes == 1) || (head_dim == 32),
              "flash attention supports head_dim 32/64 (tf32 and fp32 modes) and 128 (tf32 mode)");
  TORCH_CHECK(q.size(0) == batch * lq && k.size(0) == batch * lk && v.size(0) == batch * lk, "row counts");
  TORCH_CHECK(q.size(1) >= heads * head_dim && k.size(1) >= heads * head_dim && v.size(1) >= heads * head_dim,
              "head columns");
  TORCH_CHECK(out.is_contiguous() && out.size(0) == batch * lq && out.size(1) == heads * head_dim, "out shape");
  TORCH_CHECK(lse.is_contiguous() && lse.numel() == batch * heads * lq, "lse shape");
  TORCH_CHECK((q_pos.has_value() == k_pos.has_value()), "pass both position arrays or neither");
  TORCH_CHECK(q_pos.has_value() || lq == lk, "plain causal attention needs Lq == Lk");
  TORCH_CHECK((lk + kBlockN - 1) / kBlockN <= 2048, "sequence too long for one attention call");
  if (batch == 0 || lq == 0) return;
  FwdParams p;
  memset(&p, 0, sizeof(p));
  p.tma_q = map2d(q, kBlockM, false);
  p.tma_k = map2d(k, kBlockN, false);
  p.tma_v = map2d(v, kBlockN, true);
  p.out = out.data_ptr<float>();
  p.ld_o = out.stride(0);
  p.lse = lse.data_ptr<float>();
  p.q_pos = positions_ptr(q_pos, lq, "q_pos");
  p.k_pos = positions_ptr(k_pos, lk, "k_pos");
  p.batch = static_cast<int>(batch);
  p.heads = static_cast<int>(heads);
  p.lq = static_cast<int>(lq);
  p.lk = static_cast<int>(lk);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.status = host::status_ptr(q.device().index());
  p.trace = g_fwd_trace;
  if (!wait.empty()) {
    TORCH_CHECK(wait[2] >= 1 && wait[2] <= 8 && wait[3] >= 0 && wait[3] < wait[2], "bad wait spec");
    p.wait_flags = reinterpret_cast<const int*>(wait[0]);
    p.wait_epoch = static_cast<int>(wait[1]);
    p.wait_world = static_cast<int>(wait[2]);
    p.wait_self = static_cast<int>(wait[3]);
  }
  dim3 grid(static_cast<unsigned>((lq + kBlockM - 1) / kBlockM), static_cast<unsigned>(heads),
            static_cast<unsigned>(batch));
  auto s = at::cuda::getCurrentCUDAStream();
  if (head_dim == 64) {
    if (passes == 3) launch_fwd<64, 3>(p, grid, s);
    else launch_fwd<64, 1>(p, grid, s);
  } else if (head_dim == 32) {
    if (passes == 3) launch_fwd<32, 3>(p, grid, s);
    else launch_fwd<32, 1>(p, grid, s);
  } else {
    launch_fwd<128, 1>(p, grid, s);
  }
}
}  // namespace

namespace {

// Delta[b, h, q] = sum_d dO[b*L+q, h*D+d] * O[b*L+q, h*D+d]; one warp per (row, head).
__global__ void attn_delta_kernel(const float* __restrict__ out, long long ld_o, const float* __restrict__ dout,
                                  long long ld_do, float* __restrict__ delta, int batch, int heads, int lq, int hd) {
  const long long item = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const long long total = static_cast<long long>(batch) * lq * heads;
  if (item >= total) return;
  const int lane = threadIdx.x % 32;
  const int h = static_cast<int>(item % heads);
  const long long row = item / heads;  // b * lq + q
  const float* o = out + row * ld_o + h * hd;
  const float* g = dout + row * ld_do + h * hd;
  float s = 0.f;
  for (int d = lane; d < hd; d += 32) s += o[d] * g[d];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    const long long b = row / lq, q = row % lq;
    delta[(b * heads + h) * lq + q] = s;
  }
}

template <int D, int PASSES>
void prepare_bwd(BwdParams& p, const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                 const torch::Tensor& dout) {
  constexpr int inner = DkdvCfg<D, PASSES>::kInner;
  // dkdv: K, V tiles of 128 keys; Q / dO tiles of `inner` queries in both layouts.
  // dq:   Q, dO tiles of 128 queries; K (both layouts) and V tiles of `inner` keys.
  p.tma_k_k = map2d(k, 128, false);
  p.tma_v_k = map2d(v, 128, false);
  p.tma_q_k = map2d(q, inner, false);
  p.tma_q_mn = map2d(q, inner, true);
  p.tma_do_k = map2d(dout, inner, false);
  p.tma_do_mn = map2d(dout, inner, true);
}

template <int D, int PASSES>
void prepare_bwd_dq(BwdParams& p, const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                    const torch::Tensor& dout) {
  constexpr int inner = DqCfg<D, PASSES>::kInner;
  p.tma_q_k = map2d(q, 128, false);
  p.tma_do_k = map2d(dout, 128, false);
  p.tma_k_k = map2d(k, inner, false);
  p.tma_k_mn = map2d(k, inner, true);
  p.tma_v_k = map2d(v, inner, false);
}

template <int D, int PASSES>
void run_bwd(BwdParams p, const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
             const torch::Tensor& dout, int lq, int lk, cudaStream_t s) {
  using A = DkdvCfg<D, PASSES>;
  using Q = DqCfg<D, PASSES>;
  static host::PerDeviceOnce once;
  once.run([&] {
    C10_CUDA_CHECK(cudaFuncSetAttribute(flash_bwd_dkdv_kernel<D, PASSES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        A::kSmemBytes));
    C10_CUDA_CHECK(cudaFuncSetAttribute(flash_bwd_dq_kernel<D, PASSES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        Q::kSmemBytes));
  });
  BwdParams pa = p;
  prepare_bwd<D, PASSES>(pa, q, k, v, dout);
  dim3 ga(static_cast<unsigned>((lk + 127) / 128), static_cast<unsigned>(p.heads), static_cast<unsigned>(p.batch));
  flash_bwd_dkdv_kernel<D, PASSES><<<ga, A::kThreads, A::kSmemBytes, s>>>(pa);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
  BwdParams pq = p;
  prepare_bwd_dq<D, PASSES>(pq, q, k, v, dout);
  dim3 gq(static_cast<unsigned>((lq + 127) / 128), static_cast<unsigned>(p.heads), static_cast<unsigned>(p.batch));
  flash_bwd_dq_kernel<D, PASSES><<<gq, Q::kThreads, Q::kSmemBytes, s>>>(pq);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
}

}  // namespace

void flash_attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor dout,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, int64_t batch,
                    int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes) {
  flash_bwd_impl(q, k, v, out, dout, lse, dq, dk, dv, batch, heads, head_dim, lq, lk, scale, q_pos, k_pos, passes,
                 {});
}

// Context-parallel backward: dK / dV of the gathered keys are stored straight
// into their owners' staging slots (dk / dv here are this rank's slot views,
// which fix the row stride); scatter = [chunk, dk_0.., dv_0.., counter_0..].
void flash_attn_bwd_cp(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor dout,
                       torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, int64_t batch,
                       int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                       c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes,
                       std::vector<int64_t> scatter) {
  TORCH_CHECK(scatter.size() >= 4 && (scatter.size() - 1) % 3 == 0, "scatter = [chunk, dk.., dv.., counters..]");
  flash_bwd_impl(q, k, v, out, dout, lse, dq, dk, dv, batch, heads, head_dim, lq, lk, scale, q_pos, k_pos, passes,
                 scatter);
}

namespace {
void flash_bwd_impl(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor dout,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, int64_t batch,
                    int64_t heads, int64_t head_dim, int64_t lq, int64_t lk, double scale,
                    c10::optional<torch::Tensor> q_pos, c10::optional<torch::Tensor> k_pos, int64_t passes,
                    const std::vector<int64_t>& scatter) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(passes == 1 || passes == 3, "passes must be 1 or 3");
  TORCH_CHECK(head_dim == 64 || head_dim == 32 || (head_dim == 128 && passes == 1),
              "flash attention backward supports head_dim 32/64 (tf32 and fp32 modes) and 128 (tf32 mode)");
  TORCH_CHECK(q_pos.has_value() == k_pos.has_value(), "pass both position arrays or neither");
  TORCH_CHECK(q_pos.has_value() || lq == lk, "plain causal attention needs Lq == Lk");
  TORCH_CHECK(dout.stride(1) == 1 && dout.size(0) == batch * lq, "dout layout");
  for (auto* t : {&dq, &dk, &dv}) TORCH_CHECK(t->stride(1) == 1 && t->stride(0) % 4 == 0, "gradient layouts");
  if (batch == 0 || lq == 0) return;
  auto delta = torch::empty({batch, heads, lq}, q.options());
  auto s = at::cuda::getCurrentCUDAStream();
  {
    const long long items = batch * lq * heads;
    attn_delta_kernel<<<static_cast<unsigned>((items + 7) / 8), 256, 0, s>>>(
        out.data_ptr<float>(), out.stride(0), dout.data_ptr<float>(), dout.stride(0), delta.data_ptr<float>(),
        static_cast<int>(batch), static_cast<int>(heads), static_cast<int>(lq), static_cast<int>(head_dim));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  abacus::host::note_launch();
  }
  BwdParams p;
  memset(&p, 0, sizeof(p));
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq = dq.data_ptr<float>();
  p.ld_dq = dq.stride(0);
  p.dk = dk.data_ptr<float>();
  p.ld_dk = dk.stride(0);
  p.dv = dv.data_ptr<float>();
  p.ld_dv = dv.stride(0);
  p.q_pos = positions_ptr(q_pos, lq, "q_pos");
  p.k_pos = positions_ptr(k_pos, lk, "k_pos");
  p.batch = static_cast<int>(batch);
  p.heads = static_cast<int>(heads);
  p.lq = static_cast<int>(lq);
  p.lk = static_cast<int>(lk);
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.status = host::status_ptr(q.device().index());
  p.trace = g_bwd_trace;
  if (!scatter.empty()) {
    const size_t world = (scatter.size() - 1) / 3;
    TORCH_CHECK(world >= 1 && world <= 8, "scatter over 1..8 ranks");
    TORCH_CHECK(scatter[0] % 128 == 0 && scatter[0] * static_cast<int64_t>(world) == lk,
                "key chunk must be a multiple of 128 and cover the gathered keys");
    p.scatter_chunk = static_cast<int>(scatter[0]);
    for (size_t i = 0; i < world; ++i) {
      p.scatter_dk[i] = reinterpret_cast<float*>(scatter[1 + i]);
      p.scatter_dv[i] = reinterpret_cast<float*>(scatter[1 + world + i]);
      p.scatter_counter[i] = reinterpret_cast<unsigned*>(scatter[1 + 2 * world + i]);
    }
  }
  const int LQ = static_cast<int>(lq), LK = static_cast<int>(lk);
  if (head_dim == 64) {
    if (passes == 3) run_bwd<64, 3>(p, q, k, v, dout, LQ, LK, s);
    else run_bwd<64, 1>(p, q, k, v, dout, LQ, LK, s);
  } else if (head_dim == 32) {
    if (passes == 3) run_bwd<32, 3>(p, q, k, v, dout, LQ, LK, s);
    else run_bwd<32, 1>(p, q, k, v, dout, LQ, LK, s);
  } else {
    run_bwd<128, 1>(p, q, k, v, dout, LQ, LK, s);
  }
}
}  // namespace

}  // namespace attn
}  // namespace abacus
