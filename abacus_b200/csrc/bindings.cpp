// Python bindings of the abacus_b200._C extension (sm_100a kernels).
#include <torch/extension.h>
#include "api.h"
#include "common/host.h"
#include "ops/router.h"
#include "ops/transpose.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm_out", &abacus::gemm::gemm_out, "tcgen05 tf32 / 3xTF32 GEMM into C");
  m.def("gemm_n_tiles", &abacus::gemm::gemm_n_tiles, "N tiles of a single-B GEMM of the given output width");
  m.def("gemm_pair_clusters", &abacus::gemm::gemm_pair_clusters, "CTA pairs of the last CTA-pair GEMM launch");
  m.def("gemm_qkv_norm_rope", &abacus::gemm::gemm_qkv_norm_rope,
        "QKV projection with QK-norm + RoPE fused into the GEMM epilogue");
  m.def("gemm_trace", &abacus::gemm::gemm_trace, "phase trace of the following GEMM launches (None: off)");
  m.def("gemm_grouped", &abacus::gemm::gemm_grouped, "one GEMM launch over (experts, rows, cols) operands");
  m.def("gemm_swiglu_grouped", &abacus::gemm::gemm_swiglu_grouped, "grouped gate/up GEMM with SwiGLU epilogue");
  m.def("gemm_swiglu_bwd_grouped", &abacus::gemm::gemm_swiglu_bwd_grouped,
        "grouped down-projection dgrad with SwiGLU backward epilogue");
  m.def("gemm_out_tp", &abacus::gemm::gemm_out_tp, "GEMM with a peer-gathered operand and/or row-scattered output");
  m.def("gemm_swiglu_tp", &abacus::gemm::gemm_swiglu_tp, "SwiGLU up-projection over a peer-gathered input");
  m.def("gemm_swiglu_bwd_tp", &abacus::gemm::gemm_swiglu_bwd_tp, "SwiGLU backward GEMM over a peer-gathered dy");
  m.def("gemm_batched", &abacus::gemm::gemm_batched, "batched tcgen05 GEMM over (B, H, rows, cols) views");
  m.def("gemm_swiglu", &abacus::gemm::gemm_swiglu, "gate/up GEMM with SwiGLU epilogue");
  m.def("gemm_swiglu_bwd", &abacus::gemm::gemm_swiglu_bwd, "down-projection dgrad with SwiGLU backward epilogue");
  m.def("router_logits", &abacus::ops::router_logits, "MoE router scores x @ w (E <= 64)");
  m.def("router_logits_bwd", &abacus::ops::router_logits_bwd, "gradients of the router scores");
  m.def("route_topk", &abacus::ops::route_topk, "MoE routing: probabilities, top-k experts and weights (E <= 64)");
  m.def("route_topk_bwd", &abacus::ops::route_topk_bwd, "gradient of the routing logits");
  m.def("expert_rank", &abacus::ops::expert_rank, "per-expert rank of each assignment (capacity slots)");
  m.def("transpose2d", &abacus::ops::transpose2d, "out = in^T (fp32, tiled)");
  m.def("rmsnorm_fwd", &abacus::ops::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &abacus::ops::rmsnorm_bwd);
  m.def("qk_prologue_fwd", &abacus::ops::qk_prologue_fwd);
  m.def("qk_prologue_bwd", &abacus::ops::qk_prologue_bwd);
  m.def("embedding_fwd", &abacus::ops::embedding_fwd);
  m.def("embedding_bwd", &abacus::ops::embedding_bwd);
  m.def("cross_entropy_fwd_bwd", &abacus::ops::cross_entropy_fwd_bwd);
  m.def("cross_entropy_grad", &abacus::ops::cross_entropy_grad);
  m.def("adamw_step", &abacus::ops::adamw_step);
  m.def("causal_softmax_fwd", &abacus::attn::causal_softmax_fwd, "in-place causal row softmax (materialised attention)");
  m.def("causal_softmax_bwd", &abacus::attn::causal_softmax_bwd, "in-place dS from P and dP (materialised attention)");
  m.def("flash_attn_fwd_cp", &abacus::attn::flash_attn_fwd_cp, "flash forward over peer-pushed K/V (context parallel)");
  m.def("flash_attn_bwd_cp", &abacus::attn::flash_attn_bwd_cp, "flash backward scattering dK/dV to their owners");
  m.def("flash_attn_fwd", &abacus::attn::flash_attn_fwd);
  m.def("flash_fwd_trace", &abacus::attn::flash_fwd_trace, "phase trace of the flash forward (debugging)");
  m.def("flash_attn_bwd", &abacus::attn::flash_attn_bwd);
  m.def("launch_count", &abacus::host::launch_count, "number of abacus kernels launched by this process");
  m.def("wait_flag", &abacus::comm::wait_flag, "bounded device wait for a flag (error status on timeout)");
  m.def("set_flag", &abacus::comm::set_flag, "release-store a device flag");
  m.def("symm_barrier", &abacus::comm::symm_barrier, "bounded system-scope barrier over peer signal pads");
  m.def("tp_push_rows", &abacus::comm::tp_push_rows, "SP shard -> every rank's gathered buffer + epoch flags");
  m.def("tp_reduce_rows", &abacus::comm::tp_reduce_rows, "sum of scattered partial slots (+ residual) after arrival");
  m.def("ep_push_rows", &abacus::comm::ep_push_rows, "expert-parallel dispatch: rows into their experts' slabs on peers");
  m.def("ep_credit", &abacus::comm::ep_credit, "credit rows that will never return to an expert-parallel counter");
  m.def("ep_combine", &abacus::comm::ep_combine, "expert-parallel combine: weighted sum of returned rows");
  m.def("ar_adamw", &abacus::comm::ar_adamw, "peer-memory gradient reduce + AdamW + parameter broadcast");
  m.def("read_status", &abacus::host::read_status, "device status word (0 = healthy)");
  m.def("reset_status", &abacus::host::reset_status, "clear the device status word");
  m.def(
      "status_tensor",
      [](int64_t device) {
        // A one-element int32 view of the status word, for asynchronous reads.
        return torch::from_blob(abacus::host::status_ptr(static_cast<int>(device)), {1},
                                torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, device));
      },
      "device status word as a 1-element CUDA tensor (no copy)");
}
