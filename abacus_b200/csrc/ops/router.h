// Router scores of a mixture-of-experts layer: logits = x @ w (w is (D, E),
// E <= 64 experts) and its backward, without a library GEMM; the routing
// (probabilities, top-k, weights) and its backward.
#pragma once
#include <torch/extension.h>

namespace abacus {
namespace ops {
void router_logits(torch::Tensor x, torch::Tensor w, torch::Tensor logits);
void router_logits_bwd(torch::Tensor dlogits, torch::Tensor x, torch::Tensor w, torch::Tensor dx, torch::Tensor dw);
// Routing: probabilities (softmax or sigmoid), top-k selection and the
// renormalised, scaled weights, and the gradient of the logits.
void route_topk(torch::Tensor logits, c10::optional<torch::Tensor> bias, int64_t mode, int64_t top_k,
                double route_scale, torch::Tensor probs, torch::Tensor weights, torch::Tensor indices);
void route_topk_bwd(torch::Tensor probs, torch::Tensor indices, torch::Tensor dweights,
                    c10::optional<torch::Tensor> dprobs, int64_t mode, int64_t top_k, double route_scale,
                    torch::Tensor dlogits);
// rank[a] = number of earlier assignments (in list order) to the same expert
// as assignment a: the capacity slot of static expert slabs.
void expert_rank(torch::Tensor experts, int64_t n_experts, torch::Tensor rank);
}  // namespace ops
}  // namespace abacus
