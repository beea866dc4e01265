// Router scores of a mixture-of-experts layer: logits = x @ w (w is (D, E),
// E <= 64 experts) and its backward, without a library GEMM.
#pragma once
#include <torch/extension.h>

namespace abacus {
namespace ops {
void router_logits(torch::Tensor x, torch::Tensor w, torch::Tensor logits);
void router_logits_bwd(torch::Tensor dlogits, torch::Tensor x, torch::Tensor w, torch::Tensor dx, torch::Tensor dw);
}  // namespace ops
}  // namespace abacus
