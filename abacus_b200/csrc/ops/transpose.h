// Tiled 2-D transpose (fp32): out (N, M) contiguous = in (M, N)^T, in with any
// row stride. Used to give the weight-gradient GEMM x^T @ dy a K-major A.
#pragma once
#include <torch/extension.h>

namespace abacus {
namespace ops {
void transpose2d(torch::Tensor in, torch::Tensor out);
}  // namespace ops
}  // namespace abacus
