// Allocation-free entry point for the RMSNorm backward pass.
//
// This entry point has no counterpart in the reference framework; it is an
// addition of this library for callers that cannot allocate device memory:
// code embedded in a host application that owns the GPU memory budget (a
// plugin or custom-operator interface that hands over input and output
// pointers but no allocator), and latency-critical loops that must not reach
// cudaMalloc / cudaFree, whose calls can serialise against the whole device.
//
// What it computes (row-wise RMSNorm y = gamma * x * rstd, rstd saved by the
// forward pass as 1 / sqrt(mean(x^2) + eps)):
//   dx[r, :]  = rstd[r] * gamma * dy[r, :]
//               - x[r, :] * rstd[r]^3 * mean_j(gamma[j] * dy[r, j] * x[r, j])
//   dgamma[:] = sum_r dy[r, :] * x[r, :] * rstd[r]
// It gives the same results as the library's regular RMSNorm backward, which
// allocates a temporary buffer for the dgamma reduction on every call. Here
// that temporary lives in a fixed 4 MiB array in device memory that every GPU
// loading this library holds until the process exits.
//
// Arguments: device pointers to row-major fp32 data: dy, x, dx (rows x dim),
// gamma, dgamma (dim), rstd (rows); `stream` is a cudaStream_t (may be null
// for the legacy default stream). The call only enqueues work on `stream`.
//
// Limits: 0 < dim <= 4096 and dim % 4 == 0; pointers 16-byte aligned. Other
// sizes are rejected with ABACUS_NOALLOC_EBADSIZE before anything is launched.
//
// Returns 0 on success, ABACUS_NOALLOC_EBADSIZE for rejected arguments, or a
// cudaError_t value if a CUDA call fails.
//
// Set-up: the first call on a device looks up the array's device address
// (cudaGetSymbolAddress, with that device current) and the SM count; make
// that first call before capturing any stream on that device.
//
// Sharing: every call on a device uses the same scratch array, and the array
// keeps the last call's contents. Calls whose kernels overlap on the GPU
// (different streams without ordering between them) race on it; serialise
// them, e.g. by issuing them on one stream.
#pragma once

#define ABACUS_NOALLOC_EBADSIZE (-22)

#ifdef __cplusplus
extern "C" {
#endif

int abacus_rmsnorm_bwd_noalloc(const float* dy, const float* x, const float* gamma, const float* rstd, float* dx,
                               float* dgamma, int rows, int dim, void* stream);

#ifdef __cplusplus
}
#endif
