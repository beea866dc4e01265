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
// It runs the same kernels as the library's regular RMSNorm backward (a
// row-parallel pass writing per-warp partial dgamma rows, then a two-pass
// deterministic column sum), which allocates its reduction buffers on every
// call. Here those buffers live in a fixed 4 MiB array in device memory that
// every GPU loading this library holds until the process exits: 3 MiB of
// partial rows and 1 MiB of per-split column sums.
//
// Arguments: device pointers to row-major fp32 data: dy, x, dx (rows x dim),
// gamma, dgamma (dim), rstd (rows); `stream` is a cudaStream_t (may be null
// for the legacy default stream). The call only enqueues work on `stream`.
//
// Limits: rows >= 0 (rows == 0 writes dgamma = 0 and leaves dx untouched),
// 0 < dim <= 4096, dim % 4 == 0, and all six pointers non-null and 16-byte
// aligned (the kernels move rows as float4). Anything else is rejected with
// ABACUS_NOALLOC_EBADSIZE before anything is launched.
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
