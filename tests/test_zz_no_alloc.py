"""The allocation-free RMSNorm backward entry point (``abacus_rmsnorm_bwd_noalloc``).

Some callers of this library cannot allocate device memory: a host application
that owns the GPU memory budget and exposes only input / output pointers to
its plugins, or a latency-critical loop that must stay clear of cudaMalloc /
cudaFree. For them the library exports one C function that runs the RMSNorm
backward with its reduction scratch in a fixed device array instead of a
per-call buffer. This test calls that function through its exported C symbol
(ctypes, raw device pointers, the current stream) and checks it against the
library's regular backward and against a plain fp32 PyTorch autograd RMSNorm,
on two calls in a row, since every call reuses the same scratch array.
"""
import ctypes

import pytest
import torch

from abacus_b200.ops._ext import check_status, ext

pytestmark = pytest.mark.gpu

EBADSIZE = -22


def _entry_point():
    lib = ctypes.CDLL(ext().__file__)
    fn = lib.abacus_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _call(fn, dy, x, gamma, rstd, dx, dgamma):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return fn(dy.data_ptr(), x.data_ptr(), gamma.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dgamma.data_ptr(),
              x.shape[0], x.shape[1], stream)


def _case(rows, dim, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, dim, device="cuda", generator=g)
    dy = torch.randn(rows, dim, device="cuda", generator=g)
    gamma = torch.rand(dim, device="cuda", generator=g) + 0.5
    rstd = torch.rsqrt(x.square().mean(-1) + 1e-5)
    return dy, x, gamma, rstd


def _autograd_oracle(dy, x, gamma, eps=1e-5):
    """dx, dgamma of y = gamma * x * rsqrt(mean(x^2) + eps) by fp32 autograd."""
    xr = x.detach().clone().requires_grad_(True)
    gr = gamma.detach().clone().requires_grad_(True)
    y = gr * xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + eps)
    y.backward(dy)
    return xr.grad, gr.grad


def _close(a, b, tol=1e-5):
    err = ((a.double() - b.double()).abs().max() / b.double().abs().max()).item()
    assert err < tol, f"rel err {err:.3e}"


@pytest.mark.parametrize("rows,dim", [(4096, 768), (37, 2048), (1, 8)])
def test_no_alloc_entry_point_matches_regular_backward(rows, dim):
    fn = _entry_point()
    for call in range(2):  # the second call runs on the array the first one left behind
        dy, x, gamma, rstd = _case(rows, dim, seed=10 * call + dim)
        dx_ref, dg_ref = torch.empty_like(x), torch.empty_like(gamma)
        ext().rmsnorm_bwd(dy, x, gamma, rstd, dx_ref, dg_ref)
        dx, dg = torch.full_like(x, float("nan")), torch.full_like(gamma, float("nan"))
        torch.cuda.synchronize()
        allocated = torch.cuda.memory_allocated()
        assert _call(fn, dy, x, gamma, rstd, dx, dg) == 0
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == allocated
        check_status()
        _close(dx, dx_ref)
        _close(dg, dg_ref)
        dx_ag, dg_ag = _autograd_oracle(dy, x, gamma)
        _close(dx, dx_ag, tol=1e-4)
        _close(dg, dg_ag, tol=1e-4)


def test_no_alloc_entry_point_zero_rows():
    fn = _entry_point()
    dim = 768
    # Real buffers (an empty tensor has no address), passed with rows = 0.
    x = torch.zeros(1, dim, device="cuda")
    dx = torch.full((1, dim), 7.0, device="cuda")
    rstd = torch.ones(4, device="cuda")
    gamma = torch.ones(dim, device="cuda")
    dg = torch.full((dim,), float("nan"), device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        ptrs = [t.data_ptr() for t in (x, x, gamma, rstd, dx, dg)]
        assert fn(*ptrs, 0, dim, stream) == 0
        torch.cuda.synchronize()
        check_status()
        assert torch.equal(dg, torch.zeros_like(dg))
        assert torch.equal(dx, torch.full_like(dx, 7.0))  # dx untouched


def test_no_alloc_entry_point_rejects_unsupported_sizes():
    fn = _entry_point()
    for dim in (4100, 6, 8192):
        x = torch.zeros(2, dim, device="cuda")
        vec = torch.zeros(dim, device="cuda")
        rstd = torch.ones(2, device="cuda")
        assert _call(fn, x, x, vec, rstd, x, vec) == EBADSIZE


def test_no_alloc_entry_point_rejects_misaligned_pointers():
    """A row view starting 4 bytes into a buffer is refused before launch."""
    fn = _entry_point()
    rows, dim = 8, 64
    buf = torch.zeros(rows * dim + 4, device="cuda")
    x = buf[1:1 + rows * dim].view(rows, dim)  # 4-byte offset
    good = torch.zeros(rows, dim, device="cuda")
    vec = torch.ones(dim, device="cuda")
    rstd = torch.ones(rows, device="cuda")
    assert x.data_ptr() % 16 == 4
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for args in ((x, good, vec, rstd, good, vec), (good, good, vec, rstd, x, vec)):
        ptrs = [a.data_ptr() for a in args]
        assert fn(*ptrs, rows, dim, stream) == EBADSIZE
    torch.cuda.synchronize()
    check_status()
