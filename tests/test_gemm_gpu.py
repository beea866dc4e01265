"""tcgen05 GEMM numerics against an fp64 PyTorch reference of the same op."""
import itertools

import pytest
import torch

from abacus_b200.ops import gemm, precision
from abacus_b200.ops._ext import check_status

pytestmark = pytest.mark.gpu


def _ref(a, b, trans_a, trans_b):
    lhs = a.double().t() if trans_a else a.double()
    rhs = b.double().t() if trans_b else b.double()
    return lhs @ rhs


def _rel_err(out, ref):
    return ((out.double() - ref).abs().max() / ref.abs().max()).item()


SHAPES = [(128, 128, 32), (256, 256, 64), (200, 136, 72), (384, 512, 768), (1000, 2304, 768), (132, 300, 1028)]


@pytest.mark.parametrize("mode", ["tf32", "fp32"])
@pytest.mark.parametrize("trans_a,trans_b", list(itertools.product([False, True], repeat=2)))
@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_layouts(mode, trans_a, trans_b, shape):
    m, n, k = shape
    torch.manual_seed(0)
    a = torch.randn(k, m, device="cuda") if trans_a else torch.randn(m, k, device="cuda")
    b = torch.randn(n, k, device="cuda") if trans_b else torch.randn(k, n, device="cuda")
    precision.set_precision(mode)
    try:
        out = gemm.matmul(a, b, trans_a=trans_a, trans_b=trans_b)
    finally:
        precision.set_precision("fp32")
    torch.cuda.synchronize()
    check_status()
    ref = _ref(a, b, trans_a, trans_b)
    err = _rel_err(out, ref)
    if mode == "tf32":
        tol = 2e-3
    else:
        # 3xTF32 must be within a small factor of true fp32 SGEMM accuracy.
        torch.backends.cuda.matmul.allow_tf32 = False
        lhs = a.t() if trans_a else a
        rhs = b.t() if trans_b else b
        tol = 8 * _rel_err(lhs @ rhs, ref) + 1e-6
    assert err < tol, f"{mode} {shape} ta={trans_a} tb={trans_b}: rel err {err:.3e} (tol {tol:.3e})"


@pytest.mark.parametrize("trans_a,trans_b", list(itertools.product([False, True], repeat=2)))
@pytest.mark.parametrize("shape", [(256, 128, 64), (384, 200, 96), (1000, 640, 768), (512, 256, 8192)])
def test_cta_pair_gemm_matches_single_cta(monkeypatch, trans_a, trans_b, shape):
    """fp32 mode on CTA pairs (one cta_group::2 MMA over 256 rows; a ragged
    last pair; split-K at K = 8192) against fp64 and against one CTA per tile."""
    m, n, k = shape
    torch.manual_seed(11)
    a = torch.randn(k, m, device="cuda") if trans_a else torch.randn(m, k, device="cuda")
    b = torch.randn(n, k, device="cuda") if trans_b else torch.randn(k, n, device="cuda")
    outs = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("ABACUS_GEMM_PAIR", flag)
        outs[flag] = gemm.matmul(a, b, trans_a=trans_a, trans_b=trans_b)
        torch.cuda.synchronize()
        check_status()
    ref = _ref(a, b, trans_a, trans_b)
    assert _rel_err(outs["1"], ref) < 2e-6
    assert _rel_err(outs["1"], outs["0"].double()) < 1e-6


@pytest.mark.parametrize("tokens", [256, 300, 1024])
def test_cta_pair_swiglu_matches_single_cta(monkeypatch, tokens):
    torch.manual_seed(12)
    dim, hidden = 256, 512
    x = torch.randn(tokens, dim, device="cuda")
    wg = torch.randn(dim, hidden, device="cuda") / dim**0.5
    wu = torch.randn(dim, hidden, device="cuda") / dim**0.5
    wd = torch.randn(hidden, dim, device="cuda") / hidden**0.5
    gy = torch.randn(tokens, dim, device="cuda")
    res = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("ABACUS_GEMM_PAIR", flag)
        leaves = [t.clone().requires_grad_() for t in (x, wg, wu, wd)]
        y = gemm.swiglu_mlp(*leaves)
        y.backward(gy)
        torch.cuda.synchronize()
        check_status()
        res[flag] = [y.detach()] + [t.grad for t in leaves]
    xd, wgd, wud, wdd = [t.double().requires_grad_() for t in (x, wg, wu, wd)]
    yd = (torch.nn.functional.silu(xd @ wgd) * (xd @ wud)) @ wdd
    yd.backward(gy.double())
    for got, single, ref in zip(res["1"], res["0"], [yd.detach(), xd.grad, wgd.grad, wud.grad, wdd.grad]):
        assert _rel_err(got, ref) < 1e-5
        assert _rel_err(got, single.double()) < 1e-6


def test_fp32_mode_matches_sgemm_accuracy():
    torch.manual_seed(1)
    a = torch.randn(512, 768, device="cuda")
    b = torch.randn(768, 2048, device="cuda")
    ref = _ref(a, b, False, False)
    torch.backends.cuda.matmul.allow_tf32 = False
    sgemm_err = _rel_err(a @ b, ref)
    out = gemm.matmul(a, b)
    ours = _rel_err(out, ref)
    assert ours < 4 * sgemm_err + 1e-7, f"3xTF32 err {ours:.3e} vs SGEMM {sgemm_err:.3e}"


def test_gemm_epilogue_residual_accumulate_alpha():
    torch.manual_seed(2)
    a = torch.randn(300, 256, device="cuda")
    b = torch.randn(256, 384, device="cuda")
    r = torch.randn(300, 384, device="cuda")
    c0 = torch.randn(300, 384, device="cuda")
    out = c0.clone()
    gemm.matmul(a, b, alpha=0.5, residual=r, out=out, accumulate=True)
    ref = 0.5 * _ref(a, b, False, False) + r.double() + c0.double()
    assert _rel_err(out, ref) < 5e-6


def test_gemm_segmented_n_and_k():
    torch.manual_seed(3)
    x = torch.randn(260, 768, device="cuda")
    ws = [torch.randn(768, 768, device="cuda") for _ in range(3)]
    out = gemm.matmul(x, ws, b_mode=gemm.B_SEG_N)
    ref = x.double() @ torch.cat(ws, 1).double()
    assert _rel_err(out, ref) < 5e-6
    dq = torch.randn(260, 3 * 768, device="cuda")
    out = gemm.matmul(dq, ws, trans_b=True, b_mode=gemm.B_SEG_K)
    ref = dq.double() @ torch.cat([w.t() for w in ws], 0).double()
    assert _rel_err(out, ref) < 5e-6


@pytest.mark.parametrize("tokens,dim,hidden", [(256, 128, 256), (300, 256, 688), (1024, 768, 2048)])
def test_swiglu_mlp_forward_backward(tokens, dim, hidden):
    torch.manual_seed(4)
    x = torch.randn(tokens, dim, device="cuda", requires_grad=True)
    wg = (torch.randn(dim, hidden, device="cuda") / dim**0.5).requires_grad_()
    wu = (torch.randn(dim, hidden, device="cuda") / dim**0.5).requires_grad_()
    wd = (torch.randn(hidden, dim, device="cuda") / hidden**0.5).requires_grad_()
    r = torch.randn(tokens, dim, device="cuda", requires_grad=True)
    y = gemm.swiglu_mlp(x, wg, wu, wd, residual=r)
    gy = torch.randn_like(y)
    y.backward(gy)
    leaves = [x, wg, wu, wd, r]
    ours = [t.grad.clone() for t in leaves]
    xd, wgd, wud, wdd, rd = [t.detach().double().requires_grad_() for t in leaves]
    yd = rd + (torch.nn.functional.silu(xd @ wgd) * (xd @ wud)) @ wdd
    yd.backward(gy.double())
    assert _rel_err(y, yd.detach()) < 1e-5
    for got, ref in zip(ours, [xd.grad, wgd.grad, wud.grad, wdd.grad, rd.grad]):
        assert _rel_err(got, ref) < 1e-5


def test_linear_autograd_matches_fp64():
    torch.manual_seed(5)
    x = torch.randn(4, 64, 256, device="cuda", requires_grad=True)
    w = (torch.randn(256, 512, device="cuda") / 16).requires_grad_()
    y = gemm.linear(x, w)
    gy = torch.randn_like(y)
    y.backward(gy)
    xd, wd = x.detach().double().requires_grad_(), w.detach().double().requires_grad_()
    (xd @ wd).backward(gy.double())
    assert _rel_err(x.grad, xd.grad) < 1e-5
    assert _rel_err(w.grad, wd.grad) < 1e-5


@pytest.mark.parametrize("mode", ["tf32", "fp32"])
def test_split_k_wgrad_shape_with_epilogue(mode):
    # Few output tiles and a long K: runs as split-K with a deterministic reduce.
    torch.manual_seed(6)
    x = torch.randn(16384, 768, device="cuda")
    dy = torch.randn(16384, 2048, device="cuda")
    r = torch.randn(768, 2048, device="cuda")
    c0 = torch.randn(768, 2048, device="cuda")
    precision.set_precision(mode)
    try:
        out = c0.clone()
        gemm.matmul(x, dy, trans_a=True, alpha=0.25, residual=r, out=out, accumulate=True)
        again = c0.clone()
        gemm.matmul(x, dy, trans_a=True, alpha=0.25, residual=r, out=again, accumulate=True)
    finally:
        precision.set_precision("fp32")
    torch.cuda.synchronize()
    check_status()
    assert torch.equal(out, again)  # deterministic
    ref = 0.25 * (x.double().t() @ dy.double()) + r.double() + c0.double()
    tol = 2e-3 if mode == "tf32" else 2e-6
    assert _rel_err(out, ref) < tol


@pytest.mark.parametrize("mode", ["tf32", "fp32"])
@pytest.mark.parametrize("trans_a,trans_b", [(False, True), (False, False), (True, False)])
def test_batched_gemm_strided_heads(mode, trans_a, trans_b):
    """(B, H, rows, cols) strided views (heads of a packed projection)."""
    from abacus_b200.ops._ext import check_status, ext

    torch.manual_seed(5)
    b, h, m, n, k = 2, 3, 192, 160, 96
    def packed(rows, cols):
        base = torch.randn(b, rows, h, cols + 4, device="cuda")[..., :cols]  # padded row stride
        return base.permute(0, 2, 1, 3)
    a = packed(k, m) if trans_a else packed(m, k)
    bb = packed(n, k) if trans_b else packed(k, n)
    c = torch.empty(b, h, m, n, device="cuda")
    precision.set_precision(mode)
    try:
        ext().gemm_batched(c, a, bb, trans_a, trans_b, 0.5, 0, precision.passes())
    finally:
        precision.set_precision("fp32")
    torch.cuda.synchronize()
    check_status()
    aa = a.double().transpose(-1, -2) if trans_a else a.double()
    bm = bb.double().transpose(-1, -2) if trans_b else bb.double()
    ref = 0.5 * aa @ bm
    err = ((c.double() - ref).abs().max() / ref.abs().max()).item()
    assert err < (3e-3 if mode == "tf32" else 2e-6)


@pytest.mark.parametrize("trans_a,trans_b", list(itertools.product([False, True], repeat=2)))
@pytest.mark.parametrize("experts,m,n,k", [(3, 200, 136, 72), (4, 256, 384, 512), (2, 132, 128, 1024)])
def test_grouped_gemm_matches_per_expert(trans_a, trans_b, experts, m, n, k):
    """One launch over E experts (3-D operands) against fp64 per expert."""
    from abacus_b200.ops._ext import ext

    torch.manual_seed(13)
    a = torch.randn(experts, k, m, device="cuda") if trans_a else torch.randn(experts, m, k, device="cuda")
    b = torch.randn(experts, n, k, device="cuda") if trans_b else torch.randn(experts, k, n, device="cuda")
    c = torch.empty(experts, m, n, device="cuda")
    ext().gemm_grouped(c, a, [b], trans_a, trans_b, gemm.B_SINGLE, 1.0, False, precision.passes(), None)
    torch.cuda.synchronize()
    check_status()
    ref = torch.stack([_ref(a[e], b[e], trans_a, trans_b) for e in range(experts)])
    assert _rel_err(c, ref) < 2e-6
    # accumulate and K segments
    c2 = torch.randn(experts, m, n, device="cuda")
    base = c2.double()
    if not trans_a and trans_b and k % 64 == 0:
        halves = [b[..., : k // 2].contiguous(), b[..., k // 2 :].contiguous()]
        ext().gemm_grouped(c2, a, halves, False, True, gemm.B_SEG_K, 0.5, True, precision.passes(), None)
        torch.cuda.synchronize()
        check_status()
        assert _rel_err(c2, base + 0.5 * ref) < 2e-6


@pytest.mark.parametrize("experts,rows,dim,hidden", [(4, 160, 128, 256), (3, 300, 256, 688), (8, 512, 768, 1536)])
def test_grouped_swiglu_matches_fp64(experts, rows, dim, hidden):
    torch.manual_seed(14)
    x = torch.randn(experts, rows, dim, device="cuda", requires_grad=True)
    wg = (torch.randn(experts, dim, hidden, device="cuda") / dim**0.5).requires_grad_()
    wu = (torch.randn(experts, dim, hidden, device="cuda") / dim**0.5).requires_grad_()
    wd = (torch.randn(experts, hidden, dim, device="cuda") / hidden**0.5).requires_grad_()
    y = gemm.grouped_swiglu_mlp(x, wg, wu, wd)
    gy = torch.randn_like(y)
    y.backward(gy)
    torch.cuda.synchronize()
    check_status()
    leaves = [x, wg, wu, wd]
    xd, wgd, wud, wdd = [t.detach().double().requires_grad_() for t in leaves]
    yd = torch.bmm(torch.nn.functional.silu(torch.bmm(xd, wgd)) * torch.bmm(xd, wud), wdd)
    yd.backward(gy.double())
    assert _rel_err(y, yd.detach()) < 1e-5
    for got, ref in zip([t.grad for t in leaves], [xd.grad, wgd.grad, wud.grad, wdd.grad]):
        assert _rel_err(got, ref) < 1e-5
