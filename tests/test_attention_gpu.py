"""tcgen05 flash attention against an fp64 PyTorch reference of the same op."""
import math

import pytest
import torch

from abacus_b200.ops import attention as attn_ops
from abacus_b200.ops import precision
from abacus_b200.ops._ext import check_status
from abacus_b200.parallel.context_parallel import gathered_positions, zigzag_positions

pytestmark = pytest.mark.gpu


def _ref(q, k, v, batch, heads, hd, q_pos, k_pos):
    lq, lk = q.shape[0] // batch, k.shape[0] // batch
    qh = q.double().view(batch, lq, heads, hd).transpose(1, 2)
    kh = k.double().view(batch, lk, heads, hd).transpose(1, 2)
    vh = v.double().view(batch, lk, heads, hd).transpose(1, 2)
    s = qh @ kh.transpose(-1, -2) / math.sqrt(hd)
    s = s.masked_fill(q_pos.view(-1, 1).cpu().to(s.device) < k_pos.view(1, -1).to(s.device), float("-inf"))
    pr = torch.softmax(s, -1)
    o = pr @ vh
    lse = torch.logsumexp(s, -1)
    return o.transpose(1, 2).reshape(batch * lq, heads * hd), lse


def _err(a, b):
    return ((a.double() - b.double()).abs().max() / b.double().abs().max()).item()


@pytest.mark.parametrize("mode", ["tf32", "fp32"])
@pytest.mark.parametrize("batch,length,heads,hd", [(1, 64, 1, 64), (2, 128, 2, 64), (1, 200, 3, 64), (2, 1024, 2, 64), (1, 300, 2, 32)])
def test_flash_forward_causal(mode, batch, length, heads, hd):
    torch.manual_seed(0)
    t = batch * length
    q = torch.randn(t, heads * hd, device="cuda")
    k = torch.randn(t, heads * hd, device="cuda")
    qkv = torch.randn(t, 3 * heads * hd, device="cuda")
    v = qkv[:, 2 * heads * hd :]  # strided like the real prologue output
    precision.set_precision(mode)
    try:
        out = attn_ops.flash_attention(q, k, v, batch, heads, hd)
    finally:
        precision.set_precision("fp32")
    torch.cuda.synchronize()
    check_status()
    pos = torch.arange(length)
    ref, _ = _ref(q, k, v, batch, heads, hd, pos, pos)
    tol = 3e-3 if mode == "tf32" else 2e-5
    assert _err(out, ref) < tol


@pytest.mark.parametrize("mode", ["tf32", "fp32"])
def test_flash_forward_with_zigzag_positions(mode):
    torch.manual_seed(1)
    batch, heads, hd, world, total = 2, 2, 64, 4, 1024
    local = total // world
    rank = 1
    q_pos = zigzag_positions(total, rank, world).cuda()
    k_pos = gathered_positions(local, world).cuda()
    q = torch.randn(batch * local, heads * hd, device="cuda")
    k = torch.randn(batch * total, heads * hd, device="cuda")
    v = torch.randn(batch * total, heads * hd, device="cuda")
    precision.set_precision(mode)
    try:
        out = attn_ops.flash_attention(q, k, v, batch, heads, hd, q_pos=q_pos, k_pos=k_pos)
    finally:
        precision.set_precision("fp32")
    torch.cuda.synchronize()
    check_status()
    ref, _ = _ref(q, k, v, batch, heads, hd, q_pos.cpu(), k_pos.cpu())
    assert _err(out, ref) < (3e-3 if mode == "tf32" else 2e-5)


def _ref_grads(q, k, v, batch, heads, hd, q_pos, k_pos, gout):
    qd, kd, vd = [t.detach().double().cpu().requires_grad_() for t in (q, k, v)]
    o, _ = _ref(qd, kd, vd, batch, heads, hd, q_pos.cpu(), k_pos.cpu())
    o.backward(gout.double().cpu())
    return o.detach(), qd.grad, kd.grad, vd.grad


@pytest.mark.parametrize("mode", ["tf32", "fp32"])
@pytest.mark.parametrize("batch,length,heads,hd", [(1, 64, 1, 64), (2, 256, 2, 64), (1, 200, 2, 64), (1, 512, 1, 32)])
def test_flash_backward_causal(mode, batch, length, heads, hd):
    torch.manual_seed(2)
    t = batch * length
    q = torch.randn(t, heads * hd, device="cuda", requires_grad=True)
    k = torch.randn(t, heads * hd, device="cuda", requires_grad=True)
    v = torch.randn(t, heads * hd, device="cuda", requires_grad=True)
    precision.set_precision(mode)
    try:
        out = attn_ops.flash_attention(q, k, v, batch, heads, hd)
        gout = torch.randn_like(out)
        out.backward(gout)
    finally:
        precision.set_precision("fp32")
    torch.cuda.synchronize()
    check_status()
    pos = torch.arange(length)
    o_ref, dq_ref, dk_ref, dv_ref = _ref_grads(q, k, v, batch, heads, hd, pos, pos, gout)
    tol = 5e-3 if mode == "tf32" else 5e-5
    assert _err(out.detach().cpu(), o_ref) < tol
    assert _err(v.grad.cpu(), dv_ref) < tol
    assert _err(k.grad.cpu(), dk_ref) < tol
    assert _err(q.grad.cpu(), dq_ref) < tol


@pytest.mark.parametrize("mode", ["tf32", "fp32"])
def test_flash_backward_with_zigzag_positions(mode):
    torch.manual_seed(3)
    batch, heads, hd, world, total = 1, 2, 64, 2, 512
    local = total // world
    q_pos = zigzag_positions(total, 0, world).cuda()
    k_pos = gathered_positions(local, world).cuda()
    q = torch.randn(batch * local, heads * hd, device="cuda", requires_grad=True)
    k = torch.randn(batch * total, heads * hd, device="cuda", requires_grad=True)
    v = torch.randn(batch * total, heads * hd, device="cuda", requires_grad=True)
    precision.set_precision(mode)
    try:
        out = attn_ops.flash_attention(q, k, v, batch, heads, hd, q_pos=q_pos, k_pos=k_pos)
        gout = torch.randn_like(out)
        out.backward(gout)
    finally:
        precision.set_precision("fp32")
    torch.cuda.synchronize()
    check_status()
    _, dq_ref, dk_ref, dv_ref = _ref_grads(q, k, v, batch, heads, hd, q_pos, k_pos, gout)
    tol = 5e-3 if mode == "tf32" else 5e-5
    assert _err(q.grad.cpu(), dq_ref) < tol
    assert _err(k.grad.cpu(), dk_ref) < tol
    assert _err(v.grad.cpu(), dv_ref) < tol


@pytest.mark.parametrize("batch,length,heads", [(1, 256, 1), (2, 384, 2), (1, 200, 2)])
def test_dense_head_dim_128_fp32_forward_backward(batch, length, heads):
    """head_dim 128 in fp32 mode: materialised attention on the batched GEMM
    (causal tile skipping) + the in-place softmax kernels, against fp64."""
    torch.manual_seed(3)
    hd = 128
    t = batch * length
    q = torch.randn(t, heads * hd, device="cuda", requires_grad=True)
    k = torch.randn(t, heads * hd, device="cuda", requires_grad=True)
    qkv = torch.randn(t, 3 * heads * hd, device="cuda")
    v = qkv[:, 2 * heads * hd :].clone().requires_grad_()
    gout = torch.randn(t, heads * hd, device="cuda")
    precision.set_precision("fp32")
    out = attn_ops.flash_attention(q, k, v, batch, heads, hd)
    out.backward(gout)
    torch.cuda.synchronize()
    check_status()
    pos = torch.arange(length)
    ref_o, rq, rk, rv = _ref_grads(q, k, v, batch, heads, hd, pos, pos, gout)
    assert _err(out.detach().cpu(), ref_o) < 2e-5
    for got, want in ((q.grad, rq), (k.grad, rk), (v.grad, rv)):
        assert _err(got.cpu(), want) < 5e-5
