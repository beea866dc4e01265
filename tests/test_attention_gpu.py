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


@pytest.mark.parametrize("heads,hd,length", [(4, 64, 256), (2, 128, 384)])
def test_qkv_gemm_with_fused_qk_norm_rope(monkeypatch, heads, hd, length):
    """QK-norm + RoPE in the QKV GEMM epilogue against the separate prologue
    kernel (outputs and all gradients) and against the fp64 reference."""
    precision.set_precision("fp32")
    torch.manual_seed(21)
    batch, dim = 2, 256
    x = torch.randn(batch, length, dim, device="cuda")
    w = [torch.randn(dim, heads, hd, device="cuda") / dim**0.5 for _ in range(3)]
    gq = 1 + 0.1 * torch.randn(hd, device="cuda")
    gk = 1 + 0.1 * torch.randn(hd, device="cuda")
    inv_freq = 1.0 / (10000 ** (torch.arange(0, hd, 2, device="cuda").float() / hd))
    gout = torch.randn(batch * length, heads * hd, device="cuda")
    results = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("ABACUS_FUSED_QK", flag)
        leaves = [t.clone().requires_grad_() for t in [x, *w, gq, gk]]
        out = attn_ops.qkv_attention(leaves[0], leaves[1], leaves[2], leaves[3], batch, heads, hd, leaves[4],
                                     leaves[5], inv_freq)
        out.backward(gout)
        torch.cuda.synchronize()
        check_status()
        results[flag] = [out.detach()] + [t.grad for t in leaves]
    for fused, split in zip(results["1"], results["0"]):
        assert _err(fused, split) < 1e-5
    # fp64 reference of the whole path
    xd, wqd, wkd, wvd, gqd, gkd = [t.double() for t in [x, *w, gq, gk]]
    qkv = torch.cat([xd.reshape(-1, dim) @ m.reshape(dim, -1) for m in (wqd, wkd, wvd)], dim=1)
    pos = torch.arange(length, device="cuda")
    ref = attn_ops.attention_reference(qkv, batch, heads, hd, gqd, gkd, inv_freq.double(), pos, pos)
    assert _err(results["1"][0], ref) < 2e-5
