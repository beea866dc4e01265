"""Memory-bound CUDA kernels against plain PyTorch fp32 references of the same op."""
import pytest
import torch

from abacus_b200.ops import attention as attn_ops
from abacus_b200.ops import cross_entropy as ce_ops
from abacus_b200.ops import embedding as emb_ops
from abacus_b200.ops._ext import check_status, ext
from abacus_b200.ops.norm import rmsnorm, rmsnorm_reference
from abacus_b200.optim.adamw import AdamW

pytestmark = pytest.mark.gpu


def _close(a, b, tol=1e-5):
    err = ((a.double() - b.double()).abs().max() / b.double().abs().max().clamp(min=1e-30)).item()
    assert err < tol, f"rel err {err:.3e}"


@pytest.mark.parametrize("rows,dim", [(1, 8), (37, 256), (4096, 768), (300, 2048)])
def test_rmsnorm_forward_backward(rows, dim):
    torch.manual_seed(0)
    x = torch.randn(rows, dim, device="cuda", requires_grad=True)
    g = (torch.rand(dim, device="cuda") + 0.5).requires_grad_()
    y = rmsnorm(x, g)
    gy = torch.randn_like(y)
    y.backward(gy)
    xr, gr = x.detach().cpu().requires_grad_(), g.detach().cpu().requires_grad_()
    yr = rmsnorm_reference(xr, gr)
    yr.backward(gy.cpu())
    check_status()
    _close(y.cpu(), yr.detach())
    _close(x.grad.cpu(), xr.grad, 1e-4)
    _close(g.grad.cpu(), gr.grad, 1e-4)


@pytest.mark.parametrize("batch,length,heads,head_dim", [(2, 16, 2, 64), (1, 130, 3, 64), (2, 64, 2, 128)])
def test_qk_prologue_forward_backward(batch, length, heads, head_dim):
    torch.manual_seed(1)
    hk = heads * head_dim
    t = batch * length
    qkv = torch.randn(t, 3 * hk, device="cuda", requires_grad=True)
    gq = (torch.rand(head_dim, device="cuda") + 0.5).requires_grad_()
    gk = (torch.rand(head_dim, device="cuda") + 0.5).requires_grad_()
    inv_freq = 1.0 / (10000 ** (torch.arange(0, head_dim, 2, device="cuda").float() / head_dim))
    q, k, v = attn_ops.qk_prologue(qkv, heads, head_dim, gq, gk, inv_freq, length)
    gq_out, gk_out, gv_out = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    (q * gq_out + k * gk_out + v * gv_out).sum().backward()

    def ref(qkv_c, gq_c, gk_c):
        pos = torch.arange(length)
        freqs = torch.outer(pos.float(), inv_freq.cpu())
        emb = torch.cat((freqs, freqs), -1)
        out = []
        for i, gam in ((0, gq_c), (1, gk_c)):
            x = qkv_c[:, i * hk : (i + 1) * hk].reshape(batch, length, heads, head_dim)
            x = rmsnorm_reference(x, gam)
            rot = torch.cat((-x[..., head_dim // 2 :], x[..., : head_dim // 2]), -1)
            x = x * emb.cos()[None, :, None] + rot * emb.sin()[None, :, None]
            out.append(x.reshape(t, hk))
        return out[0], out[1], qkv_c[:, 2 * hk :]

    qc = qkv.detach().cpu().requires_grad_()
    gqc, gkc = gq.detach().cpu().requires_grad_(), gk.detach().cpu().requires_grad_()
    qr, kr, vr = ref(qc, gqc, gkc)
    (qr * gq_out.cpu() + kr * gk_out.cpu() + vr * gv_out.cpu()).sum().backward()
    check_status()
    _close(q.detach().cpu(), qr.detach())
    _close(k.detach().cpu(), kr.detach())
    _close(qkv.grad.cpu(), qc.grad, 1e-4)
    _close(gq.grad.cpu(), gqc.grad, 1e-4)
    _close(gk.grad.cpu(), gkc.grad, 1e-4)


def test_embedding_forward_backward_deterministic():
    torch.manual_seed(2)
    w = torch.randn(1000, 64, device="cuda", requires_grad=True)
    tok = torch.randint(0, 1000, (4, 300), device="cuda")
    tok[0, :50] = 7  # a long run of one id
    y = emb_ops.embedding(tok, w)
    gy = torch.randn_like(y)
    y.backward(gy)
    g1 = w.grad.clone()
    w.grad = None
    emb_ops.embedding(tok, w).backward(gy)
    assert torch.equal(g1, w.grad)
    ref = torch.zeros(1000, 64, dtype=torch.float64).index_add_(0, tok.cpu().reshape(-1), gy.cpu().double().reshape(-1, 64))
    torch.testing.assert_close(y.detach().cpu(), w.detach().cpu()[tok.cpu()])
    _close(g1.cpu(), ref, 1e-5)


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
def test_cross_entropy_matches_torch(reduction):
    torch.manual_seed(3)
    logits = torch.randn(257, 50304, device="cuda") * 3
    logits.requires_grad_()
    tgt = torch.randint(0, 50304, (257,), device="cuda")
    tgt[::7] = -100
    loss = ce_ops.cross_entropy(logits, tgt, reduction=reduction)
    g = torch.randn_like(loss) if reduction == "none" else torch.tensor(1.7, device="cuda")
    loss.backward(g)
    lc = logits.detach().cpu().requires_grad_()
    ref = torch.nn.functional.cross_entropy(lc, tgt.cpu(), ignore_index=-100, reduction=reduction)
    ref.backward(g.cpu())
    _close(loss.detach().cpu(), ref.detach())
    _close(logits.grad.cpu(), lc.grad, 1e-4)


def test_fused_linear_cross_entropy_matches_unfused():
    torch.manual_seed(4)
    h = torch.randn(3000, 256, device="cuda", requires_grad=True)
    w = (torch.randn(256, 5000, device="cuda") / 16).requires_grad_()
    tgt = torch.randint(0, 5000, (3000,), device="cuda")
    tgt[:100] = -100
    loss = ce_ops.fused_linear_cross_entropy(h, w, tgt, chunk_rows=1024)
    loss.backward(torch.tensor(0.5, device="cuda"))
    hc, wc = h.detach().double().cpu().requires_grad_(), w.detach().double().cpu().requires_grad_()
    ref = torch.nn.functional.cross_entropy(hc @ wc, tgt.cpu(), ignore_index=-100)
    (0.5 * ref).backward()
    _close(loss.detach().cpu(), ref.detach(), 1e-5)
    _close(h.grad.cpu(), hc.grad, 1e-4)
    _close(w.grad.cpu(), wc.grad, 1e-4)


def test_multi_tensor_adamw_matches_reference_sequence():
    torch.manual_seed(5)
    shapes = [(3, 5), (4096,), (7,), (300, 129)] * 12  # > 36 tensors: several launches
    params = [torch.nn.Parameter(torch.randn(s, device="cuda")) for s in shapes]
    cpu = [torch.nn.Parameter(p.detach().cpu().clone()) for p in params]
    opt = AdamW(params, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    ref = AdamW(cpu, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    for step in range(4):
        for p, c in zip(params, cpu):
            c.grad = torch.randn(c.shape)
            p.grad = c.grad.cuda()
        opt.step()
        ref.step()
    check_status()
    for p, c in zip(params, cpu):
        _close(p.detach().cpu(), c.detach(), 1e-6)
        _close(opt.state[id(p)]["exp_avg_sq"].cpu(), ref.state[id(c)]["exp_avg_sq"], 1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", [(65536, 768), (333, 130), (64, 64), (7, 1)])
def test_transpose_kernel(rows, cols):
    from abacus_b200.ops import gemm

    x = torch.randn(rows, cols, device="cuda")
    assert torch.equal(gemm.transpose(x), x.t())
    view = torch.randn(rows, cols + 3, device="cuda")[:, 1 : cols + 1]  # unaligned, strided rows
    assert torch.equal(gemm.transpose(view), view.t())


@pytest.mark.gpu
@pytest.mark.parametrize("tokens,dim,experts", [(4096, 768, 8), (333, 256, 2), (64, 128, 64)])
def test_router_logits_kernels_match_fp64(tokens, dim, experts):
    from abacus_b200.models.moe import router_logits

    g = torch.Generator(device="cuda").manual_seed(tokens)
    x = torch.randn(2, tokens // 2 + tokens % 2, dim, device="cuda", generator=g)[:, : tokens // 2]
    w = torch.randn(dim, experts, device="cuda", generator=g) / dim**0.5
    x.requires_grad_(True)
    w.requires_grad_(True)
    out = router_logits(x, w)
    gout = torch.randn_like(out)
    out.backward(gout)
    xd, wd = x.detach().double().requires_grad_(True), w.detach().double().requires_grad_(True)
    ref = xd @ wd
    ref.backward(gout.double())
    rel = lambda a, b: ((a.double() - b).abs().max() / b.abs().max()).item()  # noqa: E731
    assert rel(out, ref) < 1e-5
    assert rel(x.grad, xd.grad) < 1e-5
    assert rel(w.grad, wd.grad) < 1e-5
    check_status()


@pytest.mark.parametrize("mode", ["softmax", "sigmoid"])
@pytest.mark.parametrize("experts,top_k", [(8, 2), (16, 4)])
def test_routing_kernels_match_aten_router(mode, experts, top_k):
    """Routing kernels (probabilities, top-k, weights and their backward)
    against the same Router on CPU (ATen ops): indices equal, weights,
    auxiliary loss and the x / w gradients close."""
    import copy

    from abacus_b200.models.moe import Router

    torch.manual_seed(31)
    cpu = Router(64, experts, top_k, router=mode, route_scale=2.5)
    cpu.expert_bias_E.copy_(0.01 * torch.randn(experts))
    gpu = copy.deepcopy(cpu).cuda()
    x = torch.randn(3, 100, 64)
    g = torch.randn(3, 100, top_k)
    res = {}
    for name, r, dev in (("cpu", cpu, "cpu"), ("gpu", gpu, "cuda")):
        xi = x.to(dev).clone().requires_grad_()
        w, idx = r(xi)
        loss = (w * g.to(dev)).sum()
        if r.aux_loss is not None:
            loss = loss + 10 * r.aux_loss
        loss.backward()
        res[name] = (w.detach().cpu(), idx.cpu(), xi.grad.cpu(), r.w_DE.grad.cpu(), r.expert_bias_E.cpu())
    wc, ic, gxc, gwc, bc = res["cpu"]
    wg, ig, gxg, gwg, bg = res["gpu"]
    assert torch.equal(ic, ig)
    assert (wc - wg).abs().max().item() < 1e-5 * max(1.0, wc.abs().max().item())
    assert (gxc - gxg).abs().max().item() < 1e-4 * gxc.abs().max().item()
    assert (gwc - gwg).abs().max().item() < 1e-4 * gwc.abs().max().item()
    assert torch.allclose(bc, bg)


@pytest.mark.parametrize("n,experts", [(100003, 8), (4097, 64), (5, 3)])
def test_expert_rank_kernel_matches_prefix_count(n, experts):
    """Capacity-slot ranks from the scan kernel against the CPU one-hot prefix sum."""
    from abacus_b200.ops.routing import expert_rank

    torch.manual_seed(41)
    flat = torch.randint(0, experts, (n,))
    got = expert_rank(flat.cuda(), experts).cpu()
    want = expert_rank(flat, experts)
    assert torch.equal(got, want)


def test_static_expert_parallel_plan_on_device():
    """The fused EP path's slab placement (ranks from the scan kernel) against
    the same plan computed on CPU."""
    from types import SimpleNamespace

    from abacus_b200.parallel import ep_fused

    torch.manual_seed(43)
    idx = torch.randint(0, 8, (500, 2))
    ws = SimpleNamespace(world=2, rank=1)
    got = ep_fused._static_plan(idx.cuda(), 8, 4, 100, ws)
    want = ep_fused._static_plan(idx, 8, 4, 100, ws)
    for g, w in zip(got, want):
        assert torch.equal(g.cpu(), w)
