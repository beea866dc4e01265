"""AdamW and WSD semantics (CPU)."""
import pytest
import torch

from abacus_b200.optimizers.adamw import AdamW
from abacus_b200.optimizers.lr_scheduler import WSD


@pytest.mark.parametrize("wd", [0.0, 1e-2])
def test_adamw_tracks_torch_adamw(wd):
    torch.manual_seed(0)
    ours, ref = torch.nn.Linear(5, 3), torch.nn.Linear(5, 3)
    ref.load_state_dict(ours.state_dict())
    opt = AdamW(ours, lr=3e-3, betas=(0.8, 0.95), weight_decay=wd)
    ref_opt = torch.optim.AdamW(ref.parameters(), lr=3e-3, betas=(0.8, 0.95), weight_decay=wd)
    for step in range(8):
        g = torch.Generator().manual_seed(step)
        for p, rp in zip(ours.parameters(), ref.parameters()):
            p.grad = torch.randn(p.shape, generator=g)
            rp.grad = p.grad.clone()
        opt.step()
        ref_opt.step()
    for p, rp in zip(ours.parameters(), ref.parameters()):
        torch.testing.assert_close(p, rp)
        st, rst = opt.state[id(p)], ref_opt.state[rp]
        assert st["step"] == 8
        torch.testing.assert_close(st["exp_avg"], rst["exp_avg"])
        torch.testing.assert_close(st["exp_avg_sq"], rst["exp_avg_sq"])


def test_owned_slice_steps_like_full_and_leaves_rest():
    torch.manual_seed(1)
    sliced, full = torch.nn.Linear(4, 5), torch.nn.Linear(4, 5)
    full.load_state_dict(sliced.state_dict())
    before = [p.detach().clone() for p in sliced.parameters()]
    owned = {id(p): (2, 5) for p in sliced.parameters()}
    opt, full_opt = AdamW(sliced, owned=owned), AdamW(full)
    for step in range(3):
        g = torch.Generator().manual_seed(10 + step)
        for p, fp in zip(sliced.parameters(), full.parameters()):
            p.grad = torch.randn(p.shape, generator=g)
            fp.grad = p.grad.clone()
        opt.step()
        full_opt.step()
    for p, fp, b in zip(sliced.parameters(), full.parameters(), before):
        torch.testing.assert_close(p.view(-1)[2:5], fp.view(-1)[2:5])
        torch.testing.assert_close(p.view(-1)[:2], b.view(-1)[:2])
        torch.testing.assert_close(p.view(-1)[5:], b.view(-1)[5:])
        torch.testing.assert_close(opt.state[id(p)]["exp_avg"], full_opt.state[id(fp)]["exp_avg"].view(-1)[2:5])


def test_owned_parameter_without_gradient_is_an_error():
    lin = torch.nn.Linear(2, 2)
    opt = AdamW(lin, owned={id(lin.weight): (0, 2)})
    lin.bias.grad = torch.zeros(2)
    with pytest.raises(RuntimeError, match="missing a gradient"):
        opt.step()


def test_invalid_hyperparameters_rejected():
    lin = torch.nn.Linear(2, 2)
    for kwargs in ({"lr": -1}, {"eps": -1}, {"betas": (1.0, 0.9)}, {"weight_decay": -1}):
        with pytest.raises(ValueError):
            AdamW(lin, **kwargs)


def test_wsd_warmup_stable_decay():
    s = WSD(100, lr=1.0)
    assert (s.warmup_steps, s.decay_steps) == (2, 10)
    lrs = [s.step() for _ in range(100)]
    assert lrs[0] == 0.5 and lrs[1] == 1.0
    assert all(v == 1.0 for v in lrs[2:90])
    assert lrs[90] == pytest.approx(0.9) and lrs[99] == 0.0
    with pytest.raises(ValueError):
        s.learning_rate(101)


def test_wsd_short_runs_have_no_warmup():
    s = WSD(20, lr=5e-4)
    assert s.warmup_steps == 0 and s.decay_steps == 2
    assert [s.learning_rate(i) for i in (1, 18, 19, 20)] == [5e-4, 5e-4, 2.5e-4, 0.0]
