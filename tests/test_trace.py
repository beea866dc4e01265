"""Per-phase tracing of Trainer.step (NVTX ranges + per-phase times)."""
import torch

from abacus_b200.trainer import Trainer
from abacus_b200.transformer import Transformer
from abacus_b200.utils.trace import PhaseTracer


def test_trainer_reports_every_phase():
    torch.manual_seed(0)
    model = Transformer(dim=16, n_heads=2, head_dim=8, n_blocks=1, vocab_size=20, hidden_dim=24)
    tracer = PhaseTracer(nvtx=False, timing=True)
    trainer = Trainer(model, total_steps=4, device="cpu", tracer=tracer)
    trainer.step(torch.randint(0, 20, (2, 9)))
    times = tracer.times_ms()
    assert set(times) == {"forward", "backward", "optimizer"}
    assert all(t >= 0 for t in times.values())
    assert tracer.times_ms() == {}  # cleared by the read


def test_nested_phases_accumulate():
    tracer = PhaseTracer(nvtx=False, timing=True)
    for _ in range(3):
        with tracer.phase("a"):
            with tracer.phase("b"):
                pass
    times = tracer.times_ms()
    assert set(times) == {"a", "b"} and times["a"] >= times["b"]
