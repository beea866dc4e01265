"""Pipeline-parallel GPT training (GPipe), cf. the reference's
``examples/train_gpt_pp.py``. ``--cp C`` makes every stage context parallel
over C ranks (world = PP x C; the reference forbids PP + CP).

torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node=4 examples/train_gpt_pp.py --synthetic 32
torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node=4 examples/train_gpt_pp.py --synthetic 32 --cp 2
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from abacus_b200.distributed.pipeline_parallel import PipelineParallel  # noqa: E402
from abacus_b200.parallel import mesh  # noqa: E402
from abacus_b200.trainer import Trainer  # noqa: E402
from abacus_b200.utils.trace import PhaseTracer  # noqa: E402
from abacus_b200.transformer import PipelineStage  # noqa: E402
from abacus_b200.utils import cli  # noqa: E402


def main():
    p = cli.base_parser("Train a Transformer with pipeline parallelism.")
    p.add_argument("--cp", type=int, default=1)
    p.add_argument("--microbatches", type=int, default=2)
    p.add_argument("--dim", type=int, default=128)
    p.add_argument("--heads", type=int, default=4)
    p.add_argument("--head-dim", type=int, default=32)
    p.add_argument("--blocks", type=int, default=4)
    p.add_argument("--hidden", type=int, default=None)
    p.add_argument("--batch", type=int, default=2)
    args = p.parse_args()
    device, distributed = cli.setup(args)
    if not distributed:
        raise ValueError("pipeline parallel needs torchrun with at least 2 processes")
    try:
        world = cli.world_size()
        m = mesh.init_mesh(pp=world // args.cp, cp=args.cp)
        c = m.coords(cli.rank())
        docs, vocab = cli.documents(args)
        total_steps = len(docs) // args.batch
        torch.manual_seed(0)
        stage = PipelineStage(args.dim, args.heads, args.head_dim, args.blocks, vocab, rank=c["pp"], world_size=m.pp,
                              hidden_dim=args.hidden, context_parallel=args.cp > 1).to(device)
        trainer = Trainer(stage, pipeline=PipelineParallel(stage, n_microbatches=args.microbatches),
                          total_steps=total_steps, tracer=PhaseTracer(timing=args.phase_times))
        batches = cli.padded_batches(docs, args.batch, multiple_of=2 * args.cp)

        def on_step(step, loss, local, tokens):
            if c["pp"] == m.pp - 1 and c["cp"] == 0:
                print(f"step {step}/{total_steps} loss {loss.item():.4f} batch {tokens.shape[0]} "
                      f"length {tokens.shape[1]}", flush=True)

        cli.run_loop(trainer, batches, total_steps, device, True, on_step=on_step, max_steps=args.steps)
    finally:
        cli.shutdown()


if __name__ == "__main__":
    main()
