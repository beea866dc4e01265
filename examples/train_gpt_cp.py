"""Context-parallel GPT training (Llama-3 all-gather KV with zigzag sharding),
cf. the reference's ``examples/train_gpt_cp.py``.

torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node=2 examples/train_gpt_cp.py --synthetic 32
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from abacus_b200.model_config import DIM, HEAD_DIM, N_BLOCKS, N_HEADS  # noqa: E402
from abacus_b200.trainer import Trainer  # noqa: E402
from abacus_b200.utils.trace import PhaseTracer  # noqa: E402
from abacus_b200.transformer import Transformer  # noqa: E402
from abacus_b200.utils import cli  # noqa: E402


def main():
    p = cli.base_parser("Train a Transformer with context parallelism.")
    p.add_argument("--batch", type=int, default=2)
    args = p.parse_args()
    device, distributed = cli.setup(args)
    try:
        world = cli.world_size() if distributed else 1
        docs, vocab = cli.documents(args)
        total_steps = len(docs) // args.batch
        torch.manual_seed(0)
        model = Transformer(dim=DIM, n_heads=N_HEADS, head_dim=HEAD_DIM, n_blocks=N_BLOCKS, vocab_size=vocab,
                            context_parallel=True).to(device)
        trainer = Trainer(model, total_steps=total_steps, tracer=PhaseTracer(timing=args.phase_times))
        batches = cli.padded_batches(docs, args.batch, multiple_of=2 * world)
        cli.run_loop(trainer, batches, total_steps, device, distributed, max_steps=args.steps)
    finally:
        if distributed:
            cli.shutdown()


if __name__ == "__main__":
    main()
