"""Tensor-parallel GPT training (Megatron TP, optional sequence parallel),
cf. the reference's ``examples/train_gpt_tp.py``. ``--dp D`` combines TP with
data parallelism over a 2-D mesh (world = D x TP), which the reference cannot
express.

torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node=4 examples/train_gpt_tp.py --synthetic 32 --sequence-parallel
torchrun --nproc_per_node=8 --master-addr 127.0.0.1 examples/train_gpt_tp.py --synthetic 64 --dp 2 --sequence-parallel
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from abacus_b200.distributed.data_parallel import DataParallel  # noqa: E402
from abacus_b200.parallel import mesh  # noqa: E402
from abacus_b200.trainer import Trainer  # noqa: E402
from abacus_b200.utils.trace import PhaseTracer  # noqa: E402
from abacus_b200.transformer import Transformer  # noqa: E402
from abacus_b200.utils import cli  # noqa: E402


def main():
    p = cli.base_parser("Train a Transformer with tensor parallelism.")
    p.add_argument("--sequence-parallel", action="store_true")
    p.add_argument("--dp", type=int, default=1, help="data-parallel replicas of the TP group")
    p.add_argument("--dim", type=int, default=128)
    p.add_argument("--heads", type=int, default=4)
    p.add_argument("--head-dim", type=int, default=32)
    p.add_argument("--blocks", type=int, default=2)
    p.add_argument("--hidden", type=int, default=None)
    p.add_argument("--batch", type=int, default=2)
    args = p.parse_args()
    device, distributed = cli.setup(args)
    try:
        world = cli.world_size() if distributed else 1
        if distributed:
            mesh.init_mesh(dp=args.dp, tp=world // args.dp)
        m = mesh.get_mesh()
        dp_rank = m.coords(cli.rank())["dp"] if m else 0
        docs, vocab = cli.documents(args, dp_rank, args.dp)
        total_steps = len(docs) // args.batch
        torch.manual_seed(0)
        model = Transformer(dim=args.dim, n_heads=args.heads, head_dim=args.head_dim, n_blocks=args.blocks,
                            vocab_size=vocab, hidden_dim=args.hidden, tensor_parallel=True,
                            sequence_parallel=args.sequence_parallel).to(device)
        parallel = DataParallel(model) if args.dp > 1 else None
        trainer = Trainer(model, parallel, total_steps=total_steps, tracer=PhaseTracer(timing=args.phase_times))
        tp = m.tp if m else 1
        multiple = tp if args.sequence_parallel else 1
        cli.run_loop(trainer, cli.padded_batches(docs, args.batch, multiple_of=multiple), total_steps, device,
                     distributed, max_steps=args.steps)
    finally:
        if distributed:
            cli.shutdown()


if __name__ == "__main__":
    main()
