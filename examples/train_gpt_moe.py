"""Mixture-of-experts GPT training, cf. the reference's
``examples/train_gpt_moe.py``. ``--expert-parallel`` shards the experts over
the ranks (one expert each, replicated batch, as in the reference);
``--expert-data-parallel`` instead gives every rank its own data and
synchronises the non-expert weights (DP over the expert-parallel ranks).

python examples/train_gpt_moe.py --synthetic 32
torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node=4 examples/train_gpt_moe.py --synthetic 32 --expert-parallel
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402

from abacus_b200.distributed.data_parallel import DataParallel  # noqa: E402
from abacus_b200.model_config import DIM, HEAD_DIM, N_BLOCKS, N_HEADS  # noqa: E402
from abacus_b200.parallel import mesh  # noqa: E402
from abacus_b200.trainer import Trainer  # noqa: E402
from abacus_b200.utils.trace import PhaseTracer  # noqa: E402
from abacus_b200.transformer_moe import TransformerMoe  # noqa: E402
from abacus_b200.utils import cli  # noqa: E402


def main():
    p = cli.base_parser("Train a mixture-of-experts Transformer.")
    p.add_argument("--expert-parallel", action="store_true")
    p.add_argument("--expert-data-parallel", action="store_true")
    p.add_argument("--experts", type=int, default=4)
    p.add_argument("--top-k", type=int, default=1)
    p.add_argument("--router", choices=("sigmoid", "softmax"), default="sigmoid")
    p.add_argument("--capacity-factor", type=float, default=None)
    p.add_argument("--batch", type=int, default=2)
    p.add_argument("--wandb", action="store_true")
    args = p.parse_args()
    device, distributed = cli.setup(args)
    if distributed and not (args.expert_parallel or args.expert_data_parallel):
        raise ValueError("multi-process MoE training needs --expert-parallel or --expert-data-parallel")
    try:
        world = cli.world_size() if distributed else 1
        edp = args.expert_data_parallel
        if distributed:
            mesh.init_mesh(dp=world, ep=world)
        rank_ = cli.rank() if distributed else 0
        docs, vocab = cli.documents(args, rank_ if edp else 0, world if edp else 1)
        total_steps = len(docs) // args.batch
        experts = args.experts if not (args.expert_parallel and not edp) else max(world, 1)
        torch.manual_seed(0)
        model = TransformerMoe(DIM, N_HEADS, HEAD_DIM, N_BLOCKS, vocab, experts, args.top_k,
                               expert_parallel=args.expert_parallel or edp, expert_data_parallel=edp,
                               router=args.router, capacity_factor=args.capacity_factor).to(device)
        parallel = None
        if edp:
            expert_params = [p for n, p in model.named_parameters() if ".moe.w_" in n]
            parallel = DataParallel(model, exclude=expert_params, token_weighted=False)
        trainer = Trainer(model, parallel, total_steps=total_steps, tracer=PhaseTracer(timing=args.phase_times))
        cli.run_loop(trainer, cli.padded_batches(docs, args.batch), total_steps, device, distributed,
                     max_steps=args.steps)
    finally:
        if distributed:
            cli.shutdown()


if __name__ == "__main__":
    main()
