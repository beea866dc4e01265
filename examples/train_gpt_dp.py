"""Data-parallel GPT training (DDP or ZeRO-1/2/3), cf. the reference's
``examples/train_gpt_dp.py``.

One process:            python examples/train_gpt_dp.py --synthetic 64
CPU ranks (gloo):       torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node=4 examples/train_gpt_dp.py --synthetic 64 --zero 3
GPUs (NCCL, one/GPU):   torchrun --nproc_per_node=8 --master-addr 127.0.0.1 examples/train_gpt_dp.py --preset config2 --synthetic 4096
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from abacus_b200.distributed.data_parallel import DataParallel  # noqa: E402
from abacus_b200.trainer import Trainer  # noqa: E402
from abacus_b200.utils.trace import PhaseTracer  # noqa: E402
from abacus_b200.transformer import Transformer  # noqa: E402
from abacus_b200.utils import cli  # noqa: E402

PRESETS = {
    # The reference example's dimensions.
    "tiny": dict(dim=64, n_heads=4, head_dim=16, n_blocks=2, hidden_dim=None, batch=2),
    # ~125M GPT (benchmark config 2): per-rank batch of 8 sequences.
    "config2": dict(dim=768, n_heads=12, head_dim=64, n_blocks=12, hidden_dim=2048, batch=8),
}


def main():
    p = cli.base_parser("Train a Transformer with data parallelism.")
    p.add_argument("--zero", type=int, choices=(0, 1, 2, 3), default=0)
    p.add_argument("--preset", choices=sorted(PRESETS), default="tiny")
    p.add_argument("--wandb", action="store_true", help="log cumulative loss to Weights & Biases")
    p.add_argument("--wandb-project", default="abacus")
    args = p.parse_args()
    device, distributed = cli.setup(args)
    if args.zero > 0 and not distributed:
        raise ValueError("--zero above 0 needs more than one process")
    run = None
    try:
        rank_ = cli.rank() if distributed else 0
        world = cli.world_size() if distributed else 1
        cfg = PRESETS[args.preset]
        docs, vocab = cli.documents(args, rank_, world)
        batch = cfg["batch"]
        per_rank = (len(docs) // batch) * batch
        total_steps = per_rank // batch
        torch.manual_seed(0)
        model = Transformer(dim=cfg["dim"], n_heads=cfg["n_heads"], head_dim=cfg["head_dim"], n_blocks=cfg["n_blocks"],
                            vocab_size=vocab, hidden_dim=cfg["hidden_dim"]).to(device)
        parallel = DataParallel(model, stage=args.zero) if distributed else None
        trainer = Trainer(model, parallel, total_steps=total_steps, tracer=PhaseTracer(timing=args.phase_times))
        if args.wandb and rank_ == 0:
            import wandb

            run = wandb.init(project=args.wandb_project, config=vars(args))

        def on_step(step, loss, local, tokens):
            if distributed:
                print(f"step {step} rank {rank_} loss {local.item():.4f} batch {tokens.shape[0]} length {tokens.shape[1]}",
                      flush=True)
                dist.barrier()
                if rank_ == 0:
                    print(f"step {step} cumulative loss {loss.item():.4f} {step * world * batch}/{per_rank * world}",
                          flush=True)
            else:
                print(f"step {step}/{total_steps} loss {loss.item():.4f} batch {tokens.shape[0]} "
                      f"length {tokens.shape[1]}", flush=True)
            if run is not None:
                run.log({"cumulative_loss": loss.item()}, step=step)

        cli.run_loop(trainer, cli.padded_batches(docs, batch), total_steps, device, distributed, on_step=on_step,
                     max_steps=args.steps)
    finally:
        if run is not None:
            run.finish()
        if distributed:
            cli.shutdown()


if __name__ == "__main__":
    main()
