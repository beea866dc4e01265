"""GPipe pipeline parallelism (``abacus/distributed/pipeline_parallel.py``).

All microbatch forwards run first, then all backwards in reverse order; the
last stage's loss is each microbatch's summed cross entropy divided by the
batch's total target count, so the returned loss (sum over microbatches, last
rank only) is the token mean.

Transfers stay on NCCL p2p but are overlapped with compute: the receive of
microbatch i+1 is posted before microbatch i is computed, and sends are
asynchronous (completed before the next phase). The last stage computes the
loss with the fused linear + cross-entropy kernel path instead of
materialising logits.

With a mesh, stages talk over the "pp" group and the stage may be context
parallel: the token count is then summed over the "cp" group and targets are
taken at each rank's zigzag positions.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from abacus_b200.ops.cross_entropy import fused_linear_cross_entropy
from abacus_b200.parallel import mesh
from abacus_b200.parallel.context_parallel import zigzag_positions

IGNORE = -100


def shifted_targets(tokens_BL: torch.Tensor) -> torch.Tensor:
    """targets[b, l] = tokens[b, l+1]; the last position is ignored."""
    pad = torch.full_like(tokens_BL[:, :1], IGNORE)
    return torch.cat([tokens_BL[:, 1:], pad], dim=1)


def context_parallel_targets(tokens_BL: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Targets at this rank's zigzag positions (next global token, -100 past the end)."""
    length = tokens_BL.shape[1]
    positions = zigzag_positions(length, rank, world).to(tokens_BL.device)
    next_pos = positions + 1
    valid = next_pos < length
    targets = tokens_BL.index_select(1, next_pos.clamp(max=length - 1))
    return torch.where(valid.unsqueeze(0), targets, torch.full_like(targets, IGNORE))


class PipelineParallel:
    """GPipe: all microbatch forwards, then all microbatch backwards."""

    def __init__(self, model: torch.nn.Module, n_microbatches: int = 2):
        if n_microbatches < 1:
            raise ValueError(f"n_microbatches must be at least 1, got {n_microbatches}")
        self.model = model
        self.n_microbatches = n_microbatches

    def _peer(self, index: int) -> int:
        return mesh.global_rank("pp", index)

    def forward_backward(self, tokens_BL: torch.Tensor) -> torch.Tensor:
        rank, world = mesh.rank_and_world_size("pp")
        group = mesh.group_for("pp")
        batch, length = tokens_BL.shape
        if batch % self.n_microbatches != 0:
            raise ValueError(f"batch {batch} is not divisible by n_microbatches {self.n_microbatches}")
        cp_rank, cp_world = mesh.rank_and_world_size("cp")
        cp = getattr(self.model, "context_parallel", False) and cp_world > 1
        if cp:
            targets_all = context_parallel_targets(tokens_BL, cp_rank, cp_world)
            local_len = length // cp_world
        else:
            targets_all = shifted_targets(tokens_BL)
            local_len = length
        total = (targets_all != IGNORE).sum().to(torch.float32)
        if cp:
            dist.all_reduce(total, op=dist.ReduceOp.SUM, group=mesh.group_for("cp"))
            if tokens_BL.is_cuda:
                from abacus_b200.parallel import cp_fused

                # Fused CP buffers are keyed per microbatch call and reused every
                # step: bounded device barrier over the CP group first.
                cp_fused.begin_step(tokens_BL.device)
        if not tokens_BL.is_cuda and total.item() < 1:
            raise ValueError("batch has no target tokens")

        dim = self.model.dim
        dtype = next(self.model.parameters()).dtype
        device = tokens_BL.device
        first, last = rank == 0, rank == world - 1
        micro = batch // self.n_microbatches
        token_chunks = tokens_BL.chunk(self.n_microbatches, dim=0)
        target_chunks = targets_all.chunk(self.n_microbatches, dim=0)
        inputs, outputs, losses, sends = [], [], [], []

        def post_recv(index):
            buf = torch.empty(micro, local_len, dim, device=device, dtype=dtype)
            return buf, dist.irecv(buf, src=self._peer(rank - 1), group=group, tag=index)

        pending = post_recv(0) if not first else None
        for index in range(self.n_microbatches):
            if first:
                incoming = token_chunks[index].clamp(min=0)
            else:
                buf, work = pending
                work.wait()
                if index + 1 < self.n_microbatches:
                    pending = post_recv(index + 1)
                incoming = buf.requires_grad_(True)
                inputs.append(incoming)
            hidden = self.model.hidden_states(incoming)
            if last:
                losses.append(fused_linear_cross_entropy(hidden, self.model.w_D_vocab, target_chunks[index], total))
            else:
                outputs.append(hidden)
                sends.append(dist.isend(hidden.detach().contiguous(), dst=self._peer(rank + 1), group=group, tag=index))
        for work in sends:
            work.wait()
        sends.clear()

        # Backward: the last microbatch's gradient flows first.
        n = self.n_microbatches

        def post_grad_recv(index):
            grad = torch.empty(micro, local_len, dim, device=device, dtype=dtype)
            return grad, dist.irecv(grad, src=self._peer(rank + 1), group=group, tag=n + index)

        pending = post_grad_recv(n - 1) if not last else None
        for index in reversed(range(n)):
            if last:
                losses[index].backward()
            else:
                grad, work = pending
                work.wait()
                if index > 0:
                    pending = post_grad_recv(index - 1)
                outputs[index].backward(grad)
            if not first:
                grad_in = inputs[index].grad
                if grad_in is None:
                    raise RuntimeError("stage input received no gradient")
                sends.append(dist.isend(grad_in.contiguous(), dst=self._peer(rank - 1), group=group, tag=n + index))
        for work in sends:
            work.wait()
        if not last:
            return torch.zeros((), device=device, dtype=dtype)
        return torch.stack([loss.detach() for loss in losses]).sum()
