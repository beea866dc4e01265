"""Training loop (``abacus/trainer.py``): forward -> cross entropy ->
zero_grad -> backward -> data-parallel sync -> WSD learning rate -> AdamW ->
ZeRO parameter gather; plus the pipeline and context-parallel branches. With
the fused data-parallel optimizer the learning rate is taken before backward
and the reduction + AdamW run per gradient bucket under backward.

Differences from the reference, none of which change the maths:

* The loss is computed by the fused linear + cross-entropy path
  (``model(inputs, targets=..., normalizer=...)``), so the (T, V) logits are
  never materialised; targets are ``tokens[:, 1:]`` with the last position
  ignored, which equals the reference's ``logits[:, :-1]`` slicing.
* The target-token count stays on the device (no host sync per step). The
  reference's "batch has no target tokens" check therefore runs only for CPU
  tensors.
* Optional optimizer / schedule hyper-parameters (the reference hard-codes
  AdamW's defaults and ``WSD(total_steps)``); defaults are the reference's.
* MoE models with the softmax router add their load-balancing loss.
* Pipeline and context parallel may be combined through a mesh (the
  reference forbids PP + CP).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from abacus_b200.optim.adamw import AdamW
from abacus_b200.optim.lr_scheduler import WSD
from abacus_b200.parallel import mesh
from abacus_b200.parallel.context_parallel import sum_parameter_gradients
from abacus_b200.parallel.data_parallel import DataParallel
from abacus_b200.parallel.pipeline_parallel import (
    PipelineParallel,
    context_parallel_targets,
    shifted_targets,
)
from abacus_b200.utils.dist import print_peak_memory
from abacus_b200.utils.trace import PhaseTracer

IGNORE = -100


def get_device() -> torch.device:
    if not torch.cuda.is_available():
        return torch.device("cpu")
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    return torch.device("cuda", local_rank)


class Trainer:
    def __init__(
        self,
        model: torch.nn.Module,
        parallel: DataParallel | None = None,
        pipeline: PipelineParallel | None = None,
        total_steps: int | None = None,
        lr: float | None = None,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 1e-2,
        schedule_lr: float = 5e-4,
        print_memory: bool = False,
        device: torch.device | str | None = None,
        tracer: PhaseTracer | None = None,
    ):
        if parallel is not None and pipeline is not None and mesh.get_mesh() is None:
            raise ValueError("pipeline parallel does not use DataParallel")
        if pipeline is not None and getattr(model, "context_parallel", False) and mesh.get_mesh() is None:
            raise ValueError("pipeline parallel does not combine with context parallel")
        self.device = get_device() if device is None else torch.device(device)
        self.model = model.to(self.device)
        self.parallel = parallel
        self.pipeline = pipeline
        self.print_memory = print_memory
        # NVTX range (and optional device timing) per phase of a step.
        self.tracer = tracer if tracer is not None else PhaseTracer()
        owned = grad_shards = None
        if parallel is not None:
            parallel.broadcast_parameters()
            owned = parallel.owned
            grad_shards = parallel.grad_shards
        self.optimizer = AdamW(
            self.model, lr=1e-3 if lr is None else lr, betas=betas, eps=eps, weight_decay=weight_decay,
            owned=owned, grad_shards=grad_shards,
        )
        self._fused = bool(getattr(parallel, "fused_optimizer", False))
        if self._fused and pipeline is not None:
            raise ValueError("the fused data-parallel optimizer does not combine with pipeline parallel")
        if self._fused:
            parallel.bind_optimizer(self.optimizer)
        self.scheduler = WSD(total_steps, lr=schedule_lr) if total_steps is not None else None
        if self.scheduler is not None:
            self.optimizer.lr = self.scheduler.learning_rate(1)

    # ------------------------------------------------------------------ steps
    def step(self, tokens_BL: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        self.model.train()
        tokens_BL = tokens_BL.to(self.device, non_blocking=True)
        phase = self.tracer.phase
        if self.pipeline is not None:
            self.optimizer.zero_grad()
            with phase("pipeline_forward_backward", self.device):
                loss = self.pipeline.forward_backward(tokens_BL).detach()
            if getattr(self.model, "context_parallel", False) and mesh.rank_and_world_size("cp")[1] > 1:
                with phase("cp_sync", self.device):
                    sum_parameter_gradients(self.model)
                    # Each CP rank of the last stage holds its shard's share of the loss.
                    loss = loss.clone()
                    dist.all_reduce(loss, op=dist.ReduceOp.SUM, group=mesh.group_for("cp"))
            with phase("optimizer", self.device):
                self._optimizer_step()
            return loss, loss
        inputs_BL = tokens_BL.clamp(min=0)  # -100 is padding; the embedding has no row for it
        if self._context_parallel_active():
            return self._context_parallel_step(tokens_BL, inputs_BL)
        with phase("forward", self.device):
            targets = shifted_targets(tokens_BL)
            token_count = (targets != IGNORE).sum()
            if not tokens_BL.is_cuda and int(token_count) < 1:
                raise ValueError("batch has no target tokens")
            normalizer = token_count.to(torch.float32)
            if self.parallel is not None and not self.parallel.token_weighted:
                # Loss divided by the global token count; gradients are then summed.
                normalizer = normalizer.clone()
                dist.all_reduce(normalizer, op=dist.ReduceOp.SUM, group=self.parallel.group)
            loss = self.model(inputs_BL, targets=targets, normalizer=normalizer)
            loss = self._with_aux_loss(loss)
        self.optimizer.zero_grad()
        if self.print_memory:
            print_peak_memory()
        if self.parallel is not None:
            self.parallel.set_token_count(token_count)
        if self._fused:
            # The fused data-parallel path reduces and updates each gradient
            # bucket while backward runs, so this step's learning rate and
            # token count are fixed before backward.
            self._advance_lr()
            self.parallel.prepare_step(self.optimizer, token_count)
        with phase("backward", self.device):
            loss.backward()
        local_loss = loss.detach()
        if self.parallel is not None:
            with phase("dp_sync", self.device):
                loss = self.parallel.synchronize(loss, token_count)
        if not self._fused:
            with phase("optimizer", self.device):
                self._optimizer_step()
        if self.parallel is not None:
            with phase("dp_gather", self.device):
                self.parallel.gather_parameters()
        return loss.detach(), local_loss

    def _with_aux_loss(self, loss):
        aux = getattr(self.model, "aux_loss", None)
        if callable(aux):
            extra = aux()
            if extra is not None:
                loss = loss + extra
        return loss

    def _advance_lr(self) -> None:
        if self.scheduler is not None:
            self.optimizer.lr = self.scheduler.step()

    def _optimizer_step(self) -> None:
        self._advance_lr()
        self.optimizer.step()

    def _context_parallel_active(self) -> bool:
        if not getattr(self.model, "context_parallel", False):
            return False
        if self.parallel is not None:
            raise ValueError("context parallel does not use DataParallel")
        return mesh.rank_and_world_size("cp")[1] > 1

    def _context_parallel_step(self, tokens_BL, inputs_BL):
        """Global token-weighted loss across CP ranks (``abacus/trainer.py:115-148``);
        parameter gradients are summed over the CP group after backward."""
        phase = self.tracer.phase
        rank, world = mesh.rank_and_world_size("cp")
        group = mesh.group_for("cp")
        with phase("forward", self.device):
            targets = context_parallel_targets(tokens_BL, rank, world)
            local_count = (targets != IGNORE).sum()
            total_count = local_count.to(torch.float32)
            dist.all_reduce(total_count, op=dist.ReduceOp.SUM, group=group)
            if not tokens_BL.is_cuda and total_count.item() < 1:
                raise ValueError("batch has no target tokens")
            loss = self.model(inputs_BL, targets=targets, normalizer=total_count)
            local_sum = loss.detach() * total_count
        self.optimizer.zero_grad()
        if self.print_memory:
            print_peak_memory()
        with phase("backward", self.device):
            loss.backward()
        with phase("cp_sync", self.device):
            sum_parameter_gradients(self.model)
        with phase("optimizer", self.device):
            self._optimizer_step()
        reported = local_sum.clone()
        dist.all_reduce(reported, op=dist.ReduceOp.SUM, group=group)
        global_loss = (reported / total_count).detach()
        local_loss = local_sum / local_count.to(torch.float32).clamp(min=1)
        return global_loss, local_loss

    def train(self, batches) -> None:
        for tokens_BL in batches:
            self.step(tokens_BL)
