"""Checkpoint save / load in the reference's ``state_dict`` layout.

The reference has no checkpointing; its implicit format is the module
``state_dict`` (fp32, (in, out) weights). This module writes that layout for
the *full* model from any parallel configuration:

* tensor-parallel shards (heads / MLP hidden) and expert-parallel shards are
  all-gathered and concatenated back to the 1-rank shapes;
* ZeRO-3 parameters are gathered with ``DataParallel.full_parameters``;
* AdamW state is stored per parameter name (``step``, ``exp_avg``,
  ``exp_avg_sq``; full tensors for replicated parameters) together with the
  WSD step.

Pipeline stages keep their local block indices (reference semantics) and are
saved per stage as ``<path>.stage<k>``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from abacus_b200.parallel import mesh

# name suffix -> (mesh dim, concat axis) of sharded parameters
_TP_AXES = {
    "attention.w_q_DHK": 1,
    "attention.w_k_DHK": 1,
    "attention.w_v_DHK": 1,
    "attention.w_o_HKD": 0,
    "mlp.w_gate_DM": 1,
    "mlp.w_up_DM": 1,
    "mlp.w_down_MD": 0,
}
_EP_AXES = {"moe.w_gate_EDM": 0, "moe.w_up_EDM": 0, "moe.w_down_EMD": 0}


def _gather_along(t: torch.Tensor, dim_name: str, axis: int) -> torch.Tensor:
    _, world = mesh.rank_and_world_size(dim_name)
    if world == 1:
        return t
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous(), group=mesh.group_for(dim_name))
    return torch.cat(parts, dim=axis)


def _axis_for(name: str, model) -> tuple[str, int] | None:
    if getattr(model, "tensor_parallel", False) or any(
        getattr(m, "tensor_parallel", False) for m in model.modules() if hasattr(m, "tensor_parallel")
    ):
        for suffix, axis in _TP_AXES.items():
            if name.endswith(suffix):
                return "tp", axis
    if getattr(model, "expert_parallel", False):
        for suffix, axis in _EP_AXES.items():
            if name.endswith(suffix):
                return "ep", axis
    return None


def full_state_dict(model: torch.nn.Module, parallel=None) -> dict[str, torch.Tensor]:
    """Model state in the single-rank layout (collective: call on every rank)."""
    params = dict(model.named_parameters())
    values = {}
    if parallel is not None and getattr(parallel, "stage", 0) == 3:
        for (name, _), full in zip(model.named_parameters(), parallel.full_parameters()):
            values[name] = full
    state = {}
    for name, tensor in model.state_dict().items():
        t = values.get(name, tensor.detach())
        if name in params:
            spec = _axis_for(name, model)
            if spec is not None:
                t = _gather_along(t, *spec)
        state[name] = t.detach().cpu().clone()
    return state


def save_checkpoint(path, model, optimizer=None, scheduler=None, parallel=None, extra=None) -> None:
    """Collective. Rank 0 writes ``path`` (``path.stage<k>`` for pipeline stages)."""
    state = {"model": full_state_dict(model, parallel)}
    if optimizer is not None:
        opt = {}
        for name, st in optimizer.state_dict_by_name(model).items():
            opt[name] = {"step": st["step"], "exp_avg": st["exp_avg"].cpu(), "exp_avg_sq": st["exp_avg_sq"].cpu()}
        state["optimizer"] = opt
        state["lr"] = optimizer.lr
    if scheduler is not None:
        state["scheduler"] = scheduler.state_dict()
    if extra:
        state["extra"] = extra
    rank = dist.get_rank() if dist.is_initialized() else 0
    stage = getattr(model, "rank", None) if hasattr(model, "is_last") else None
    target = f"{path}.stage{stage}" if stage is not None else str(path)
    pp_rank = mesh.rank_and_world_size("pp")[0] if stage is not None else 0
    writer = rank == 0 or (stage is not None and _is_stage_writer(pp_rank))
    if writer:
        torch.save(state, target)
    if dist.is_initialized():
        dist.barrier()


def _is_stage_writer(pp_rank: int) -> bool:
    # The first rank of every non-PP coordinate group writes its stage.
    m = mesh.get_mesh()
    if m is None:
        return True
    c = m.coords(dist.get_rank())
    return all(v == 0 for k, v in c.items() if k != "pp")


def _shard_of(full: torch.Tensor, name: str, model) -> torch.Tensor:
    spec = _axis_for(name, model)
    if spec is None:
        return full
    dim_name, axis = spec
    rank, world = mesh.rank_and_world_size(dim_name)
    if world == 1:
        return full
    return full.chunk(world, dim=axis)[rank]


def load_checkpoint(path, model, optimizer=None, scheduler=None) -> dict:
    """Load a full-layout checkpoint into a (possibly sharded) model."""
    stage = getattr(model, "rank", None) if hasattr(model, "is_last") else None
    target = f"{path}.stage{stage}" if stage is not None else str(path)
    state = torch.load(target, map_location="cpu", weights_only=False)
    own = model.state_dict()
    with torch.no_grad():
        for name, t in own.items():
            src = _shard_of(state["model"][name], name, model)
            t.copy_(src.to(t.device, t.dtype))
    if optimizer is not None and "optimizer" in state:
        optimizer.load_state_dict_by_name(model, state["optimizer"])
        optimizer.lr = state.get("lr", optimizer.lr)
    if scheduler is not None and "scheduler" in state:
        scheduler.load_state_dict(state["scheduler"])
    return state.get("extra", {})
