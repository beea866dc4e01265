"""Checkpoint save / load in the reference's ``state_dict`` layout.

The reference has no checkpointing; its implicit format is the module
``state_dict`` (fp32, (in, out) weights). This module writes that layout for
the *full* model from any parallel configuration:

* tensor-parallel shards (heads / MLP hidden) and expert-parallel shards are
  all-gathered and concatenated back to the 1-rank shapes;
* ZeRO-3 parameters are gathered with ``DataParallel.full_parameters``;
* AdamW state is stored per parameter name (``step``, ``exp_avg``,
  ``exp_avg_sq``) in the same full layout: moments sharded by ZeRO (or by the
  fused data-parallel kernel, which keeps moments for its owned slice only)
  are all-gathered over the data-parallel group, then tensor- / expert-parallel
  moments are concatenated like their weights. Loading re-shards them the
  same way (TP / EP shard, then this rank's owned ZeRO range), so a run may
  resume under a different TP, EP or ZeRO layout;
* the WSD step.

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


def _full_shapes(model, parallel) -> dict[str, tuple]:
    """Local (TP / EP-sharded, ZeRO-unsharded) shape of every parameter."""
    shapes = {}
    recorded = {}
    for unit in getattr(parallel, "units", None) or []:
        for p, shape in zip(unit.params, unit.shapes):
            recorded[id(p)] = shape
    for name, p in model.named_parameters():
        shapes[name] = recorded.get(id(p), tuple(p.shape))
    return shapes


def full_optimizer_state(model, optimizer, parallel=None) -> dict[str, dict]:
    """AdamW state of every parameter in the single-rank layout (collective)."""
    owned = getattr(parallel, "owned", None)
    by_id = {id(p): name for name, p in model.named_parameters()}
    states = {id(p): optimizer.state.get(id(p)) for _, p in model.named_parameters()}
    step = max([int(st["step"]) for st in states.values() if st is not None] or [0])
    if dist.is_initialized() and parallel is not None:
        t = torch.tensor([step], dtype=torch.int64, device=_device_of(model))
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=parallel.group)
        step = int(t.item())
    moments = {}
    for key in ("exp_avg", "exp_avg_sq"):
        pieces = {pid: st[key] for pid, st in states.items() if st is not None}
        if owned is not None:
            # ZeRO-sharded moments: every rank holds only its owned range.
            gathered = parallel.gather_owned(pieces)
            pieces = {pid: gathered.get(pid, t) for pid, t in pieces.items()} | {
                pid: t for pid, t in gathered.items() if pid not in pieces}
        moments[key] = pieces
    shapes = _full_shapes(model, parallel)
    out = {}
    for name, p in model.named_parameters():
        m, v = moments["exp_avg"].get(id(p)), moments["exp_avg_sq"].get(id(p))
        if m is None or v is None:
            continue
        spec = _axis_for(name, model)
        m, v = m.reshape(shapes[name]), v.reshape(shapes[name])
        if spec is not None:
            m, v = _gather_along(m, *spec), _gather_along(v, *spec)
        out[by_id[id(p)]] = {"step": step, "exp_avg": m.detach().cpu().clone(), "exp_avg_sq": v.detach().cpu().clone()}
    return out


def _device_of(model) -> torch.device:
    p = next(model.parameters(), None)
    return p.device if p is not None else torch.device("cpu")


def save_checkpoint(path, model, optimizer=None, scheduler=None, parallel=None, extra=None) -> None:
    """Collective. Rank 0 writes ``path`` (``path.stage<k>`` for pipeline stages)."""
    state = {"model": full_state_dict(model, parallel)}
    if optimizer is not None:
        state["optimizer"] = full_optimizer_state(model, optimizer, parallel)
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


def load_checkpoint(path, model, optimizer=None, scheduler=None, parallel=None) -> dict:
    """Load a full-layout checkpoint into a (possibly sharded) model.

    With ``parallel`` (a ZeRO ``DataParallel`` or ``FusedDataParallel`` whose
    ``broadcast_parameters`` has run) the optimizer moments are cut to this
    rank's owned range, and ZeRO-3 parameters receive this rank's piece."""
    stage = getattr(model, "rank", None) if hasattr(model, "is_last") else None
    target = f"{path}.stage{stage}" if stage is not None else str(path)
    state = torch.load(target, map_location="cpu", weights_only=False)
    own = model.state_dict()
    # ZeRO-3: parameters hold only this rank's piece of their unit's chunk.
    pieces = {}
    for unit in getattr(parallel, "units", None) or []:
        if getattr(unit, "local", None) is not None:
            for q, (lo, hi, _), view in zip(unit.params, unit.pieces, unit.piece_views(unit.local)):
                pieces[id(q)] = (lo, hi, view)
    params = dict(model.named_parameters())
    with torch.no_grad():
        for name, t in own.items():
            src = _shard_of(state["model"][name], name, model)
            piece = pieces.get(id(params[name])) if name in params else None
            if piece is not None:
                lo, hi, view = piece
                view.copy_(src.reshape(-1)[lo:hi].to(view.device, view.dtype))
            else:
                t.copy_(src.to(t.device, t.dtype))
    if optimizer is not None and "optimizer" in state:
        owned = getattr(parallel, "owned", None)
        local = {}
        for name, param in model.named_parameters():
            saved = state["optimizer"].get(name)
            if saved is None:
                continue
            entry = {"step": saved["step"]}
            for key in ("exp_avg", "exp_avg_sq"):
                t = _shard_of(saved[key], name, model)
                if owned is not None:
                    span = owned.get(id(param))
                    if span is None:
                        entry = None
                        break
                    t = t.reshape(-1)[span[0] : span[1]]
                entry[key] = t
            if entry is not None:
                local[name] = entry
        optimizer.load_state_dict_by_name(model, local)
        optimizer.lr = state.get("lr", optimizer.lr)
    if scheduler is not None and "scheduler" in state:
        scheduler.load_state_dict(state["scheduler"])
    return state.get("extra", {})
