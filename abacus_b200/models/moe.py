"""Mixture of SwiGLU experts: router, single-process MoE, expert-parallel MoE.

Reference semantics:

* ``Router`` (``abacus/moe/router.py:12-70``): sigmoid scores; top-k chosen
  on ``scores + expert_bias`` (bias used for the choice only); weights = the
  chosen scores normalised to sum 1, times ``route_scale``; in training the
  DeepSeek-V3 aux-loss-free update ``b += gamma * sign(mean_load - load)``.
* ``load_balancing_loss`` (``abacus/moe/load_balancing.py:8-41``): Switch
  Transformer ``coeff * E * sum_e f_e p_e``.
* ``MoE`` (``abacus/moe/moe.py:22-86``): dense combine of every expert's
  weighted output (no capacity limit).
* ``MoEExpertParallel`` (``abacus/moe/moe.py:89-189``): one expert per rank,
  replicated batch, contiguous token shards, all-to-all dispatch/combine and an
  all-gather-v of the shard outputs.

Options beyond the reference (defaults reproduce it):

* ``router="softmax"``: softmax scores with top-k on the scores, weights
  renormalised over the chosen experts, and the load-balancing auxiliary loss
  recorded on ``Router.aux_loss`` (added to the training loss by the trainer).
* ``capacity_factor``: per-expert capacity ``ceil(cf * tokens * k / E)``;
  assignments beyond it (in token order) are dropped.
* ``MoEExpertParallel(data_parallel=True)``: every rank routes its *own*
  tokens (DP over the non-expert parameters) instead of a shard of a
  replicated batch; no gather-v is needed and non-expert gradients are
  averaged by the data-parallel wrapper.

Without a capacity factor, tokens are permuted by expert with one stable
sort, each expert's contiguous slab runs the fused SwiGLU GEMM path, and the
combine is a weighted ``index_add`` in sorted order (deterministic). With a
capacity factor (CUDA), every expert owns a static slab of C rows and all
experts run as one grouped launch per product (``gemm.grouped_swiglu_mlp``),
with no host sync.
"""
from __future__ import annotations

import math
import os

import torch

from abacus_b200.ops import gemm
from abacus_b200.ops._ext import ext
from abacus_b200.ops.routing import expert_rank
from abacus_b200.parallel import ep_fused, mesh, tp_fused
from abacus_b200.parallel.expert_parallel import (
    _AllToAll,
    _GatherTokenShards,
    _SumReplicatedGrads,
    exchange_counts,
    shard_counts,
)


def load_balancing_loss(router_probs: torch.Tensor, expert_indices: torch.Tensor, coeff: float = 1e-2) -> torch.Tensor:
    """Switch Transformer auxiliary loss."""
    if router_probs.ndim < 1:
        raise ValueError("router_probs must include an expert dimension")
    n_experts = router_probs.shape[-1]
    if n_experts < 1:
        raise ValueError(f"router_probs has no experts, got shape {tuple(router_probs.shape)}")
    batch = router_probs.shape[:-1]
    if expert_indices.shape[: len(batch)] != batch:
        raise ValueError(
            f"expert_indices shape {tuple(expert_indices.shape)} does not match router_probs batch {tuple(batch)}"
        )
    extra = expert_indices.ndim - len(batch)
    if extra > 1:
        raise ValueError(f"expert_indices has {extra} expert-choice dimensions, expected 0 or 1")
    probs_TE = router_probs.reshape(-1, n_experts).float()
    tokens = probs_TE.shape[0]
    if tokens == 0:
        return router_probs.new_zeros(())
    slots_TK = expert_indices.reshape(tokens, -1).to(dtype=torch.long)
    # A token counts once per expert even if its slot list repeats it.
    dispatch_TE = torch.zeros(tokens, n_experts, device=probs_TE.device).scatter_(1, slots_TK, 1.0)
    k = slots_TK.shape[-1]
    f_E = dispatch_TE.sum(dim=0) / (tokens * k)
    p_E = probs_TE.sum(dim=0) / tokens
    return (torch.sum(f_E * p_E) * (coeff * n_experts)).to(dtype=router_probs.dtype)


class _RouterLogits(torch.autograd.Function):
    """``x @ w_DE`` on the router kernels (one read of x; no library GEMM)."""

    @staticmethod
    def forward(ctx, x2, w):
        out = torch.empty(x2.shape[0], w.shape[1], device=x2.device, dtype=torch.float32)
        ext().router_logits(x2, w.contiguous(), out)
        ctx.save_for_backward(x2, w)
        return out

    @staticmethod
    def backward(ctx, grad):
        x2, w = ctx.saved_tensors
        dx = torch.empty_like(x2)
        dw = torch.empty_like(w)
        ext().router_logits_bwd(grad.contiguous(), x2, w.contiguous(), dx, dw)
        return dx, dw


def router_logits(x_BLD: torch.Tensor, w_DE: torch.Tensor) -> torch.Tensor:
    """Router scores (B, L, E) = x @ w_DE: the router kernels for fp32 CUDA
    inputs with a power-of-two expert count up to 64, ATen otherwise."""
    e = w_DE.shape[1]
    if x_BLD.is_cuda and x_BLD.dtype == torch.float32 and e <= 64 and (e & (e - 1)) == 0:
        x2 = x_BLD.reshape(-1, x_BLD.shape[-1])
        if x2.stride(1) != 1:
            x2 = x2.contiguous()
        return _RouterLogits.apply(x2, w_DE).view(*x_BLD.shape[:-1], e)
    return x_BLD @ w_DE


class _RouteTopK(torch.autograd.Function):
    """Routing on one kernel per direction: probabilities, top-k selection and
    renormalised weights (forward); d logits from d weights and d probs
    (backward). Returns (weights, indices, probs)."""

    @staticmethod
    def forward(ctx, logits_TE, bias_E, mode, top_k, route_scale):
        t, e = logits_TE.shape
        probs = torch.empty_like(logits_TE)
        weights = torch.empty(t, top_k, device=logits_TE.device, dtype=torch.float32)
        indices = torch.empty(t, top_k, device=logits_TE.device, dtype=torch.int64)
        ext().route_topk(logits_TE, bias_E, mode, top_k, route_scale, probs, weights, indices)
        ctx.save_for_backward(probs, indices)
        ctx.meta = (mode, top_k, route_scale)
        ctx.mark_non_differentiable(indices)
        return weights, indices, probs

    @staticmethod
    def backward(ctx, d_weights, _d_indices, d_probs):
        probs, indices = ctx.saved_tensors
        mode, top_k, route_scale = ctx.meta
        if d_weights is None:
            d_weights = torch.zeros(indices.shape, device=probs.device, dtype=torch.float32)
        d_logits = torch.empty_like(probs)
        ext().route_topk_bwd(probs, indices, d_weights.contiguous(), None if d_probs is None else d_probs.contiguous(),
                             mode, top_k, route_scale, d_logits)
        return d_logits, None, None, None, None


def _route_kernel_usable(logits_BLE: torch.Tensor) -> bool:
    e = logits_BLE.shape[-1]
    return logits_BLE.is_cuda and logits_BLE.dtype == torch.float32 and e <= 64 and (e & (e - 1)) == 0


class Router(torch.nn.Module):
    def __init__(
        self,
        dim: int,
        n_experts: int,
        top_k: int,
        bias_update_speed: float = 1e-3,
        route_scale: float = 1.0,
        expert_parallel: bool = False,
        router: str = "sigmoid",
        aux_loss_coeff: float = 1e-2,
        sync_dim: str = "ep",
    ):
        super().__init__()
        if n_experts < 1:
            raise ValueError(f"n_experts must be at least 1, got {n_experts}")
        if not 1 <= top_k <= n_experts:
            raise ValueError(f"top_k must be in [1, {n_experts}], got {top_k}")
        if router not in ("sigmoid", "softmax"):
            raise ValueError(f"router must be 'sigmoid' or 'softmax', got {router!r}")
        self.dim = dim
        self.n_experts = n_experts
        self.top_k = top_k
        self.bias_update_speed = bias_update_speed
        self.route_scale = route_scale
        self.expert_parallel = expert_parallel
        self.router = router
        self.aux_loss_coeff = aux_loss_coeff
        self.sync_dim = sync_dim
        self.aux_loss: torch.Tensor | None = None
        self.w_DE = torch.nn.Parameter(torch.empty(dim, n_experts))
        torch.nn.init.xavier_uniform_(self.w_DE)
        self.register_buffer("expert_bias_E", torch.zeros(n_experts, dtype=self.w_DE.dtype))

    def forward(self, x_BLD: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        w_DE = _SumReplicatedGrads.apply(self.w_DE, self.sync_dim) if self.expert_parallel else self.w_DE
        logits_BLE = router_logits(x_BLD, w_DE)
        if _route_kernel_usable(logits_BLE):
            lead = logits_BLE.shape[:-1]
            softmax = self.router == "softmax"
            bias = None if softmax else self.expert_bias_E.to(torch.float32).contiguous()
            weights_TK, indices_TK, probs_TE = _RouteTopK.apply(
                logits_BLE.reshape(-1, self.n_experts).contiguous(), bias, 0 if softmax else 1, self.top_k,
                float(self.route_scale))
            weights_BLK = weights_TK.view(*lead, self.top_k)
            indices_BLK = indices_TK.view(*lead, self.top_k)
            if softmax:
                probs_BLE = probs_TE.view(*lead, self.n_experts)
                self.aux_loss = load_balancing_loss(probs_BLE, indices_BLK, self.aux_loss_coeff) if self.training else None
            elif self.training:
                self.update_bias(indices_BLK)
            return weights_BLK, indices_BLK
        if self.router == "softmax":
            probs_BLE = torch.softmax(logits_BLE, dim=-1)
            indices_BLK = torch.topk(probs_BLE.detach(), self.top_k, dim=-1).indices
            weights_BLK = probs_BLE.gather(dim=-1, index=indices_BLK)
            weights_BLK = weights_BLK / weights_BLK.sum(dim=-1, keepdim=True) * self.route_scale
            self.aux_loss = load_balancing_loss(probs_BLE, indices_BLK, self.aux_loss_coeff) if self.training else None
            return weights_BLK, indices_BLK
        scores_BLE = torch.sigmoid(logits_BLE)
        selection_BLE = scores_BLE.detach() + self.expert_bias_E
        indices_BLK = torch.topk(selection_BLE, self.top_k, dim=-1).indices
        weights_BLK = scores_BLE.gather(dim=-1, index=indices_BLK)
        weights_BLK = weights_BLK / weights_BLK.sum(dim=-1, keepdim=True)
        weights_BLK = weights_BLK * self.route_scale
        if self.training:
            self.update_bias(indices_BLK)
        return weights_BLK, indices_BLK

    @torch.no_grad()
    def update_bias(self, indices_BLK: torch.Tensor) -> None:
        """DeepSeek-V3: b_i += gamma * sign(average load - load_i)."""
        if self.bias_update_speed == 0:
            return
        counts_E = torch.bincount(indices_BLK.reshape(-1), minlength=self.n_experts)
        counts_E = counts_E.to(device=self.expert_bias_E.device)
        violation_E = counts_E.sum() - counts_E * self.n_experts
        step_E = torch.sign(violation_E.to(dtype=self.expert_bias_E.dtype))
        self.expert_bias_E.add_(self.bias_update_speed * step_E)


def _capacity_keep(indices_TK: torch.Tensor, n_experts: int, capacity: int) -> torch.Tensor:
    """Mask (T, K) of kept assignments: the first `capacity` per expert in
    (token, slot) order."""
    rank_in_expert = expert_rank(indices_TK.reshape(-1), n_experts)
    return (rank_in_expert < capacity).reshape(indices_TK.shape)


def _expert_forward(x_SD, w_gate_DM, w_up_DM, w_down_MD):
    return gemm.swiglu_mlp(x_SD, w_gate_DM, w_up_DM, w_down_MD)


def _grouped_experts(x_TD, weights_TK, indices_TK, w_gate_EDM, w_up_EDM, w_down_EMD, expert_offset=0):
    """Weighted sum over each token's chosen experts. Tokens are sorted by
    expert once; each expert runs on its contiguous slab."""
    t, k = indices_TK.shape
    flat_e = indices_TK.reshape(-1) - expert_offset
    order = torch.argsort(flat_e, stable=True)
    token_of = torch.arange(t, device=x_TD.device).repeat_interleave(k)[order]
    counts = torch.bincount(flat_e, minlength=w_gate_EDM.shape[0]).tolist()
    xs = x_TD.index_select(0, token_of)
    w_sorted = weights_TK.reshape(-1)[order]
    outs = []
    start = 0
    for e, n in enumerate(counts):
        # Empty slabs still run, so an idle expert gets a zero gradient rather
        # than none (expert-parallel ranks compare shard by shard).
        outs.append(_expert_forward(xs[start : start + n], w_gate_EDM[e], w_up_EDM[e], w_down_EMD[e]))
        start += n
    y = torch.cat(outs, dim=0) * w_sorted.unsqueeze(-1)
    return x_TD.new_zeros(x_TD.shape).index_add(0, token_of, y)


def _grouped_experts_capacity(x_TD, weights_TK, indices_TK, w_gate_EDM, w_up_EDM, w_down_EMD, capacity):
    """``_grouped_experts`` with static capacity slabs: expert e's rows are
    slots [e*C, (e+1)*C) of one (E*C, D) slab, filled in (token, slot) order;
    assignments past an expert's capacity go to a discarded extra row (the
    router has already given them weight 0). Every expert GEMM has C rows, so
    nothing about the routing reaches the host."""
    t, k = indices_TK.shape
    n_experts = w_gate_EDM.shape[0]
    flat_e = indices_TK.reshape(-1)
    within = expert_rank(flat_e, n_experts)
    keep = within < capacity
    spill = n_experts * capacity
    slot = torch.where(keep, flat_e * capacity + within, spill)
    token_of = torch.arange(t, device=x_TD.device).repeat_interleave(k)
    slab = x_TD.new_zeros(spill + 1, x_TD.shape[1]).index_copy(0, slot, x_TD.index_select(0, token_of))
    # All experts in one grouped launch per product (every slab has C rows).
    y_ECD = gemm.grouped_swiglu_mlp(slab[:spill].view(n_experts, capacity, -1), w_gate_EDM, w_up_EDM, w_down_EMD)
    y_slab = torch.cat((y_ECD.reshape(spill, -1), x_TD.new_zeros(1, x_TD.shape[1])), dim=0)
    y_TKD = y_slab.index_select(0, slot).view(t, k, -1)
    return (y_TKD * (weights_TK * keep.view(t, k)).unsqueeze(-1)).sum(dim=1)


class MoE(torch.nn.Module):
    """Top-k mixture of SwiGLU experts (single process)."""

    def __init__(
        self,
        dim: int,
        n_experts: int,
        top_k: int,
        hidden_dim: int | None = None,
        bias_update_speed: float = 1e-3,
        route_scale: float = 1.0,
        router: str = "sigmoid",
        capacity_factor: float | None = None,
        aux_loss_coeff: float = 1e-2,
    ):
        super().__init__()
        self.dim = dim
        self.n_experts = n_experts
        self.top_k = top_k
        self.hidden_dim = dim if hidden_dim is None else hidden_dim
        self.capacity_factor = capacity_factor
        if self.hidden_dim < 1:
            raise ValueError(f"hidden_dim must be at least 1, got {self.hidden_dim}")
        self.router = Router(
            dim, n_experts, top_k, bias_update_speed=bias_update_speed, route_scale=route_scale,
            router=router, aux_loss_coeff=aux_loss_coeff,
        )
        gate_EDM = torch.empty(n_experts, dim, self.hidden_dim)
        up_EDM = torch.empty(n_experts, dim, self.hidden_dim)
        down_EMD = torch.empty(n_experts, self.hidden_dim, dim)
        for expert in range(n_experts):
            torch.nn.init.xavier_uniform_(gate_EDM[expert])
            torch.nn.init.xavier_uniform_(up_EDM[expert])
            torch.nn.init.xavier_uniform_(down_EMD[expert])
        self.w_gate_EDM = torch.nn.Parameter(gate_EDM)
        self.w_up_EDM = torch.nn.Parameter(up_EDM)
        self.w_down_EMD = torch.nn.Parameter(down_EMD)

    def _route(self, x_BLD):
        weights_BLK, indices_BLK = self.router(x_BLD)
        tokens = x_BLD.shape[0] * x_BLD.shape[1]
        weights_TK = weights_BLK.reshape(tokens, self.top_k)
        indices_TK = indices_BLK.reshape(tokens, self.top_k)
        capacity = self._capacity(tokens)
        if capacity is not None:
            weights_TK = weights_TK * _capacity_keep(indices_TK, self.n_experts, capacity)
        return weights_TK, indices_TK

    def forward(self, x_BLD: torch.Tensor) -> torch.Tensor:
        batch, length, _ = x_BLD.shape
        weights_TK, indices_TK = self._route(x_BLD)
        x_TD = x_BLD.reshape(batch * length, self.dim)
        if x_TD.shape[0] == 0:
            return x_BLD
        capacity = self._capacity(x_TD.shape[0])
        if capacity is not None and x_TD.is_cuda:
            out_TD = _grouped_experts_capacity(x_TD, weights_TK, indices_TK, self.w_gate_EDM, self.w_up_EDM,
                                               self.w_down_EMD, capacity)
        else:
            out_TD = _grouped_experts(x_TD, weights_TK, indices_TK, self.w_gate_EDM, self.w_up_EDM, self.w_down_EMD)
        return out_TD.reshape(batch, length, self.dim)

    def _capacity(self, tokens: int) -> int | None:
        """Per-expert capacity of this rank's tokens (None without a capacity factor)."""
        if self.capacity_factor is None or tokens == 0:
            return None
        return math.ceil(self.capacity_factor * tokens * self.top_k / self.n_experts)


class MoEExpertParallel(torch.nn.Module):
    """Top-k SwiGLU experts, ``n_experts / ep`` experts on each rank."""

    def __init__(
        self,
        dim: int,
        n_experts: int,
        top_k: int,
        hidden_dim: int | None = None,
        bias_update_speed: float = 1e-3,
        route_scale: float = 1.0,
        router: str = "sigmoid",
        capacity_factor: float | None = None,
        aux_loss_coeff: float = 1e-2,
        data_parallel: bool = False,
    ):
        super().__init__()
        self.dim = dim
        self.n_experts = n_experts
        self.top_k = top_k
        self.hidden_dim = dim if hidden_dim is None else hidden_dim
        self.capacity_factor = capacity_factor
        self.data_parallel = data_parallel
        if self.hidden_dim < 1:
            raise ValueError(f"hidden_dim must be at least 1, got {self.hidden_dim}")
        self.rank, self.world_size = mesh.rank_and_world_size("ep")
        if self.world_size > 1 and not data_parallel and self.n_experts != self.world_size:
            raise ValueError(
                f"expert parallel keeps 1 expert on each rank, "
                f"got {self.n_experts} experts and world size {self.world_size}"
            )
        if self.world_size > 1 and n_experts % self.world_size != 0:
            raise ValueError(f"{n_experts} experts do not divide over {self.world_size} ranks")
        # A replicated batch needs the router grad summed; DP routes local tokens
        # and the data-parallel wrapper averages the router like any replica param.
        self.router = Router(
            dim, n_experts, top_k, bias_update_speed=bias_update_speed, route_scale=route_scale,
            expert_parallel=self.world_size > 1 and not data_parallel, router=router, aux_loss_coeff=aux_loss_coeff,
        )
        gate_EDM = torch.empty(n_experts, dim, self.hidden_dim)
        up_EDM = torch.empty(n_experts, dim, self.hidden_dim)
        down_EMD = torch.empty(n_experts, self.hidden_dim, dim)
        for expert in range(n_experts):
            torch.nn.init.xavier_uniform_(gate_EDM[expert])
            torch.nn.init.xavier_uniform_(up_EDM[expert])
            torch.nn.init.xavier_uniform_(down_EMD[expert])
        self.local_experts = n_experts // self.world_size if self.world_size > 1 else n_experts
        start = self.rank * self.local_experts if self.world_size > 1 else 0
        self.expert_offset = start
        self.w_gate_EDM = torch.nn.Parameter(gate_EDM[start : start + self.local_experts].clone())
        self.w_up_EDM = torch.nn.Parameter(up_EDM[start : start + self.local_experts].clone())
        self.w_down_EMD = torch.nn.Parameter(down_EMD[start : start + self.local_experts].clone())
        self._ep_key = tp_fused.new_key("moe")

    _route = MoE._route
    _capacity = MoE._capacity

    def forward(self, x_BLD: torch.Tensor) -> torch.Tensor:
        if self.world_size == 1:
            return MoE.forward(self, x_BLD)
        if not self.data_parallel:
            x_BLD = _SumReplicatedGrads.apply(x_BLD, "ep")
        weights_TK, indices_TK = self._route(x_BLD)
        batch, length, _ = x_BLD.shape
        tokens = batch * length
        if tokens == 0:
            return x_BLD
        x_TD = x_BLD.reshape(tokens, self.dim)
        if self.data_parallel:
            out_TD = self._dispatch(x_TD, weights_TK, indices_TK)
            return out_TD.reshape(batch, length, self.dim)
        counts = shard_counts(tokens, self.world_size)
        offset = sum(counts[: self.rank])
        local_n = counts[self.rank]
        local_SD = self._dispatch(
            x_TD[offset : offset + local_n], weights_TK[offset : offset + local_n], indices_TK[offset : offset + local_n]
        )
        counts_E = torch.tensor(counts, device=x_BLD.device, dtype=torch.long)
        out_TD = _GatherTokenShards.apply(local_SD, counts_E, "ep")
        return out_TD.reshape(batch, length, self.dim)

    def _dispatch(self, local_SD, weights_SK, indices_SK):
        """Send each (token, slot) row to the rank owning its expert, run the
        local experts, send results back, weight and sum the K slots."""
        if ep_fused.usable(local_SD, self.hidden_dim):
            # Dispatch fused with the permutation, combine fused into the
            # expert down-projection's epilogue (NVLink peer memory). With a
            # capacity and every routed token local (EP over DP ranks), the
            # slabs are static and the routing never reaches the host.
            static = os.environ.get("ABACUS_EP_STATIC", "1") != "0"
            capacity = self._capacity(local_SD.shape[0]) if self.data_parallel and static else None
            if capacity is not None:
                return ep_fused.dispatch_combine_capacity(local_SD, weights_SK, indices_SK, self.w_gate_EDM,
                                                          self.w_up_EDM, self.w_down_EMD, self.n_experts, capacity,
                                                          self._ep_key)
            return ep_fused.dispatch_combine(local_SD, weights_SK, indices_SK, self.w_gate_EDM, self.w_up_EDM,
                                             self.w_down_EMD, self.n_experts, self._ep_key)
        n_local = local_SD.shape[0]
        flat_ids = indices_SK.reshape(-1)
        flat_weights = weights_SK.reshape(-1)
        dest = torch.div(flat_ids, self.local_experts, rounding_mode="floor")
        order = torch.argsort(flat_ids, stable=True)  # grouped by destination rank, then expert
        repeated_SD = local_SD.repeat_interleave(self.top_k, dim=0)
        input_splits = torch.bincount(dest, minlength=self.world_size)
        output_splits = exchange_counts(input_splits, "ep")
        # Expert ids travel with the rows so the receiver can group them.
        send_ids = flat_ids[order].to(local_SD.dtype).unsqueeze(-1)
        payload = torch.cat([repeated_SD[order], send_ids], dim=-1)
        received = _AllToAll.apply(payload, input_splits, output_splits, "ep")
        recv_SD, recv_ids = received[:, :-1], received[:, -1].detach().round().long() - self.expert_offset
        ones = torch.ones(recv_SD.shape[0], 1, device=recv_SD.device, dtype=recv_SD.dtype)
        expert_SD = _grouped_experts(recv_SD, ones, recv_ids.unsqueeze(-1), self.w_gate_EDM, self.w_up_EDM, self.w_down_EMD)
        returned_SD = _AllToAll.apply(expert_SD, output_splits, input_splits, "ep")
        inverse = torch.empty_like(order)
        inverse[order] = torch.arange(order.shape[0], device=order.device)
        restored_SD = returned_SD.index_select(0, inverse)
        weighted_SD = restored_SD * flat_weights.unsqueeze(-1)
        return weighted_SD.reshape(n_local, self.top_k, self.dim).sum(dim=1)
