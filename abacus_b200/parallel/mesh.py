"""Rank grid with one process group per parallel dimension.

The reference runs every collective on the implicit world group
(``abacus/distributed/tensor_parallel.py:5-8``), so its parallel modes cannot
be combined (``abacus/trainer.py:38-41``). Here each dimension owns a
sub-group, which is what TP x DP, CP x PP and EP + DP need.

Without an installed mesh every dimension resolves to the world group, which
reproduces the reference's single-mode behaviour exactly.

Rank layout (outermost to innermost): ``pp, dp, cp, tp``. Tensor parallel is
innermost so a TP group is a run of consecutive local ranks. Expert parallel
reuses the data-parallel ranks (experts are sharded across the replicas that
see different data), so ``ep`` must divide ``dp``.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass, field

import torch.distributed as dist

DIMS = ("pp", "dp", "cp", "tp")


@dataclass
class Mesh:
    pp: int = 1
    dp: int = 1
    cp: int = 1
    tp: int = 1
    ep: int = 1
    groups: dict = field(default_factory=dict, repr=False)
    ranks: dict = field(default_factory=dict, repr=False)

    @property
    def size(self) -> int:
        return self.pp * self.dp * self.cp * self.tp

    def shape(self) -> dict[str, int]:
        return {"pp": self.pp, "dp": self.dp, "cp": self.cp, "tp": self.tp}

    def coords(self, rank: int) -> dict[str, int]:
        out = {}
        for dim in reversed(DIMS):
            size = getattr(self, dim)
            out[dim] = rank % size
            rank //= size
        return out

    def rank_of(self, coords: dict[str, int]) -> int:
        rank = 0
        for dim in DIMS:
            rank = rank * getattr(self, dim) + coords.get(dim, 0)
        return rank

    def group_ranks(self, dim: str, rank: int) -> list[int]:
        """Ranks that share every coordinate with `rank` except `dim`."""
        if dim == "ep":
            dp_ranks = self.group_ranks("dp", rank)
            pos = dp_ranks.index(rank)
            start = (pos // self.ep) * self.ep
            return dp_ranks[start : start + self.ep]
        base = self.coords(rank)
        out = []
        for value in range(getattr(self, dim)):
            c = dict(base)
            c[dim] = value
            out.append(self.rank_of(c))
        return out


_MESH: Mesh | None = None


def init_mesh(pp: int = 1, dp: int = 1, cp: int = 1, tp: int = 1, ep: int = 1) -> Mesh:
    """Create every sub-group (collectively, on all ranks) and install the mesh."""
    global _MESH
    mesh = Mesh(pp=pp, dp=dp, cp=cp, tp=tp, ep=ep)
    world = dist.get_world_size() if dist.is_initialized() else 1
    if mesh.size != world:
        raise ValueError(f"mesh {mesh.shape()} has {mesh.size} ranks, world size is {world}")
    if ep > 1 and dp % ep != 0:
        raise ValueError(f"expert parallel {ep} must divide data parallel {dp}")
    me = dist.get_rank() if dist.is_initialized() else 0
    for dim in DIMS + ("ep",):
        # new_group is collective: every rank creates every group in the same order.
        seen = set()
        for r in range(mesh.size):
            ranks = tuple(mesh.group_ranks(dim, r))
            if ranks in seen:
                continue
            seen.add(ranks)
            group = None
            if dist.is_initialized() and len(ranks) > 1:
                group = dist.new_group(list(ranks)) if len(ranks) < world else dist.group.WORLD
            if me in ranks:
                mesh.groups[dim] = group
                mesh.ranks[dim] = list(ranks)
    _MESH = mesh
    return mesh


def set_mesh(mesh: Mesh | None) -> None:
    global _MESH
    _MESH = mesh


def get_mesh() -> Mesh | None:
    return _MESH


def group_for(dim: str):
    """Process group for `dim`; the world group when no mesh is installed."""
    if _MESH is None:
        return None
    return _MESH.groups.get(dim)


def rank_and_world_size(dim: str | None = None) -> tuple[int, int]:
    """(rank, size) within `dim`'s group; world rank/size without a mesh.

    Mirrors ``_rank_and_world_size`` (``abacus/distributed/tensor_parallel.py:5-8``):
    (0, 1) when no process group is initialized.
    """
    if not (dist.is_available() and dist.is_initialized()):
        return 0, 1
    if _MESH is None or dim is None:
        return dist.get_rank(), dist.get_world_size()
    ranks = _MESH.ranks.get(dim)
    if ranks is None or len(ranks) == 1:
        return 0, 1
    return ranks.index(dist.get_rank()), len(ranks)


def global_rank(dim: str, index: int) -> int:
    """World rank of member `index` of this rank's `dim` group."""
    if _MESH is None:
        return index
    return _MESH.ranks[dim][index]


def all_combinations(mesh: Mesh):
    return itertools.product(*(range(getattr(mesh, d)) for d in DIMS))
