"""EP collectives at ``abacus/distributed/expert_parallel.py``."""
from abacus_b200.parallel.expert_parallel import (  # noqa: F401
    _AllToAll,
    _GatherTokenShards,
    _rank_and_world_size,
    _SumReplicatedGrads,
    exchange_counts,
    shard_counts,
)
