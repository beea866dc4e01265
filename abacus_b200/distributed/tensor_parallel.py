"""TP / SP collectives at ``abacus/distributed/tensor_parallel.py``."""
from abacus_b200.parallel.tensor_parallel import (  # noqa: F401
    _AllReduceGrads,
    _GatherFromSequenceParallel,
    _GatherReplicated,
    _rank_and_world_size,
    _ReduceScatterToSequenceParallel,
    _ScatterToSequenceParallel,
    _SumOutputs,
)
