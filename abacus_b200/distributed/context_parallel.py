"""CP helpers at ``abacus/distributed/context_parallel.py``."""
from abacus_b200.parallel.context_parallel import (  # noqa: F401
    _AllGatherSequenceBlock,
    all_gather_positions,
    sum_parameter_gradients,
    zigzag_positions,
)
