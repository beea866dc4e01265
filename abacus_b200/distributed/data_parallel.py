"""Data parallel (DDP, ZeRO-1/2/3) at ``abacus/distributed/data_parallel.py``."""
from abacus_b200.parallel.data_parallel import DataParallel, _Partition  # noqa: F401
