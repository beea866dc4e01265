"""Data parallel (DDP, ZeRO-1/2/3) at ``abacus/distributed/data_parallel.py``."""
from abacus_b200.parallel.data_parallel import DataParallel, _FlatUnit  # noqa: F401
from abacus_b200.parallel.fused_data_parallel import FusedDataParallel  # noqa: F401,E402
from abacus_b200.parallel.fused_zero3 import FusedZero3  # noqa: F401,E402
