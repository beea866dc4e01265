"""abacus_b200: a Blackwell (B200, sm_100a) native Transformer training framework.

Public modules mirror the reference framework's import paths
(``abacus_b200.transformer``, ``abacus_b200.trainer``,
``abacus_b200.distributed.data_parallel``, ...). Implementations live in
``models/`` (layers and models), ``ops/`` (the sm_100a kernels and their
autograd functions), ``parallel/`` (mesh, collectives, DP/TP/CP/EP/PP),
``optim/`` and ``utils/``.
"""

__version__ = "0.1.0"
