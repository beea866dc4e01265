"""WSD schedule at ``abacus/optimizers/lr_scheduler.py``."""
from abacus_b200.optim.lr_scheduler import WSD  # noqa: F401
