"""AdamW at ``abacus/optimizers/adamw.py``."""
from abacus_b200.optim.adamw import AdamW  # noqa: F401
