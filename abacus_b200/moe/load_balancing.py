"""Load-balancing loss at ``abacus/moe/load_balancing.py``."""
from abacus_b200.models.moe import load_balancing_loss  # noqa: F401
