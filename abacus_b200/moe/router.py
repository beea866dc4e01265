"""Router at ``abacus/moe/router.py``."""
from abacus_b200.models.moe import Router  # noqa: F401
