"""MoE modules at ``abacus/moe/moe.py``."""
from abacus_b200.models.moe import MoE, MoEExpertParallel  # noqa: F401
