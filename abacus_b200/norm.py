"""RMSNorm at the reference path ``abacus/norm.py``."""
from abacus_b200.models.layers import RMSNorm

__all__ = ["RMSNorm"]
