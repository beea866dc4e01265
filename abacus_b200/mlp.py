"""SwiGLU MLPs at the reference path ``abacus/mlp.py``."""
from abacus_b200.models.layers import MLP, MLPTensorParallel

__all__ = ["MLP", "MLPTensorParallel"]
