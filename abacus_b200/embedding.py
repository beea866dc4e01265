"""Embedding at the reference path ``abacus/embedding.py``."""
from abacus_b200.models.layers import Embedding

__all__ = ["Embedding"]
