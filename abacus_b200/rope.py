"""Rotary embeddings at the reference path ``abacus/rope.py``."""
from abacus_b200.models.layers import Rotary, apply_rotary_pos_emb, rotate_half

__all__ = ["Rotary", "apply_rotary_pos_emb", "rotate_half"]
