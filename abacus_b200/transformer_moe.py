"""MoE model at the reference path ``abacus/transformer_moe.py``."""
from abacus_b200.models.transformer_moe import TransformerBlockMoe, TransformerMoe

__all__ = ["TransformerBlockMoe", "TransformerMoe"]
