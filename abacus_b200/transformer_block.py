"""Blocks at the reference path ``abacus/transformer_block.py``."""
from abacus_b200.models.transformer import TransformerBlock
from abacus_b200.models.transformer_moe import TransformerBlockMoe

__all__ = ["TransformerBlock", "TransformerBlockMoe"]
