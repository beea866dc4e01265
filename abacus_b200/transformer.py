"""Dense models at the reference path ``abacus/transformer.py``."""
from abacus_b200.models.transformer import PipelineStage, Transformer, TransformerBlock

__all__ = ["PipelineStage", "Transformer", "TransformerBlock"]
