"""Attention modules at the reference path ``abacus/attention.py``."""
from abacus_b200.models.attention import MultiHeadAttention, ScaledDotProductAttention, _later_than_query

__all__ = ["MultiHeadAttention", "ScaledDotProductAttention", "_later_than_query"]
