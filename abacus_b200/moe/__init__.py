"""Mixture of experts at the reference path ``abacus/moe``."""
