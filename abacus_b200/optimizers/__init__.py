"""Optimizers at the reference path ``abacus/optimizers``."""
