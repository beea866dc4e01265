"""Kernel switches at the reference path ``abacus/kernels``."""
