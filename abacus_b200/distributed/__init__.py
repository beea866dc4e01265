"""Parallelism at the reference path ``abacus/distributed``."""
