"""Process-group helpers at ``abacus/distributed/utils.py``."""
from abacus_b200.utils.dist import dist_env_vars, init_process_group, print_peak_memory, rank, shutdown, world_size

__all__ = ["dist_env_vars", "init_process_group", "print_peak_memory", "rank", "shutdown", "world_size"]
