"""GPipe at ``abacus/distributed/pipeline_parallel.py``."""
from abacus_b200.parallel.pipeline_parallel import PipelineParallel  # noqa: F401
