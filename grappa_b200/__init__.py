"""grappa_b200: distributed GNN training for B200 (sm_100a) nodes.

Each GPU trains its own graph partition in isolation; accuracy lost by the
isolation is recovered with periodic repartitioning and coverage-corrected
gradient aggregation (the Grappa algorithm).  The data plane is resident in HBM
and runs on hand-written sm_100a kernels: neighbour sampling, block compaction,
aggregation, tcgen05 GEMMs, a fused all-reduce + Adam over NVLink peer memory and
a peer-memory repartition exchange.
"""
__version__ = "0.1.0"

from grappa_b200._native import cuda, cuda_available, host  # noqa: F401
