"""naylis_b200 — B200-native (sm_100a) Mixture-of-Memory hot path for Naylis.

Public surface:
  naylis_b200.mom_kernels   the dispatch door (preflight, resolve_mode, mom_read,
                            announce, and the added mom_route) for mode "sm100"
  naylis_b200.model.MoMLayer  drop-in MoM layer (reference constructor and keys)
  naylis_b200.data_parallel   explicit bucketed NCCL gradient all-reduce
  naylis_b200.build           in-tree nvcc build of libnaylis_mom.so
"""
from . import mom_kernels  # noqa: F401

__all__ = ["mom_kernels"]
