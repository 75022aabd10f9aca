"""rccl_b200: B200-native DeviceRadixSort (keys and stable pairs, six key types,
both directions) behind the C ABI of librsort_b200.so, plus a multi-GPU sample
sort over NCCL.

Modules:
  cub     -- rccl-cub DeviceRadixSort functions, workspaces and DoubleBuffer
  thrust  -- rccl-thrust sort()/sort_unstable()/with_values() radix lowering
  dist    -- multi-GPU sample sort (torch.distributed over NCCL)
  errors  -- DeviceAlgorithmError mirror
"""
from . import errors
from ._lib import LIB_PATH, lib

__all__ = ["errors", "lib", "LIB_PATH"]
