"""numpy front end of the CPU oracle (oracle/radix_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  The product path never imports
it.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Tuple

import numpy as np

from . import build as _build  # noqa: F401  (package-relative when imported as oracle.pyoracle)

U32, I32, F32, U64, I64, F64 = range(6)
NP_KEY = {U32: np.uint32, I32: np.int32, F32: np.float32, U64: np.uint64, I64: np.int64,
          F64: np.float64}
BITS_VIEW = {U32: np.uint32, I32: np.uint32, F32: np.uint32, U64: np.uint64, I64: np.uint64,
             F64: np.uint64}
KEY_OF_DTYPE = {np.dtype(v): k for k, v in NP_KEY.items()}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        h = ctypes.CDLL(path)
        vp, sz, u, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint, ctypes.c_int
        u64 = ctypes.c_uint64
        h.orc_to_ordered.argtypes = [i, i, u64]
        h.orc_to_ordered.restype = u64
        h.orc_from_ordered.argtypes = [i, i, u64]
        h.orc_from_ordered.restype = u64
        h.orc_fold.argtypes = [i, u64]
        h.orc_fold.restype = u64
        h.orc_single_tile_items.argtypes = [u, u]
        h.orc_single_tile_items.restype = sz
        h.orc_sort_key.argtypes = [i, i, u, u, i, u64]
        h.orc_sort_key.restype = u64
        h.orc_radix_sort.argtypes = [i, i, vp, vp, sz, u, u, u, i, ctypes.POINTER(ctypes.c_int)]
        h.orc_radix_sort.restype = i
        h.orc_stable_order.argtypes = [vp, sz, u, i, vp]
        h.orc_stable_order.restype = None
        h.orc_sample_partition.argtypes = [i, i, vp, vp, i, u, i, vp]
        h.orc_sample_partition.restype = i
        h.orc_cpu_sort.argtypes = [i, i, i, vp, vp, sz, i]
        h.orc_cpu_sort.restype = i
        _lib = h
    return _lib


def key_type_of(arr: np.ndarray) -> int:
    return KEY_OF_DTYPE[arr.dtype]


def to_ordered(key_type: int, descending: bool, raw: int) -> int:
    return lib().orc_to_ordered(key_type, int(descending), raw)


def from_ordered(key_type: int, descending: bool, ordered: int) -> int:
    return lib().orc_from_ordered(key_type, int(descending), ordered)


def fold(key_type: int, ordered: int) -> int:
    return lib().orc_fold(key_type, ordered)


def single_tile_items(key_bytes: int, value_bytes: int = 0) -> int:
    return lib().orc_single_tile_items(key_bytes, value_bytes)


def radix_sort(keys: np.ndarray, values: Optional[np.ndarray] = None, descending: bool = False,
               bit_range: Optional[Tuple[int, int]] = None, threads: int = 1,
               key_type: Optional[int] = None):
    """Return (sorted keys, sorted values or None, selector flips, status).

    Inputs are not modified.  `values` may be any 1-D array or a 2-D uint8
    array of (n, width) rows."""
    kt = key_type_of(keys) if key_type is None else key_type
    bits = 32 if kt < U64 else 64
    begin, end = (0, bits) if bit_range is None else bit_range
    k = np.ascontiguousarray(keys).copy()
    v = None
    vb = 0
    if values is not None:
        v = np.ascontiguousarray(values).copy()
        vb = v.dtype.itemsize * (v.shape[1] if v.ndim == 2 else 1)
    swaps = ctypes.c_int(0)
    st = lib().orc_radix_sort(kt, int(descending), k.ctypes.data, None if v is None else v.ctypes.data,
                              k.shape[0], vb, begin, end, threads, ctypes.byref(swaps))
    return k, v, swaps.value, st


def sample_partition(keys: np.ndarray, shard_sizes, samples_per_rank: int,
                     descending: bool = False, threads: int = 1) -> np.ndarray:
    kt = key_type_of(keys)
    k = np.ascontiguousarray(keys)
    sizes = np.asarray(shard_sizes, dtype=np.uint64)
    out = np.zeros(len(sizes), dtype=np.uint64)
    st = lib().orc_sample_partition(kt, int(descending), k.ctypes.data, sizes.ctypes.data,
                                    len(sizes), samples_per_rank, threads, out.ctypes.data)
    if st != 0:
        raise ValueError(f"oracle sample partition failed: {st}")
    return out


def cpu_sort(keys: np.ndarray, values: Optional[np.ndarray] = None, descending: bool = False,
             stable: bool = False, threads: int = 1):
    """The CPU baseline stand-ins (std::sort / std::stable_sort, chunked over
    `threads` threads).  Returns sorted copies (keys, values or None)."""
    kt = key_type_of(keys)
    k = np.ascontiguousarray(keys).copy()
    v = None if values is None else np.ascontiguousarray(values, dtype=np.uint32).copy()
    st = lib().orc_cpu_sort(kt, int(descending), int(stable), k.ctypes.data,
                            None if v is None else v.ctypes.data, k.shape[0], threads)
    if st != 0:
        raise ValueError(f"cpu sort failed: {st}")
    return k, v


def bits_of(arr: np.ndarray) -> np.ndarray:
    """Raw bit pattern view (for bit-exact float comparisons)."""
    return arr.view(BITS_VIEW[key_type_of(arr)])
