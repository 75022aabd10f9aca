"""ctypes binding of librsort_b200.so (the C ABI declared in include/rsort_b200.h).

The shared library is the only compute path: if it is missing, loading fails
loudly instead of falling back to any CPU or library sort.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
LIB_PATH = os.path.join(LIB_DIR, "librsort_b200.so")

# rsort_key_t
RSORT_U32, RSORT_I32, RSORT_F32, RSORT_U64, RSORT_I64, RSORT_F64 = range(6)
# small keys (no reference counterpart)
RSORT_U8, RSORT_I8, RSORT_U16, RSORT_I16, RSORT_F16, RSORT_BF16 = range(6, 12)

# rsort_status
RSORT_OK = 0
RSORT_INVALID_BIT_RANGE = 1
RSORT_LENGTH_MISMATCH = 2
RSORT_WORKSPACE_TOO_SMALL = 3
RSORT_UNSUPPORTED_TARGET = 4
RSORT_SIZE_OVERFLOW = 5
RSORT_CUDA_ERROR = 6
RSORT_TIMEOUT = 7
RSORT_BAD_ARGUMENT = 8

# kernel ids of rsort_profile_read
KERNEL_NAMES = {0: "init", 1: "histogram", 2: "onesweep", 3: "single_tile", 4: "dist",
                5: "merge", 6: "gather", 7: "records", 8: "onesweep_runs"}
IPC_HANDLE_BYTES = 64
GATHER_MAX_SEGMENTS = 64
MAX_ITEMS = 1 << 40  # RSORT_MAX_ITEMS

EXPORTED_SYMBOLS = (
    "rsort_controls_query",
    "rsort_keys_buffer",
    "rsort_pairs_buffer",
    "rsort_keys",
    "rsort_pairs",
    "rsort_check_device_status",
    "rsort_single_tile_items",
    "rsort_selector_flips",
    "rsort_status_string",
    "rsort_last_error",
    "rsort_launch_count",
    "rsort_launch_count_reset",
    "rsort_profile_enable",
    "rsort_profile_read",
    "rsort_dist_samples",
    "rsort_dist_splitters",
    "rsort_dist_bounds",
    "rsort_merge_partition_words",
    "rsort_merge",
    "rsort_merge_runs",
    "rsort_keys_static",
    "rsort_selftest_lookback_timeout",
    "rsort_ipc_export",
    "rsort_ipc_import",
    "rsort_ipc_release",
    "rsort_gather_segments",
    "rsort_merge_segments",
    "rsort_merge_sort_keys",
    "rsort_merge_sort_pairs",
    "rsort_merge_ordered",
    "rsort_rows_scratch_bytes",
    "rsort_rows_lexicographic",
    "rsort_segmented_scratch_bytes",
    "rsort_segmented_sort",
    "rsort_dist_scratch_bytes",
    "rsort_dist_pairs",
    "rsort_dist_pairs_rank",
    "rsort_multiway_scratch_bytes",
    "rsort_merge_multiway",
    "rsort_sort_by_scratch_bytes",
    "rsort_sort_by",
)

# rsort_exchange_t
RSORT_EXCHANGE_NCCL = 0
RSORT_EXCHANGE_PEER = 1


# rsort_projection_t and the comparator-program limit
RSORT_PROJ_IDENTITY, RSORT_PROJ_AND, RSORT_PROJ_SHR, RSORT_PROJ_DIV, RSORT_PROJ_REM = range(5)
RSORT_MAX_TERMS = 16


class CompareTerm(ctypes.Structure):
    """rsort_compare_term"""
    _fields_ = [("offset", ctypes.c_uint32), ("type", ctypes.c_int32),
                ("projection", ctypes.c_int32), ("order", ctypes.c_int32),
                ("operand", ctypes.c_int64)]


class Controls(ctypes.Structure):
    _fields_ = [("bins", ctypes.c_size_t), ("lookback", ctypes.c_size_t),
                ("counters", ctypes.c_size_t)]


class ErrorInfo(ctypes.Structure):
    _fields_ = [("status", ctypes.c_int), ("role", ctypes.c_char_p),
                ("expected", ctypes.c_size_t), ("actual", ctypes.c_size_t),
                ("begin_bit", ctypes.c_uint), ("end_bit", ctypes.c_uint),
                ("key_bits", ctypes.c_uint)]


_lock = threading.Lock()
_lib = None


def _declare(lib: ctypes.CDLL) -> None:
    vp, sz, u, i, pi = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint, ctypes.c_int, ctypes.POINTER(ctypes.c_int)
    lib.rsort_controls_query.argtypes = [i, sz, sz, ctypes.POINTER(Controls)]
    lib.rsort_controls_query.restype = i
    lib.rsort_keys_buffer.argtypes = [i, i, vp, vp, sz, u, u, pi, vp, sz, vp, sz, vp, sz, vp]
    lib.rsort_keys_buffer.restype = i
    lib.rsort_pairs_buffer.argtypes = [i, i, vp, vp, vp, vp, sz, sz, u, u, pi, vp, sz, vp, sz,
                                       vp, sz, vp]
    lib.rsort_pairs_buffer.restype = i
    lib.rsort_keys.argtypes = [i, i, vp, vp, sz, sz, vp, sz, vp, sz, vp, sz, vp]
    lib.rsort_keys.restype = i
    lib.rsort_pairs.argtypes = [i, i, vp, vp, sz, vp, sz, vp, sz, sz, vp, sz, vp, sz, vp, sz, vp]
    lib.rsort_pairs.restype = i
    lib.rsort_check_device_status.argtypes = [vp, sz, vp]
    lib.rsort_check_device_status.restype = i
    lib.rsort_single_tile_items.argtypes = [i, sz]
    lib.rsort_single_tile_items.restype = sz
    lib.rsort_selector_flips.argtypes = [i, sz, sz, u, u]
    lib.rsort_selector_flips.restype = i
    lib.rsort_status_string.argtypes = [i]
    lib.rsort_status_string.restype = ctypes.c_char_p
    lib.rsort_last_error.argtypes = [ctypes.POINTER(ErrorInfo)]
    lib.rsort_last_error.restype = None
    lib.rsort_launch_count.argtypes = []
    lib.rsort_launch_count.restype = ctypes.c_uint64
    lib.rsort_launch_count_reset.argtypes = []
    lib.rsort_launch_count_reset.restype = None
    lib.rsort_profile_enable.argtypes = [i]
    lib.rsort_profile_enable.restype = None
    lib.rsort_profile_read.argtypes = [ctypes.POINTER(ctypes.c_int32),
                                       ctypes.POINTER(ctypes.c_float), sz]
    lib.rsort_profile_read.restype = sz
    lib.rsort_dist_samples.argtypes = [i, i, vp, sz, u, u, vp, vp]
    lib.rsort_dist_samples.restype = i
    lib.rsort_dist_splitters.argtypes = [vp, sz, u, vp, vp]
    lib.rsort_dist_splitters.restype = i
    lib.rsort_dist_bounds.argtypes = [i, i, vp, sz, u, vp, u, vp, vp]
    lib.rsort_dist_bounds.restype = i
    lib.rsort_merge_partition_words.argtypes = [sz]
    lib.rsort_merge_partition_words.restype = sz
    lib.rsort_merge.argtypes = [i, i, vp, vp, sz, vp, vp, sz, vp, vp, sz, vp, sz, vp]
    lib.rsort_merge.restype = i
    lib.rsort_merge_runs.argtypes = [i, i, vp, vp, sz, ctypes.POINTER(sz), u, vp, vp, vp, sz, pi,
                                     vp]
    lib.rsort_merge_runs.restype = i
    lib.rsort_keys_static.argtypes = [i, i, vp, sz, vp]
    lib.rsort_keys_static.restype = i
    lib.rsort_selftest_lookback_timeout.argtypes = [vp]
    lib.rsort_selftest_lookback_timeout.restype = i
    lib.rsort_ipc_export.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_uint64)]
    lib.rsort_ipc_export.restype = i
    lib.rsort_ipc_import.argtypes = [vp, ctypes.POINTER(vp)]
    lib.rsort_ipc_import.restype = i
    lib.rsort_ipc_release.argtypes = [vp]
    lib.rsort_ipc_release.restype = i
    lib.rsort_gather_segments.argtypes = [u, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_uint64),
                                          vp, vp]
    lib.rsort_gather_segments.restype = i
    lib.rsort_merge_segments.argtypes = [i, i, u, ctypes.POINTER(vp), ctypes.POINTER(vp),
                                         ctypes.POINTER(sz), sz, vp, vp, vp, vp, vp, sz, pi, u,
                                         vp]
    lib.rsort_merge_segments.restype = i
    lib.rsort_merge_sort_keys.argtypes = [i, i, vp, vp, sz, sz, vp, sz, vp, sz, vp, sz, vp]
    lib.rsort_merge_sort_keys.restype = i
    lib.rsort_merge_sort_pairs.argtypes = [i, i, vp, vp, sz, vp, sz, vp, sz, sz, vp, sz, vp, sz,
                                           vp, sz, vp]
    lib.rsort_merge_sort_pairs.restype = i
    lib.rsort_merge_ordered.argtypes = [i, i, vp, vp, sz, vp, vp, sz, vp, vp, sz, vp, sz, vp]
    lib.rsort_merge_ordered.restype = i
    lib.rsort_rows_scratch_bytes.argtypes = [sz, sz, sz]
    lib.rsort_rows_scratch_bytes.restype = sz
    lib.rsort_rows_lexicographic.argtypes = [sz, vp, vp, sz, sz, vp, sz, vp]
    lib.rsort_rows_lexicographic.restype = i
    lib.rsort_sort_by_scratch_bytes.argtypes = [sz, sz, sz]
    lib.rsort_sort_by_scratch_bytes.restype = sz
    lib.rsort_sort_by.argtypes = [ctypes.POINTER(CompareTerm), sz, vp, sz, vp, sz, sz, vp, sz, vp]
    lib.rsort_sort_by.restype = i
    lib.rsort_segmented_scratch_bytes.argtypes = [i, sz, sz, sz]
    lib.rsort_segmented_scratch_bytes.restype = sz
    lib.rsort_segmented_sort.argtypes = [i, i, vp, vp, vp, vp, sz, sz, sz, vp, vp, u, u, vp, sz,
                                         vp]
    lib.rsort_segmented_sort.restype = i
    lib.rsort_dist_scratch_bytes.argtypes = [i, sz, sz, sz, u]
    lib.rsort_dist_scratch_bytes.restype = sz
    pvp = ctypes.POINTER(vp)
    psz = ctypes.POINTER(sz)
    lib.rsort_dist_pairs.argtypes = [i, i, sz, i, ctypes.POINTER(i), pvp, pvp, pvp, pvp, psz, pvp,
                                     pvp, psz, pvp, psz, i, psz]
    lib.rsort_dist_pairs.restype = i
    lib.rsort_dist_pairs_rank.argtypes = [i, i, sz, i, i, vp, vp, vp, vp, sz, vp, vp, sz, vp, sz,
                                          psz]
    lib.rsort_dist_pairs_rank.restype = i
    lib.rsort_multiway_scratch_bytes.argtypes = [i, sz, u, sz]
    lib.rsort_multiway_scratch_bytes.restype = sz
    lib.rsort_merge_multiway.argtypes = [i, i, u, pvp, pvp, psz, sz, vp, vp, vp, sz, vp]
    lib.rsort_merge_multiway.restype = i


def lib() -> ctypes.CDLL:
    """Load librsort_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with "
                        "`python -c 'import __graft_entry__ as g; g.build()'` "
                        "(there is no fallback sort)")
                handle = ctypes.CDLL(LIB_PATH)
                _declare(handle)
                _lib = handle
    return _lib


def last_error() -> ErrorInfo:
    info = ErrorInfo()
    lib().rsort_last_error(ctypes.byref(info))
    return info
