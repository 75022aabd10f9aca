"""The whole-sort multi-GPU C entry points (rsort_dist_pairs,
rsort_dist_pairs_rank): exported, sized, and their argument checks, which run
before any device or NCCL call (CPU)."""
import ctypes

from rccl_b200 import _lib

L = _lib.lib()


def test_scratch_sizing():
    small = L.rsort_dist_scratch_bytes(_lib.RSORT_U64, 4, 1000, 1000, 2)
    big = L.rsort_dist_scratch_bytes(_lib.RSORT_U64, 4, 1 << 24, 1 << 24, 8)
    assert 0 < small < big
    # holds the sort scratch for max(n_local, capacity) items of key + value
    assert big >= (1 << 24) * 12
    assert L.rsort_dist_scratch_bytes(_lib.RSORT_U8, 0, 1000, 1000, 2) == 0
    assert L.rsort_dist_scratch_bytes(_lib.RSORT_U32, 3, 1000, 1000, 2) == 0
    assert L.rsort_dist_scratch_bytes(_lib.RSORT_U32, 0, 1000, 1000, 0) == 0


def test_multi_device_argument_checks():
    W = 2
    VP, SZ = ctypes.c_void_p * W, ctypes.c_size_t * W
    devs = (ctypes.c_int * W)(0, 1)
    n = SZ(10, 10)
    out = SZ()
    ptrs = VP(4096, 8192)

    def call(key=_lib.RSORT_U32, vb=0, world=W, comms=ptrs, exchange=0, keys=ptrs):
        return L.rsort_dist_pairs(key, 0, vb, world, devs, comms, ptrs, keys, None, n, ptrs, None,
                                  n, ptrs, SZ(1 << 30, 1 << 30), exchange, out)

    assert call(key=_lib.RSORT_I16) == _lib.RSORT_BAD_ARGUMENT
    assert b"key type" in _lib.last_error().role
    assert call(vb=3) == _lib.RSORT_BAD_ARGUMENT
    assert call(world=0) == _lib.RSORT_BAD_ARGUMENT
    assert call(world=65) == _lib.RSORT_BAD_ARGUMENT
    assert call(exchange=7) == _lib.RSORT_BAD_ARGUMENT
    assert call(comms=None) == _lib.RSORT_BAD_ARGUMENT
    assert b"null" in _lib.last_error().role
    # values requested (value_bytes 4) but no value arrays
    assert call(vb=4) == _lib.RSORT_BAD_ARGUMENT
    # a scratch that is not 256-byte aligned
    st = L.rsort_dist_pairs(_lib.RSORT_U32, 0, 0, W, devs, ptrs, ptrs, ptrs, None, n, ptrs, None,
                            n, VP(4096 + 8, 8192), SZ(1 << 30, 1 << 30), 0, out)
    assert st == _lib.RSORT_BAD_ARGUMENT and b"alignment" in _lib.last_error().role
    # a scratch that is too small reports the size it needs
    need = L.rsort_dist_scratch_bytes(_lib.RSORT_U32, 0, 10, 10, W)
    st = L.rsort_dist_pairs(_lib.RSORT_U32, 0, 0, W, devs, ptrs, ptrs, ptrs, None, n, ptrs, None,
                            n, ptrs, SZ(need - 1, need), 0, out)
    assert st == _lib.RSORT_WORKSPACE_TOO_SMALL
    err = _lib.last_error()
    assert err.expected == need and err.actual == need - 1


def test_rank_entry_argument_checks():
    out = ctypes.c_size_t()
    args = (4096, None, 10, 8192, None, 10, 1 << 20, 1 << 30, ctypes.byref(out))
    assert L.rsort_dist_pairs_rank(_lib.RSORT_U32, 0, 0, 2, 2, 1, None, *args) == \
        _lib.RSORT_BAD_ARGUMENT
    assert L.rsort_dist_pairs_rank(_lib.RSORT_U32, 0, 0, -1, 2, 1, None, *args) == \
        _lib.RSORT_BAD_ARGUMENT
    # no communicator
    assert L.rsort_dist_pairs_rank(_lib.RSORT_U32, 0, 0, 0, 2, None, None, *args) == \
        _lib.RSORT_BAD_ARGUMENT
