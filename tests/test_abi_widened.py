"""CPU tests of the widened C ABI: argument validation and sizing of the
named-order merge sort, small keys, the segmented and record sorts and the
exchange entry points.  Every call here is rejected or sized on the host
before any device work, so no GPU is needed."""
import ctypes

from rccl_b200 import _lib

L = _lib.lib()
vp = ctypes.c_void_p


def test_merge_sort_rejects_unknown_order():
    st = L.rsort_merge_sort_keys(_lib.RSORT_U32, 7, 4096, 8192, 10, 10, None, 0, None, 0, None,
                                 0, None)
    assert st == _lib.RSORT_BAD_ARGUMENT
    st = L.rsort_merge_ordered(_lib.RSORT_U32, -1, 16, None, 1, 32, None, 1, 64, None, 0, 4096,
                               8, None)
    assert st == _lib.RSORT_BAD_ARGUMENT


def test_small_keys_rejected_by_distributed_steps_and_merges():
    for key in (_lib.RSORT_U8, _lib.RSORT_I16, _lib.RSORT_F16, _lib.RSORT_BF16):
        assert L.rsort_dist_samples(key, 0, 16, 100, 0, 4, 64, None) == _lib.RSORT_BAD_ARGUMENT
        assert L.rsort_merge(key, 0, 16, None, 1, 32, None, 1, 64, None, 0, 4096, 8,
                             None) == _lib.RSORT_BAD_ARGUMENT
        assert L.rsort_keys_static(key, 0, 16, 100, None) == _lib.RSORT_BAD_ARGUMENT


def test_small_key_controls_and_routes():
    out = _lib.Controls()
    assert L.rsort_controls_query(_lib.RSORT_U16, 0, 1 << 20, ctypes.byref(out)) == 0
    assert out.bins == 2 * 256 and out.lookback > 0 and out.counters >= 10
    assert L.rsort_controls_query(_lib.RSORT_U8, 0, 1 << 20, ctypes.byref(out)) == 0
    assert out.bins == 1 * 256
    # small keys take the 4-byte single-tile extent
    assert L.rsort_single_tile_items(_lib.RSORT_U16, 0) == L.rsort_single_tile_items(
        _lib.RSORT_U32, 0)
    assert L.rsort_selector_flips(_lib.RSORT_I8, 0, 1 << 20, 0, 8) == 1
    assert L.rsort_selector_flips(_lib.RSORT_BF16, 0, 1 << 20, 0, 16) == 2
    assert L.rsort_selector_flips(_lib.RSORT_U16, 0, 1 << 20, 0, 17) == 0  # invalid window


def test_record_sort_sizing_and_validation():
    small = L.rsort_rows_scratch_bytes(3, 8, 1000)
    big = L.rsort_rows_scratch_bytes(3, 8, 100_000)
    assert 0 < small < big
    assert L.rsort_rows_scratch_bytes(6, 0, 100_000) > L.rsort_rows_scratch_bytes(2, 0, 100_000)
    # n <= 1 and zero-width rows are no-ops
    assert L.rsort_rows_lexicographic(3, None, None, 0, 1, None, 0, None) == _lib.RSORT_OK
    assert L.rsort_rows_lexicographic(0, None, None, 0, 100, None, 0, None) == _lib.RSORT_OK
    no_payload = L.rsort_rows_scratch_bytes(3, 0, 1000)
    st = L.rsort_rows_lexicographic(3, 4096, None, 0, 1000, 8192, no_payload - 1, None)
    assert st == _lib.RSORT_WORKSPACE_TOO_SMALL
    st = L.rsort_rows_lexicographic(3, 4096, None, 8, 1000, 8192, small, None)
    assert st == _lib.RSORT_BAD_ARGUMENT  # payload bytes without a payload pointer


def test_segmented_sort_validation():
    n, nseg = 10_000, 4
    need = L.rsort_segmented_scratch_bytes(_lib.RSORT_U32, 4, n, nseg)
    assert need > L.rsort_segmented_scratch_bytes(_lib.RSORT_U32, 0, n, nseg) > 0
    st = L.rsort_segmented_sort(_lib.RSORT_U32, 0, 4096, 8192, None, None, 0, n, nseg, 16, 32,
                                20, 12, 65536, need, None)
    assert st == _lib.RSORT_INVALID_BIT_RANGE
    st = L.rsort_segmented_sort(_lib.RSORT_U32, 0, 4096, 8192, None, None, 0, 0, nseg, 16, 32,
                                0, 32, None, 0, None)
    assert st == _lib.RSORT_OK  # nothing to sort
    st = L.rsort_segmented_sort(_lib.RSORT_U32, 0, 4096, 8192, None, None, 0, n, nseg, 16, 32,
                                0, 32, 65536, 16, None)
    assert st == _lib.RSORT_WORKSPACE_TOO_SMALL
    st = L.rsort_segmented_sort(_lib.RSORT_U32, 0, 4096, 8192, None, None, 3, n, nseg, 16, 32,
                                0, 32, 65536, need, None)
    assert st == _lib.RSORT_BAD_ARGUMENT  # value width 3
    # (the pointers above are never dereferenced: validation rejects first)


def test_exchange_entry_points_validate_arguments():
    n = _lib.GATHER_MAX_SEGMENTS + 1
    st = L.rsort_gather_segments(n, (vp * n)(), (ctypes.c_uint64 * n)(), 4096, None)
    assert st == _lib.RSORT_BAD_ARGUMENT
    assert L.rsort_gather_segments(0, None, None, None, None) == _lib.RSORT_OK
    assert L.rsort_ipc_export(None, None, None) == _lib.RSORT_BAD_ARGUMENT
    assert L.rsort_ipc_import(None, None) == _lib.RSORT_BAD_ARGUMENT
    assert L.rsort_ipc_release(None) == _lib.RSORT_BAD_ARGUMENT
    flag = ctypes.c_int(0)
    st = L.rsort_merge_segments(_lib.RSORT_U64, 0, 2, None, None, None, 4, None, None, None,
                                None, None, 0, ctypes.byref(flag), 0, None)
    assert st == _lib.RSORT_BAD_ARGUMENT


def test_static_entry_point_errors_set_last_error():
    """rsort_keys_static's argument errors are recorded like every other entry
    point's, before any device work."""
    n = (1 << 20) + 1
    assert L.rsort_keys_static(_lib.RSORT_U64, 0, 16, n, None) == _lib.RSORT_WORKSPACE_TOO_SMALL
    err = _lib.last_error()
    assert err.status == _lib.RSORT_WORKSPACE_TOO_SMALL
    assert err.expected == 1 << 20 and err.actual == n
    assert b"RSORT_STATIC_MAX_ITEMS" in err.role
    assert L.rsort_keys_static(_lib.RSORT_U8, 0, 16, 100, None) == _lib.RSORT_BAD_ARGUMENT
    assert _lib.last_error().status == _lib.RSORT_BAD_ARGUMENT
    assert L.rsort_keys_static(_lib.RSORT_U32, 0, None, 100, None) == _lib.RSORT_BAD_ARGUMENT
    assert b"null" in _lib.last_error().role
