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


def _last_role():
    return _lib.last_error().role or b""


def test_misaligned_buffers_rejected_before_any_launch():
    """Keys, values and merge inputs must be aligned to their element size:
    the kernels move whole elements, and a misaligned address would fault the
    GPU.  Every entry point rejects one on the host (the addresses here are
    never dereferenced)."""
    n = 100_000
    c = _lib.Controls()
    assert L.rsort_controls_query(_lib.RSORT_U64, 0, n, ctypes.byref(c)) == 0
    st = L.rsort_keys(_lib.RSORT_U64, 0, 0x10004, 0x200000, n, n, 0x300000, c.bins, 0x400000,
                      c.lookback, 0x500000, c.counters, None)
    assert st == _lib.RSORT_BAD_ARGUMENT
    err = _lib.last_error()
    assert b"alignment" in err.role and err.expected == 8 and err.actual == 4
    # the single-tile route checks too
    st = L.rsort_keys(_lib.RSORT_F32, 0, 0x10002, 0x200000, 100, 100, None, 0, None, 0, None, 0,
                      None)
    assert st == _lib.RSORT_BAD_ARGUMENT and b"keys alignment" in _last_role()
    assert L.rsort_controls_query(_lib.RSORT_U32, 8, n, ctypes.byref(c)) == 0
    st = L.rsort_pairs(_lib.RSORT_U32, 0, 0x10000, 0x20004, 8, 0x200000, n, 0x300000, n, n,
                       0x400000, c.bins, 0x500000, c.lookback, 0x600000, c.counters, None)
    assert st == _lib.RSORT_BAD_ARGUMENT and b"values alignment" in _last_role()
    st = L.rsort_merge(_lib.RSORT_U64, 0, 0x10004, None, 10, 0x20000, None, 10, 0x30000, None, 0,
                       0x40000, 1000, None)
    assert st == _lib.RSORT_BAD_ARGUMENT and b"merge keys alignment" in _last_role()
    st = L.rsort_rows_lexicographic(3, 0x10002, None, 0, 1000, 0x100000,
                                    L.rsort_rows_scratch_bytes(3, 0, 1000), None)
    assert st == _lib.RSORT_BAD_ARGUMENT and b"rows alignment" in _last_role()
    st = L.rsort_dist_samples(_lib.RSORT_U64, 0, 0x10004, 1000, 0, 4, 0x20000, None)
    assert st == _lib.RSORT_BAD_ARGUMENT


def test_scratch_blobs_must_be_256_byte_aligned():
    n, nseg = 10_000, 4
    need = L.rsort_segmented_scratch_bytes(_lib.RSORT_U32, 0, n, nseg)
    st = L.rsort_segmented_sort(_lib.RSORT_U32, 0, 0x10000, 0x20000, None, None, 0, n, nseg,
                                0x30000, 0x40000, 0, 32, 0x100040, need, None)
    assert st == _lib.RSORT_BAD_ARGUMENT
    err = _lib.last_error()
    assert b"scratch alignment" in err.role and err.expected == 256 and err.actual == 0x40
    need = L.rsort_rows_scratch_bytes(3, 0, 1000)
    st = L.rsort_rows_lexicographic(3, 0x10000, None, 0, 1000, 0x100008, need, None)
    assert st == _lib.RSORT_BAD_ARGUMENT and b"scratch alignment" in _last_role()
    term = (_lib.CompareTerm * 1)()
    term[0].offset, term[0].type, term[0].projection, term[0].order, term[0].operand = (
        0, _lib.RSORT_U32, _lib.RSORT_PROJ_IDENTITY, 0, 0)
    need = L.rsort_sort_by_scratch_bytes(8, 0, 1000)
    st = L.rsort_sort_by(term, 1, 0x10000, 8, None, 0, 1000, 0x100010, need, None)
    assert st == _lib.RSORT_BAD_ARGUMENT and b"scratch alignment" in _last_role()


def test_item_count_and_scratch_size_limits():
    c = _lib.Controls()
    big = _lib.MAX_ITEMS + 1
    assert L.rsort_controls_query(_lib.RSORT_U32, 0, big, ctypes.byref(c)) == (
        _lib.RSORT_SIZE_OVERFLOW)
    assert L.rsort_controls_query(_lib.RSORT_U32, 0, _lib.MAX_ITEMS, ctypes.byref(c)) == 0
    st = L.rsort_keys(_lib.RSORT_U32, 0, 0x10000, 0x20000, big, big, 0x30000, 1024, 0x40000, 16,
                      0x50000, 16, None)
    assert st == _lib.RSORT_SIZE_OVERFLOW
    # scratch regions that would wrap a size_t size as 0 (no valid layout)
    assert L.rsort_sort_by_scratch_bytes(1 << 30, 0, 1 << 30) == 0
    assert L.rsort_rows_scratch_bytes(3, 1 << 40, 1 << 20) == 0
