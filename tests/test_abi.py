"""CPU tests of the C ABI: the library loads, exports every declared symbol,
sizes the control regions and validates arguments exactly as the reference's
pass control does -- all without launching anything."""
import ctypes
import os
import re

import pytest

from rccl_b200 import _lib
from rccl_b200.errors import raise_for, InvalidBitRange, LengthMismatch, WorkspaceTooSmall

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "rsort_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(rsort_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert "rsort_keys_buffer" in names and "rsort_pairs" in names
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)


def q(key, vb, n):
    out = _lib.Controls()
    assert _lib.lib().rsort_controls_query(key, vb, n, ctypes.byref(out)) == 0
    return out.bins, out.lookback, out.counters


def test_controls_zero_on_single_tile_route():
    # rccl-cub/src/workspace.rs:96-106 and the 4,864 / 4,865 boundary test
    # (workspace.rs:776-806).
    assert q(_lib.RSORT_U32, 0, 4864) == (0, 0, 0)
    b, l, c = q(_lib.RSORT_U32, 0, 4865)
    assert b == 4 * 256 and l > 0 and c >= 8
    assert q(_lib.RSORT_U64, 0, 2304) == (0, 0, 0)
    assert q(_lib.RSORT_U64, 0, 2305)[0] == 8 * 256
    assert q(_lib.RSORT_U32, 8, 2304) == (0, 0, 0)
    assert q(_lib.RSORT_U32, 8, 2305) != (0, 0, 0)


def test_lookback_scales_with_tiles():
    # lookback = ceil(n / tile) * 256 words of 64 bits (512 i32)
    b1, l1, _ = q(_lib.RSORT_U32, 0, 1 << 20)
    b2, l2, _ = q(_lib.RSORT_U32, 0, 1 << 21)
    assert b1 == b2 and l1 % 512 == 0 and l2 % 512 == 0
    assert 2 * l1 - 512 <= l2 <= 2 * l1


def test_selector_flips_follow_reference_routes():
    f = _lib.lib().rsort_selector_flips
    assert f(_lib.RSORT_U32, 0, 0, 0, 32) == 0
    assert f(_lib.RSORT_U32, 0, 10, 12, 12) == 0
    assert f(_lib.RSORT_U32, 0, 4864, 0, 32) == 1
    assert f(_lib.RSORT_U32, 0, 4865, 0, 32) == 4
    assert f(_lib.RSORT_U32, 0, 10_003, 0, 24) == 3
    assert f(_lib.RSORT_U64, 4, 1 << 20, 0, 64) == 8
    assert _lib.lib().rsort_single_tile_items(_lib.RSORT_F64, 16) == 1024


def test_invalid_bit_range_leaves_selector():
    sel = ctypes.c_int(1)
    st = _lib.lib().rsort_keys_buffer(_lib.RSORT_U32, 0, 16, 32, 4, 25, 17, ctypes.byref(sel),
                                      None, 0, None, 0, None, 0, None)
    assert st == _lib.RSORT_INVALID_BIT_RANGE and sel.value == 1
    with pytest.raises(InvalidBitRange) as e:
        raise_for(st)
    assert (e.value.begin, e.value.end, e.value.key_bits) == (25, 17, 32)
    st = _lib.lib().rsort_keys_buffer(_lib.RSORT_U64, 0, 16, 32, 4, 0, 65, ctypes.byref(sel),
                                      None, 0, None, 0, None, 0, None)
    assert st == _lib.RSORT_INVALID_BIT_RANGE


def test_empty_input_and_empty_window_are_noops():
    sel = ctypes.c_int(1)
    lib = _lib.lib()
    assert lib.rsort_keys_buffer(_lib.RSORT_U32, 0, None, None, 0, 0, 32, ctypes.byref(sel),
                                 None, 0, None, 0, None, 0, None) == 0
    assert lib.rsort_keys_buffer(_lib.RSORT_U32, 0, 16, 32, 4, 12, 12, ctypes.byref(sel),
                                 None, 0, None, 0, None, 0, None) == 0
    assert sel.value == 1


def test_control_validation_errors():
    lib = _lib.lib()
    sel = ctypes.c_int(1)
    n = 100_000
    b, l, c = q(_lib.RSORT_U32, 0, n)
    st = lib.rsort_keys_buffer(_lib.RSORT_U32, 0, 256, 512, n, 0, 32, ctypes.byref(sel),
                               4096, b - 1, 8192, l, 65536, c, None)
    assert st == _lib.RSORT_WORKSPACE_TOO_SMALL
    with pytest.raises(WorkspaceTooSmall) as e:
        raise_for(st)
    assert e.value.role == "radix bins" and e.value.required == b
    st = lib.rsort_keys_buffer(_lib.RSORT_U32, 0, 256, 512, n, 0, 32, ctypes.byref(sel),
                               4096, b, 8192, l + 2, 65536, c, None)
    assert st == _lib.RSORT_LENGTH_MISMATCH
    with pytest.raises(LengthMismatch) as e:
        raise_for(st)
    assert e.value.role == "radix lookback" and e.value.expected == l
    st = lib.rsort_keys_buffer(_lib.RSORT_U32, 0, 256, 512, n, 0, 32, ctypes.byref(sel),
                               4096, b, 8192, l, 65536, c - 1, None)
    assert st == _lib.RSORT_WORKSPACE_TOO_SMALL
    assert sel.value == 1


def test_scratch_length_mismatch():
    st = _lib.lib().rsort_keys(_lib.RSORT_U32, 0, 256, 512, 9, 10, None, 0, None, 0, None, 0,
                               None)
    assert st == _lib.RSORT_LENGTH_MISMATCH
    with pytest.raises(LengthMismatch) as e:
        raise_for(st)
    assert e.value.role == "radix scratch keys"


def test_status_strings():
    for s in range(9):
        assert _lib.lib().rsort_status_string(s)
