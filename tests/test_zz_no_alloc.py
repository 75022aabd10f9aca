"""The allocation-free entry point rsort_keys_static, called through the C ABI.

It exists for callers that cannot allocate device memory where they sort:
code recording a CUDA graph by stream capture (cudaMalloc is not allowed
while capturing), plugins whose host framework owns all device memory through
its own pool, and latency-critical loops.  Its scratch is one static device
array inside the library, shared by every call on a device.

The tests compare its output bit-exactly with the CPU oracle and with the
regular rsort_keys entry point (which takes caller-owned scratch) on two calls
in a row, so the second call runs on the leftovers of the first.  This file is
named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import pyoracle
from rccl_b200 import _lib, cub

pytestmark = pytest.mark.gpu

MAX_ITEMS = 1 << 20


def regular_sort(keys_np, descending):
    launch = cub.Program.load("cuda:0").on()
    t = torch.from_numpy(keys_np.copy()).cuda()
    ws = cub.device_radix_sort_workspace(launch, t.dtype, t.numel())
    (cub.device_radix_sort_keys_descending if descending else cub.device_radix_sort_keys)(
        launch, t, ws)
    torch.cuda.synchronize()
    return t.cpu().numpy()


def static_sort(keys_np, descending):
    t = torch.from_numpy(keys_np.copy()).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    st = _lib.lib().rsort_keys_static(cub.key_code(t.dtype), int(descending), t.data_ptr(),
                                      t.numel(), stream)
    assert st == _lib.RSORT_OK, _lib.lib().rsort_status_string(st)
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    return a.view(np.uint32 if a.dtype.itemsize == 4 else np.uint64)


def oracle_sort(keys_np, descending):
    out, _, _, st = pyoracle.radix_sort(keys_np, None, descending, threads=4)
    assert st == 0
    return out


def test_static_entry_point_matches_regular_sort_twice():
    rng = np.random.default_rng(77)
    # Two calls in a row on the shared static scratch: first a large u64
    # descending sort, then a u32 ascending sort of a different size.
    first = rng.integers(0, 2**64, MAX_ITEMS, dtype=np.uint64)
    second = rng.integers(0, 2**32, 300_001, dtype=np.uint64).astype(np.uint32)
    got1 = static_sort(first, True)
    got2 = static_sort(second, False)
    assert np.array_equal(got1, oracle_sort(first, True))
    assert np.array_equal(got2, oracle_sort(second, False))
    assert np.array_equal(got1, regular_sort(first, True))
    assert np.array_equal(got2, regular_sort(second, False))


def test_static_entry_point_float_keys_and_small_inputs():
    rng = np.random.default_rng(5)
    f = rng.normal(0, 100, 200_003).astype(np.float32)
    f[::37] = -0.0
    f[::41] = 0.0
    f[::43] = np.nan
    for desc in (False, True):
        got = bits(static_sort(f, desc))
        assert np.array_equal(got, bits(oracle_sort(f, desc)))
        assert np.array_equal(got, bits(regular_sort(f, desc)))
    small = rng.integers(-50, 50, 4000, dtype=np.int64)
    assert np.array_equal(static_sort(small, False), oracle_sort(small, False))


def test_static_entry_point_rejects_oversized_input():
    t = torch.zeros(MAX_ITEMS + 1, dtype=torch.uint32, device="cuda")
    st = _lib.lib().rsort_keys_static(_lib.RSORT_U32, 0, t.data_ptr(), t.numel(),
                                      torch.cuda.current_stream().cuda_stream)
    assert st == _lib.RSORT_WORKSPACE_TOO_SMALL
    err = _lib.last_error()
    assert err.status == _lib.RSORT_WORKSPACE_TOO_SMALL
    assert err.expected == MAX_ITEMS and err.actual == MAX_ITEMS + 1
