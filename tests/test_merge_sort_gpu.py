"""DeviceMergeSort / DeviceMerge for named orders.

The reference's merge sort takes a comparator closure (device code); this
library takes the comparators such closures almost always are, by name
(rccl_b200.cub.Order).  A stable sort's output is fixed by its order, so the
expected output is numpy's stable argsort of each order's unsigned image:
ASCENDING/DESCENDING use the radix image (-0.0 == +0.0), TOTAL_* use Rust's
total_cmp image (-0.0 < +0.0, NaNs by sign and payload).  CPU tests cover the
host-side order handling; the rest need a GPU."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import NP_OF, bits, order_image, to_dev, to_host
from rccl_b200 import cub, thrust

TORCH_OF = {"uint32": torch.uint32, "int32": torch.int32, "float32": torch.float32,
            "uint64": torch.uint64, "int64": torch.int64, "float64": torch.float64}


def total_image(keys: np.ndarray, descending: bool) -> np.ndarray:
    """total_cmp order image (f32::total_cmp / f64::total_cmp): the float bit
    transform without the zero fold; integers as their natural order."""
    w = keys.dtype.itemsize * 8
    ut = np.uint32 if w == 32 else np.uint64
    u = np.ascontiguousarray(keys).view(ut)
    sign = ut(1 << (w - 1))
    if keys.dtype.kind == "f":
        o = np.where((u & sign) != 0, ~u, u ^ sign)
    elif keys.dtype.kind == "i":
        o = u ^ sign
    else:
        o = u.copy()
    if descending:
        o = ~o
    return o.astype(np.uint64)


def expected(keys, values, order):
    desc = order in (cub.Order.DESCENDING, cub.Order.TOTAL_DESCENDING)
    total = order in (cub.Order.TOTAL_ASCENDING, cub.Order.TOTAL_DESCENDING)
    img = total_image(keys, desc) if total else order_image(keys, desc)
    perm = np.argsort(img, kind="stable")
    return keys[perm], None if values is None else values[perm]


def gen(rng, dtype, n):
    if dtype in (np.float32, np.float64):
        x = rng.normal(0, 100, n).astype(dtype)
        x[rng.integers(0, n, max(1, n // 20))] = 0.0
        x[rng.integers(0, n, max(1, n // 20))] = -0.0
        specials = np.array([np.inf, -np.inf], dtype=dtype)
        x[rng.integers(0, n, max(1, n // 50))] = specials[rng.integers(0, 2, max(1, n // 50))]
        ut = np.uint32 if dtype == np.float32 else np.uint64
        nan_bits = np.array([0x7fc00001, 0xffc00002, 0x7f800003, 0xff800004], dtype=np.uint64)
        if dtype == np.float64:
            nan_bits = np.array([0x7ff8000000000001, 0xfff8000000000002, 0x7ff0000000000003,
                                 0xfff0000000000004], dtype=np.uint64)
        idx = rng.integers(0, n, max(1, n // 100))
        x.view(ut)[idx] = nan_bits.astype(ut)[rng.integers(0, 4, idx.size)]
        return x
    info = np.iinfo(dtype)
    return rng.integers(info.min // 2, info.max // 2, n, dtype=dtype)


ORDERS = list(cub.Order)
KEYS = ["uint32", "int32", "float32", "uint64", "int64", "float64"]


def test_order_codes_on_host():
    assert cub.order_code(cub.Order.TOTAL_DESCENDING) == 3
    assert cub.order_code("descending") == 1
    with pytest.raises(NotImplementedError):
        cub.order_code(lambda a, b: (a > b) - (a < b))
    with pytest.raises(cub.BadArgument):
        cub.order_code("sideways")


@pytest.mark.gpu
@pytest.mark.parametrize("kname", KEYS)
@pytest.mark.parametrize("order", ORDERS, ids=[o.name for o in ORDERS])
@pytest.mark.parametrize("n", [3000, 70_001])
def test_merge_sort_pairs_named_orders(kname, order, n):
    rng = np.random.default_rng(n + int(order))
    dt = NP_OF[kname]
    k = gen(rng, dt, n)
    v = np.arange(n, dtype=np.uint32)
    launch = cub.Program.load("cuda:0").on()
    dk, dv = to_dev(k), to_dev(v)
    ws = cub.device_merge_sort_pairs_workspace(launch, TORCH_OF[kname], torch.uint32, n)
    cub.device_merge_sort_pairs(launch, dk, dv, ws, order)
    cub.check_device_status(launch, ws.controls)
    ek, ev = expected(k, v, order)
    assert np.array_equal(bits(to_host(dk)), bits(ek))
    assert np.array_equal(to_host(dv), ev)


@pytest.mark.gpu
@pytest.mark.parametrize("kname", ["float32", "float64", "int64"])
@pytest.mark.parametrize("order", ORDERS, ids=[o.name for o in ORDERS])
def test_merge_sort_keys_and_thrust_sort_by(kname, order):
    rng = np.random.default_rng(int(order) * 7 + len(kname))
    dt = NP_OF[kname]
    n = 100_003
    k = gen(rng, dt, n)
    ek, _ = expected(k, None, order)
    launch = cub.Program.load("cuda:0").on()
    dk = to_dev(k)
    ws = cub.device_merge_sort_keys_workspace(launch, TORCH_OF[kname], n)
    cub.device_merge_sort_keys(launch, dk, ws, order)
    assert np.array_equal(bits(to_host(dk)), bits(ek))
    # Thrust: sort_by on a buffer and on with_values pairs
    execution = thrust.Program.load("cuda:0").par()
    dk2 = to_dev(k)
    thrust.sort_by(execution, dk2, order)
    assert np.array_equal(bits(to_host(dk2)), bits(ek))
    v = np.arange(n, dtype=np.int32)
    dk3, dv3 = to_dev(k), to_dev(v)
    thrust.with_values(dk3, dv3).sort_by(execution, order)
    ek3, ev3 = expected(k, v, order)
    assert np.array_equal(bits(to_host(dk3)), bits(ek3))
    assert np.array_equal(to_host(dv3), ev3)


@pytest.mark.gpu
def test_total_order_separates_zeros_and_nans():
    k = np.array([0.0, -0.0, 1.0, -0.0, 0.0, -1.0], dtype=np.float32)
    nan_bits = np.array([0x7fc00001, 0xffc00001, 0x7f800001, 0xff800001], dtype=np.uint32)
    k = np.concatenate([k, nan_bits.view(np.float32)])
    v = np.arange(k.size, dtype=np.uint32)
    launch = cub.Program.load("cuda:0").on()
    for order in ORDERS:
        dk, dv = to_dev(k), to_dev(v)
        ws = cub.device_merge_sort_pairs_workspace(launch, torch.float32, torch.uint32, k.size)
        cub.device_merge_sort_pairs(launch, dk, dv, ws, order)
        ek, ev = expected(k, v, order)
        assert np.array_equal(bits(to_host(dk)), bits(ek)), order
        assert np.array_equal(to_host(dv), ev), order
    # total order: -qNaN, -sNaN, -1, -0, -0, +0, +0, 1, +sNaN, +qNaN
    dk, dv = to_dev(k), to_dev(v)
    ws = cub.device_merge_sort_pairs_workspace(launch, torch.float32, torch.uint32, k.size)
    cub.device_merge_sort_pairs(launch, dk, dv, ws, cub.Order.TOTAL_ASCENDING)
    assert to_host(dv).tolist() == [7, 9, 5, 1, 3, 0, 4, 2, 8, 6]


@pytest.mark.gpu
@pytest.mark.parametrize("kname", ["uint32", "float32", "int64", "float64"])
@pytest.mark.parametrize("order", ORDERS, ids=[o.name for o in ORDERS])
@pytest.mark.parametrize("sizes", [(0, 1000), (1, 1), (5000, 70_000), (33_333, 12_345)])
def test_device_merge_named_orders(kname, order, sizes):
    rng = np.random.default_rng(sizes[0] + sizes[1] + int(order))
    dt = NP_OF[kname]
    na, nb = sizes
    a, b = gen(rng, dt, max(na, 1))[:na], gen(rng, dt, max(nb, 1))[:nb]
    a, _ = expected(a, None, order)
    b, _ = expected(b, None, order)
    av = np.arange(na, dtype=np.uint32)
    bv = np.arange(na, na + nb, dtype=np.uint32)
    launch = cub.Program.load("cuda:0").on()
    ws = cub.device_merge_workspace(launch, na, nb)
    ok = torch.empty(na + nb, dtype=TORCH_OF[kname], device="cuda")
    ov = torch.empty(na + nb, dtype=torch.uint32, device="cuda")
    cub.device_merge_pairs(launch, to_dev(a), to_dev(av), to_dev(b), to_dev(bv), ws, ok, ov, order)
    # a stable merge with ties taking `first` = the stable sort of a ++ b
    ek, ev = expected(np.concatenate([a, b]), np.concatenate([av, bv]), order)
    assert np.array_equal(bits(to_host(ok)), bits(ek))
    assert np.array_equal(to_host(ov), ev)
    ok2 = torch.empty(na + nb, dtype=TORCH_OF[kname], device="cuda")
    cub.device_merge_keys(launch, to_dev(a), to_dev(b), ws, ok2, order)
    assert np.array_equal(bits(to_host(ok2)), bits(ek))
