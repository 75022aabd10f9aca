"""Small keys (no reference counterpart; rccl-cub lists them as missing):
u8/i8/u16/i16 and IEEE half / bfloat16, in the radix sorts and the
named-order sorts.  They follow the reference's ordering rules, so the
expected output is numpy's stable argsort of the same order image the 32- and
64-bit keys use: sign flip for integers; flip all bits of negative floats and
the sign bit of the others; descending = NOT; and the radix order folds -0.0
onto +0.0 (the total order does not)."""
import numpy as np
import pytest
import torch

from rccl_b200 import cub

pytestmark = pytest.mark.gpu

# name: (numpy storage dtype, torch dtype, kind)
SMALL = {
    "uint8": (np.uint8, torch.uint8, "u"),
    "int8": (np.int8, torch.int8, "i"),
    "uint16": (np.uint16, torch.uint16, "u"),
    "int16": (np.int16, torch.int16, "i"),
    "float16": (np.float16, torch.float16, "f"),
    "bfloat16": (np.uint16, torch.bfloat16, "f"),  # held as raw 16-bit patterns
}


def raw_bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint8 if a.dtype.itemsize == 1 else np.uint16)


def image(a: np.ndarray, kind: str, descending: bool, fold: bool = True) -> np.ndarray:
    u = raw_bits(a).astype(np.uint64)
    w = a.dtype.itemsize * 8
    full = (1 << w) - 1
    sign = 1 << (w - 1)
    if kind == "f":
        o = np.where((u & sign) != 0, ~u & full, u ^ sign)
    elif kind == "i":
        o = u ^ sign
    else:
        o = u
    if descending:
        o = ~o & full
    if kind == "f" and fold:
        o = np.where(o == sign - 1, sign, o)
    return o


def gen(rng, name, n):
    np_t, _, kind = SMALL[name]
    if kind == "f":
        if name == "float16":
            x = rng.normal(0, 30, n).astype(np.float16)
        else:  # bfloat16: the top half of float32 bit patterns
            x = (rng.normal(0, 30, n).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
        b = raw_bits(x)
        b[rng.integers(0, n, max(1, n // 20))] = 0x0000  # +0
        b[rng.integers(0, n, max(1, n // 20))] = 0x8000  # -0
        nans = np.array([0x7e01, 0xfe02, 0x7c03, 0xfc04] if name == "float16"
                        else [0x7fc1, 0xffc2, 0x7f83, 0xff84], dtype=np.uint16)
        b[rng.integers(0, n, max(1, n // 50))] = nans[rng.integers(0, 4, max(1, n // 50))]
        return x
    info = np.iinfo(np_t)
    return rng.integers(info.min, info.max, n, dtype=np_t, endpoint=True)


def to_dev(a, name):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.view(torch.bfloat16) if name == "bfloat16" else t


def to_host(t):
    if t.dtype == torch.bfloat16:
        t = t.view(torch.uint16)
    return t.cpu().numpy()


@pytest.mark.parametrize("name", list(SMALL))
@pytest.mark.parametrize("n", [1, 777, 4865, 70_001])
def test_small_keys_radix_keys_and_pairs(name, n):
    rng = np.random.default_rng(n * 3 + len(name))
    _, tdt, kind = SMALL[name]
    k = gen(rng, name, n)
    v = np.arange(n, dtype=np.uint32)
    launch = cub.Program.load("cuda:0").on()
    for desc in (False, True):
        perm = np.argsort(image(k, kind, desc), kind="stable")
        dk = to_dev(k, name)
        ws = cub.device_radix_sort_workspace(launch, tdt, n)
        (cub.device_radix_sort_keys_descending if desc else cub.device_radix_sort_keys)(
            launch, dk, ws)
        assert np.array_equal(raw_bits(to_host(dk)), raw_bits(k[perm])), (name, desc)
        dk, dv = to_dev(k, name), torch.from_numpy(v).cuda()
        wsp = cub.device_radix_sort_pairs_workspace(launch, tdt, torch.uint32, n)
        (cub.device_radix_sort_pairs_descending if desc else cub.device_radix_sort_pairs)(
            launch, dk, dv, wsp)
        cub.check_device_status(launch, wsp.controls)
        assert np.array_equal(raw_bits(to_host(dk)), raw_bits(k[perm])), (name, desc)
        assert np.array_equal(to_host(dv), v[perm]), (name, desc)


@pytest.mark.parametrize("name", ["uint16", "int16", "float16", "bfloat16"])
def test_small_keys_bit_window(name):
    rng = np.random.default_rng(9)
    _, tdt, kind = SMALL[name]
    n = 30_000
    k = gen(rng, name, n)
    launch = cub.Program.load("cuda:0").on()
    for begin, end in [(0, 8), (3, 14), (8, 16)]:
        for desc in (False, True):
            img = image(k, kind, desc)
            # the onesweep route orders by the digits of the window of the
            # (descending) image
            mask = (1 << (end - begin)) - 1
            perm = np.argsort((img >> begin) & mask, kind="stable")
            first, second = to_dev(k, name), torch.zeros_like(to_dev(k, name))
            buffers = cub.DoubleBuffer.new(first, second)
            ws = cub.device_radix_sort_keys_buffer_workspace(launch, tdt, n)
            (cub.device_radix_sort_keys_buffer_descending if desc
             else cub.device_radix_sort_keys_buffer)(launch, buffers, range(begin, end), ws)
            assert np.array_equal(raw_bits(to_host(buffers.current())), raw_bits(k[perm])), \
                (name, begin, end, desc)


@pytest.mark.parametrize("name", ["float16", "bfloat16", "int8"])
@pytest.mark.parametrize("order", list(cub.Order), ids=[o.name for o in cub.Order])
def test_small_keys_named_orders(name, order):
    rng = np.random.default_rng(int(order) + 40)
    _, tdt, kind = SMALL[name]
    n = 50_001
    k = gen(rng, name, n)
    v = np.arange(n, dtype=np.uint32)
    desc = order in (cub.Order.DESCENDING, cub.Order.TOTAL_DESCENDING)
    total = order in (cub.Order.TOTAL_ASCENDING, cub.Order.TOTAL_DESCENDING)
    perm = np.argsort(image(k, kind, desc, fold=not total), kind="stable")
    launch = cub.Program.load("cuda:0").on()
    dk, dv = to_dev(k, name), torch.from_numpy(v).cuda()
    ws = cub.device_merge_sort_pairs_workspace(launch, tdt, torch.uint32, n)
    cub.device_merge_sort_pairs(launch, dk, dv, ws, order)
    assert np.array_equal(raw_bits(to_host(dk)), raw_bits(k[perm]))
    assert np.array_equal(to_host(dv), v[perm])


def test_small_keys_rejected_by_merge():
    launch = cub.Program.load("cuda:0").on()
    a = torch.zeros(10, dtype=torch.uint16, device="cuda")
    out = torch.zeros(20, dtype=torch.uint16, device="cuda")
    ws = cub.device_merge_workspace(launch, 10, 10)
    with pytest.raises(cub.BadArgument):
        cub.device_merge_keys(launch, a, a, ws, out, cub.Order.ASCENDING)
