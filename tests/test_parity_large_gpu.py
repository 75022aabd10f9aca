"""GPU parity at the benchmark sizes: the workloads of bench.py sorted through
the C ABI and compared bit-exactly with the CPU oracle (configs 1-3, 2^20 to
2^28 items) or with an independent stable sort of the input's order image
(config 4's 2^30 keys; the oracle checks a 2^24-key sample of it as well), and
2^31 + 12,345-item sorts whose offsets pass 2^31, checked bit-exactly through
the input indices the items carry.

These cover what the small-size suite cannot: the 64-bit offsets that lift
the reference's one-portion limit (rccl-cub/src/radix.rs:377-384), the 48-bit
look-back counts, the -0.0/+0.0 input order and NaN placement of config 3
(rccl-cub/src/ordering_backend/radix.rs:257-337;
rccl-cub/examples/device_radix_sort_keys_probe.rs:121-173) at full size, and
the skewed digits of config 4."""
import os

import numpy as np
import pytest
import torch

import bench
from helpers import bits
from oracle import pyoracle as O
from rccl_b200 import cub

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1


@pytest.fixture(scope="module")
def launch():
    return cub.Program.load("cuda:0").on()


def sort_device(launch, keys, values, descending):
    if values is None:
        ws = cub.device_radix_sort_workspace(launch, keys.dtype, keys.numel())
        (cub.device_radix_sort_keys_descending if descending else cub.device_radix_sort_keys)(
            launch, keys, ws)
    else:
        ws = cub.device_radix_sort_pairs_workspace(launch, keys.dtype, values.dtype, keys.numel())
        (cub.device_radix_sort_pairs_descending if descending else cub.device_radix_sort_pairs)(
            launch, keys, values, ws)
    cub.check_device_status(launch, ws.controls)
    torch.cuda.synchronize()


def release():
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


@pytest.mark.parametrize("config", [1, 2, 3])
def test_benchmark_config_matches_oracle(config, launch):
    w = bench.Workload(config)
    keys, values = w.generate(0, w.n, "cuda:0")
    host_k = keys.cpu().numpy()
    host_v = values.cpu().numpy() if values is not None else None
    sort_device(launch, keys, values, w.desc)
    exp_k, exp_v, _, st = O.radix_sort(host_k, host_v, w.desc, threads=THREADS)
    assert st == 0
    assert np.array_equal(bits(keys.cpu().numpy()), bits(exp_k))
    if values is not None:
        assert np.array_equal(values.cpu().numpy(), exp_v)
    if config == 3:
        # the special values are present in the expected numbers
        b = bits(host_k)
        assert np.count_nonzero((b & 0x7FFFFFFF) == 0) > w.n // 2000
        assert np.count_nonzero(np.isnan(host_k)) > w.n // 20000
        assert np.count_nonzero((b & 0x7FFFFFFF) == 0x7F800000) > w.n // 20000
    del keys, values
    release()


def test_u32_2p28_plus_3_matches_oracle(launch):
    """2^28 + 3 uniform u32 keys (a partial last tile) against the oracle."""
    n = (1 << 28) + 3
    w = bench.Workload(1, n)
    keys, _ = w.generate(0, n, "cuda:0")
    host = keys.cpu().numpy()
    sort_device(launch, keys, None, False)
    exp, _, _, st = O.radix_sort(host, None, False, threads=THREADS)
    assert st == 0 and np.array_equal(keys.cpu().numpy(), exp)
    del keys
    release()


def test_config4_skewed_2p30(launch):
    w = bench.Workload(4)
    src, _ = w.generate(0, w.n, "cuda:0")
    keys = src.clone()
    sort_device(launch, keys, None, False)
    assert bench.check_keys_only(src, keys, "u", False)
    del keys
    release()
    # and a 2^24-key sample of the same distribution against the oracle
    sample = src[: 1 << 24].clone()
    host = sample.cpu().numpy()
    sort_device(launch, sample, None, False)
    exp, _, _, _ = O.radix_sort(host, None, False, threads=THREADS)
    assert np.array_equal(sample.cpu().numpy(), exp)
    del src, sample
    release()


def test_offsets_beyond_2p31_pairs(launch):
    """2^31 + 12,345 u32 keys with u32 values = input index: destination
    offsets and look-back prefixes above 2^31 (the reference stops at one
    2^28-item portion).  Bit-exact without a second sort: every output key is
    the key its value's index generated, the order never decreases, equal keys
    keep ascending indices, and every index appears once."""
    n = (1 << 31) + 12_345
    w = bench.Workload(1, n)
    keys, _ = w.generate(0, n, "cuda:0")
    values = torch.empty(n, dtype=torch.uint32, device="cuda:0")
    for a in range(0, n, bench.CHUNK):
        b = min(n, a + bench.CHUNK)
        values.view(torch.int32)[a:b] = bench._to_i32(
            torch.arange(a, b, dtype=torch.int64, device="cuda:0"))
    sort_device(launch, keys, values, False)
    mark = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    assert bench.check_pairs_index(w, keys, values, mark)
    assert bool(torch.all(mark == 1))
    del keys, values, mark
    release()


def test_offsets_beyond_2p31_keys_only(launch):
    """Keys-only at 2^31 + 12,345 u64 keys whose low 32 bits are the input
    index (all keys distinct): the sorted keys' index bits name a permutation,
    their high bits are the generated ones, and the order never decreases."""
    n = (1 << 31) + 12_345
    keys = torch.empty(n, dtype=torch.uint64, device="cuda:0")
    kv = keys.view(torch.int64)
    for a in range(0, n, bench.CHUNK):
        b = min(n, a + bench.CHUNK)
        idx = torch.arange(a, b, dtype=torch.int64, device="cuda:0")
        kv[a:b] = (bench.splitmix64(idx, 9) & ~0xFFFFFFFF) | idx
    sort_device(launch, keys, None, False)
    mark = torch.zeros(n, dtype=torch.uint8, device="cuda:0")
    prev = None
    ok = True
    for a in range(0, n, bench.CHUNK):
        b = min(n, a + bench.CHUNK)
        k = kv[a:b]
        idx = k & 0xFFFFFFFF
        ok &= bool(torch.equal(bench.splitmix64(idx, 9) & ~0xFFFFFFFF, k & ~0xFFFFFFFF))
        img = k ^ (-(1 << 63))  # unsigned order as signed
        if prev is not None:
            img = torch.cat([prev, img])
        ok &= bool(torch.all(img[1:] > img[:-1]))
        prev = img[-1:]
        mark[idx] = 1
    assert ok
    assert bool(torch.all(mark == 1))
    del keys, mark
    release()


def test_pairs_2p28_descending_stable(launch):
    """Config 2's pairs sorted descending: the value indices of equal keys
    stay ascending (stability), checked against the oracle on the host."""
    n = 1 << 28
    w = bench.Workload(2)
    keys, values = w.generate(0, n, "cuda:0")
    # few distinct keys, so almost every key has ties
    keys.view(torch.int64).bitwise_and_(0xFFF)
    host_k, host_v = keys.cpu().numpy(), values.cpu().numpy()
    sort_device(launch, keys, values, True)
    exp_k, exp_v, _, _ = O.radix_sort(host_k, host_v, True, threads=THREADS)
    assert np.array_equal(keys.cpu().numpy(), exp_k)
    assert np.array_equal(values.cpu().numpy(), exp_v)
    del keys, values
    release()
