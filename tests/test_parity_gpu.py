"""GPU parity: the CUDA path (through the C ABI, via the rccl_cub / rccl_thrust
mirrors) against the reference's golden vectors and against the CPU oracle on
seeded inputs.  Integer, byte and index work: every comparison is bit-exact."""
import os

import numpy as np
import pytest
import torch

from helpers import NP_OF, bits, load_cases, to_dev, to_host
from oracle import pyoracle as O
from rccl_b200 import cub, thrust
from rccl_b200.errors import InvalidBitRange

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 1

CASES = load_cases()
TORCH_OF = {"uint32": torch.uint32, "int32": torch.int32, "float32": torch.float32,
            "uint64": torch.uint64, "int64": torch.int64, "float64": torch.float64}


@pytest.fixture(scope="module")
def launch():
    return cub.Program.load("cuda:0").on()


@pytest.fixture(scope="module")
def execution():
    return thrust.Program.load("cuda:0").par()


def run_case(case, launch, execution):
    api, kd = case["api"], TORCH_OF[case["key_dtype"]]
    keys = to_dev(case["keys"])
    values = to_dev(case["values"]) if case["has_values"] else None
    desc = case["descending"]
    n = keys.numel()
    if api == "keys":
        ws = cub.device_radix_sort_workspace(launch, kd, n)
        f = cub.device_radix_sort_keys_descending if desc else cub.device_radix_sort_keys
        f(launch, keys, ws)
        return keys, None, None
    if api == "pairs":
        ws = cub.device_radix_sort_pairs_workspace(launch, kd, values.dtype, n)
        f = cub.device_radix_sort_pairs_descending if desc else cub.device_radix_sort_pairs
        f(launch, keys, values, ws)
        return keys, values, None
    if api in ("thrust_sort", "thrust_sort_unstable"):
        getattr(thrust, api.split("_", 1)[1])(execution, keys)
        return keys, None, None
    if api in ("thrust_pairs_sort", "thrust_pairs_sort_unstable"):
        r = thrust.with_values(keys, values)
        r.sort(execution) if api.endswith("_sort") else r.sort_unstable(execution)
        return keys, values, None
    rng = range(*case["bit_range"])
    if api == "keys_buffer":
        second = to_dev(case["second"])
        buffers = cub.DoubleBuffer.new(keys, second)
        ws = cub.device_radix_sort_keys_buffer_workspace(launch, kd, n)
        f = (cub.device_radix_sort_keys_buffer_descending if desc
             else cub.device_radix_sort_keys_buffer)
        f(launch, buffers, rng, ws)
        return buffers.current(), None, buffers
    if api == "pairs_buffer":
        second_k = to_dev(case["second"])
        second_v = torch.zeros_like(values)
        buffers = cub.DoubleBuffer.paired((keys, values), (second_k, second_v))
        ws = cub.device_radix_sort_pairs_buffer_workspace(launch, kd, values.dtype, n)
        f = (cub.device_radix_sort_pairs_buffer_descending if desc
             else cub.device_radix_sort_pairs_buffer)
        f(launch, buffers, rng, ws)
        k, v = buffers.current()
        return k, v, buffers
    raise AssertionError(api)


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_golden_probe(case, launch, execution):
    if case["expect_error"]:
        keys = to_dev(case["keys"])
        buffers = cub.DoubleBuffer.new(keys, to_dev(case["second"]))
        ws = cub.device_radix_sort_keys_buffer_workspace(launch, torch.uint32, keys.numel())
        with pytest.raises(InvalidBitRange) as e:
            cub.device_radix_sort_keys_buffer(launch, buffers, range(*case["bit_range"]), ws)
        assert [e.value.begin, e.value.end, e.value.key_bits] == case["expect_error"][1:]
        assert buffers.current_is_first()
        assert np.array_equal(to_host(buffers.current()), case["keys"])
        return
    k, v, buffers = run_case(case, launch, execution)
    torch.cuda.synchronize()
    assert np.array_equal(bits(to_host(k)), bits(case["expected_keys"]))
    if v is not None:
        assert np.array_equal(to_host(v), case["expected_values"])
    if case["expect_current_is_first"] is not None:
        assert buffers.current_is_first() == case["expect_current_is_first"]


# ---------------------------------------------------------------------------
# Seeded random parity against the oracle
# ---------------------------------------------------------------------------
def gen_keys(rng, dtype, n, mode):
    if mode == "uniform":
        if dtype in (np.float32, np.float64):
            x = rng.normal(0, 1e3, n).astype(dtype)
            if n:
                idx = rng.choice(n, size=max(1, n // 50), replace=False)
                specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan], dtype=dtype)
                x[idx] = specials[rng.integers(0, 5, idx.size)]
            return x
        info = np.iinfo(dtype)
        return rng.integers(info.min, info.max, n, dtype=dtype, endpoint=True)
    if mode == "low_entropy":
        base = rng.integers(0, 7, n)
        return np.asarray(base * 977 - 1000, dtype=np.float64).astype(dtype) if dtype in (
            np.float32, np.float64) else np.asarray(base * 977, dtype=dtype)
    return np.full(n, 5, dtype=dtype)


def gen_values(rng, vb, n):
    if vb == 16:
        return rng.integers(0, 256, (n, 16), dtype=np.uint8)
    return np.arange(n, dtype={1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[vb])


def gpu_sort(launch, keys_np, values_np, desc, bit_range=None):
    kd = torch.from_numpy(keys_np[:0]).dtype
    n = keys_np.shape[0]
    keys = to_dev(keys_np)
    second = torch.zeros_like(keys)
    bits_total = keys.element_size() * 8
    rng = range(*(bit_range or (0, bits_total)))
    if values_np is None:
        buffers = cub.DoubleBuffer.new(keys, second)
        ws = cub.device_radix_sort_keys_buffer_workspace(launch, kd, n)
        (cub.device_radix_sort_keys_buffer_descending if desc
         else cub.device_radix_sort_keys_buffer)(launch, buffers, rng, ws)
        out = buffers.current()
        cub.check_device_status(launch, ws)
        return to_host(out), None, buffers.current_is_first()
    values = to_dev(values_np)
    buffers = cub.DoubleBuffer.paired((keys, values), (second, torch.zeros_like(values)))
    ws = cub.device_radix_sort_pairs_buffer_workspace(launch, kd, cub.value_bytes_of(values), n)
    (cub.device_radix_sort_pairs_buffer_descending if desc
     else cub.device_radix_sort_pairs_buffer)(launch, buffers, rng, ws)
    k, v = buffers.current()
    cub.check_device_status(launch, ws)
    return to_host(k), to_host(v), buffers.current_is_first()


def check_against_oracle(launch, keys_np, values_np, desc, bit_range=None):
    gk, gv, cur_first = gpu_sort(launch, keys_np, values_np, desc, bit_range)
    ok, ov, swaps, st = O.radix_sort(keys_np, values_np, desc, bit_range)
    assert st == 0
    assert np.array_equal(bits(gk), bits(ok)), "keys differ from the oracle"
    if values_np is not None:
        assert np.array_equal(gv, ov), "values differ from the oracle"
    assert cur_first == (swaps % 2 == 0)


KEY_NAMES = ["uint32", "int32", "float32", "uint64", "int64", "float64"]
SIZES = [1, 2, 31, 4864, 4865, 8191, 8193, 100_003, (1 << 17) + 3]


@pytest.mark.parametrize("kname", KEY_NAMES)
@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("n", SIZES)
def test_keys_random_parity(launch, kname, desc, n):
    rng = np.random.default_rng(1000 + n)
    k = gen_keys(rng, NP_OF[kname], n, "uniform")
    check_against_oracle(launch, k, None, desc)


@pytest.mark.parametrize("kname", KEY_NAMES)
@pytest.mark.parametrize("mode", ["low_entropy", "constant"])
def test_keys_skewed_parity(launch, kname, mode):
    rng = np.random.default_rng(11)
    for desc in (False, True):
        check_against_oracle(launch, gen_keys(rng, NP_OF[kname], 70_001, mode), None, desc)


@pytest.mark.parametrize("kname", KEY_NAMES)
@pytest.mark.parametrize("with_values", [False, True])
def test_one_bucket_passes(launch, kname, with_values):
    """Keys whose high digits are the same for every key: those passes take
    the one-bucket identity path (a transformed copy), the others sort."""
    rng = np.random.default_rng(17)
    dt = NP_OF[kname]
    n = 100_003
    if dt in (np.float32, np.float64):
        k = rng.uniform(1.0, 1.5, n).astype(dt)  # one sign, one exponent
    elif np.issubdtype(dt, np.signedinteger):
        k = rng.integers(0, 3000, n).astype(dt)  # non-negative: top digits constant
    else:
        k = rng.integers(0, 3000, n).astype(dt)
    k[::101] = k[5]  # duplicates: stability through identity passes
    v = np.arange(n, dtype=np.uint32) if with_values else None
    for desc in (False, True):
        check_against_oracle(launch, k, v, desc)
        # a partial window whose every pass is a single bucket
        width = np.dtype(dt).itemsize * 8
        check_against_oracle(launch, k, v, desc, (width - 4, width))


@pytest.mark.parametrize("kname", ["uint32", "float32", "uint64", "int64"])
@pytest.mark.parametrize("vb", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("n", [777, 2305, 4865, 50_001])
def test_pairs_random_parity(launch, kname, vb, n):
    rng = np.random.default_rng(n * 31 + vb)
    k = gen_keys(rng, NP_OF[kname], n, "low_entropy" if n % 2 else "uniform")
    v = gen_values(rng, vb, n)
    for desc in (False, True):
        check_against_oracle(launch, k, v, desc)


@pytest.mark.parametrize("kname", KEY_NAMES)
@pytest.mark.parametrize("n", [3000, 30_000])
def test_bit_windows(launch, kname, n):
    rng = np.random.default_rng(5)
    k = gen_keys(rng, NP_OF[kname], n, "uniform")
    width = np.dtype(NP_OF[kname]).itemsize * 8
    for begin, end in [(0, 8), (3, 19), (5, 6), (0, width - 1), (width - 9, width),
                       (7, 7 + min(24, width - 7))]:
        for desc in (False, True):
            check_against_oracle(launch, k, None, desc, (begin, end))


def test_zero_order_partial_window_follows_route(launch):
    pattern = np.array([0.0, 1.0, -0.0], np.float32)
    for reps in (1, 1622):
        k = np.tile(pattern, reps)
        check_against_oracle(launch, k, None, True, (0, 8))
        check_against_oracle(launch, k, np.arange(k.size, dtype=np.uint32), True, (0, 8))


def test_selector_on_odd_pass_counts(launch):
    rng = np.random.default_rng(9)
    k = rng.integers(0, 2**32, 20_000, dtype=np.uint64).astype(np.uint32)
    for rngs, first in [((0, 8), False), ((0, 16), True), ((0, 24), False), ((0, 32), True)]:
        _, _, cur = gpu_sort(launch, k, None, False, rngs)
        assert cur == first


def test_doublebuffer_started_on_second(launch):
    # A selector already pointing at `second` sorts the data held there.
    rng = np.random.default_rng(4)
    k = rng.integers(0, 2**32, 30_000, dtype=np.uint64).astype(np.uint32)
    first = torch.zeros(k.size, dtype=torch.uint32, device="cuda")
    second = to_dev(k)
    buffers = cub.DoubleBuffer(first, second, current_is_first=False)
    ws = cub.device_radix_sort_keys_buffer_workspace(launch, torch.uint32, k.size)
    cub.device_radix_sort_keys_buffer(launch, buffers, range(0, 32), ws)
    assert not buffers.current_is_first()
    assert np.array_equal(to_host(buffers.current()), np.sort(k))


def test_workspace_reuse_across_directions_and_sizes(launch):
    rng = np.random.default_rng(2)
    k = rng.integers(0, 2**32, 60_000, dtype=np.uint64).astype(np.uint32)
    ws = cub.device_radix_sort_workspace(launch, torch.uint32, k.size)
    t = to_dev(k)
    cub.device_radix_sort_keys(launch, t, ws)
    assert np.array_equal(to_host(t), np.sort(k))
    cub.device_radix_sort_keys_descending(launch, t, ws)
    assert np.array_equal(to_host(t), np.sort(k)[::-1])
    cub.device_radix_sort_keys(launch, t, ws)
    assert np.array_equal(to_host(t), np.sort(k))


def test_non_default_stream(launch):
    s = torch.cuda.Stream()
    l2 = cub.Program.load("cuda:0").on(s)
    rng = np.random.default_rng(8)
    k = rng.integers(0, 2**64, 200_000, dtype=np.uint64)
    with torch.cuda.stream(s):
        t = to_dev(k)
        ws = cub.device_radix_sort_workspace(l2, torch.uint64, k.size)
    cub.device_radix_sort_keys(l2, t, ws)
    s.synchronize()
    assert np.array_equal(to_host(t), np.sort(k))


# The uniform-step form of a pass (RANK_RUNS) takes passes after the first
# when the pass and the one before each have a digit holding 1/16 of the
# keys, in sorts of at least 2^25 items.
RUNS_MIN_ITEMS = 1 << 25


@pytest.mark.parametrize("kname", KEY_NAMES)
@pytest.mark.parametrize("with_values", [False, True])
def test_runs_of_equal_keys_parity(launch, kname, with_values):
    """Duplicate-heavy input at 2^25 + 4321 items: six heavy values holding
    30% down to 6.5% of the keys over a uniform rest, so every pass is hot
    and, after the first, sorted runs of equal keys fill whole warp steps.
    Checked bit-exactly against the oracle; value indices check stability."""
    rng = np.random.default_rng(23)
    dt = NP_OF[kname]
    n = RUNS_MIN_ITEMS + 4321
    k = gen_keys(rng, dt, n, "uniform")
    heavy = gen_keys(rng, dt, 6, "uniform")
    which = np.searchsorted(np.cumsum([0.30, 0.15, 0.08, 0.07, 0.065, 0.065]), rng.random(n))
    for h in range(heavy.size):
        k[which == h] = heavy[h]
    v = np.arange(n, dtype=np.uint32) if with_values else None
    desc = with_values  # both directions across the parametrization
    gk, gv, cur_first = gpu_sort(launch, k, v, desc)
    ok, ov, swaps, st = O.radix_sort(k, v, desc, threads=THREADS)
    assert st == 0
    assert np.array_equal(bits(gk), bits(ok))
    if v is not None:
        assert np.array_equal(gv, ov)
    assert cur_first == (swaps % 2 == 0)


def test_runs_form_below_threshold_parity(launch):
    """The same kind of input below 2^25 items (plain passes only)."""
    rng = np.random.default_rng(29)
    n = (1 << 20) + 77
    k = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    k[rng.random(n) < 0.4] = 123456789
    v = np.arange(n, dtype=np.uint32)
    for desc in (False, True):
        check_against_oracle(launch, k, v, desc)
