"""CPU tests: pin the oracle against the reference's golden vectors and host
unit tests before it is trusted as the checker of the CUDA path."""
import numpy as np
import pytest

from helpers import bits, load_cases, order_image
from oracle import pyoracle as O

CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_golden(case):
    keys = case["keys"]
    values = case.get("values")
    rng = tuple(case["bit_range"]) if case["bit_range"] else None
    out_k, out_v, swaps, status = O.radix_sort(keys, values, case["descending"], rng)
    if case["expect_error"]:
        assert status == 1  # InvalidBitRange
        assert np.array_equal(bits(out_k), bits(keys))
        return
    assert status == 0
    assert np.array_equal(bits(out_k), bits(case["expected_keys"]))
    if values is not None:
        assert np.array_equal(out_v, case["expected_values"])
    if case["expect_current_is_first"] is not None:
        # Selector after the call: flipped once per swap.
        assert (swaps % 2 == 0) == case["expect_current_is_first"]


# rccl-cub/src/radix.rs:884-893
def test_i32_ascending_image_of_minus_one():
    assert O.to_ordered(O.I32, False, 0xFFFFFFFF) == 0x7FFFFFFF
    assert O.to_ordered(O.U32, False, 7) == 7
    raw = int(np.array([-3.5], np.float32).view(np.uint32)[0])
    assert O.from_ordered(O.F32, False, O.to_ordered(O.F32, False, raw)) == raw


# rccl-cub/src/ordering_backend/tests.rs:29-111
@pytest.mark.parametrize("kt,samples", [
    (O.U32, [0, 1, 0xFFFFFFFF, 0x80000000, 0x12345678]),
    (O.I32, [0x80000000, 0xFFFFFFFF, 0, 1, 0x7FFFFFFF]),
    (O.F32, [0, 0x80000000, 0x3F800000, 0xBF800000, 0x7F800000, 0x7FC00000]),
    (O.U64, [0, 1, 2**64 - 1, 2**63, 0x123456789ABCDEF0]),
    (O.I64, [2**63, 2**64 - 1, 0, 1, 2**63 - 1]),
    (O.F64, [0, 2**63, 0x3FF0000000000000, 0xBFF0000000000000, 0x7FF0000000000000,
             0x7FF8000000000000]),
])
def test_transforms_round_trip(kt, samples):
    for raw in samples:
        for desc in (False, True):
            assert O.from_ordered(kt, desc, O.to_ordered(kt, desc, raw)) == raw


# rccl-cub/src/ordering_backend/tests.rs:137-177
@pytest.mark.parametrize("kt,width", [(O.F32, 32), (O.F64, 64)])
def test_signed_zero_digits_equal_in_both_directions(kt, width):
    neg_zero = 1 << (width - 1)
    for desc in (False, True):
        pos = O.fold(kt, O.to_ordered(kt, desc, 0))
        neg = O.fold(kt, O.to_ordered(kt, desc, neg_zero))
        for bit in range(width):
            for nbits in range(1, min(8, width - bit) + 1):
                mask = (1 << nbits) - 1
                assert (pos >> bit) & mask == (neg >> bit) & mask


# rccl-cub/src/radix.rs:895-905 and rccl-cub/src/workspace.rs:776-806
def test_policy800_single_tile_extents():
    assert O.single_tile_items(4, 0) == 4864
    assert O.single_tile_items(8, 0) == 2304
    assert O.single_tile_items(4, 8) == 2304
    assert O.single_tile_items(4, 4) == 4864
    assert O.single_tile_items(8, 16) == 1024


def test_oracle_route_dependent_zero_order_under_partial_window():
    # Single-tile route: descending by the ascending-space window of
    # fold(to_ordered_ascending); onesweep route: ascending by the window of
    # fold(to_ordered_descending) (ordering_kernels.rs:1229-1234 vs :1309-1314).
    # Under window 0..8 the images are: single tile 0.0, 1.0 and -0.0 all
    # 0x00 (tie, input order kept); onesweep +-0.0 -> 0x00, 1.0 -> 0xff.
    pattern = np.array([0.0, 1.0, -0.0], np.float32)
    small, _, swaps, _ = O.radix_sort(pattern, descending=True, bit_range=(0, 8))
    assert swaps == 1
    assert np.array_equal(bits(small), bits(pattern))
    big = np.tile(pattern, 1622)  # 4866 items > 4864: onesweep route
    out, _, swaps_big, _ = O.radix_sort(big, descending=True, bit_range=(0, 8))
    assert swaps_big == 1
    zeros = big[bits(big) != 0x3F800000]
    assert np.array_equal(bits(out[:zeros.size]), bits(zeros))
    assert np.all(bits(out[zeros.size:]) == 0x3F800000)


def test_oracle_threads_agree():
    rng = np.random.default_rng(7)
    k = rng.integers(0, 2**64, 300_000, dtype=np.uint64)
    v = np.arange(k.size, dtype=np.uint32)
    a = O.radix_sort(k, v, threads=1)
    b = O.radix_sort(k, v, threads=4)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert np.array_equal(a[0], np.sort(k))


def test_sample_partition_sums_to_total():
    rng = np.random.default_rng(3)
    k = rng.integers(0, 2**32, 40_000, dtype=np.uint64).astype(np.uint32)
    counts = O.sample_partition(k, [10_000] * 4, 256)
    assert counts.sum() == k.size
    assert counts.min() > 5_000  # regular sampling balances uniform keys
    # Constant keys still split evenly: ties break by (rank, position).
    c = np.full(40_000, 9, np.uint32)
    counts_c = O.sample_partition(c, [10_000] * 4, 256)
    assert counts_c.sum() == c.size and counts_c.max() - counts_c.min() < 200


@pytest.mark.parametrize("dtype", [np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64])
@pytest.mark.parametrize("threads", [1, 3])
def test_cpu_baseline_stand_ins_agree_with_the_oracle(dtype, threads):
    """The std::stable_sort stand-ins of the CPU baseline produce the oracle's
    output (stable radix order); the std::sort one the same order image."""
    rng = np.random.default_rng(7)
    n = 50_001
    if np.dtype(dtype).kind == "f":
        k = rng.normal(0, 10, n).astype(dtype)
        k[::9] = -0.0
        k[::10] = 0.0
        k[::23] = np.nan
    else:
        k = rng.integers(-1000, 1000, n).astype(dtype)
    v = np.arange(n, dtype=np.uint32)
    for desc in (False, True):
        ok, ov, _, _ = O.radix_sort(k, v, desc)
        ck, cv = O.cpu_sort(k, v, desc, stable=True, threads=threads)
        assert np.array_equal(O.bits_of(ck), O.bits_of(ok)) and np.array_equal(cv, ov)
        sk, _ = O.cpu_sort(k, None, desc, stable=True, threads=threads)
        assert np.array_equal(O.bits_of(sk), O.bits_of(ok))
        uk, _ = O.cpu_sort(k, None, desc, stable=False, threads=threads)
        img = order_image(uk, desc)
        assert np.array_equal(img, order_image(ok, desc))
