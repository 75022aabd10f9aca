"""Segmented radix sort (no reference counterpart): every segment is sorted
as the non-segmented radix sort would sort an array of its length -- small
segments through the one-CTA route, large ones through onesweep -- checked
against the oracle per segment (keys and stable values), with empty, single,
boundary-sized and large segments, gaps between segments and both
directions."""
import numpy as np
import pytest
import torch

from helpers import NP_OF, bits
from oracle import pyoracle as O
from rccl_b200 import cub

pytestmark = pytest.mark.gpu

TORCH_OF = {"uint32": torch.uint32, "int32": torch.int32, "float32": torch.float32,
            "uint64": torch.uint64, "int64": torch.int64, "float64": torch.float64}


def gen(rng, dt, n):
    if dt in (np.float32, np.float64):
        x = rng.normal(0, 50, n).astype(dt)
        x[rng.integers(0, n, max(1, n // 30))] = -0.0
        x[rng.integers(0, n, max(1, n // 30))] = 0.0
        return x
    info = np.iinfo(dt)
    return rng.integers(info.min, info.max, n, dtype=dt, endpoint=True)


@pytest.mark.parametrize("kname", ["uint32", "float32", "int64", "float64"])
@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("with_values", [False, True])
def test_segmented_matches_per_segment_oracle(kname, desc, with_values):
    rng = np.random.default_rng(len(kname) * 10 + desc * 2 + with_values)
    dt = NP_OF[kname]
    lens = [0, 1, 2, 31, 4864, 4865, 2304, 2305, 50_000, 7, 0, 3000]
    gaps = [int(x) for x in rng.integers(0, 5, len(lens))]
    begins, ends, pos = [], [], 0
    for L, g in zip(lens, gaps):
        pos += g
        begins.append(pos)
        ends.append(pos + L)
        pos += L
    n = pos + 3
    k = gen(rng, dt, n)
    v = np.arange(n, dtype=np.uint32)
    launch = cub.Program.load("cuda:0").on()
    kin = torch.from_numpy(k).cuda()
    kout = torch.from_numpy(k.copy()).cuda()  # items outside segments keep these
    b = torch.tensor(begins, dtype=torch.int64, device="cuda")
    e = torch.tensor(ends, dtype=torch.int64, device="cuda")
    if with_values:
        vin = torch.from_numpy(v).cuda()
        vout = torch.from_numpy(v.copy()).cuda()
        f = (cub.device_segmented_radix_sort_pairs_descending if desc
             else cub.device_segmented_radix_sort_pairs)
        f(launch, kin, kout, vin, vout, b, e)
    else:
        f = (cub.device_segmented_radix_sort_keys_descending if desc
             else cub.device_segmented_radix_sort_keys)
        f(launch, kin, kout, b, e)
    gk = kout.cpu().numpy()
    assert np.array_equal(bits(kin.cpu().numpy()), bits(k))  # input untouched
    for bb, ee in zip(begins, ends):
        ek, ev, _, st = O.radix_sort(k[bb:ee], v[bb:ee] if with_values else None, desc)
        assert st == 0
        assert np.array_equal(bits(gk[bb:ee]), bits(ek)), (bb, ee)
        if with_values:
            assert np.array_equal(vout.cpu().numpy()[bb:ee], ev), (bb, ee)
    covered = np.zeros(n, bool)
    for bb, ee in zip(begins, ends):
        covered[bb:ee] = True
    assert np.array_equal(bits(gk[~covered]), bits(k[~covered]))


def test_segmented_bit_window_and_bad_offsets():
    rng = np.random.default_rng(3)
    n = 20_000
    k = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    launch = cub.Program.load("cuda:0").on()
    kin = torch.from_numpy(k).cuda()
    kout = torch.empty_like(kin)
    b = torch.tensor([0, 100, 9000], dtype=torch.int64, device="cuda")
    e = torch.tensor([100, 9000, n], dtype=torch.int64, device="cuda")
    cub.device_segmented_radix_sort_keys(launch, kin, kout, b, e, range(4, 20))
    gk = kout.cpu().numpy()
    for bb, ee in [(0, 100), (100, 9000), (9000, n)]:
        ek, _, _, st = O.radix_sort(k[bb:ee], None, False, (4, 20))
        assert np.array_equal(gk[bb:ee], ek)
    bad_e = torch.tensor([100, 9000, n + 1], dtype=torch.int64, device="cuda")
    with pytest.raises(cub.BadArgument):
        cub.device_segmented_radix_sort_keys(launch, kin, kout, b, bad_e)
