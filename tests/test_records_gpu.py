"""Lexicographic record sort (rccl-thrust/src/record_sort.rs): stable
ascending order of [u32; N] rows (word 0 most significant), payloads in
lockstep, arities 2..6.  Expected: numpy's stable lexsort of the rows.
CPU: the arity and payload checks; GPU: the sorts."""
import numpy as np
import pytest
import torch

from rccl_b200 import thrust
from rccl_b200.errors import UnsupportedTarget


def expected(rows: np.ndarray):
    # np.lexsort sorts by the last key first: pass the columns reversed
    return np.lexsort(rows.T[::-1])


@pytest.mark.gpu
@pytest.mark.parametrize("arity", [2, 3, 4, 5, 6])
@pytest.mark.parametrize("n", [1, 2, 1000, 4865, 60_001])
def test_rows_lexicographic(arity, n):
    rng = np.random.default_rng(arity * 100 + n)
    # small value ranges so rows share prefixes and duplicates occur
    rows = rng.integers(0, 6, (n, arity), dtype=np.uint32)
    rows[:, -1] = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    rows[::7] = rows[3 % max(n, 1)]  # exact duplicates: stability
    payload = np.arange(n, dtype=np.uint64) * 3 + 1
    perm = expected(rows)
    execution = thrust.Program.load("cuda:0").par()
    dr = torch.from_numpy(rows.copy()).cuda()
    dp = torch.from_numpy(payload.copy()).cuda()
    thrust.sort_rows_with_payload_lexicographic(execution, dr, dp)
    assert np.array_equal(dr.cpu().numpy(), rows[perm])
    assert np.array_equal(dp.cpu().numpy(), payload[perm])
    dr2 = torch.from_numpy(rows.copy()).cuda()
    thrust.sort_rows_lexicographic(execution, dr2)
    assert np.array_equal(dr2.cpu().numpy(), rows[perm])


@pytest.mark.gpu
@pytest.mark.parametrize("arity", [2, 4])
def test_rows_at_four_byte_offset(arity):
    """Rows whose base address is 4-byte but not 8-byte aligned (a view that
    starts one u32 into its allocation): the row permutation must use 4-byte
    accesses, not the 8-byte accesses an even word count would allow."""
    rng = np.random.default_rng(11 + arity)
    n = 30_001
    rows = rng.integers(0, 5, (n, arity), dtype=np.uint32)
    perm = expected(rows)
    flat = torch.zeros(n * arity + 1, dtype=torch.uint32, device="cuda")
    view = flat[1:].view(n, arity)
    assert view.data_ptr() % 8 == 4
    view.copy_(torch.from_numpy(rows))
    thrust.sort_rows_lexicographic(thrust.Program.load("cuda:0").par(), view)
    assert np.array_equal(view.cpu().numpy(), rows[perm])
    assert int(flat[0].item()) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float64, torch.bool])
def test_rows_into_with_payload_types(dtype):
    rng = np.random.default_rng(5)
    n, arity = 20_000, 3
    rows = rng.integers(0, 4, (n, arity), dtype=np.uint32)
    pay = (rng.random(n) if dtype == torch.float64 else rng.random(n) < 0.5)
    perm = expected(rows)
    execution = thrust.Program.load("cuda:0").par()
    dr = torch.from_numpy(rows.copy()).cuda()
    dp = torch.from_numpy(pay.copy()).cuda()
    out_r, out_p = torch.empty_like(dr), torch.empty_like(dp)
    thrust.sort_rows_with_payload_lexicographic_into(execution, dr, dp, out_r, out_p)
    assert np.array_equal(out_r.cpu().numpy(), rows[perm])
    assert np.array_equal(out_p.cpu().numpy(), pay[perm])
    assert np.array_equal(dr.cpu().numpy(), rows)  # input untouched
    out2 = torch.empty_like(dr)
    thrust.sort_rows_lexicographic_into(execution, dr, out2)
    assert np.array_equal(out2.cpu().numpy(), rows[perm])


def test_rows_arity_and_payload_checks():
    # the checks run before any device use
    for arity in (1, 7):
        rows = torch.zeros((4, arity), dtype=torch.uint32)
        with pytest.raises(UnsupportedTarget):
            thrust._sort_rows(_FakeExec(), rows, None)
    with pytest.raises(thrust.BadArgument):
        thrust._sort_rows(_FakeExec(), torch.zeros((4, 3), dtype=torch.uint32),
                          torch.zeros(4, dtype=torch.int32))


class _FakeLaunch:
    device = torch.device("cpu")

    def check(self, *tensors):
        pass


class _FakeExec:
    launch = _FakeLaunch()
