"""Comparator-program sort (rsort_sort_by) on the GPU: the reference's own
comparator-sort cases through the Thrust and CUB mirrors, and seeded records
with fields at aligned and unaligned offsets against the CPU oracle
(oracle/compare_oracle.py).  Index and byte work: every comparison is
bit-exact on the record bytes."""
import numpy as np
import pytest
import torch

from helpers import load_compare_cases, oracle_terms, program_of
from oracle import compare_oracle as CO
from rccl_b200 import compare, cub, thrust
from test_compare import LAYOUT, random_records, random_terms

pytestmark = pytest.mark.gpu

CASES = load_compare_cases()


@pytest.fixture(scope="module")
def execution():
    return thrust.Program.load("cuda:0").par()


@pytest.fixture(scope="module")
def launch():
    return cub.Program.load("cuda:0").on()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_reference_cases_thrust(case, execution):
    order = program_of(case["terms"])
    keys = torch.from_numpy(case["records"].copy()).cuda()
    if case["has_values"]:
        values = torch.from_numpy(case["values"].copy()).cuda()
        thrust.with_values(keys, values).sort_by(execution, order)
        assert np.array_equal(values.cpu().numpy(), case["expected_values"])
    else:
        thrust.sort_by(execution, keys, order)
    assert np.array_equal(keys.cpu().numpy(), case["expected"])


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_reference_cases_cub(case, launch):
    order = program_of(case["terms"])
    keys = torch.from_numpy(case["records"].copy()).cuda()
    values = torch.from_numpy(case["values"].copy()).cuda() if case["has_values"] else None
    ws = cub.device_merge_sort_by_workspace(launch, keys, values)
    if values is None:
        cub.device_merge_sort_keys(launch, keys, ws, order)
    else:
        cub.device_merge_sort_pairs(launch, keys, values, ws, order)
        assert np.array_equal(values.cpu().numpy(), case["expected_values"])
    torch.cuda.synchronize()
    assert np.array_equal(keys.cpu().numpy(), case["expected"])


def program_from_oracle(terms):
    keys = []
    for t in terms:
        k = compare.Key(torch.from_numpy(np.zeros(0, t.dtype)).dtype, t.offset)
        if t.projection != "identity":
            k = getattr(k, {"and": "and_"}.get(t.projection, t.projection))(t.operand)
        if t.descending:
            k = k.reverse()
        if t.total:
            k = k.total()
        keys.append(k)
    return compare.Comparator(tuple(keys))


def gpu_sort_rows(rows, values, terms, execution):
    dr = torch.from_numpy(rows.copy()).cuda()
    if values is None:
        thrust.sort_by(execution, dr, program_from_oracle(terms))
        return dr.cpu().numpy(), None
    dv = torch.from_numpy(values.copy()).cuda()
    thrust.with_values(dr, dv).sort_by(execution, program_from_oracle(terms))
    return dr.cpu().numpy(), dv.cpu().numpy()


@pytest.mark.parametrize("n", [2, 777, 4865, 70_001])
@pytest.mark.parametrize("seed", range(6))
def test_random_programs_on_records(n, seed, execution):
    """19-byte records, 1-4 random terms over fields at offsets 0, 4, 6, 10
    and 18 (unaligned 16-, 32- and 64-bit fields), 8-byte values."""
    rng = np.random.default_rng(100 * seed + n % 97)
    rows = random_records(rng, n, LAYOUT, 19)
    terms = random_terms(rng, int(rng.integers(1, 5)), LAYOUT)
    values = np.arange(n, dtype=np.uint64) * 7 + 3
    order = CO.order_by_terms(rows, terms)
    if n <= 5000:
        assert np.array_equal(order, CO.sort_by_cmp(rows, terms))
    got_r, got_v = gpu_sort_rows(rows, values if seed % 2 else None, terms, execution)
    assert np.array_equal(got_r, rows[order]), terms
    if got_v is not None:
        assert np.array_equal(got_v, values[order])


@pytest.mark.parametrize("dt", [np.int8, np.uint8, np.int16, np.uint16, np.int32, np.uint32,
                                np.int64, np.uint64, np.float32, np.float64])
def test_every_projection_per_type(dt, execution):
    """Scalar records of each type under each projection, both directions
    (floats: partial and total order), against the oracle."""
    rng = np.random.default_rng(int(np.dtype(dt).num))
    n = 30_011
    rows = random_records(rng, n, [(dt, 0)], np.dtype(dt).itemsize)
    d = np.dtype(dt)
    if d.kind == "f":
        programs = [[CO.Term(d, 0, "identity", 0, desc, tot)] for desc in (False, True)
                    for tot in (False, True)]
    else:
        info = np.iinfo(d)
        w = 8 * d.itemsize
        programs = [[CO.Term(d, 0, "identity", 0, desc)] for desc in (False, True)]
        programs += [[CO.Term(d, 0, "and", op), CO.Term(d, 0, "identity", 0, True)]
                     for op in (1, info.max, -2 if d.kind == "i" else info.max - 1)]
        programs += [[CO.Term(d, 0, "shr", s)] for s in (1, w // 2, w - 1)]
        programs += [[CO.Term(d, 0, p, op, desc)] for p in ("div", "rem")
                     for op in (3, 1000 % (int(info.max) + 1) or 7, -5 if d.kind == "i" else 250)
                     for desc in (False, True)]
    for terms in programs:
        got, _ = gpu_sort_rows(rows, None, terms, execution)
        assert np.array_equal(got, rows[CO.order_by_terms(rows, terms)]), terms


def test_many_terms_span_several_key_groups(execution):
    """Sixteen terms (three 64-bit and mixed narrower fields: well over 64
    bits of key) sort as several LSD groups."""
    rng = np.random.default_rng(5)
    n = 50_003
    layout = [(np.uint64, 0), (np.int64, 8), (np.float64, 16), (np.uint32, 24), (np.int16, 28),
              (np.uint8, 30)]
    rows = random_records(rng, n, layout, 31)
    rows[:, :8] = rows[rng.integers(0, 40, n), :8]  # few distinct leading keys: later terms decide
    terms = [CO.Term(np.dtype(dt), off, "identity", 0, bool(i % 2))
             for i, (dt, off) in enumerate(layout)]
    terms += random_terms(rng, 10, layout)
    got, _ = gpu_sort_rows(rows, None, terms, execution)
    assert np.array_equal(got, rows[CO.order_by_terms(rows, terms)])


def test_large_records_2p20(execution):
    """2^20 + 7 records of 16 bytes (key u32 / tag u16 / payload), sorted by
    (tag >> 4, key descending), values moving in lockstep."""
    rng = np.random.default_rng(9)
    n = (1 << 20) + 7
    layout = [(np.uint32, 0), (np.uint16, 4), (np.int64, 8)]
    rows = random_records(rng, n, layout, 16)
    terms = [CO.Term(np.dtype(np.uint16), 4, "shr", 4), CO.Term(np.dtype(np.uint32), 0, "identity",
                                                               0, True)]
    values = np.arange(n, dtype=np.uint32)
    got_r, got_v = gpu_sort_rows(rows, values, terms, execution)
    order = CO.order_by_terms(rows, terms)
    assert np.array_equal(got_r, rows[order])
    assert np.array_equal(got_v, values[order])
