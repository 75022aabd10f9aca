"""Comparator-program sort (rsort_sort_by), CPU side: the oracle pinned to
the reference's own comparator-sort outputs, its two forms against each
other, the term builder, and the C ABI's argument checks (which run before
any device use)."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import load_compare_cases, oracle_terms, program_of
from oracle import compare_oracle as CO
from rccl_b200 import _lib, compare
from rccl_b200.errors import BadArgument, WorkspaceTooSmall, raise_for, SizeOverflow

CASES = load_compare_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_outputs(case):
    rows = CO.as_rows(case["records"])
    terms = oracle_terms(case["terms"])
    for form in (CO.order_by_terms, CO.sort_by_cmp):
        order = form(rows, terms)
        assert np.array_equal(case["records"][order], case["expected"]), form.__name__
        if case["has_values"]:
            assert np.array_equal(case["values"][order], case["expected_values"])


INT_TYPES = [np.int8, np.uint8, np.int16, np.uint16, np.int32, np.uint32, np.int64, np.uint64]


def random_terms(rng, n_terms, layout):
    """layout: list of (dtype, offset); a random projection per term."""
    terms = []
    for _ in range(n_terms):
        dt, off = layout[rng.integers(len(layout))]
        dt = np.dtype(dt)
        desc = bool(rng.integers(2))
        if dt.kind == "f":
            terms.append(CO.Term(dt, off, "identity", 0, desc, bool(rng.integers(2))))
            continue
        info = np.iinfo(dt)
        proj = ["identity", "and", "shr", "div", "rem"][rng.integers(5)]
        op = 0
        if proj == "and":
            op = int(rng.integers(info.min, info.max, dtype=dt, endpoint=True))
        elif proj == "shr":
            op = int(rng.integers(0, 8 * dt.itemsize))
        elif proj in ("div", "rem"):
            while op == 0 or (dt.kind == "i" and op == -1):
                op = int(rng.integers(max(info.min, -300), min(info.max, 300), endpoint=True))
        terms.append(CO.Term(dt, off, proj, op, desc))
    return terms


def random_records(rng, n, layout, record_bytes):
    rows = rng.integers(0, 256, (n, record_bytes), dtype=np.uint8)
    for dt, off in layout:
        dt = np.dtype(dt)
        if dt.kind == "f":
            v = rng.normal(0, 4, n).astype(dt)
            v[rng.integers(0, n, max(1, n // 20))] = 0.0
            v[rng.integers(0, n, max(1, n // 20))] = -0.0
            v[rng.integers(0, n, max(1, n // 50))] = np.nan
            v[rng.integers(0, n, max(1, n // 50))] = -np.inf
        else:
            info = np.iinfo(dt)
            v = rng.integers(info.min, info.max, n, dtype=dt, endpoint=True)
            v[::3] = v[1]  # ties: stability
            v[::7] = rng.integers(-3, 4, v[::7].size).astype(dt)
        rows[:, off:off + dt.itemsize] = v.view(np.uint8).reshape(n, dt.itemsize)
    return rows


# a 19-byte record with fields at aligned and unaligned offsets
LAYOUT = [(np.uint32, 0), (np.int16, 4), (np.float32, 6), (np.int64, 10), (np.uint8, 18)]


def test_oracle_forms_agree():
    rng = np.random.default_rng(7)
    for trial in range(60):
        rows = random_records(rng, 300, LAYOUT, 19)
        terms = random_terms(rng, int(rng.integers(0, 4)), LAYOUT)
        assert np.array_equal(CO.order_by_terms(rows, terms), CO.sort_by_cmp(rows, terms)), terms
    for dt in INT_TYPES + [np.float32, np.float64]:
        rows = random_records(rng, 400, [(dt, 0)], np.dtype(dt).itemsize)
        for terms in ([CO.Term(np.dtype(dt), 0)], random_terms(rng, 2, [(dt, 0)])):
            assert np.array_equal(CO.order_by_terms(rows, terms), CO.sort_by_cmp(rows, terms))


def test_truncating_division_and_remainder():
    # Rust: -15 / 10 == -1, -15 % 10 == -5, 15 / -10 == -1, 15 % -10 == 5
    v = np.array([-15, 15, -5, 5], np.int32)
    rows = CO.as_rows(v)
    img = CO.term_images(rows, [CO.Term(np.dtype(np.int32), 0, "div", 10)])[0]
    assert (img ^ np.uint64(1 << 31)).astype(np.uint32).view(np.int32).tolist() == [-1, 1, 0, 0]
    img = CO.term_images(rows, [CO.Term(np.dtype(np.int32), 0, "rem", 10)])[0]
    assert (img ^ np.uint64(1 << 31)).astype(np.uint32).view(np.int32).tolist() == [-5, 5, -5, 5]
    assert CO._py_project(15, CO.Term(np.dtype(np.int32), 0, "div", -10)) == -1
    assert CO._py_project(15, CO.Term(np.dtype(np.int32), 0, "rem", -10)) == 5


def test_builder_terms():
    c = compare.Key(torch.int32).and_(1).then(compare.Key(torch.int32))
    t = compare.c_terms(c)
    assert [(t[i].type, t[i].projection, t[i].order, t[i].operand) for i in range(2)] == [
        (_lib.RSORT_I32, _lib.RSORT_PROJ_AND, 0, 1), (_lib.RSORT_I32, _lib.RSORT_PROJ_IDENTITY, 0, 0)]
    r = compare.Key(torch.float64, offset=8).total().reverse()
    t = compare.c_terms(r)
    assert (t[0].offset, t[0].order) == (8, 3)
    assert compare.c_terms(compare.Key(torch.uint64).and_(2 ** 64 - 1))[0].operand == -1
    assert c.reverse().terms[0].descending and c.reverse().terms[1].descending
    with pytest.raises(BadArgument):
        compare.Key(torch.int32).div(3).rem(2)
    with pytest.raises(BadArgument):
        compare.c_terms(compare.Comparator(tuple(compare.Key(torch.int32) for _ in range(17))))
    with pytest.raises(BadArgument):
        compare.c_terms(compare.Key(torch.uint64).and_(2 ** 64))
    assert compare.record_bytes_of(torch.zeros((5, 3), dtype=torch.int32)) == 12
    assert compare.record_bytes_of(torch.zeros(5, dtype=torch.float64)) == 8
    assert program_of(CASES[1]["terms"]).terms[0].projection == "and"


def sort_by_status(terms, record_bytes=8, n=1000, scratch=1, nterms=None):
    arr = (_lib.CompareTerm * max(len(terms), 1))()
    for i, (off, ty, proj, order, op) in enumerate(terms):
        arr[i].offset, arr[i].type, arr[i].projection, arr[i].order, arr[i].operand = (
            off, ty, proj, order, op)
    return _lib.lib().rsort_sort_by(arr, len(terms) if nterms is None else nterms,
                                    ctypes.c_void_p(0x1000), record_bytes, None, 0, n,
                                    ctypes.c_void_p(0x100000), scratch, None)


def test_c_abi_argument_checks():
    U32, I32, F32 = _lib.RSORT_U32, _lib.RSORT_I32, _lib.RSORT_F32
    P = _lib
    bad = [
        [(0, 99, P.RSORT_PROJ_IDENTITY, 0, 0)],            # type
        [(0, U32, P.RSORT_PROJ_IDENTITY, 7, 0)],           # order
        [(6, U32, P.RSORT_PROJ_IDENTITY, 0, 0)],           # field past the record
        [(0, U32, 9, 0, 0)],                               # projection
        [(0, F32, P.RSORT_PROJ_AND, 0, 1)],                # float projection
        [(0, U32, P.RSORT_PROJ_SHR, 0, 32)],               # shift >= width
        [(0, I32, P.RSORT_PROJ_SHR, 0, -1)],               # negative shift
        [(0, U32, P.RSORT_PROJ_DIV, 0, 0)],                # divide by zero
        [(0, I32, P.RSORT_PROJ_REM, 0, -1)],               # MIN % -1
        [(0, U32, P.RSORT_PROJ_AND, 0, 1 << 32)],          # mask outside u32
        [(0, I32, P.RSORT_PROJ_DIV, 0, 1 << 31)],          # divisor outside i32
    ]
    for terms in bad:
        assert sort_by_status(terms) == _lib.RSORT_BAD_ARGUMENT, terms
    assert sort_by_status([(0, U32, 0, 0, 0)] * 17) == _lib.RSORT_BAD_ARGUMENT
    assert sort_by_status([(0, U32, 0, 0, 0)], n=1 << 32) == _lib.RSORT_SIZE_OVERFLOW
    with pytest.raises(SizeOverflow):
        raise_for(sort_by_status([(0, U32, 0, 0, 0)], n=1 << 32))
    # valid terms: a too-small scratch is reported before any device use
    st = sort_by_status([(0, U32, P.RSORT_PROJ_AND, 0, 1), (4, I32, 0, 1, 0)])
    assert st == _lib.RSORT_WORKSPACE_TOO_SMALL
    with pytest.raises(WorkspaceTooSmall):
        raise_for(st)
    # nothing to do: one record, no terms, or only terms that compare equal
    assert sort_by_status([(0, U32, 0, 0, 0)], n=1) == _lib.RSORT_OK
    assert sort_by_status([], n=1000) == _lib.RSORT_OK
    assert sort_by_status([(0, U32, P.RSORT_PROJ_AND, 0, 0), (0, U32, P.RSORT_PROJ_REM, 0, 1)],
                          n=1000) == _lib.RSORT_OK


def test_scratch_bytes():
    lib = _lib.lib()
    small = lib.rsort_sort_by_scratch_bytes(12, 0, 1000)
    big = lib.rsort_sort_by_scratch_bytes(12, 8, 1000)
    assert small >= 1000 * (8 + 8 + 4 + 4 + 12)
    assert big >= small + 8 * 1000
