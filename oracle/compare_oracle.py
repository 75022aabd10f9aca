"""CPU restatement of the sort by a comparator program (rsort_sort_by).

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker.  The product
path never imports it.

What it restates: rccl-cub's DeviceMergeSort (rccl-cub/src/dispatch.rs:170-193,
1113-1146) is a stable sort by a `Fn(&K, &K) -> Ordering` closure, and the
closures its callers write (rccl-thrust/examples/sort.rs:101-113,
rccl-thrust/examples/set_operations_tests.rs:145-152,
rccl-cub/examples/device_ordering_benchmark.rs:162) compare projected fields
with `Ord::cmp`, chain them with `Ordering::then_with` and reverse them by
swapping the arguments.  A term is (dtype, offset, projection, operand,
descending, total): the field of `dtype` at byte `offset` of the record,
projected with Rust integer semantics in the field's type (`&`, arithmetic
`>>` for signed, truncating `/`, `%` with the dividend's sign), compared
ascending or descending; floats compare by partial_cmp with -0.0 == +0.0 (NaNs
by their bit image, as the radix order places them) or, with `total`, by
total_cmp.

Two forms:
  sort_by_cmp   literal: Python's stable sort (like Rust's slice::sort_by)
                with functools.cmp_to_key over a term-by-term comparison;
                small inputs only
  order_by_terms  vectorised: one order image per term, np.lexsort (stable)
The tests check the two against each other and against the reference's own
expected outputs before using either as the checker.
"""
from __future__ import annotations

import functools
from typing import List, NamedTuple, Sequence

import numpy as np


class Term(NamedTuple):
    dtype: np.dtype
    offset: int = 0
    projection: str = "identity"   # identity / and / shr / div / rem
    operand: int = 0
    descending: bool = False
    total: bool = False


def _field(rows: np.ndarray, t: Term) -> np.ndarray:
    """The field column of (n, record_bytes) uint8 rows."""
    dt = np.dtype(t.dtype)
    raw = np.ascontiguousarray(rows[:, t.offset:t.offset + dt.itemsize])
    return raw.view(dt).reshape(-1)


def _project(v: np.ndarray, t: Term) -> np.ndarray:
    dt = v.dtype
    if t.projection == "identity":
        return v
    if dt.kind == "f":
        raise ValueError("float fields take the identity projection only")
    op = np.array(t.operand).astype(dt) if dt.kind == "i" else np.array(
        t.operand & ((1 << (8 * dt.itemsize)) - 1), dtype=np.uint64).astype(dt)
    if t.projection == "and":
        return v & op
    if t.projection == "shr":
        return v >> np.array(t.operand).astype(dt)
    if t.projection == "div":
        if dt.kind == "u":
            return v // op
        q = v // op  # floor; truncation differs when the signs differ and a remainder exists
        fix = (v % op != 0) & ((v < 0) != (op < 0))
        return (q + fix.astype(dt)).astype(dt)
    if t.projection == "rem":
        return np.fmod(v, op) if dt.kind == "i" else v % op
    raise ValueError(t.projection)


def _image(p: np.ndarray, t: Term) -> np.ndarray:
    """Order image as uint64: unsigned as is, signed with the sign bit
    flipped, floats sign-magnitude to unsigned (-0.0 folded onto +0.0 unless
    total); complemented when descending."""
    dt = p.dtype
    w = 8 * dt.itemsize
    u = p.view(np.dtype(f"u{dt.itemsize}")).astype(np.uint64)
    sign = np.uint64(1 << (w - 1))
    full = np.uint64((1 << w) - 1)
    if dt.kind == "i":
        img = u ^ sign
    elif dt.kind == "f":
        neg = (u & sign) != 0
        img = np.where(neg, u ^ full, u ^ sign)
        if not t.total:
            img = np.where(img == sign - np.uint64(1), sign, img)
    else:
        img = u
    return (img ^ full) if t.descending else img


def term_images(rows: np.ndarray, terms: Sequence[Term]) -> List[np.ndarray]:
    return [_image(_project(_field(rows, t), t), t) for t in terms]


def order_by_terms(rows: np.ndarray, terms: Sequence[Term]) -> np.ndarray:
    """Stable order (a permutation) of the records under the comparator."""
    n = rows.shape[0]
    if not terms:
        return np.arange(n)
    imgs = term_images(rows, terms)
    return np.lexsort(imgs[::-1])  # lexsort's last key is the primary one


def _py_project(v: int, t: Term) -> int:
    """One projection on a Python int, Rust semantics in the field's type."""
    op = t.operand
    if t.projection == "identity":
        return v
    if t.projection == "and":
        w = 8 * np.dtype(t.dtype).itemsize
        r = v & (op & ((1 << w) - 1))
        if np.dtype(t.dtype).kind == "i" and r >> (w - 1):
            r -= 1 << w
        return r
    if t.projection == "shr":
        return v >> op  # arithmetic for negative v, as Rust's i32 >>
    q = abs(v) // abs(op)
    if (v < 0) != (op < 0):
        q = -q  # truncating division
    return q if t.projection == "div" else v - op * q


def _total_key(bits: int, w: int) -> int:
    """f32::total_cmp / f64::total_cmp: flip the magnitude bits of negatives,
    then compare as signed integers."""
    s = bits - (1 << w) if bits >> (w - 1) else bits
    if s < 0:
        s ^= (1 << (w - 1)) - 1
    return s


def _cmp_term(a, b, t: Term) -> int:
    dt = np.dtype(t.dtype)
    if dt.kind != "f":
        c = (a > b) - (a < b)
    elif t.total:
        w = 8 * dt.itemsize
        ka, kb = _total_key(a[1], w), _total_key(b[1], w)
        c = (ka > kb) - (ka < kb)
    elif a[0] < b[0]:
        c = -1
    elif a[0] > b[0]:
        c = 1
    elif a[0] == b[0]:
        c = 0  # partial_cmp: -0.0 == +0.0
    else:
        # NaN: the radix order's place for it (its order image)
        ia, ib = a[2], b[2]
        c = (ia > ib) - (ia < ib)
    return -c if t.descending else c


def sort_by_cmp(rows: np.ndarray, terms: Sequence[Term]) -> np.ndarray:
    """Literal form: Python's stable sort (like Rust's slice::sort_by) with a
    comparator that walks the terms in order (Ordering::then_with).  Field
    values are projected with Python integers; floats compare as floats."""
    cols = []
    for t in terms:
        f = _field(rows, t)
        if f.dtype.kind == "f":
            bits = f.view(np.dtype(f"u{f.dtype.itemsize}")).tolist()
            img = _image(f, t._replace(descending=False)).tolist()
            cols.append(list(zip(f.astype(np.float64).tolist(), bits, img)))
        else:
            cols.append([_py_project(int(v), t) for v in f.tolist()])

    def cmp(i: int, j: int) -> int:
        for t, col in zip(terms, cols):
            c = _cmp_term(col[i], col[j], t)
            if c:
                return c
        return 0

    return np.array(sorted(range(rows.shape[0]), key=functools.cmp_to_key(cmp)), dtype=np.int64)


def as_rows(records: np.ndarray) -> np.ndarray:
    """(n, record_bytes) uint8 view of a record array (1-D scalars, 2-D rows
    or a structured array)."""
    a = np.ascontiguousarray(records)
    n = a.shape[0]
    return a.view(np.uint8).reshape(n, -1) if n else np.zeros((0, a.itemsize), np.uint8)
