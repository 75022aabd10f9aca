"""Comparator programs for DeviceMergeSort / Thrust sort_by.

rccl-cub's merge sort (rccl-cub/src/dispatch.rs:170-193, 1113-1146) and
rccl-thrust's sort_by lowering (rccl-thrust/src/backend.rs:39-63) take any
`Fn(&K, &K) -> Ordering` closure.  A closure is device code and cannot cross
the C ABI, but the closures the reference's callers write are key projections
chained with `then_with` and optionally reversed.  A comparator program states
such a closure as data, and `rsort_sort_by` sorts by it stably:

    |l, r| (l & 1).cmp(&(r & 1)).then_with(|| l.cmp(r))
        Key(torch.int32).and_(1).then(Key(torch.int32))
    |l, r| (l / 10).cmp(&(r / 10))        Key(torch.int32).div(10)
    |l, r| r.cmp(l)                       Key(torch.int32).reverse()
    |l, r| l.total_cmp(r)                 Key(torch.float32).total()
    |l, r| l.key.cmp(&r.key)   (KeyValue<u32, u32>, #[repr(C)])
        Key(torch.uint32, offset=0)      records: an (n, 2) uint32 tensor

Records are the rows of a tensor: a 1-D tensor's elements, or the rows of an
(n, ...) tensor (any dtype; one row = one record of row bytes).  Fields may
sit at any byte offset.  Integer projections follow Rust's integer semantics
in the field's type (`>>` is arithmetic for signed fields, `/` and `%`
truncate); floats compare by partial_cmp (-0.0 == +0.0) or total_cmp.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace
from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from .errors import BadArgument, LengthMismatch, raise_for

PROJECTIONS = {"identity": _lib.RSORT_PROJ_IDENTITY, "and": _lib.RSORT_PROJ_AND,
               "shr": _lib.RSORT_PROJ_SHR, "div": _lib.RSORT_PROJ_DIV,
               "rem": _lib.RSORT_PROJ_REM}
# rsort_order_t
_ASC, _DESC, _TOTAL_ASC, _TOTAL_DESC = 0, 1, 2, 3


@dataclass(frozen=True)
class Key:
    """One term: the `dtype` field at byte `offset` of the record, projected,
    compared ascending unless reversed."""
    dtype: torch.dtype
    offset: int = 0
    projection: str = "identity"
    operand: int = 0
    descending: bool = False
    total_order: bool = False

    def _project(self, name: str, operand: int) -> "Key":
        if self.projection != "identity":
            raise BadArgument(f"one projection per term ({self.projection} then {name})")
        return replace(self, projection=name, operand=int(operand))

    def and_(self, mask: int) -> "Key":
        """(v & mask)"""
        return self._project("and", mask)

    def shr(self, shift: int) -> "Key":
        """(v >> shift)"""
        return self._project("shr", shift)

    def div(self, divisor: int) -> "Key":
        """(v / divisor), truncating"""
        return self._project("div", divisor)

    def rem(self, divisor: int) -> "Key":
        """(v % divisor), the dividend's sign"""
        return self._project("rem", divisor)

    def reverse(self) -> "Key":
        """r.cmp(l): this term descending"""
        return replace(self, descending=not self.descending)

    def total(self) -> "Key":
        """total_cmp instead of partial_cmp (floats: -0.0 < +0.0)"""
        return replace(self, total_order=True)

    def then(self, *more) -> "Comparator":
        """.then_with(|| more...)"""
        return Comparator((self,)).then(*more)

    @property
    def terms(self) -> Tuple["Key", ...]:
        return (self,)

    def order_code(self) -> int:
        if self.total_order:
            return _TOTAL_DESC if self.descending else _TOTAL_ASC
        return _DESC if self.descending else _ASC


@dataclass(frozen=True)
class Comparator:
    """A chain of terms, most significant first (nothing = all equal)."""
    terms: Tuple[Key, ...] = ()

    def then(self, *more) -> "Comparator":
        out = list(self.terms)
        for m in more:
            if not isinstance(m, (Key, Comparator)):
                raise BadArgument(f"not a comparator term: {m!r}")
            out.extend(m.terms)
        return Comparator(tuple(out))

    def reverse(self) -> "Comparator":
        """|l, r| cmp(r, l): every term reversed"""
        return Comparator(tuple(t.reverse() for t in self.terms))


def is_program(order) -> bool:
    return isinstance(order, (Key, Comparator))


def _type_code(dtype: torch.dtype) -> int:
    from .cub import key_code
    return key_code(dtype)


def c_terms(order) -> ctypes.Array:
    """The rsort_compare_term array of a Key or Comparator."""
    terms = order.terms
    if len(terms) > _lib.RSORT_MAX_TERMS:
        raise BadArgument(f"at most {_lib.RSORT_MAX_TERMS} comparator terms, got {len(terms)}")
    arr = (_lib.CompareTerm * max(len(terms), 1))()
    for i, t in enumerate(terms):
        if t.offset < 0:
            raise BadArgument("negative field offset")
        arr[i].offset = t.offset
        arr[i].type = _type_code(t.dtype)
        arr[i].projection = PROJECTIONS[t.projection]
        arr[i].order = t.order_code()
        arr[i].operand = _as_i64(t.operand)
    return arr


def _as_i64(v: int) -> int:
    """Operands up to 2^64 - 1 (u64 masks) travel as their 64-bit pattern."""
    if not -(1 << 63) <= v < (1 << 64):
        raise BadArgument(f"operand {v} does not fit 64 bits")
    return v - (1 << 64) if v >= (1 << 63) else v


def record_bytes_of(records: torch.Tensor) -> int:
    if records.dim() == 0:
        raise BadArgument("records must have a leading record dimension")
    if not records.is_contiguous():
        raise BadArgument("records must be contiguous")
    n = records.shape[0]
    per = records[0].numel() if n else int(torch.Size(records.shape[1:]).numel())
    return per * records.element_size()


def scratch_bytes(records: torch.Tensor, values: Optional[torch.Tensor] = None) -> int:
    vb = record_bytes_of(values) if values is not None else 0
    return _lib.lib().rsort_sort_by_scratch_bytes(record_bytes_of(records), vb,
                                                  records.shape[0])


def sort_by(records: torch.Tensor, values: Optional[torch.Tensor], order, scratch: torch.Tensor,
            stream_handle: int) -> None:
    """Stable in-place sort of `records` (and `values` in lockstep) by the
    comparator program `order` through rsort_sort_by; `scratch` holds at
    least scratch_bytes(records, values) bytes on the records' device."""
    if not is_program(order):
        raise BadArgument(f"not a comparator program: {order!r}")
    n = records.shape[0] if records.dim() else 0
    rb = record_bytes_of(records)
    vb = 0
    if values is not None:
        if values.shape[0] != n:
            raise LengthMismatch("sort_by values", n, values.shape[0])
        vb = record_bytes_of(values)
    terms = c_terms(order)
    raise_for(_lib.lib().rsort_sort_by(
        terms, len(order.terms), records.data_ptr() if n else None, rb,
        values.data_ptr() if values is not None and n else None, vb, n,
        scratch.data_ptr() if scratch.numel() else None, scratch.numel() * scratch.element_size(),
        stream_handle))


__all__ = ["Key", "Comparator", "is_program", "sort_by", "scratch_bytes", "record_bytes_of",
           "c_terms"]
