"""Host-side mirror of rccl-thrust's radix lowering over the B200 C ABI.

`sort` / `sort_unstable` on a key buffer and on `with_values(...)` pairs lower
to DeviceRadixSort exactly as in rccl-thrust/src/ordering.rs:46-168 and
rccl-thrust/src/backend.rs:8-110: one temporary byte block split into aligned
regions (scratch keys[, scratch values], bins, lookback, counters), the CUB
sort, release of the block, then a stream synchronization.  The comparator
forms `sort_by` / `sort_unstable_by` lower to DeviceMergeSort in the reference
(backend.rs:39-63, 112-150); here they take a named order (rccl_b200.cub.Order:
the comparator closure itself is device code) and give the stable sort by it.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib, compare
from .cub import (KEY_TYPES, BadArgument, ContextMismatch, Launch, Order, Program as CubProgram,
                  controls_counts, key_code, order_code, value_bytes_of)
from .errors import LengthMismatch, UnsupportedTarget, raise_for


def _align(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class Execution:
    """Stream + allocator binding (rccl_thrust::cuda::Execution)."""

    def __init__(self, launch: Launch):
        self.launch = launch

    @property
    def stream(self) -> torch.cuda.Stream:
        return self.launch.stream

    def synchronize(self) -> None:
        self.launch.stream.synchronize()


class Program:
    """rccl_thrust::cuda::Program (rccl-thrust/src/cuda.rs:80-122)."""

    def __init__(self, cub: CubProgram):
        self.cub = cub

    @staticmethod
    def load(device=None) -> "Program":
        return Program(CubProgram.load(device))

    def par(self, stream: Optional[torch.cuda.Stream] = None) -> Execution:
        return Execution(self.cub.on(stream))


class _Temporary:
    """One byte allocation split into aligned regions
    (rccl-memory TemporaryWorkspaceN, rccl-memory/src/temporary.rs:200-290)."""

    def __init__(self, device, sizes, alignments):
        offsets, off = [], 0
        for size, align in zip(sizes, alignments):
            off = _align(off, align)
            offsets.append(off)
            off += size
        self.block = torch.empty(max(off, 1), dtype=torch.uint8, device=device)
        self.base = self.block.data_ptr()
        self.offsets = offsets

    def ptr(self, i: int) -> int:
        return self.base + self.offsets[i]

    def zero(self, i: int, nbytes: int, stream: torch.cuda.Stream) -> None:
        """Zero one region on `stream` (the counters region holds the sticky
        device status word, which must start cleared)."""
        if nbytes:
            with torch.cuda.stream(stream):
                self.block[self.offsets[i]:self.offsets[i] + nbytes].zero_()


def _radix_sort(execution: Execution, keys: torch.Tensor, order: Optional[int] = None) -> None:
    """order: None for the radix lowering, else a named-order code for the
    sort_by lowering (the same temporaries and the same synchronization)."""
    launch = execution.launch
    launch.check(keys)
    code = key_code(keys.dtype)
    n, kb = keys.numel(), keys.element_size()
    nb, nl, nc = controls_counts(keys.dtype, 0, n)
    # backend.rs:16-28: regions scratch keys, bins, lookback, counters with
    # alignments 128, 256, 256, 256.
    tmp = _Temporary(launch.device, [n * kb, nb * 8, nl * 4, nc * 4], [128, 256, 256, 256])
    tmp.zero(3, nc * 4, launch.stream)
    if order is None:
        st = _lib.lib().rsort_keys(code, 0, keys.data_ptr(), tmp.ptr(0), n, n, tmp.ptr(1), nb,
                                   tmp.ptr(2), nl, tmp.ptr(3), nc, launch.handle)
    else:
        st = _lib.lib().rsort_merge_sort_keys(code, order, keys.data_ptr(), tmp.ptr(0), n, n,
                                              tmp.ptr(1), nb, tmp.ptr(2), nl, tmp.ptr(3), nc,
                                              launch.handle)
    raise_for(st)
    # backend.rs:33-36: release the block (stream-ordered by the caching
    # allocator), then synchronize.
    status = _lib.lib().rsort_check_device_status(tmp.ptr(3) if nc else None, nc, launch.handle)
    del tmp
    execution.synchronize()
    raise_for(status)


def _radix_sort_pairs(execution: Execution, keys: torch.Tensor, values: torch.Tensor,
                      order: Optional[int] = None) -> None:
    launch = execution.launch
    launch.check(keys, values)
    code = key_code(keys.dtype)
    n = keys.numel()
    # backend.rs:75-81
    if values.shape[0] != n:
        raise LengthMismatch("values", n, values.shape[0])
    kb, vb = keys.element_size(), value_bytes_of(values)
    nb, nl, nc = controls_counts(keys.dtype, vb, n)
    # backend.rs:82-96: alignments 128, 128, 256, 256, 256.
    tmp = _Temporary(launch.device, [n * kb, n * vb, nb * 8, nl * 4, nc * 4],
                     [128, 128, 256, 256, 256])
    tmp.zero(4, nc * 4, launch.stream)
    if order is None:
        st = _lib.lib().rsort_pairs(code, 0, keys.data_ptr(), values.data_ptr(), vb, tmp.ptr(0),
                                    n, tmp.ptr(1), n, n, tmp.ptr(2), nb, tmp.ptr(3), nl,
                                    tmp.ptr(4), nc, launch.handle)
    else:
        st = _lib.lib().rsort_merge_sort_pairs(code, order, keys.data_ptr(), values.data_ptr(),
                                               vb, tmp.ptr(0), n, tmp.ptr(1), n, n, tmp.ptr(2),
                                               nb, tmp.ptr(3), nl, tmp.ptr(4), nc, launch.handle)
    raise_for(st)
    status = _lib.lib().rsort_check_device_status(tmp.ptr(4) if nc else None, nc, launch.handle)
    del tmp
    execution.synchronize()
    raise_for(status)


def sort(execution: Execution, keys: torch.Tensor) -> None:
    """Stable in-place ascending sort (DeviceSortExt::sort, ordering.rs:70-76)."""
    _radix_sort(execution, keys)


def sort_unstable(execution: Execution, keys: torch.Tensor) -> None:
    """In-place ascending sort (DeviceSortExt::sort_unstable, ordering.rs:47-56)."""
    _radix_sort(execution, keys)


def _sort_by_program(execution: Execution, records: torch.Tensor,
                     values: Optional[torch.Tensor], order) -> None:
    """sort_by with a comparator program: one temporary block (the
    rsort_sort_by scratch), the sort, release, synchronization -- the same
    lowering shape as backend.rs:39-63."""
    launch = execution.launch
    launch.check(records, values)
    tmp = _Temporary(launch.device, [compare.scratch_bytes(records, values)], [256])
    compare.sort_by(records, values, order, tmp.block, launch.handle)
    del tmp
    execution.synchronize()


def sort_by(execution: Execution, keys: torch.Tensor, order) -> None:
    """Stable in-place sort by a comparator (DeviceSortExt::sort_by,
    ordering.rs:78-87; the reference lowers it to DeviceMergeSort).  `order`
    is a named order (rccl_b200.cub.Order) or a comparator program
    (rccl_b200.compare.Key / Comparator) over the rows of `keys`: the closure
    itself is device code."""
    if compare.is_program(order):
        _sort_by_program(execution, keys, None, order)
    else:
        _radix_sort(execution, keys, order_code(order))


def sort_unstable_by(execution: Execution, keys: torch.Tensor, order) -> None:
    """DeviceSortExt::sort_unstable_by (ordering.rs:58-68); stable here."""
    sort_by(execution, keys, order)


class KeyValueRangeMut:
    """with_values() pair range (rccl-thrust/src/range.rs:315-351)."""

    def __init__(self, keys: torch.Tensor, values: torch.Tensor):
        self.keys = keys
        self.values = values

    def sort(self, execution: Execution) -> None:
        _radix_sort_pairs(execution, self.keys, self.values)

    def sort_unstable(self, execution: Execution) -> None:
        _radix_sort_pairs(execution, self.keys, self.values)

    def sort_by(self, execution: Execution, order) -> None:
        """DeviceKeyValueSortExt::sort_by (ordering.rs:170-181) by a named
        order or a comparator program over the key rows."""
        if compare.is_program(order):
            _sort_by_program(execution, self.keys, self.values, order)
        else:
            _radix_sort_pairs(execution, self.keys, self.values, order_code(order))

    def sort_unstable_by(self, execution: Execution, order) -> None:
        self.sort_by(execution, order)


class RangeError(ValueError):
    def __init__(self, first: int, second: int):
        self.first, self.second = first, second
        super().__init__(f"range lengths differ: {first} vs {second}")


def with_values(keys: torch.Tensor, values: torch.Tensor) -> KeyValueRangeMut:
    """DeviceViewMut::with_values (range.rs:158-163, length check :320-334).
    Keys may be record rows (an (n, ...) tensor) for a comparator program."""
    n = keys.shape[0] if keys.dim() else keys.numel()
    if n != values.shape[0]:
        raise RangeError(n, values.shape[0])
    return KeyValueRangeMut(keys, values)


# ---------------------------------------------------------------------------
# Lexicographic record sort (rccl-thrust/src/record_sort.rs:144-300)
# ---------------------------------------------------------------------------
_ROW_PAYLOADS = (torch.uint64, torch.int64, torch.float64, torch.bool, torch.uint8)


def _sort_rows(execution: Execution, rows: torch.Tensor,
               payload: Optional[torch.Tensor]) -> None:
    """Stable ascending lexicographic sort of (n, N) uint32 rows in place,
    payload rows in lockstep: multi-word LSD radix (rsort_rows_lexicographic)
    with a temporary block, then a stream synchronization."""
    launch = execution.launch
    launch.check(rows, payload)
    if rows.dim() != 2 or rows.dtype not in (torch.uint32, torch.int32):
        raise BadArgument("rows must be an (n, N) uint32 tensor")
    n, arity = rows.shape
    # record_sort.rs:118-126
    if not 2 <= arity <= 6:
        raise UnsupportedTarget("record sort supports audited workload arities 2 through 6; "
                                "use radix sort for scalar keys")
    pb = 0
    if payload is not None:
        # record_sort.rs:128-141 and the sealed payload set (:24-31)
        if payload.shape[0] != n:
            raise LengthMismatch("record payloads", n, payload.shape[0])
        if payload.dtype not in _ROW_PAYLOADS or payload.dim() != 1:
            raise BadArgument("payloads: u64, f64 or Boolean provenance, one per row")
        pb = payload.element_size()
    lib = _lib.lib()
    nbytes = lib.rsort_rows_scratch_bytes(arity, pb, n)
    tmp = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=launch.device)
    st = lib.rsort_rows_lexicographic(arity, rows.data_ptr(),
                                      None if payload is None else payload.data_ptr(), pb, n,
                                      tmp.data_ptr(), nbytes, launch.handle)
    raise_for(st)
    del tmp
    execution.synchronize()


def sort_rows_lexicographic(execution: Execution, rows: torch.Tensor) -> None:
    """record_sort.rs:176-184"""
    _sort_rows(execution, rows, None)


def sort_rows_lexicographic_into(execution: Execution, input: torch.Tensor,
                                 output: torch.Tensor) -> None:
    """Stable out-of-place row sort (record_sort.rs:186-221)."""
    if output.shape != input.shape:
        raise LengthMismatch("record output", input.shape[0], output.shape[0])
    with torch.cuda.stream(execution.stream):
        output.copy_(input)
    _sort_rows(execution, output, None)


def sort_rows_with_payload_lexicographic(execution: Execution, rows: torch.Tensor,
                                         payloads: torch.Tensor) -> None:
    """record_sort.rs:223-271"""
    _sort_rows(execution, rows, payloads)


def sort_rows_with_payload_lexicographic_into(execution: Execution, rows: torch.Tensor,
                                              payloads: torch.Tensor, rows_out: torch.Tensor,
                                              payloads_out: torch.Tensor) -> None:
    """Stable out-of-place row/payload sort (record_sort.rs:273-300)."""
    if rows_out.shape != rows.shape:
        raise LengthMismatch("record output", rows.shape[0], rows_out.shape[0])
    if payloads_out.shape != payloads.shape:
        raise LengthMismatch("record payload output", payloads.shape[0], payloads_out.shape[0])
    with torch.cuda.stream(execution.stream):
        rows_out.copy_(rows)
        payloads_out.copy_(payloads)
    _sort_rows(execution, rows_out, payloads_out)
