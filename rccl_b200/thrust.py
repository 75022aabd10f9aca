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

from . import _lib
from .cub import (KEY_TYPES, BadArgument, ContextMismatch, Launch, Order, Program as CubProgram,
                  controls_counts, key_code, order_code, value_bytes_of)
from .errors import LengthMismatch, raise_for


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


def sort_by(execution: Execution, keys: torch.Tensor, order) -> None:
    """Stable in-place sort by a named order (DeviceSortExt::sort_by,
    ordering.rs:78-87; the reference lowers it to DeviceMergeSort).  `order`
    is a rccl_b200.cub.Order: the comparator closure itself is device code."""
    _radix_sort(execution, keys, order_code(order))


def sort_unstable_by(execution: Execution, keys: torch.Tensor, order) -> None:
    """DeviceSortExt::sort_unstable_by (ordering.rs:58-68); stable here."""
    _radix_sort(execution, keys, order_code(order))


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
        """DeviceKeyValueSortExt::sort_by (ordering.rs:170-181) by a named order."""
        _radix_sort_pairs(execution, self.keys, self.values, order_code(order))

    def sort_unstable_by(self, execution: Execution, order) -> None:
        _radix_sort_pairs(execution, self.keys, self.values, order_code(order))


class RangeError(ValueError):
    def __init__(self, first: int, second: int):
        self.first, self.second = first, second
        super().__init__(f"range lengths differ: {first} vs {second}")


def with_values(keys: torch.Tensor, values: torch.Tensor) -> KeyValueRangeMut:
    """DeviceViewMut::with_values (range.rs:158-163, length check :320-334)."""
    if keys.numel() != values.shape[0]:
        raise RangeError(keys.numel(), values.shape[0])
    return KeyValueRangeMut(keys, values)
