"""Host-side mirror of rccl-cub's DeviceRadixSort API over the B200 C ABI.

Same function names, argument meaning and error behaviour as the reference's
public radix functions (rccl-cub/src/dispatch.rs:2091-2942), workspace types
(rccl-cub/src/workspace.rs:126-174, 581-706), DoubleBuffer
(rccl-cub/src/double_buffer.rs:6-130) and Program/Launch binding
(rccl-cub/src/cuda.rs:741-771).  Device memory is torch CUDA storage; every
sort runs in librsort_b200.so on the launch's stream and is asynchronous, as
in the reference.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _lib, compare
from .errors import (BadArgument, DeviceAlgorithmError, LengthMismatch, raise_for)

KEY_TYPES = {
    torch.uint32: _lib.RSORT_U32,
    torch.int32: _lib.RSORT_I32,
    torch.float32: _lib.RSORT_F32,
    torch.uint64: _lib.RSORT_U64,
    torch.int64: _lib.RSORT_I64,
    torch.float64: _lib.RSORT_F64,
}
# Small keys (no reference counterpart; the reference lists them as missing):
# accepted by the single-GPU radix and named-order sorts.
SMALL_KEY_TYPES = {
    torch.uint8: _lib.RSORT_U8,
    torch.int8: _lib.RSORT_I8,
    torch.uint16: _lib.RSORT_U16,
    torch.int16: _lib.RSORT_I16,
    torch.float16: _lib.RSORT_F16,
    torch.bfloat16: _lib.RSORT_BF16,
}
KEY_BITS = {k: torch.empty(0, dtype=k).element_size() * 8
            for k in list(KEY_TYPES) + list(SMALL_KEY_TYPES)}


class ContextMismatch(DeviceAlgorithmError):
    """A buffer or stream belongs to another device (rccl-cub/src/cuda.rs:763-765)."""


def key_code(dtype: torch.dtype) -> int:
    try:
        return KEY_TYPES[dtype] if dtype in KEY_TYPES else SMALL_KEY_TYPES[dtype]
    except KeyError:
        raise BadArgument(f"{dtype} is not a RadixKey (u32/i32/f32/u64/i64/f64, or "
                          "u8/i8/u16/i16/f16/bf16)") from None


def value_bytes_of(t: torch.Tensor) -> int:
    """Width of one value item: a 1-D tensor's element size, or the row bytes
    of a 2-D (n, w) uint8 tensor (w = 1, 2, 4, 8 or 16)."""
    if t.dim() == 1:
        return t.element_size()
    if t.dim() == 2 and t.dtype == torch.uint8:
        return t.shape[1]
    raise BadArgument("values must be 1-D, or 2-D uint8 rows")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


class Launch:
    """A stream bound to a loaded program (rccl_cub::cuda::Launch)."""

    def __init__(self, device: torch.device, stream: torch.cuda.Stream):
        self.device = device
        self.stream = stream

    @property
    def handle(self) -> int:
        return self.stream.cuda_stream

    def check(self, *tensors: Optional[torch.Tensor]) -> None:
        for t in tensors:
            if t is None:
                continue
            if t.device != self.device:
                raise ContextMismatch(f"tensor on {t.device}, launch on {self.device}")
            if not t.is_contiguous():
                raise BadArgument("device ranges must be contiguous")


class Program:
    """The loaded radix-sort library bound to one device (rccl_cub::cuda::Program)."""

    def __init__(self, device: torch.device):
        self.device = device

    @staticmethod
    def load(device=None) -> "Program":
        _lib.lib()
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        if device.type != "cuda":
            raise ContextMismatch(f"{device} is not a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        return Program(device)

    def on(self, stream: Optional[torch.cuda.Stream] = None) -> Launch:
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        if stream.device != self.device:
            raise ContextMismatch(f"stream on {stream.device}, program on {self.device}")
        return Launch(self.device, stream)


# ---------------------------------------------------------------------------
# DoubleBuffer
# ---------------------------------------------------------------------------
class DoubleBuffer:
    """Two same-shaped ranges used by ping-pong sorts.  For pairs each side is
    a (keys, values) tuple and one selector covers both."""

    def __init__(self, first, second, current_is_first: bool = True):
        self.first = first
        self.second = second
        self._current_is_first = bool(current_is_first)

    @staticmethod
    def new(first: torch.Tensor, second: torch.Tensor) -> Optional["DoubleBuffer"]:
        if first.numel() != second.numel():
            return None
        return DoubleBuffer(first, second)

    @staticmethod
    def paired(first: Tuple[torch.Tensor, torch.Tensor],
               second: Tuple[torch.Tensor, torch.Tensor]) -> Optional["DoubleBuffer"]:
        n = first[0].shape[0]
        if first[1].shape[0] != n or second[0].shape[0] != n or second[1].shape[0] != n:
            return None
        return DoubleBuffer(tuple(first), tuple(second))

    def __len__(self) -> int:
        side = self.first[0] if isinstance(self.first, tuple) else self.first
        return side.shape[0]

    def current_is_first(self) -> bool:
        return self._current_is_first

    def current(self):
        return self.first if self._current_is_first else self.second

    def alternate(self):
        return self.second if self._current_is_first else self.first

    def swap(self) -> None:
        self._current_is_first = not self._current_is_first


# ---------------------------------------------------------------------------
# Workspaces (caller-owned device memory; the sort itself never allocates)
# ---------------------------------------------------------------------------
def controls_counts(key_dtype: torch.dtype, value_bytes: int, n: int) -> Tuple[int, int, int]:
    out = _lib.Controls()
    raise_for(_lib.lib().rsort_controls_query(key_code(key_dtype), value_bytes, n,
                                              ctypes.byref(out)))
    return out.bins, out.lookback, out.counters


@dataclass
class DeviceRadixSortBufferWorkspace:
    """bins (u64), lookback (i32), counters (i32): workspace.rs:581-610."""
    bins: torch.Tensor
    lookback: torch.Tensor
    counters: torch.Tensor

    def args(self):
        return (self.bins.data_ptr(), self.bins.numel(), self.lookback.data_ptr(),
                self.lookback.numel(), self.counters.data_ptr(), self.counters.numel())


@dataclass
class DeviceRadixSortKeysWorkspace:
    scratch_keys: torch.Tensor
    controls: DeviceRadixSortBufferWorkspace


@dataclass
class DeviceRadixSortPairsWorkspace:
    scratch_keys: torch.Tensor
    scratch_values: torch.Tensor
    controls: DeviceRadixSortBufferWorkspace


def _controls_for(launch: Launch, key_dtype, value_bytes: int, n: int):
    nb, nl, nc = controls_counts(key_dtype, value_bytes, n)
    dev = launch.device
    return DeviceRadixSortBufferWorkspace(
        bins=torch.zeros(nb, dtype=torch.int64, device=dev),
        lookback=torch.zeros(nl, dtype=torch.int32, device=dev),
        counters=torch.zeros(nc, dtype=torch.int32, device=dev))


def device_radix_sort_keys_buffer_workspace(launch: Launch, key_dtype: torch.dtype,
                                            n: int) -> DeviceRadixSortBufferWorkspace:
    return _controls_for(launch, key_dtype, 0, n)


def device_radix_sort_pairs_buffer_workspace(launch: Launch, key_dtype: torch.dtype,
                                             value_dtype, n: int) -> DeviceRadixSortBufferWorkspace:
    return _controls_for(launch, key_dtype, _value_width(value_dtype), n)


def device_radix_sort_workspace(launch: Launch, key_dtype: torch.dtype,
                                n: int) -> DeviceRadixSortKeysWorkspace:
    """In-place keys workspace (rccl_cub::device_radix_sort_workspace)."""
    return DeviceRadixSortKeysWorkspace(
        scratch_keys=torch.zeros(n, dtype=key_dtype, device=launch.device),
        controls=_controls_for(launch, key_dtype, 0, n))


device_radix_sort_keys_workspace = device_radix_sort_workspace


def device_radix_sort_pairs_workspace(launch: Launch, key_dtype: torch.dtype, value_dtype,
                                      n: int) -> DeviceRadixSortPairsWorkspace:
    vb = _value_width(value_dtype)
    if isinstance(value_dtype, torch.dtype):
        sv = torch.zeros(n, dtype=value_dtype, device=launch.device)
    else:
        sv = torch.zeros((n, vb), dtype=torch.uint8, device=launch.device)
    return DeviceRadixSortPairsWorkspace(
        scratch_keys=torch.zeros(n, dtype=key_dtype, device=launch.device),
        scratch_values=sv,
        controls=_controls_for(launch, key_dtype, vb, n))


def _value_width(value_dtype) -> int:
    if isinstance(value_dtype, torch.dtype):
        return torch.empty(0, dtype=value_dtype).element_size()
    return int(value_dtype)  # raw byte width for (n, w) uint8 rows


# ---------------------------------------------------------------------------
# Sorts
# ---------------------------------------------------------------------------
def _keys_inplace(launch: Launch, keys: torch.Tensor, ws: DeviceRadixSortKeysWorkspace,
                  descending: bool) -> None:
    launch.check(keys, ws.scratch_keys)
    code = key_code(keys.dtype)
    st = _lib.lib().rsort_keys(code, int(descending), keys.data_ptr(), ws.scratch_keys.data_ptr(),
                               ws.scratch_keys.numel(), keys.numel(), *ws.controls.args(),
                               launch.handle)
    raise_for(st)


def device_radix_sort_keys(launch: Launch, keys: torch.Tensor,
                           workspace: DeviceRadixSortKeysWorkspace) -> None:
    """Sort keys in ascending radix order (dispatch.rs:2091-2114)."""
    _keys_inplace(launch, keys, workspace, False)


def device_radix_sort_keys_descending(launch: Launch, keys: torch.Tensor,
                                      workspace: DeviceRadixSortKeysWorkspace) -> None:
    """Sort keys in descending radix order (dispatch.rs:2117-2140)."""
    _keys_inplace(launch, keys, workspace, True)


def _keys_buffer(launch: Launch, buffers: DoubleBuffer, bit_range: range,
                 ws: DeviceRadixSortBufferWorkspace, descending: bool) -> None:
    first, second = buffers.first, buffers.second
    launch.check(first, second)
    code = key_code(first.dtype)
    if second.dtype != first.dtype:
        raise BadArgument("DoubleBuffer sides differ in key type")
    sel = ctypes.c_int(1 if buffers.current_is_first() else 0)
    st = _lib.lib().rsort_keys_buffer(code, int(descending), first.data_ptr(), second.data_ptr(),
                                      len(buffers), bit_range.start, bit_range.stop,
                                      ctypes.byref(sel), *ws.args(), launch.handle)
    raise_for(st)
    buffers._current_is_first = bool(sel.value)


def device_radix_sort_keys_buffer(launch: Launch, buffers: DoubleBuffer, bit_range: range,
                                  workspace: DeviceRadixSortBufferWorkspace) -> None:
    """DoubleBuffer keys sort over bits [start, stop) (dispatch.rs:2251-2274)."""
    _keys_buffer(launch, buffers, bit_range, workspace, False)


def device_radix_sort_keys_buffer_descending(launch: Launch, buffers: DoubleBuffer,
                                             bit_range: range,
                                             workspace: DeviceRadixSortBufferWorkspace) -> None:
    _keys_buffer(launch, buffers, bit_range, workspace, True)


def _pairs_inplace(launch: Launch, keys: torch.Tensor, values: torch.Tensor,
                   ws: DeviceRadixSortPairsWorkspace, descending: bool) -> None:
    launch.check(keys, values, ws.scratch_keys, ws.scratch_values)
    code = key_code(keys.dtype)
    # rccl-cub/src/radix.rs:823-831
    if values.shape[0] != keys.numel():
        raise LengthMismatch("radix values", keys.numel(), values.shape[0])
    vb = value_bytes_of(values)
    if value_bytes_of(ws.scratch_values) != vb:
        raise BadArgument("scratch values width differs from values")
    st = _lib.lib().rsort_pairs(code, int(descending), keys.data_ptr(), values.data_ptr(), vb,
                                ws.scratch_keys.data_ptr(), ws.scratch_keys.numel(),
                                ws.scratch_values.data_ptr(), ws.scratch_values.shape[0],
                                keys.numel(), *ws.controls.args(), launch.handle)
    raise_for(st)


def device_radix_sort_pairs(launch: Launch, keys: torch.Tensor, values: torch.Tensor,
                            workspace: DeviceRadixSortPairsWorkspace) -> None:
    """Stable key/value sort, ascending (dispatch.rs:2546-2576)."""
    _pairs_inplace(launch, keys, values, workspace, False)


def device_radix_sort_pairs_descending(launch: Launch, keys: torch.Tensor, values: torch.Tensor,
                                       workspace: DeviceRadixSortPairsWorkspace) -> None:
    _pairs_inplace(launch, keys, values, workspace, True)


def _pairs_buffer(launch: Launch, buffers: DoubleBuffer, bit_range: range,
                  ws: DeviceRadixSortBufferWorkspace, descending: bool) -> None:
    (fk, fv), (sk, sv) = buffers.first, buffers.second
    launch.check(fk, fv, sk, sv)
    code = key_code(fk.dtype)
    vb = value_bytes_of(fv)
    if value_bytes_of(sv) != vb or sk.dtype != fk.dtype:
        raise BadArgument("DoubleBuffer sides differ in layout")
    sel = ctypes.c_int(1 if buffers.current_is_first() else 0)
    st = _lib.lib().rsort_pairs_buffer(code, int(descending), fk.data_ptr(), sk.data_ptr(),
                                       fv.data_ptr(), sv.data_ptr(), vb, len(buffers),
                                       bit_range.start, bit_range.stop, ctypes.byref(sel),
                                       *ws.args(), launch.handle)
    raise_for(st)
    buffers._current_is_first = bool(sel.value)


def device_radix_sort_pairs_buffer(launch: Launch, buffers: DoubleBuffer, bit_range: range,
                                   workspace: DeviceRadixSortBufferWorkspace) -> None:
    """Paired DoubleBuffer sort over bits [start, stop) (dispatch.rs:2846-2894)."""
    _pairs_buffer(launch, buffers, bit_range, workspace, False)


def device_radix_sort_pairs_buffer_descending(launch: Launch, buffers: DoubleBuffer,
                                              bit_range: range,
                                              workspace: DeviceRadixSortBufferWorkspace) -> None:
    _pairs_buffer(launch, buffers, bit_range, workspace, True)


def check_device_status(launch: Launch, controls: DeviceRadixSortBufferWorkspace) -> None:
    """Synchronize the launch's stream and raise DeviceTimeout if a bounded
    device wait of an earlier sort on these controls gave up."""
    st = _lib.lib().rsort_check_device_status(
        controls.counters.data_ptr() if controls.counters.numel() else None,
        controls.counters.numel(), launch.handle)
    raise_for(st)


def single_tile_items(key_dtype: torch.dtype, value_bytes: int = 0) -> int:
    return _lib.lib().rsort_single_tile_items(key_code(key_dtype), value_bytes)


def selector_flips(key_dtype: torch.dtype, value_bytes: int, n: int, bit_range: range) -> int:
    return _lib.lib().rsort_selector_flips(key_code(key_dtype), value_bytes, n,
                                           bit_range.start, bit_range.stop)


# ---------------------------------------------------------------------------
# DeviceMergeSort / DeviceMerge for named orders
# ---------------------------------------------------------------------------
class Order(enum.IntEnum):
    """The comparators rccl-cub's merge sort is almost always given
    (its `order: F` closure, dispatch.rs:170-175), by name:
      ASCENDING         |a, b| a.cmp(b); floats partial_cmp, -0.0 == +0.0
      DESCENDING        |a, b| b.cmp(a)
      TOTAL_ASCENDING   |a, b| a.total_cmp(b): -0.0 < +0.0, NaNs by sign/payload
      TOTAL_DESCENDING  |a, b| b.total_cmp(a)
    A closure itself is device code and cannot cross the C ABI."""
    ASCENDING = 0
    DESCENDING = 1
    TOTAL_ASCENDING = 2
    TOTAL_DESCENDING = 3


def order_code(order) -> int:
    if isinstance(order, Order):
        return int(order)
    if isinstance(order, str):
        try:
            return int(Order[order.upper()])
        except KeyError:
            pass
    if callable(order):
        raise NotImplementedError(
            "a comparator closure is device code; pass one of rccl_b200.cub.Order "
            "(ASCENDING, DESCENDING, TOTAL_ASCENDING, TOTAL_DESCENDING) or a comparator "
            "program (rccl_b200.compare.Key / Comparator)")
    raise BadArgument(f"unknown sort order {order!r}")


def device_merge_sort_keys_workspace(launch: Launch, key_dtype: torch.dtype,
                                     n: int) -> DeviceRadixSortKeysWorkspace:
    """Workspace of device_merge_sort_keys (workspace.rs:253-267): scratch keys
    and the radix controls (the named orders run on the radix path)."""
    return device_radix_sort_workspace(launch, key_dtype, n)


def device_merge_sort_pairs_workspace(launch: Launch, key_dtype: torch.dtype, value_dtype,
                                      n: int) -> DeviceRadixSortPairsWorkspace:
    """Workspace of device_merge_sort_pairs (workspace.rs:269-286)."""
    return device_radix_sort_pairs_workspace(launch, key_dtype, value_dtype, n)


@dataclass
class DeviceMergeSortByWorkspace:
    """Scratch of a sort by a comparator program (rsort_sort_by_scratch_bytes):
    packed term keys, the index permutation, radix controls and the staging
    of records and values."""
    scratch: torch.Tensor


def device_merge_sort_by_workspace(launch: Launch, records: torch.Tensor,
                                   values: Optional[torch.Tensor] = None
                                   ) -> DeviceMergeSortByWorkspace:
    """Workspace of device_merge_sort_keys / _pairs with a comparator program
    (rccl_b200.compare) over these records (and values)."""
    nbytes = compare.scratch_bytes(records, values)
    return DeviceMergeSortByWorkspace(
        torch.empty(max(nbytes, 1), dtype=torch.uint8, device=launch.device))


def _sort_by_program(launch: Launch, keys, values, workspace, order) -> None:
    if not isinstance(workspace, DeviceMergeSortByWorkspace):
        raise BadArgument("a comparator program needs device_merge_sort_by_workspace")
    launch.check(keys, values, workspace.scratch)
    compare.sort_by(keys, values, order, workspace.scratch, launch.handle)


def device_merge_sort_keys(launch: Launch, keys: torch.Tensor, workspace, order) -> None:
    """Stable in-place sort by a named order or a comparator program
    (dispatch.rs:170-193).  Records of a comparator program are the rows of
    `keys` (any dtype and row shape)."""
    if compare.is_program(order):
        _sort_by_program(launch, keys, None, workspace, order)
        return
    code = order_code(order)
    launch.check(keys, workspace.scratch_keys)
    raise_for(_lib.lib().rsort_merge_sort_keys(
        key_code(keys.dtype), code, keys.data_ptr(), workspace.scratch_keys.data_ptr(),
        workspace.scratch_keys.numel(), keys.numel(), *workspace.controls.args(), launch.handle))


def device_merge_sort_pairs(launch: Launch, keys: torch.Tensor, values: torch.Tensor,
                            workspace, order) -> None:
    """Stable in-place key/value sort by a named order or a comparator program
    (dispatch.rs:1113-1146)."""
    if compare.is_program(order):
        _sort_by_program(launch, keys, values, workspace, order)
        return
    code = order_code(order)
    launch.check(keys, values, workspace.scratch_keys, workspace.scratch_values)
    if values.shape[0] != keys.numel():
        raise LengthMismatch("merge sort values", keys.numel(), values.shape[0])
    vb = value_bytes_of(values)
    if value_bytes_of(workspace.scratch_values) != vb:
        raise BadArgument("scratch values width differs from values")
    raise_for(_lib.lib().rsort_merge_sort_pairs(
        key_code(keys.dtype), code, keys.data_ptr(), values.data_ptr(), vb,
        workspace.scratch_keys.data_ptr(), workspace.scratch_keys.numel(),
        workspace.scratch_values.data_ptr(), workspace.scratch_values.shape[0], keys.numel(),
        *workspace.controls.args(), launch.handle))


@dataclass
class DeviceMergeWorkspace:
    """Merge-path partitions of a two-run merge (workspace.rs:223-233, 413-420)."""
    partitions: torch.Tensor


def device_merge_workspace(launch: Launch, first_len: int, second_len: int) -> DeviceMergeWorkspace:
    words = _lib.lib().rsort_merge_partition_words(first_len + second_len)
    return DeviceMergeWorkspace(torch.zeros(max(words, 1), dtype=torch.int64, device=launch.device))


def _merge(launch, fk, fv, sk, sv, ws, ok, ov, order) -> None:
    code = order_code(order)
    launch.check(fk, sk, ok, fv, sv, ov)
    if fk.dtype != sk.dtype or ok.dtype != fk.dtype:
        raise BadArgument("merge inputs and output differ in key type")
    na, nb = fk.numel(), sk.numel()
    if ok.numel() != na + nb:
        raise LengthMismatch("merge output", na + nb, ok.numel())
    vb = 0
    if fv is not None:
        vb = value_bytes_of(fv)
        if fv.shape[0] != na or sv.shape[0] != nb or ov.shape[0] != na + nb:
            raise LengthMismatch("merge values", na + nb, ov.shape[0])
    raise_for(_lib.lib().rsort_merge_ordered(
        key_code(fk.dtype), code, fk.data_ptr() if na else None, _ptr(fv) if na else None, na,
        sk.data_ptr() if nb else None, _ptr(sv) if nb else None, nb, ok.data_ptr(), _ptr(ov), vb,
        ws.partitions.data_ptr(), ws.partitions.numel(), launch.handle))


def device_merge_keys(launch: Launch, first: torch.Tensor, second: torch.Tensor,
                      workspace: DeviceMergeWorkspace, output: torch.Tensor, order) -> None:
    """Merge two sorted key ranges; ties take `first` (dispatch.rs:1570-1601)."""
    _merge(launch, first, None, second, None, workspace, output, None, order)


def device_merge_pairs(launch: Launch, first_keys, first_values, second_keys, second_values,
                       workspace: DeviceMergeWorkspace, output_keys, output_values, order) -> None:
    """Merge two sorted key/value ranges (dispatch.rs:1913-1960)."""
    _merge(launch, first_keys, first_values, second_keys, second_values, workspace, output_keys,
           output_values, order)


# ---------------------------------------------------------------------------
# Segmented radix sort (no reference counterpart; listed missing there)
# ---------------------------------------------------------------------------
def _segmented(launch: Launch, keys_in, keys_out, values_in, values_out, begin_offsets,
               end_offsets, bit_range: Optional[range], descending: bool) -> None:
    launch.check(keys_in, keys_out, values_in, values_out, begin_offsets, end_offsets)
    if keys_out.dtype != keys_in.dtype or keys_out.numel() != keys_in.numel():
        raise LengthMismatch("segmented keys out", keys_in.numel(), keys_out.numel())
    code = key_code(keys_in.dtype)
    n = keys_in.numel()
    nseg = begin_offsets.numel()
    if end_offsets.numel() != nseg:
        raise LengthMismatch("segment end offsets", nseg, end_offsets.numel())
    if begin_offsets.dtype not in (torch.int64, torch.uint64) or \
            end_offsets.dtype not in (torch.int64, torch.uint64):
        raise BadArgument("segment offsets must be 64-bit")
    vb = 0
    if values_in is not None:
        vb = value_bytes_of(values_in)
        if values_in.shape[0] != n or values_out.shape[0] != n:
            raise LengthMismatch("segmented values", n, values_in.shape[0])
    bits = KEY_BITS[keys_in.dtype]
    rng = bit_range if bit_range is not None else range(0, bits)
    lib = _lib.lib()
    nbytes = lib.rsort_segmented_scratch_bytes(code, vb, n, nseg)
    tmp = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=launch.device)
    raise_for(lib.rsort_segmented_sort(
        code, int(descending), keys_in.data_ptr(), keys_out.data_ptr(), _ptr(values_in),
        _ptr(values_out), vb, n, nseg, begin_offsets.data_ptr(), end_offsets.data_ptr(),
        rng.start, rng.stop, tmp.data_ptr(), nbytes, launch.handle))
    # the launches that read the scratch are ordered before its release on
    # this stream (caching allocator)
    del tmp


def device_segmented_radix_sort_keys(launch: Launch, keys_in, keys_out, begin_offsets,
                                     end_offsets, bit_range: Optional[range] = None) -> None:
    """Stable ascending sort of every segment [begin_offsets[i], end_offsets[i])."""
    _segmented(launch, keys_in, keys_out, None, None, begin_offsets, end_offsets, bit_range, False)


def device_segmented_radix_sort_keys_descending(launch: Launch, keys_in, keys_out, begin_offsets,
                                                end_offsets, bit_range=None) -> None:
    _segmented(launch, keys_in, keys_out, None, None, begin_offsets, end_offsets, bit_range, True)


def device_segmented_radix_sort_pairs(launch: Launch, keys_in, keys_out, values_in, values_out,
                                      begin_offsets, end_offsets, bit_range=None) -> None:
    _segmented(launch, keys_in, keys_out, values_in, values_out, begin_offsets, end_offsets,
               bit_range, False)


def device_segmented_radix_sort_pairs_descending(launch: Launch, keys_in, keys_out, values_in,
                                                 values_out, begin_offsets, end_offsets,
                                                 bit_range=None) -> None:
    _segmented(launch, keys_in, keys_out, values_in, values_out, begin_offsets, end_offsets,
               bit_range, True)
