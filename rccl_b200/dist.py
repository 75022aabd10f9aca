"""Multi-GPU sample sort over NCCL (no reference counterpart: the reference is
single-GPU; this is the scale-out extension of its DeviceRadixSort).

One process per GPU.  Rank r holds a contiguous shard of the global input.
  1. local stable radix sort of the shard (librsort_b200.so)
  2. S regular samples of the sorted shard, as composites
     (order image, rank << 40 | position in the sorted shard)
  3. all-gather of the samples over NCCL
  4. W-1 splitters from the sorted sample set (device kernel)
  5. bucket bounds of every splitter in the local shard (device kernel)
  6. all-to-all of the bucket sizes, then of the key and value buckets
     (NCCL grouped send/recv inside torch.distributed.all_to_all_single)
  7. stable merge of the W received runs (device merge-path kernel)
The composite order is the global stable order, so the ranks' outputs,
concatenated in rank order, are the stable sort of the concatenated input.

The phases are separate functions so a single-process emulation (tests) can
drive W simulated ranks through exactly the same steps.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .cub import (DeviceRadixSortKeysWorkspace, DeviceRadixSortPairsWorkspace, Launch, Program,
                  key_code, value_bytes_of, device_radix_sort_keys,
                  device_radix_sort_keys_descending, device_radix_sort_pairs,
                  device_radix_sort_pairs_descending, device_radix_sort_pairs_workspace,
                  device_radix_sort_workspace)
from .errors import raise_for

MAX_SPLITTER_SAMPLES = 8192
COMPOSITE_WORDS = 2  # int64 words per composite


def default_samples_per_rank(world: int) -> int:
    """64 * W regular samples per rank, capped so the world's sample set fits
    the one-CTA splitter kernel."""
    return max(1, min(64 * world, MAX_SPLITTER_SAMPLES // world))


class CudaLocalOps:
    """The per-rank device steps, all in librsort_b200.so."""

    def __init__(self, launch: Launch):
        self.launch = launch
        self._ws = None
        self._ws_key = None

    def sort(self, keys: torch.Tensor, values: Optional[torch.Tensor], descending: bool) -> None:
        n = keys.numel()
        key = (keys.dtype, None if values is None else value_bytes_of(values), n)
        if self._ws_key != key:
            if values is None:
                self._ws = device_radix_sort_workspace(self.launch, keys.dtype, n)
            else:
                vd = values.dtype if values.dim() == 1 else value_bytes_of(values)
                self._ws = device_radix_sort_pairs_workspace(self.launch, keys.dtype, vd, n)
            self._ws_key = key
        if values is None:
            (device_radix_sort_keys_descending if descending else device_radix_sort_keys)(
                self.launch, keys, self._ws)
        else:
            (device_radix_sort_pairs_descending if descending else device_radix_sort_pairs)(
                self.launch, keys, values, self._ws)

    def samples(self, keys: torch.Tensor, rank: int, count: int, descending: bool) -> torch.Tensor:
        out = torch.empty((count, COMPOSITE_WORDS), dtype=torch.int64, device=keys.device)
        raise_for(_lib.lib().rsort_dist_samples(key_code(keys.dtype), int(descending),
                                                keys.data_ptr(), keys.numel(), rank, count,
                                                out.data_ptr(), self.launch.handle))
        return out

    def splitters(self, gathered: torch.Tensor, world: int) -> torch.Tensor:
        out = torch.empty((max(world - 1, 1), COMPOSITE_WORDS), dtype=torch.int64,
                          device=gathered.device)
        raise_for(_lib.lib().rsort_dist_splitters(gathered.data_ptr(), gathered.shape[0], world,
                                                  out.data_ptr(), self.launch.handle))
        return out

    def bounds(self, keys: torch.Tensor, rank: int, splitters: torch.Tensor, world: int,
               descending: bool) -> torch.Tensor:
        out = torch.empty(world + 1, dtype=torch.int64, device=keys.device)
        raise_for(_lib.lib().rsort_dist_bounds(key_code(keys.dtype), int(descending),
                                               keys.data_ptr(), keys.numel(), rank,
                                               splitters.data_ptr(), world, out.data_ptr(),
                                               self.launch.handle))
        return out

    def merge_runs(self, keys: torch.Tensor, values: Optional[torch.Tensor],
                   run_lengths: Sequence[int], descending: bool
                   ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        runs = len(run_lengths)
        if runs <= 1:
            return keys, values
        sk = torch.empty_like(keys)
        sv = torch.empty_like(values) if values is not None else None
        nparts = _lib.lib().rsort_merge_partition_words(keys.numel())
        parts = torch.empty(nparts, dtype=torch.int64, device=keys.device)
        lens = (ctypes.c_size_t * runs)(*[int(x) for x in run_lengths])
        in_scratch = ctypes.c_int(0)
        vb = 0 if values is None else value_bytes_of(values)
        raise_for(_lib.lib().rsort_merge_runs(
            key_code(keys.dtype), int(descending), keys.data_ptr(),
            None if values is None else values.data_ptr(), vb, lens, runs, sk.data_ptr(),
            None if sv is None else sv.data_ptr(), parts.data_ptr(), nparts,
            ctypes.byref(in_scratch), self.launch.handle))
        if in_scratch.value:
            return sk, sv
        return keys, values


# ---------------------------------------------------------------------------
# Phases (shared by the torch.distributed driver and single-process emulation)
# ---------------------------------------------------------------------------
def phase_local(ops, keys, values, rank: int, samples_per_rank: int, descending: bool):
    """Sort the shard in place and return its regular samples."""
    ops.sort(keys, values, descending)
    return ops.samples(keys, rank, samples_per_rank, descending)


def phase_partition(ops, keys, gathered, rank: int, world: int, descending: bool):
    """Splitters from the gathered samples -> per-destination bucket sizes."""
    spl = ops.splitters(gathered, world)
    b = ops.bounds(keys, rank, spl, world, descending)
    return b[1:] - b[:-1]


def phase_merge(ops, recv_keys, recv_values, recv_counts: Sequence[int], descending: bool):
    return ops.merge_runs(recv_keys, recv_values, recv_counts, descending)


def _bytes(t: torch.Tensor) -> torch.Tensor:
    if t.numel() == 0:
        return torch.empty(0, dtype=torch.uint8, device=t.device)
    return t.reshape(-1).view(torch.uint8)


def sample_sort(keys: torch.Tensor, values: Optional[torch.Tensor] = None,
                descending: bool = False, group=None, samples_per_rank: Optional[int] = None,
                ops=None, timings: Optional[dict] = None):
    """Globally sort the ranks' shards; returns this rank's (keys, values) part.

    Sorts `keys` / `values` in place as its first step.  The output partition
    sizes are data dependent."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if ops is None:
        ops = CudaLocalOps(Program.load(keys.device).on())
    S = samples_per_rank or default_samples_per_rank(world)
    ev = _Events(timings, keys.device)
    ev.mark("start")
    samples = phase_local(ops, keys, values, rank, S, descending)
    ev.mark("local_sort")
    gathered = [torch.empty_like(samples) for _ in range(world)]
    dist.all_gather(gathered, samples, group=group)
    gathered = torch.cat(gathered)
    send = phase_partition(ops, keys, gathered, rank, world, descending)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    send_l, recv_l = send.tolist(), recv.tolist()
    ev.mark("partition")
    out_k = torch.empty(sum(recv_l), dtype=keys.dtype, device=keys.device)
    out_v = None
    if values is not None:
        shape = (sum(recv_l),) + tuple(values.shape[1:])
        out_v = torch.empty(shape, dtype=values.dtype, device=values.device)
    exchange(keys, values, out_k, out_v, send_l, recv_l, rank, world, group)
    ev.mark("exchange")
    out = phase_merge(ops, out_k, out_v, recv_l, descending)
    ev.mark("merge")
    ev.finish()
    return out


def exchange(keys, values, out_k, out_v, send_l, recv_l, rank: int, world: int, group=None):
    """Bucket exchange: every (rank -> peer) key and value bucket in ONE group
    of NCCL send/recv operations (torch.distributed.batch_isend_irecv), so
    keys and values of all peers move concurrently; the bucket a rank keeps is
    a local device copy."""
    import torch.distributed as dist
    kb = keys.element_size()
    vb = value_bytes_of(values) if values is not None else 0
    src_k, dst_k = _bytes(keys), _bytes(out_k)
    src_v = _bytes(values) if values is not None else None
    dst_v = _bytes(out_v) if values is not None else None
    soff = [0] * (world + 1)
    roff = [0] * (world + 1)
    for q in range(world):
        soff[q + 1] = soff[q] + send_l[q]
        roff[q + 1] = roff[q] + recv_l[q]
    ops = []
    for q in range(world):
        if q == rank:
            continue
        if send_l[q]:
            ops.append(dist.P2POp(dist.isend, src_k[soff[q] * kb:soff[q + 1] * kb], q, group))
            if vb:
                ops.append(dist.P2POp(dist.isend, src_v[soff[q] * vb:soff[q + 1] * vb], q, group))
        if recv_l[q]:
            ops.append(dist.P2POp(dist.irecv, dst_k[roff[q] * kb:roff[q + 1] * kb], q, group))
            if vb:
                ops.append(dist.P2POp(dist.irecv, dst_v[roff[q] * vb:roff[q + 1] * vb], q, group))
    if send_l[rank]:
        dst_k[roff[rank] * kb:roff[rank + 1] * kb].copy_(src_k[soff[rank] * kb:soff[rank + 1] * kb])
        if vb:
            dst_v[roff[rank] * vb:roff[rank + 1] * vb].copy_(
                src_v[soff[rank] * vb:soff[rank + 1] * vb])
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


class _Events:
    """Optional CUDA-event phase timing (milliseconds per phase)."""

    def __init__(self, sink: Optional[dict], device):
        self.sink = sink
        self.marks: List[Tuple[str, torch.cuda.Event]] = []
        self.cuda = sink is not None and device.type == "cuda"

    def mark(self, name: str) -> None:
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.marks.append((name, e))

    def finish(self) -> None:
        if not self.cuda or not self.marks:
            return
        self.marks[-1][1].synchronize()
        for (_, a), (name, b) in zip(self.marks, self.marks[1:]):
            self.sink[name] = self.sink.get(name, 0.0) + a.elapsed_time(b)
