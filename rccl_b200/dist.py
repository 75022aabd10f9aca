"""Multi-GPU sample sort over NCCL (no reference counterpart: the reference is
single-GPU; this is the scale-out extension of its DeviceRadixSort).

One process per GPU.  Rank r holds a contiguous shard of the global input.
  1. local stable radix sort of the shard (librsort_b200.so)
  2. S regular samples of the sorted shard, as composites
     (order image, rank << 40 | position in the sorted shard)
  3. all-gather of the samples over NCCL
  4. W-1 splitters from the sorted sample set (device kernel)
  5. bucket bounds of every splitter in the local shard (device kernel)
  6. all-gather of every rank's bucket sizes and shard IPC handles, then
     each rank pulls its bucket out of every peer's shard with one copy
     kernel over NVLink peer memory (PeerExchange); NCCL grouped send/recv
     is the fallback when the shards cannot be exported
  7. stable merge of the W received runs: pairwise merge-path rounds (the
     default; in "peer" mode the first round reads the buckets straight out
     of the peers' shards) or one W-way pass (RSORT_MERGE=multiway)
The composite order is the global stable order, so the ranks' outputs,
concatenated in rank order, are the stable sort of the concatenated input.

The phases are separate functions so a single-process emulation (tests) can
drive W simulated ranks through exactly the same steps.
"""
from __future__ import annotations

import atexit
import ctypes
import os
import threading
from collections import OrderedDict
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
        """Stable merge of the runs held back to back in keys / values (ties
        keep the lower run first): one W-way merge into new tensors, or, with
        merge_method() == "tree", pairwise rounds (rsort_merge_runs)."""
        runs = len(run_lengths)
        if runs <= 1:
            return keys, values
        if merge_method() == "tree":
            return self._merge_tree(keys, values, run_lengths, descending)
        kb = keys.element_size()
        vb = 0 if values is None else value_bytes_of(values)
        kp, vp, off = [], [], 0
        for n in run_lengths:
            kp.append(keys.data_ptr() + off * kb if n else None)
            vp.append(values.data_ptr() + off * vb if (n and values is not None) else None)
            off += int(n)
        return multiway_merge(keys, values, kp, vp, run_lengths, descending, self.launch.handle)


    def _merge_tree(self, keys, values, run_lengths, descending):
        runs = len(run_lengths)
        sk = torch.empty_like(keys)
        sv = torch.empty_like(values) if values is not None else None
        nparts = _lib.lib().rsort_merge_partition_words(keys.numel())
        parts = torch.empty(max(nparts, 1), dtype=torch.int64, device=keys.device)
        lens = (ctypes.c_size_t * runs)(*[int(x) for x in run_lengths])
        in_scratch = ctypes.c_int(0)
        vb = 0 if values is None else value_bytes_of(values)
        raise_for(_lib.lib().rsort_merge_runs(
            key_code(keys.dtype), int(descending), keys.data_ptr(),
            None if values is None else values.data_ptr(), vb, lens, runs, sk.data_ptr(),
            None if sv is None else sv.data_ptr(), parts.data_ptr(), nparts,
            ctypes.byref(in_scratch), self.launch.handle))
        return (sk, sv) if in_scratch.value else (keys, values)


def merge_method() -> str:
    """How a rank merges its W received runs: "multiway" (one pass,
    rsort_merge_multiway) or "tree" (pairwise rounds; in the peer exchange the
    first round reads the peers' shards).  RSORT_MERGE overrides the
    default."""
    m = os.environ.get("RSORT_MERGE", DEFAULT_MERGE)
    if m not in ("multiway", "tree"):
        raise ValueError(f"RSORT_MERGE={m!r}: expected 'multiway' or 'tree'")
    return m


DEFAULT_MERGE = "tree"


def multiway_merge(keys: torch.Tensor, values: Optional[torch.Tensor], key_ptrs, value_ptrs,
                   run_lengths: Sequence[int], descending: bool, stream):
    """rsort_merge_multiway of runs given by device pointers (this GPU's memory
    or a peer's) into new tensors shaped like keys / values."""
    runs = len(run_lengths)
    total = int(sum(run_lengths))
    out_k = torch.empty(total, dtype=keys.dtype, device=keys.device)
    out_v = None
    vb = 0
    if values is not None:
        vb = value_bytes_of(values)
        out_v = torch.empty((total,) + tuple(values.shape[1:]), dtype=values.dtype,
                            device=values.device)
    if total == 0:
        return out_k, out_v
    lib = _lib.lib()
    kc = key_code(keys.dtype)
    nbytes = lib.rsort_multiway_scratch_bytes(kc, vb, runs, total)
    scratch = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=keys.device)
    VP, SZ = ctypes.c_void_p * runs, ctypes.c_size_t * runs
    raise_for(lib.rsort_merge_multiway(
        kc, int(descending), runs, VP(*key_ptrs), VP(*value_ptrs) if values is not None else None,
        SZ(*[int(x) for x in run_lengths]), vb, out_k.data_ptr(),
        None if out_v is None else out_v.data_ptr(), scratch.data_ptr(), nbytes, stream))
    return out_k, out_v


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
                ops=None, timings: Optional[dict] = None, exchange_mode: Optional[str] = None):
    """Globally sort the ranks' shards; returns this rank's (keys, values) part.

    Sorts `keys` / `values` in place as its first step.  The output partition
    sizes are data dependent.  exchange_mode (default: the RSORT_EXCHANGE
    environment variable, else "peer"):
      "peer"       the first merge round reads the buckets straight out of the
                   peers' shards over NVLink (CUDA IPC); no staging copy
      "peer-copy"  one copy kernel pulls the buckets over NVLink, then the
                   local merge
      "nccl"       NCCL grouped send/recv, then the local merge"""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if ops is None:
        ops = CudaLocalOps(Program.load(keys.device).on())
    mode = exchange_mode or os.environ.get("RSORT_EXCHANGE", "peer")
    if mode not in ("peer", "peer-copy", "nccl"):
        raise ValueError(f"exchange mode {mode!r}: expected 'peer', 'peer-copy' or 'nccl'")
    peer = mode in ("peer", "peer-copy") and keys.is_cuda and world > 1
    S = samples_per_rank or default_samples_per_rank(world)
    ev = _Events(timings, keys.device)
    ev.mark("start")
    samples = phase_local(ops, keys, values, rank, S, descending)
    ev.mark("local_sort")
    gathered = [torch.empty_like(samples) for _ in range(world)]
    dist.all_gather(gathered, samples, group=group)
    gathered = torch.cat(gathered)
    send = phase_partition(ops, keys, gathered, rank, world, descending)
    if peer:
        # One all-gather carries every rank's bucket sizes and shard handles;
        # it also orders the peer reads after every rank's sort.
        px = peer_exchange()
        rec = torch.cat([send, px.record(keys, values, send.device)])
        table = [torch.empty_like(rec) for _ in range(world)]
        dist.all_gather(table, rec, group=group)
        table = torch.stack(table).cpu()
        sizes = table[:, :world].tolist()
        peer = bool(table[:, world].all())
        recv_l = [sizes[q][rank] for q in range(world)]
    else:
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
        send_l, recv_l = send.tolist(), recv.tolist()
    ev.mark("partition")
    if peer and mode == "peer":
        # No separate exchange: the first merge round reads the buckets
        # straight out of the peers' shards.
        ev.mark("exchange")
        out = px.merge(keys, values, table, sizes, rank, world, ops.launch.handle, descending)
        # The peers may overwrite their shards only after every rank's merge.
        dist.all_reduce(torch.zeros(1, device=keys.device), group=group)
        ev.mark("merge")
        ev.finish()
        return out
    out_k = torch.empty(sum(recv_l), dtype=keys.dtype, device=keys.device)
    out_v = None
    if values is not None:
        shape = (sum(recv_l),) + tuple(values.shape[1:])
        out_v = torch.empty(shape, dtype=values.dtype, device=values.device)
    if peer:
        px.pull(keys, values, out_k, out_v, table, sizes, rank, world, ops.launch.handle)
        # The peers may overwrite their shards only after every rank's pull.
        dist.all_reduce(torch.zeros(1, device=keys.device), group=group)
    else:
        if mode in ("peer", "peer-copy") and keys.is_cuda and world > 1:
            send_l = [sizes[rank][q] for q in range(world)]
        exchange(keys, values, out_k, out_v, send_l, recv_l, rank, world, group)
    ev.mark("exchange")
    out = phase_merge(ops, out_k, out_v, recv_l, descending)
    ev.mark("merge")
    ev.finish()
    return out


# ---------------------------------------------------------------------------
# The whole sample sort in one C call (rsort_dist_pairs / _rank): no Python
# between the steps.
# ---------------------------------------------------------------------------
def _dist_out(keys: torch.Tensor, values: Optional[torch.Tensor], capacity: int):
    ok = torch.empty(max(capacity, 1), dtype=keys.dtype, device=keys.device)
    ov = None
    if values is not None:
        ov = torch.empty((max(capacity, 1),) + tuple(values.shape[1:]), dtype=values.dtype,
                         device=values.device)
    return ok, ov


def _first_capacity(n: int) -> int:
    """Output capacity of a first attempt: the shard size plus slack for the
    sampled splitters' imbalance; a call whose part does not fit reports the
    sizes, and is repeated with exactly those."""
    return n + n // 8 + 4096


def sample_sort_c(keys: torch.Tensor, values: Optional[torch.Tensor], descending: bool,
                  comm: int, rank: int, world: int, stream=None
                  ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """This rank's part of the global stable sort, through rsort_dist_pairs_rank
    (NCCL exchange).  `comm`: this rank's ncclComm_t (rccl_b200.nccl).  Sorts
    keys / values in place as its first step."""
    lib = _lib.lib()
    kc = key_code(keys.dtype)
    vb = 0 if values is None else value_bytes_of(values)
    n = keys.numel()
    stream = stream if stream is not None else torch.cuda.current_stream(keys.device).cuda_stream
    cap = _first_capacity(n)
    for _ in range(2):
        ok, ov = _dist_out(keys, values, cap)
        nbytes = lib.rsort_dist_scratch_bytes(kc, vb, n, cap, world)
        scratch = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=keys.device)
        n_out = ctypes.c_size_t(0)
        st = lib.rsort_dist_pairs_rank(kc, int(descending), vb, rank, world, comm, stream,
                                       keys.data_ptr(),
                                       None if values is None else values.data_ptr(), n,
                                       ok.data_ptr(), None if ov is None else ov.data_ptr(), cap,
                                       scratch.data_ptr(), nbytes, ctypes.byref(n_out))
        if st == _lib.RSORT_WORKSPACE_TOO_SMALL and _lib.last_error().role.startswith(
                b"dist sort output"):
            # every rank returned here (they all hold the same table): each
            # retries with its own part's size
            cap = max(n_out.value, 1)
            continue
        raise_for(st)
        m = n_out.value
        return ok[:m], (ov[:m] if ov is not None else None)
    raise RuntimeError("rsort_dist_pairs_rank: output capacity negotiation failed")


def sample_sort_devices(keys: Sequence[torch.Tensor], values: Optional[Sequence[torch.Tensor]],
                        descending: bool, comms: Sequence[int], exchange: str = "nccl",
                        streams: Optional[Sequence] = None):
    """All ranks' parts of the global stable sort of the shards keys[r] (one
    per device, in rank order), driven from this thread through
    rsort_dist_pairs.  comms: rccl_b200.nccl.comm_init_all(devices).
    exchange: "nccl" (grouped send/recv) or "peer" (copy kernels reading the
    peers' shards).  Returns [(keys_r, values_r or None)]."""
    lib = _lib.lib()
    W = len(keys)
    kc = key_code(keys[0].dtype)
    vb = 0 if values is None else value_bytes_of(values[0])
    devs = [k.device.index for k in keys]
    if streams is None:
        streams = [torch.cuda.current_stream(k.device).cuda_stream for k in keys]
    ns = [k.numel() for k in keys]
    caps = [_first_capacity(max(ns))] * W
    mode = {"nccl": _lib.RSORT_EXCHANGE_NCCL, "peer": _lib.RSORT_EXCHANGE_PEER}[exchange]
    VP, SZ = ctypes.c_void_p * W, ctypes.c_size_t * W
    for _ in range(2):
        outs = [_dist_out(keys[r], None if values is None else values[r], caps[r])
                for r in range(W)]
        sbytes = [lib.rsort_dist_scratch_bytes(kc, vb, ns[r], caps[r], W) for r in range(W)]
        scr = [torch.empty(max(sbytes[r], 1), dtype=torch.uint8, device=keys[r].device)
               for r in range(W)]
        n_out = SZ()
        st = lib.rsort_dist_pairs(
            kc, int(descending), vb, W, (ctypes.c_int * W)(*devs), VP(*comms), VP(*streams),
            VP(*[k.data_ptr() for k in keys]),
            VP(*[v.data_ptr() for v in values]) if values is not None else None, SZ(*ns),
            VP(*[o[0].data_ptr() for o in outs]),
            VP(*[o[1].data_ptr() for o in outs]) if values is not None else None, SZ(*caps),
            VP(*[t.data_ptr() for t in scr]), SZ(*sbytes), mode, n_out)
        if st == _lib.RSORT_WORKSPACE_TOO_SMALL and _lib.last_error().role.startswith(
                b"dist sort output"):
            caps = [max(int(n_out[r]), 1) for r in range(W)]
            continue
        raise_for(st)
        return [(outs[r][0][:n_out[r]], outs[r][1][:n_out[r]] if values is not None else None)
                for r in range(W)]
    raise RuntimeError("rsort_dist_pairs: output capacity negotiation failed")


class PeerExchange:
    """Bucket exchange by direct reads of the peers' shards over NVLink.

    Each rank exports its sorted shard (keys, values) as CUDA IPC handles; a
    peer maps a handle once (kept in a small cache, released at exit) and
    pulls its bucket with rsort_gather_segments, one SM-driven copy kernel
    that reads every peer at once.  A shard that cannot be exported (for
    example memory from a VMM-based allocator) makes every rank fall back to
    the NCCL exchange, since all ranks see the same export flags."""

    WORDS = 1 + 2 * (_lib.IPC_HANDLE_BYTES // 8 + 1)  # flag, (handle, offset) x 2
    CACHE = 256

    def __init__(self):
        self._mapped: "OrderedDict[bytes, int]" = OrderedDict()
        self._lock = threading.Lock()

    def _export(self, t: Optional[torch.Tensor]) -> Tuple[bytes, int, bool]:
        if t is None or t.numel() == 0:
            return bytes(_lib.IPC_HANDLE_BYTES), 0, True
        h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        off = ctypes.c_uint64(0)
        st = _lib.lib().rsort_ipc_export(t.data_ptr(), h, ctypes.byref(off))
        return h.raw, off.value, st == 0

    def record(self, keys, values, device) -> torch.Tensor:
        """flag, key handle + offset, value handle + offset as int64 words."""
        kh, ko, kok = self._export(keys)
        vh, vo, vok = self._export(values)
        words = [1 if (kok and vok) else 0]
        for h, o in ((kh, ko), (vh, vo)):
            words += list(memoryview(h).cast("q"))
            words.append(o)
        return torch.tensor(words, dtype=torch.int64).to(device)

    def _base(self, handle: bytes) -> int:
        with self._lock:
            if handle in self._mapped:
                self._mapped.move_to_end(handle)
                return self._mapped[handle]
            p = ctypes.c_void_p(0)
            raise_for(_lib.lib().rsort_ipc_import(handle, ctypes.byref(p)))
            self._mapped[handle] = p.value
            if len(self._mapped) > self.CACHE:
                # A kernel of an earlier call may still read the oldest
                # mappings: let the device drain before unmapping.
                torch.cuda.synchronize()
                while len(self._mapped) > self.CACHE:
                    _, old = self._mapped.popitem(last=False)
                    _lib.lib().rsort_ipc_release(ctypes.c_void_p(old))
            return p.value

    def pull(self, keys, values, out_k, out_v, table, sizes, rank: int, world: int, stream) -> None:
        hw = _lib.IPC_HANDLE_BYTES // 8
        kb = keys.element_size()
        vb = value_bytes_of(values) if values is not None else 0
        for which, local, out, width in ((0, keys, out_k, kb), (1, values, out_v, vb)):
            if width == 0:
                continue
            col = world + 1 + which * (hw + 1)
            srcs = (ctypes.c_void_p * world)()
            lens = (ctypes.c_uint64 * world)()
            for q in range(world):
                start = sum(sizes[q][:rank])
                lens[q] = sizes[q][rank] * width
                if lens[q] == 0:
                    srcs[q] = None
                elif q == rank:
                    srcs[q] = local.data_ptr() + start * width
                else:
                    handle = table[q, col:col + hw].numpy().tobytes()
                    off = int(table[q, col + hw])
                    srcs[q] = self._base(handle) + off + start * width
            raise_for(_lib.lib().rsort_gather_segments(world, srcs, lens, out.data_ptr(), stream))

    def merge(self, keys, values, table, sizes, rank: int, world: int, stream, descending):
        """One W-way merge of this rank's W buckets straight out of the shards
        (peers' over NVLink, the local one from HBM) into new tensors: each
        bucket crosses NVLink once, inside the merge."""
        hw = _lib.IPC_HANDLE_BYTES // 8
        kb = keys.element_size()
        vb = value_bytes_of(values) if values is not None else 0
        n_out = sum(sizes[q][rank] for q in range(world))
        kp = (ctypes.c_void_p * world)()
        vp = (ctypes.c_void_p * world)()
        lens = (ctypes.c_size_t * world)()
        for q in range(world):
            start = sum(sizes[q][:rank])
            lens[q] = sizes[q][rank]
            for which, local, width, arr in ((0, keys, kb, kp), (1, values, vb, vp)):
                if width == 0 or lens[q] == 0:
                    continue
                if q == rank:
                    arr[q] = local.data_ptr() + start * width
                else:
                    col = world + 1 + which * (hw + 1)
                    handle = table[q, col:col + hw].numpy().tobytes()
                    arr[q] = self._base(handle) + int(table[q, col + hw]) + start * width
        if merge_method() == "multiway":
            return multiway_merge(keys, values, list(kp), list(vp), list(lens), descending, stream)
        # Pairwise: the first round merges bucket pairs straight from the shards,
        # launched from pair rank // 2 on, so the ranks read different peers.
        out_k = torch.empty(n_out, dtype=keys.dtype, device=keys.device)
        sk = torch.empty_like(out_k)
        out_v = sv = None
        if values is not None:
            shape = (n_out,) + tuple(values.shape[1:])
            out_v = torch.empty(shape, dtype=values.dtype, device=values.device)
            sv = torch.empty_like(out_v)
        nparts = _lib.lib().rsort_merge_partition_words(n_out)
        parts = torch.empty(max(nparts, 1), dtype=torch.int64, device=keys.device)
        in_scratch = ctypes.c_int(0)
        raise_for(_lib.lib().rsort_merge_segments(
            key_code(keys.dtype), int(descending), world, kp, vp, lens, vb, out_k.data_ptr(),
            None if out_v is None else out_v.data_ptr(), sk.data_ptr(),
            None if sv is None else sv.data_ptr(), parts.data_ptr(), nparts,
            ctypes.byref(in_scratch), rank // 2, stream))
        return (sk, sv) if in_scratch.value else (out_k, out_v)

    def close(self) -> None:
        with self._lock:
            if self._mapped and torch.cuda.is_available():
                torch.cuda.synchronize()
            while self._mapped:
                _, p = self._mapped.popitem()
                _lib.lib().rsort_ipc_release(ctypes.c_void_p(p))


_PEER: Optional[PeerExchange] = None


def _close_at_exit() -> None:
    # At interpreter exit the CUDA context may already be going away; the
    # mappings die with the process either way.
    try:
        if _PEER is not None:
            _PEER.close()
    except Exception:
        pass


def release_peer_mappings() -> None:
    """Unmap every peer shard this process mapped for the peer exchange.  The
    mappings are cached across calls (up to PeerExchange.CACHE of them), so a
    peer's freed shard stays mapped, and its memory held, until it is evicted,
    this is called, or the process exits.  Call it between sorts only, after
    the collective that ends a sort; the next sort maps again."""
    if _PEER is not None:
        _PEER.close()


def peer_exchange() -> PeerExchange:
    global _PEER
    if _PEER is None:
        _PEER = PeerExchange()
        atexit.register(_close_at_exit)
    return _PEER


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
