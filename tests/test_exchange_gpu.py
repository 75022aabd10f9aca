"""Bucket exchange over NVLink peer memory.

GPU: rsort_gather_segments against torch slicing for every copy width the
kernel picks (1..16 bytes, ragged and empty segments), rsort_merge_segments
on runs in separate buffers against rsort_merge_runs on their concatenation,
rsort_ipc_export's allocation offsets, and -- on boxes with two or more GPUs
-- a two-process NCCL sample sort in each exchange mode (merge from peer
memory, peer copy, NCCL send/recv), checked against the oracle."""
import ctypes
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from helpers import bits
from oracle import pyoracle as O
from rccl_b200 import _lib
from rccl_b200 import dist as D
from rccl_b200.errors import raise_for


def gather(srcs, lens, out, stream=None):
    n = len(srcs)
    ptrs = (ctypes.c_void_p * n)(*srcs)
    ls = (ctypes.c_uint64 * n)(*lens)
    s = torch.cuda.current_stream().cuda_stream if stream is None else stream
    raise_for(_lib.lib().rsort_gather_segments(n, ptrs, ls, out.data_ptr(), s))


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_gather_segments_matches_slicing(seed):
    rng = np.random.default_rng(seed)
    src = torch.randint(0, 256, (1 << 22,), dtype=torch.uint8, device="cuda")
    nseg = int(rng.integers(1, 20))
    segs = []
    for _ in range(nseg):
        # offsets / lengths that exercise every copy width, plus empties
        width = int(rng.choice([1, 2, 4, 8, 16]))
        start = int(rng.integers(0, (1 << 22) // width - 70000)) * width
        length = int(rng.choice([0, width, int(rng.integers(0, 65536)) * width]))
        segs.append((start, length))
    total = sum(l for _, l in segs)
    # destination offset by a few bytes so destination alignments vary too
    pad = int(rng.integers(0, 16))
    big = torch.full((total + pad + 32,), 0xAB, dtype=torch.uint8, device="cuda")
    out = big[pad:pad + total]
    gather([src.data_ptr() + s if l else None for s, l in segs], [l for _, l in segs], out)
    exp = torch.cat([src[s:s + l] for s, l in segs]) if total else src[:0]
    torch.cuda.synchronize()
    assert torch.equal(out, exp)
    assert bool((big[:pad] == 0xAB).all()) and bool((big[pad + total:] == 0xAB).all())


@pytest.mark.gpu
@pytest.mark.parametrize("runs", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("desc", [False, True])
def test_merge_segments_matches_merge_runs(runs, desc):
    rng = np.random.default_rng(runs * 2 + desc)
    lens = [int(x) for x in rng.integers(0, 40_000, runs)]
    if runs > 2:
        lens[1] = 0  # an empty run
    kt = 3  # u64
    ks, vs = [], []
    base = 0
    for L in lens:
        k = rng.integers(0, 5_000, L, dtype=np.uint64)  # duplicates across runs
        k = np.sort(k)[::-1].copy() if desc else np.sort(k)
        ks.append(torch.from_numpy(k.view(np.int64)).cuda())
        vs.append(torch.arange(base, base + L, dtype=torch.int32, device="cuda"))
        base += L
    total = sum(lens)
    lib = _lib.lib()
    nparts = lib.rsort_merge_partition_words(total)
    parts = torch.empty(max(nparts, 1), dtype=torch.int64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    # reference: rsort_merge_runs on the concatenation
    ck, cv = torch.cat(ks), torch.cat(vs)
    sk, sv = torch.empty_like(ck), torch.empty_like(cv)
    flag = ctypes.c_int(0)
    raise_for(lib.rsort_merge_runs(kt, int(desc), ck.data_ptr(), cv.data_ptr(), 4,
                                   (ctypes.c_size_t * runs)(*lens), runs, sk.data_ptr(),
                                   sv.data_ptr(), parts.data_ptr(), nparts, ctypes.byref(flag), st))
    ek, ev = (sk, sv) if flag.value else (ck, cv)
    # runs in separate buffers
    ok, ov = torch.empty_like(ck), torch.empty_like(cv)
    s2k, s2v = torch.empty_like(ck), torch.empty_like(cv)
    kp = (ctypes.c_void_p * runs)(*[k.data_ptr() if k.numel() else None for k in ks])
    vp = (ctypes.c_void_p * runs)(*[v.data_ptr() if v.numel() else None for v in vs])
    for first_pair in range((runs + 1) // 2 + 1):  # launch order must not matter
        flag2 = ctypes.c_int(0)
        raise_for(lib.rsort_merge_segments(kt, int(desc), runs, kp, vp,
                                           (ctypes.c_size_t * runs)(*lens), 4, ok.data_ptr(),
                                           ov.data_ptr(), s2k.data_ptr(), s2v.data_ptr(),
                                           parts.data_ptr(), nparts, ctypes.byref(flag2),
                                           first_pair, st))
        gk, gv = (s2k, s2v) if flag2.value else (ok, ov)
        torch.cuda.synchronize()
        assert torch.equal(gk, ek) and torch.equal(gv, ev)
    # stable: equal keys keep run order, i.e. ascending original index
    k = gk.cpu().numpy().view(np.uint64)
    v = gv.cpu().numpy()
    assert np.all(np.diff(k.astype(np.float64)) <= 0) if desc else np.all(k[1:] >= k[:-1])
    ties = k[1:] == k[:-1]
    assert np.all(v[1:][ties] > v[:-1][ties])


@pytest.mark.gpu
def test_gather_rejects_too_many_segments():
    n = _lib.GATHER_MAX_SEGMENTS + 1
    out = torch.empty(16, dtype=torch.uint8, device="cuda")
    st = _lib.lib().rsort_gather_segments(n, (ctypes.c_void_p * n)(),
                                          (ctypes.c_uint64 * n)(), out.data_ptr(), None)
    assert st == _lib.RSORT_BAD_ARGUMENT


@pytest.mark.gpu
def test_ipc_export_reports_offset_in_allocation():
    t = torch.empty(1 << 20, dtype=torch.int32, device="cuda")
    h0 = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    h1 = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    o0, o1 = ctypes.c_uint64(), ctypes.c_uint64()
    raise_for(_lib.lib().rsort_ipc_export(t.data_ptr(), h0, ctypes.byref(o0)))
    raise_for(_lib.lib().rsort_ipc_export(t[37:].data_ptr(), h1, ctypes.byref(o1)))
    assert h0.raw == h1.raw
    assert o1.value - o0.value == 37 * 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _peer_worker(rank, world, port, keys_all, result_path):
    import torch.distributed as dist
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        m = keys_all.size // world
        off = rank * m
        res = {}
        for mode in ("peer", "peer-copy", "nccl"):
            k = torch.from_numpy(keys_all[off:off + m].copy()).cuda()
            v = torch.arange(off, off + m, dtype=torch.int32, device="cuda")
            ok, ov = D.sample_sort(k, v, exchange_mode=mode)
            torch.cuda.synchronize()
            res[mode + "_k"] = ok.cpu().numpy()
            res[mode + "_v"] = ov.cpu().numpy()
        np.savez(f"{result_path}.{rank}.npz", **res)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_two_gpu_peer_exchange_sample_sort(tmp_path):
    rng = np.random.default_rng(7)
    world = 2
    keys = rng.integers(0, 2**64, 2 * 300_001, dtype=np.uint64)
    keys[::97] = keys[5]  # duplicates across both shards: stability matters
    port = _free_port()
    ctx = torch.multiprocessing.get_context("spawn")
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, keys, str(tmp_path / "o")))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    parts = [np.load(str(tmp_path / f"o.{r}.npz")) for r in range(world)]
    exp_k, exp_v, _, _ = O.radix_sort(keys, np.arange(keys.size, dtype=np.int32), False)
    for mode in ("peer", "peer-copy", "nccl"):
        got_k = np.concatenate([p[mode + "_k"] for p in parts])
        got_v = np.concatenate([p[mode + "_v"] for p in parts])
        assert np.array_equal(bits(got_k), bits(exp_k)), mode
        assert np.array_equal(got_v, exp_v), mode
