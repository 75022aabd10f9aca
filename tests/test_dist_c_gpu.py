"""The whole multi-GPU sample sort behind one C call, against the oracle.

rsort_dist_pairs (one thread drives every GPU, NCCL communicators from
ncclCommInitAll) and rsort_dist_pairs_rank (one communicator per rank) are
called through ctypes; the ranks' outputs concatenated in rank order must be
the oracle's stable sort of the concatenated shards, bit for bit.  World size
1 runs on any GPU box; world size 2 needs two GPUs."""
import numpy as np
import pytest
import torch

from helpers import bits
from oracle import pyoracle as O
from rccl_b200 import dist as D
from rccl_b200 import nccl

pytestmark = pytest.mark.gpu

NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0


def shards(world, n_per, dtype, seed, pairs=True, dup=False):
    rng = np.random.default_rng(seed)
    out = []
    start = 0
    for r in range(world):
        n = n_per[r]
        if np.dtype(dtype).kind == "f":
            k = rng.normal(0, 100, n).astype(dtype)
            k[::53] = -0.0
            k[::59] = 0.0
            k[::61] = np.nan
        else:
            hi = 50 if dup else 2**63
            k = rng.integers(0, hi, n, dtype=np.uint64).astype(dtype)
        v = np.arange(start, start + n, dtype=np.uint32) if pairs else None
        start += n
        out.append((k, v))
    return out


def check(parts, host, desc):
    ks = np.concatenate([h[0] for h in host])
    vs = np.concatenate([h[1] for h in host]) if host[0][1] is not None else None
    ek, ev, _, st = O.radix_sort(ks, vs, desc, threads=4)
    assert st == 0
    gk = np.concatenate([p[0].cpu().numpy() for p in parts])
    assert np.array_equal(bits(gk), bits(ek))
    if vs is not None:
        gv = np.concatenate([p[1].cpu().numpy() for p in parts])
        assert np.array_equal(gv, ev)


def run_devices(world, n_per, dtype, desc, exchange, pairs=True, dup=False, seed=3):
    host = shards(world, n_per, dtype, seed, pairs, dup)
    comms = nccl.comm_init_all(list(range(world)))
    try:
        keys = [torch.from_numpy(h[0].copy()).to(f"cuda:{r}") for r, h in enumerate(host)]
        vals = ([torch.from_numpy(h[1].copy()).to(f"cuda:{r}") for r, h in enumerate(host)]
                if pairs else None)
        parts = D.sample_sort_devices(keys, vals, desc, comms, exchange=exchange)
        for r in range(world):
            torch.cuda.synchronize(r)
        check(parts, host, desc)
    finally:
        for r in range(world):
            torch.cuda.synchronize(r)
        for c in comms:
            nccl.comm_destroy(c)


@pytest.mark.parametrize("dtype,desc", [(np.uint64, False), (np.float32, True), (np.int32, False)])
def test_world1_multi_device_entry(dtype, desc):
    run_devices(1, [300_001], dtype, desc, "nccl")


def test_world1_rank_entry_keys_only():
    host = shards(1, [200_003], np.float64, 5, pairs=False)
    comm = nccl.comm_init_all([0])[0]
    try:
        keys = torch.from_numpy(host[0][0].copy()).cuda()
        k, v = D.sample_sort_c(keys, None, False, comm, 0, 1)
        torch.cuda.synchronize()
        assert v is None
        check([(k, None)], host, False)
    finally:
        torch.cuda.synchronize()
        nccl.comm_destroy(comm)


@pytest.mark.skipif(NGPU < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("dtype,desc,dup", [(np.uint64, False, False), (np.float32, True, False),
                                            (np.uint32, False, True)])
def test_world2_multi_device_entry(exchange, dtype, desc, dup):
    run_devices(2, [500_000, 321_123], dtype, desc, exchange, dup=dup)


@pytest.mark.skipif(NGPU < 2, reason="needs two GPUs")
def test_world2_small_and_empty_shards():
    run_devices(2, [0, 70_001], np.uint64, False, "nccl")
    run_devices(2, [5, 3], np.int64, True, "peer")
