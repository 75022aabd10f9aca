"""Sample-sort orchestration tests.

CPU: two gloo ranks drive rccl_b200.dist.sample_sort end to end with a numpy
stand-in for the per-rank device steps (the CUDA steps cannot run without a
GPU); the exchange, counts and merge order are the product code.
GPU: W simulated ranks in one process run the CUDA device steps through the
same phase functions, with the exchange done by slicing (kernels that wait on
one another never run as separate launches on one GPU, and these don't).
Both compare against the oracle's global stable sort and partition rule."""
import os
import socket

import numpy as np
import pytest
import torch

from helpers import bits, order_image
from oracle import pyoracle as O
from rccl_b200 import dist as D

POS_BITS = 40


class NumpyLocalOps:
    """Host stand-in for the device steps (test double of CudaLocalOps)."""

    def sort(self, keys, values, descending):
        k = keys.numpy()
        v = None if values is None else values.numpy()
        sk, sv, _, st = O.radix_sort(k, v, descending)
        assert st == 0
        k[:] = sk
        if v is not None:
            v[:] = sv

    def samples(self, keys, rank, count, descending):
        k = keys.numpy()
        m = k.size
        out = np.full((count, 2), -1, dtype=np.int64)
        if m:
            img = order_image(k, descending)
            p = (np.arange(count, dtype=np.uint64) + 1) * np.uint64(m) // np.uint64(count + 1)
            out[:, 0] = img[p.astype(np.int64)].view(np.int64)
            out[:, 1] = ((np.uint64(rank) << np.uint64(POS_BITS)) | p).view(np.int64)
        return torch.from_numpy(out)

    def splitters(self, gathered, world):
        g = gathered.numpy().view(np.uint64)
        order = np.lexsort((g[:, 1], g[:, 0]))
        g = g[order]
        valid = int(np.sum(g[:, 1] != np.uint64(2**64 - 1)))
        out = np.full((max(world - 1, 1), 2), -1, dtype=np.int64)
        for j in range(1, world):
            if valid:
                out[j - 1] = g[j * valid // world].view(np.int64)
        return torch.from_numpy(out)

    def bounds(self, keys, rank, splitters, world, descending):
        k = keys.numpy()
        img = order_image(k, descending)
        m = k.size
        pos = (np.uint64(rank) << np.uint64(POS_BITS)) | np.arange(m, dtype=np.uint64)
        b = [0]
        for j in range(1, world):
            sk, sp = splitters.numpy().view(np.uint64)[j - 1]
            b.append(int(np.sum((img < sk) | ((img == sk) & (pos < sp)))))
        b.append(m)
        return torch.tensor(b, dtype=torch.int64)

    def merge_runs(self, keys, values, run_lengths, descending):
        k = keys.numpy()
        order = np.argsort(order_image(k, descending), kind="stable")
        ok = torch.from_numpy(k[order].copy())
        ov = None if values is None else torch.from_numpy(values.numpy()[order].copy())
        return ok, ov


def test_order_image_matches_oracle():
    rng = np.random.default_rng(0)
    for dt in (np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64):
        if np.dtype(dt).kind == "f":
            x = rng.normal(0, 10, 500).astype(dt)
            x[:4] = [0.0, -0.0, np.inf, np.nan]
        else:
            x = rng.integers(np.iinfo(dt).min, np.iinfo(dt).max, 500, dtype=dt, endpoint=True)
        kt = O.key_type_of(x)
        for desc in (False, True):
            img = order_image(x, desc)
            raw = x.view(np.uint32 if x.itemsize == 4 else np.uint64)
            ref = [O.lib().orc_sort_key(kt, int(desc), 0, x.itemsize * 8, 0, int(r)) for r in raw]
            assert np.array_equal(img, np.array(ref, dtype=np.uint64))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, keys_all, shard_sizes, desc, result_path):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        off = sum(shard_sizes[:rank])
        k = torch.from_numpy(keys_all[off:off + shard_sizes[rank]].copy())
        v = torch.arange(off, off + shard_sizes[rank], dtype=torch.int64).to(torch.int32)
        ok, ov = D.sample_sort(k, v, descending=desc, samples_per_rank=64,
                               ops=NumpyLocalOps())
        np.savez(f"{result_path}.{rank}.npz", k=ok.numpy(), v=ov.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["uniform_u64", "constant_u32", "f32_desc", "ragged"])
def test_gloo_two_rank_sample_sort(tmp_path, kind):
    rng = np.random.default_rng(42)
    desc = False
    if kind == "uniform_u64":
        keys = rng.integers(0, 2**64, 20_000, dtype=np.uint64)
        sizes = [10_000, 10_000]
    elif kind == "constant_u32":
        keys = np.full(12_000, 7, np.uint32)
        sizes = [6_000, 6_000]
    elif kind == "f32_desc":
        keys = rng.normal(0, 5, 9_000).astype(np.float32)
        keys[::11] = -0.0
        keys[::13] = 0.0
        sizes = [4_000, 5_000]
        desc = True
    else:
        keys = rng.integers(0, 50, 7_000, dtype=np.uint64).astype(np.uint32)
        sizes = [0, 7_000]
    world = 2
    port = _free_port()
    ctx = torch.multiprocessing.get_context("spawn")
    procs = [ctx.Process(target=_gloo_worker,
                         args=(r, world, port, keys, sizes, desc, str(tmp_path / "out")))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    parts = [np.load(str(tmp_path / f"out.{r}.npz")) for r in range(world)]
    got_k = np.concatenate([p["k"] for p in parts])
    got_v = np.concatenate([p["v"] for p in parts])
    exp_k, exp_v, _, _ = O.radix_sort(keys, np.arange(keys.size, dtype=np.int32), desc)
    assert np.array_equal(bits(got_k), bits(exp_k))
    assert np.array_equal(got_v, exp_v)
    counts = O.sample_partition(keys, sizes, 64, desc)
    assert [p["k"].size for p in parts] == list(counts)


def emulate(ops, shards_k, shards_v, desc, samples_per_rank):
    """Drive W simulated ranks through dist's phases; exchange by slicing."""
    world = len(shards_k)
    samples = [D.phase_local(ops, shards_k[r], None if shards_v is None else shards_v[r], r,
                             samples_per_rank, desc) for r in range(world)]
    gathered = torch.cat(samples)
    sends = [D.phase_partition(ops, shards_k[r], gathered, r, world, desc).tolist()
             for r in range(world)]
    outs = []
    for q in range(world):
        ks, vs, counts = [], [], []
        for r in range(world):
            a = sum(sends[r][:q])
            b = a + sends[r][q]
            ks.append(shards_k[r][a:b])
            if shards_v is not None:
                vs.append(shards_v[r][a:b])
            counts.append(b - a)
        rk = torch.cat(ks)
        rv = torch.cat(vs) if shards_v is not None else None
        outs.append(D.phase_merge(ops, rk, rv, counts, desc))
    return outs


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("kind", ["u64_pairs", "u32_zipf_keys", "f32_desc_pairs", "i64_ragged"])
def test_emulated_multi_rank_device_steps(world, kind):
    from rccl_b200 import cub
    ops = D.CudaLocalOps(cub.Program.load("cuda:0").on())
    rng = np.random.default_rng(world * 7 + len(kind))
    desc = False
    n = 200_003
    vals = True
    if kind == "u64_pairs":
        keys = rng.integers(0, 2**64, n, dtype=np.uint64)
    elif kind == "u32_zipf_keys":
        keys = (rng.zipf(1.3, n) % 5000).astype(np.uint32)
        keys[::10] = 99
        vals = False
    elif kind == "f32_desc_pairs":
        keys = rng.normal(0, 1e3, n).astype(np.float32)
        keys[::97] = -0.0
        keys[::89] = 0.0
        keys[::101] = np.nan
        desc = True
    else:
        keys = rng.integers(-1000, 1000, n, dtype=np.int64)
    cuts = np.sort(rng.integers(0, n, world - 1))
    cuts[0] = 0  # one empty shard
    bounds = [0] + list(cuts) + [n]
    sizes = [bounds[i + 1] - bounds[i] for i in range(world)]
    shards_k = [torch.from_numpy(keys[bounds[i]:bounds[i + 1]].copy()).cuda()
                for i in range(world)]
    shards_v = None
    if vals:
        idx = np.arange(n, dtype=np.uint32)
        shards_v = [torch.from_numpy(idx[bounds[i]:bounds[i + 1]].copy()).cuda()
                    for i in range(world)]
    S = D.default_samples_per_rank(world)
    outs = emulate(ops, shards_k, shards_v, desc, S)
    got_k = np.concatenate([o[0].cpu().numpy() for o in outs])
    exp_k, exp_v, _, _ = O.radix_sort(keys, np.arange(n, dtype=np.uint32) if vals else None, desc)
    assert np.array_equal(bits(got_k), bits(exp_k))
    if vals:
        got_v = np.concatenate([o[1].cpu().numpy() for o in outs])
        assert np.array_equal(got_v, exp_v)
    counts = O.sample_partition(keys, sizes, S, desc)
    assert [o[0].numel() for o in outs] == list(counts)


@pytest.mark.gpu
@pytest.mark.parametrize("vb", [0, 1, 2, 4, 8, 16])
def test_merge_runs_is_stable(vb):
    from rccl_b200 import cub
    ops = D.CudaLocalOps(cub.Program.load("cuda:0").on())
    rng = np.random.default_rng(vb)
    runs = [int(x) for x in rng.integers(0, 30_000, 5)]
    parts = [np.sort(rng.integers(0, 300, r).astype(np.uint32)) for r in runs]
    keys = np.concatenate(parts)
    if vb == 16:
        values = rng.integers(0, 256, (keys.size, 16), dtype=np.uint8)
    elif vb:
        values = np.arange(keys.size).astype({1: np.uint8, 2: np.uint16, 4: np.uint32,
                                              8: np.uint64}[vb])
    else:
        values = None
    tk = torch.from_numpy(keys).cuda()
    tv = None if values is None else torch.from_numpy(values).cuda()
    ok, ov = ops.merge_runs(tk, tv, runs, False)
    order = np.argsort(keys, kind="stable")
    assert np.array_equal(ok.cpu().numpy(), keys[order])
    if values is not None:
        assert np.array_equal(ov.cpu().numpy(), values[order])
