"""Host logic of the peer-memory exchange (rccl_b200.dist.PeerExchange), on
CPU: the per-rank record layout (flag, IPC handle words, offsets) and the
bucket pointers the merge is given (peer base + shard offset + the bucket's
start inside the peer's sorted shard), with the library calls replaced by
recorders.  The device side runs in the GPU tests."""
import ctypes

import numpy as np
import pytest
import torch

from rccl_b200 import _lib
from rccl_b200 import dist as D

HW = _lib.IPC_HANDLE_BYTES // 8


def make_table(world, sizes, handles, offsets, flags):
    rows = []
    for q in range(world):
        words = list(sizes[q]) + [flags[q]]
        for which in range(2):
            words += list(np.frombuffer(handles[q][which], dtype=np.int64))
            words.append(offsets[q][which])
        rows.append(words)
    return torch.tensor(rows, dtype=torch.int64)


def test_record_words_roundtrip(monkeypatch):
    px = D.PeerExchange()
    hk, hv = bytes(range(64)), bytes(range(64, 128))

    def fake_export(t):
        return (hk, 4096, True) if t.dtype == torch.int64 else (hv, 512, True)

    monkeypatch.setattr(px, "_export", fake_export)
    rec = px.record(torch.zeros(3, dtype=torch.int64), torch.zeros(3, dtype=torch.int32), "cpu")
    assert rec.numel() == D.PeerExchange.WORDS
    assert rec[0].item() == 1
    assert rec[1:1 + HW].numpy().tobytes() == hk and rec[1 + HW].item() == 4096
    assert rec[2 + HW:2 + 2 * HW].numpy().tobytes() == hv and rec[2 + 2 * HW].item() == 512


@pytest.mark.parametrize("method", ["tree", "multiway"])
def test_merge_gets_each_peers_bucket(monkeypatch, method):
    monkeypatch.setenv("RSORT_MERGE", method)
    world, rank = 3, 1
    # sizes[q][r]: items of rank q's shard destined to rank r
    sizes = [[5, 7, 2], [3, 4, 9], [0, 6, 1]]
    handles = [(bytes([q]) * 64, bytes([q + 10]) * 64) for q in range(world)]
    offsets = [(1000 * (q + 1), 100 * (q + 1)) for q in range(world)]
    table = make_table(world, sizes, handles, offsets, [1] * world)
    bases = {handles[q][w]: (1 << 32) * (q + 1) + (1 << 20) * w for q in range(world)
             for w in range(2)}
    px = D.PeerExchange()
    monkeypatch.setattr(px, "_base", lambda h: bases[h])
    seen = {}

    class FakeLib:
        def rsort_merge_partition_words(self, n):
            return 4

        def rsort_merge_segments(self, key, desc, runs, kp, vp, lens, vb, ok, ov, sk, sv, parts,
                                 nparts, flag, first_pair, stream):
            seen.update(runs=runs, kp=[kp[i] for i in range(runs)],
                        vp=[vp[i] for i in range(runs)], lens=[lens[i] for i in range(runs)],
                        vb=vb, first_pair=first_pair)
            return 0

        def rsort_multiway_scratch_bytes(self, key, vb, runs, total):
            return 64

        def rsort_merge_multiway(self, key, desc, runs, kp, vp, lens, vb, ok, ov, scratch,
                                 nbytes, stream):
            seen.update(runs=runs, kp=[kp[i] for i in range(runs)],
                        vp=[vp[i] for i in range(runs)], lens=[lens[i] for i in range(runs)],
                        vb=vb)
            return 0

    monkeypatch.setattr(_lib, "lib", lambda: FakeLib())
    keys = torch.zeros(sum(sizes[rank]), dtype=torch.int64)  # this rank's shard (8-byte keys)
    values = torch.zeros(sum(sizes[rank]), dtype=torch.int32)
    out_k, out_v = px.merge(keys, values, table, sizes, rank, world, None, False)
    assert out_k.numel() == sum(sizes[q][rank] for q in range(world)) == 17
    assert seen["runs"] == world and seen["vb"] == 4
    if method == "tree":
        assert seen["first_pair"] == rank // 2
    assert seen["lens"] == [7, 4, 6]
    for q in range(world):
        start = sum(sizes[q][:rank])
        if q == rank:
            assert seen["kp"][q] == keys.data_ptr() + start * 8
            assert seen["vp"][q] == values.data_ptr() + start * 4
        else:
            assert seen["kp"][q] == bases[handles[q][0]] + offsets[q][0] + start * 8
            assert seen["vp"][q] == bases[handles[q][1]] + offsets[q][1] + start * 4


def test_export_failure_flag_reaches_every_rank():
    # one rank that could not export makes the table's flag column falsy
    table = make_table(2, [[1, 1], [1, 1]], [(bytes(64), bytes(64))] * 2, [(0, 0)] * 2, [1, 0])
    assert not bool(table[:, 2].all())
