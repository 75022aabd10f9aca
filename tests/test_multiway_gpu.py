"""rsort_merge_multiway: one stable W-way merge of sorted runs (ties keep the
lower run first), the last step of the sample sort.  Expected output: the
stable sort of the runs concatenated in run order (each run is sorted, so a
stable sort by the order image is the stable merge).  Bit-exact."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import bits, order_image
from rccl_b200 import _lib
from rccl_b200 import dist as D

pytestmark = pytest.mark.gpu


def make_runs(rng, lens, dtype, desc, mode):
    runs = []
    for i, n in enumerate(lens):
        if mode == "dup":
            k = rng.integers(0, 20, n).astype(dtype)
        elif mode == "disjoint":  # run i holds a key range of its own, in reverse run order
            k = (rng.integers(0, 1000, n) + 1000 * (len(lens) - i)).astype(dtype)
        elif np.dtype(dtype).kind == "f":
            k = rng.normal(0, 50, n).astype(dtype)
            k[::7] = -0.0
            k[::11] = 0.0
            k[::13] = np.nan
        else:
            k = rng.integers(np.iinfo(dtype).min // 2, np.iinfo(dtype).max // 2, n,
                             dtype=np.int64 if dtype != np.uint64 else np.uint64).astype(dtype)
        k = k[np.argsort(order_image(k, desc), kind="stable")]
        runs.append(k)
    return runs


def merge(runs, desc, vb, device="cuda:0"):
    keys = np.concatenate(runs)
    n = keys.size
    vals = None
    if vb:
        vals = np.arange(n * vb, dtype=np.uint8).reshape(n, vb) if vb != 4 else \
            np.arange(n, dtype=np.uint32)
    tk = torch.from_numpy(keys.copy()).to(device)
    tv = torch.from_numpy(vals.copy()).to(device) if vals is not None else None
    lens = [r.size for r in runs]
    kb = tk.element_size()
    kp, vp, off = [], [], 0
    for n_ in lens:
        kp.append(tk.data_ptr() + off * kb if n_ else None)
        vp.append(tv.data_ptr() + off * vb if (n_ and tv is not None) else None)
        off += n_
    ok, ov = D.multiway_merge(tk, tv, kp, vp, lens, desc,
                              torch.cuda.current_stream(device).cuda_stream)
    torch.cuda.synchronize()
    return keys, vals, ok.cpu().numpy(), (ov.cpu().numpy() if ov is not None else None)


@pytest.mark.parametrize("W", [2, 3, 5, 8, 9, 16, 64])
@pytest.mark.parametrize("mode", ["random", "dup", "disjoint"])
def test_multiway_matches_stable_merge(W, mode):
    rng = np.random.default_rng(W * 10 + len(mode))
    lens = [int(x) for x in rng.integers(0, 40_000, W)]
    lens[0] = 0 if W > 2 else lens[0]
    lens[-1] = 1
    for dtype, desc, vb in [(np.uint64, False, 4), (np.float32, True, 0), (np.int32, False, 16)]:
        if mode == "disjoint" and np.dtype(dtype).kind == "f":
            continue
        runs = make_runs(rng, lens, dtype, desc, mode)
        keys, vals, gk, gv = merge(runs, desc, vb)
        perm = np.argsort(order_image(keys, desc), kind="stable")
        assert np.array_equal(bits(gk), bits(keys[perm])), (dtype, desc)
        if vb:
            assert np.array_equal(gv, vals[perm])


def test_multiway_large_skewed_lengths():
    """Runs whose lengths differ by 1000x and a 2^24-item total."""
    rng = np.random.default_rng(1)
    lens = [1 << 23, 3, 1 << 22, 8191, (1 << 22) - 8194, 0, 5, 12345]
    runs = make_runs(rng, lens, np.uint64, False, "random")
    keys, vals, gk, gv = merge(runs, False, 4)
    perm = np.argsort(keys, kind="stable")
    assert np.array_equal(gk, keys[perm]) and np.array_equal(gv, vals[perm])


def test_multiway_argument_checks():
    L = _lib.lib()
    SZ, VP = ctypes.c_size_t * 2, ctypes.c_void_p * 2
    assert L.rsort_merge_multiway(_lib.RSORT_U8, 0, 2, VP(16, 32), None, SZ(1, 1), 0, 64, None,
                                  128, 1 << 20, None) == _lib.RSORT_BAD_ARGUMENT
    assert L.rsort_merge_multiway(_lib.RSORT_U32, 0, 0, VP(16, 32), None, SZ(1, 1), 0, 64, None,
                                  128, 1 << 20, None) == _lib.RSORT_BAD_ARGUMENT
    need = L.rsort_multiway_scratch_bytes(_lib.RSORT_U32, 0, 2, 2)
    assert L.rsort_merge_multiway(_lib.RSORT_U32, 0, 2, VP(16, 32), None, SZ(1, 1), 0, 64, None,
                                  128, need - 1, None) == _lib.RSORT_WORKSPACE_TOO_SMALL
