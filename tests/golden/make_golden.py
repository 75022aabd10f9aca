"""Generate tests/golden/probes.npz and probes.json from the reference's own
GPU probes (the golden vectors of the DeviceRadixSort path).

Each case restates one probe case of the reference: the input formula or
literal, the API form, and the expected output exactly as the probe states it
(a Rust std sort expression, or a literal).  Expected outputs are computed here
with numpy stable sorts that restate those Rust expressions (`sort_unstable` on
integer keys equals a numeric sort; `sort_by_key` / `sort_by` are stable), and
never with the oracle under test.

Sources (paths inside the reference project):
  K* rccl-cub/examples/device_radix_sort_keys_probe.rs
  P* rccl-cub/examples/device_radix_sort_pairs_probe.rs
  S* rccl-cub/examples/device_radix_sort_single_tile_probe.rs,
     rccl-cub/examples/device_radix_sort_single_tile_pairs_probe.rs
  T* rccl-thrust/examples/sort.rs

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
M32 = 0xFFFFFFFF
M64 = 0xFFFFFFFFFFFFFFFF


def rotl32(x, r):
    r &= 31
    return ((x << r) | (x >> (32 - r))) & M32 if r else x


def rotl64(x, r):
    r &= 63
    return ((x << r) | (x >> (64 - r))) & M64 if r else x


def hashed_u32(n):
    # index.wrapping_mul(2_654_435_761).rotate_left(index & 31)
    return np.array([rotl32((i * 2654435761) & M32, i & 31) for i in range(n)], dtype=np.uint32)


def main():
    arrays = {}
    cases = []

    def add(name, source, api, key_dtype, keys, expected_keys, descending=False, bit_range=None,
            values=None, expected_values=None, second=None, expect_current_is_first=None,
            expect_error=None):
        arrays[f"{name}__keys"] = np.asarray(keys)
        arrays[f"{name}__expected_keys"] = np.asarray(expected_keys)
        meta = dict(name=name, source=source, api=api, key_dtype=key_dtype,
                    descending=descending, bit_range=bit_range,
                    has_values=values is not None,
                    expect_current_is_first=expect_current_is_first,
                    expect_error=expect_error, has_second=second is not None)
        if values is not None:
            arrays[f"{name}__values"] = np.asarray(values)
            arrays[f"{name}__expected_values"] = np.asarray(expected_values)
        if second is not None:
            arrays[f"{name}__second"] = np.asarray(second)
        cases.append(meta)

    kp = "rccl-cub/examples/device_radix_sort_keys_probe.rs"
    add("K_empty", kp + ":27-31", "keys", "uint32", np.zeros(0, np.uint32), np.zeros(0, np.uint32))

    x = hashed_u32(10_003)
    x[17] = 0
    x[29] = M32
    add("K_hashed_u32", kp + ":36-46", "keys", "uint32", x, np.sort(x))
    add("K_one", kp + ":51-55", "keys", "uint32", np.array([42], np.uint32),
        np.array([42], np.uint32))
    x64 = np.array([rotl64((i * 11_400_714_819_323_198_485) & M64, i & 63)
                    for i in range(10_003)], dtype=np.uint64)
    add("K_hashed_u64", kp + ":61-73", "keys", "uint64", x64, np.sort(x64))
    si = np.array([0, -1, -2**31, 7, -9, 2**31 - 1, -1, 0], np.int32)
    add("K_i32_desc", kp + ":75-83", "keys", "int32", si,
        np.array([2**31 - 1, 7, 0, 0, -1, -1, -9, -2**31], np.int32), descending=True)
    si64 = np.array([0, -1, -2**63, 7, -9, 2**63 - 1, -1, 0], np.int64)
    add("K_i64_desc", kp + ":85-97", "keys", "int64", si64,
        np.array([2**63 - 1, 7, 0, 0, -1, -1, -9, -2**63], np.int64), descending=True)
    fin = np.array([3.0, -0.0, -np.inf, 0.0, -7.5, np.inf], np.float32)
    add("K_f32_zeros", kp + ":99-119", "keys", "float32", fin,
        np.array([-np.inf, -7.5, -0.0, 0.0, 3.0, np.inf], np.float32))
    nan32 = np.array([0x7fc00001, 0x3f800000, 0xff800001, 0xffc00001, 0xbf800000, 0x7f800001],
                     np.uint32).view(np.float32)
    asc32 = np.array([0xffc00001, 0xff800001, 0xbf800000, 0x3f800000, 0x7f800001, 0x7fc00001],
                     np.uint32).view(np.float32)
    add("K_f32_nan_asc", kp + ":121-173", "keys", "float32", nan32, asc32)
    add("K_f32_nan_desc", kp + ":121-173", "keys", "float32", nan32, asc32[::-1].copy(),
        descending=True)
    fin64 = np.array([3.0, -0.0, -np.inf, 0.0, -7.5, np.inf], np.float64)
    add("K_f64_zeros", kp + ":175-194", "keys", "float64", fin64,
        np.array([-np.inf, -7.5, -0.0, 0.0, 3.0, np.inf], np.float64))
    nan64 = np.array([0x7ff8000000000001, 0x3ff0000000000000, 0xfff0000000000001,
                      0xfff8000000000001, 0xbff0000000000000, 0x7ff0000000000001],
                     np.uint64).view(np.float64)
    asc64 = np.array([0xfff8000000000001, 0xfff0000000000001, 0xbff0000000000000,
                      0x3ff0000000000000, 0x7ff0000000000001, 0x7ff8000000000001],
                     np.uint64).view(np.float64)
    add("K_f64_nan_asc", kp + ":196-246", "keys", "float64", nan64, asc64)
    add("K_f64_nan_desc", kp + ":196-246", "keys", "float64", nan64, asc64[::-1].copy(),
        descending=True)
    ent = np.array([(i * 2654435761) & M32 & 31 for i in range((1 << 17) + 3)], np.uint32)
    add("K_entropy_asc", kp + ":251-274", "keys", "uint32", ent, np.sort(ent))
    add("K_entropy_desc", kp + ":251-274", "keys", "uint32", ent, np.sort(ent)[::-1].copy(),
        descending=True)
    uni = np.full((1 << 17) + 3, 4, np.uint32)
    add("K_uniform_asc", kp + ":279-294", "keys", "uint32", uni, uni)
    add("K_uniform_desc", kp + ":279-294", "keys", "uint32", uni, uni, descending=True)
    win = np.array([(((i & 0xff) << 24) | ((i * 2654435761) & 0x00ffffff)) & M32
                    for i in range(10_003)], np.uint32)
    field = win & 0x00ffffff
    add("K_window24_asc", kp + ":300-339", "keys_buffer", "uint32", win,
        win[np.argsort(field, kind="stable")], bit_range=[0, 24],
        second=np.zeros_like(win), expect_current_is_first=False)
    add("K_window24_desc", kp + ":300-339", "keys_buffer", "uint32", win,
        win[np.argsort(-field.astype(np.int64), kind="stable")], descending=True,
        bit_range=[0, 24], second=np.zeros_like(win), expect_current_is_first=False)
    noop = np.array([9, 1, 7, 3], np.uint32)
    add("K_empty_window", kp + ":345-358", "keys_buffer", "uint32", noop, noop,
        bit_range=[12, 12], second=np.full(4, 99, np.uint32), expect_current_is_first=True)
    add("K_invalid_window", kp + ":360-376", "keys_buffer", "uint32", noop, noop,
        bit_range=[25, 17], second=np.full(4, 99, np.uint32), expect_current_is_first=True,
        expect_error=["InvalidBitRange", 25, 17, 32])
    add("K_window8_small", kp + ":380-391", "keys_buffer", "uint32", noop,
        noop[np.argsort(noop & 0xff, kind="stable")], bit_range=[0, 8],
        second=np.full(4, 99, np.uint32), expect_current_is_first=False)
    bnd = np.arange(4_864, -1, -1, dtype=np.uint32)
    add("K_boundary_4865", kp + ":395-413", "keys_buffer", "uint32", bnd,
        bnd[np.argsort(bnd & 0xff, kind="stable")], bit_range=[0, 8],
        second=np.zeros_like(bnd), expect_current_is_first=False)

    pp = "rccl-cub/examples/device_radix_sort_pairs_probe.rs"
    add("P_empty", pp + ":18-28", "pairs", "uint32", np.zeros(0, np.uint32),
        np.zeros(0, np.uint32), values=np.zeros(0, np.int32), expected_values=np.zeros(0, np.int32))
    pk = hashed_u32(10_003) & np.uint32(0x3ff)
    pv = np.arange(10_003, dtype=np.int32)
    o = np.argsort(pk, kind="stable")
    add("P_narrow_asc", pp + ":34-70", "pairs", "uint32", pk, pk[o], values=pv,
        expected_values=pv[o])
    od = np.argsort(-pk.astype(np.int64), kind="stable")
    add("P_narrow_desc", pp + ":72-99", "pairs", "uint32", pk, pk[od], values=pv,
        expected_values=pv[od], descending=True)
    wv = np.arange(10_003, dtype=np.uint64)
    add("P_u32_u64", pp + ":105-137", "pairs", "uint32", pk, pk[o], values=wv,
        expected_values=wv[o])
    pk64 = pk.astype(np.uint64)
    add("P_u64_u64", pp + ":142-175", "pairs", "uint64", pk64, pk64[o], values=wv,
        expected_values=wv[o])
    fk = np.array([1.25, -0.0, np.inf, -3.5, 0.0, -np.inf], np.float32)
    fv = np.array([4, 2, 5, 1, 3, 0], np.int32)
    fexp = np.array([-np.inf, -3.5, -0.0, 0.0, 1.25, np.inf], np.float32)
    add("P_f32_i32", pp + ":180-207", "pairs", "float32", fk, fexp, values=fv,
        expected_values=np.arange(6, dtype=np.int32))
    add("P_f32_i32_buffer", pp + ":212-248", "pairs_buffer", "float32", fk, fexp, values=fv,
        expected_values=np.arange(6, dtype=np.int32), bit_range=[0, 32],
        second=np.zeros_like(fk), expect_current_is_first=False)
    wk = np.array([(((i & 0xff) << 24) | ((i * 97) & 0x3ff)) & M32 for i in range(10_003)],
                  np.uint32)
    wvv = np.arange(10_003, dtype=np.int32)
    f = wk & 0x00ffffff
    oa = np.argsort(f, kind="stable")
    odd = np.argsort(-f.astype(np.int64), kind="stable")
    add("P_window24_asc", pp + ":253-306", "pairs_buffer", "uint32", wk, wk[oa], values=wvv,
        expected_values=wvv[oa], bit_range=[0, 24], second=np.zeros_like(wk),
        expect_current_is_first=False)
    add("P_window24_desc", pp + ":253-306", "pairs_buffer", "uint32", wk, wk[odd], values=wvv,
        expected_values=wvv[odd], bit_range=[0, 24], descending=True, second=np.zeros_like(wk),
        expect_current_is_first=False)

    sp = "rccl-cub/examples/device_radix_sort_single_tile_probe.rs"
    st = hashed_u32(4_864)
    add("S_tile_u32", sp + ":21-34", "keys_buffer", "uint32", st, np.sort(st), bit_range=[0, 32],
        second=np.zeros_like(st), expect_current_is_first=False)
    sw = np.array([(((i % 37) << 3) | ((i * 97) & 0xfff80007)) & M32 for i in range(4_097)],
                  np.uint32)
    sf = (sw >> 3) & ((1 << 16) - 1)
    add("S_window_3_19_desc", sp + ":38-67", "keys_buffer", "uint32", sw,
        sw[np.argsort(-sf.astype(np.int64), kind="stable")], descending=True, bit_range=[3, 19],
        second=np.zeros_like(sw), expect_current_is_first=False)
    spp = "rccl-cub/examples/device_radix_sort_single_tile_pairs_probe.rs"
    stk = np.array([(i * 17) % 113 for i in range(4_864)], np.uint32)
    stv = np.arange(4_864, dtype=np.uint32)
    so = np.argsort(stk, kind="stable")
    add("S_tile_pairs", spp + ":15-48", "pairs_buffer", "uint32", stk, stk[so], values=stv,
        expected_values=stv[so], bit_range=[0, 32], second=np.zeros_like(stk),
        expect_current_is_first=False)

    tp = "rccl-thrust/examples/sort.rs"
    up = np.array([79, 78, 62, 78, 94, 40, 86, 57, 40, 16, 28, 54, 77, 87, 93, 98], np.int32)
    add("T_upstream_sort_unstable", tp + ":16-26", "thrust_sort_unstable", "int32", up,
        np.array([16, 28, 40, 40, 54, 57, 62, 77, 78, 78, 79, 86, 87, 93, 94, 98], np.int32))
    add("T_upstream_pairs", tp + ":52-70", "thrust_pairs_sort_unstable", "int32", up,
        np.array([16, 28, 40, 40, 54, 57, 62, 77, 78, 78, 79, 86, 87, 93, 94, 98], np.int32),
        values=np.arange(16, dtype=np.int32),
        expected_values=np.array([9, 10, 5, 8, 11, 7, 2, 12, 1, 3, 0, 6, 13, 14, 4, 15],
                                 np.int32))
    small = np.array([1, 3, 6, 5, 2, 0, 4], np.int32)
    add("T_small_sort_unstable", tp + ":92-94", "thrust_sort_unstable", "int32", small,
        np.arange(7, dtype=np.int32))
    add("T_natural_stable", tp + ":116-118", "thrust_sort", "int32",
        np.array([3, 1, 2, 1], np.int32), np.array([1, 1, 2, 3], np.int32))
    add("T_pairs_sort", tp + ":120-127", "thrust_pairs_sort", "int32", small,
        np.arange(7, dtype=np.int32), values=np.arange(7, dtype=np.int32),
        expected_values=np.array([5, 0, 4, 1, 6, 3, 2], np.int32))
    add("T_pairs_sort_unstable", tp + ":141-148", "thrust_pairs_sort_unstable", "int32", small,
        np.arange(7, dtype=np.int32), values=np.arange(7, dtype=np.int32),
        expected_values=np.array([5, 0, 4, 1, 6, 3, 2], np.int32))
    add("T_f32_pairs", tp + ":167-191", "thrust_pairs_sort", "float32", fk, fexp, values=fv,
        expected_values=np.arange(6, dtype=np.int32))

    np.savez_compressed(os.path.join(HERE, "probes.npz"), **arrays)
    with open(os.path.join(HERE, "probes.json"), "w") as fh:
        json.dump(cases, fh, indent=1)
    print(f"{len(cases)} cases")


if __name__ == "__main__":
    main()
