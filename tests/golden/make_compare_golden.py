"""Generate tests/golden/compare_probes.npz and compare_probes.json: the
reference's own comparator-sort cases (DeviceMergeSort / Thrust sort_by with a
closure), as golden vectors for the comparator-program sort (rsort_sort_by).

Each case restates one call of the reference: its input (a literal, or the
example's own formula), the closure as comparator-program terms, and the
expected output exactly as the example states it (a literal assert, or the
Rust std expression the example compares against, restated here with numpy
stable sorts: `sort_by` / `sort_by_key` are stable).  The oracle under test
is never used here.

Sources (paths inside the reference project):
  rccl-thrust/examples/sort.rs                      literal asserts
  rccl-thrust/examples/set_operations_tests.rs      KeyValue<T, T> records, sort_by
  rccl-cub/examples/device_ordering_benchmark.rs    sort_by_key(|k| k & 0x00ff_ffff)

    python tests/golden/make_compare_golden.py
"""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def term(dtype, offset=0, projection="identity", operand=0, descending=False, total=False):
    return dict(dtype=np.dtype(dtype).name, offset=offset, projection=projection,
                operand=operand, descending=descending, total=total)


def random_u32(count):
    # device_ordering_benchmark.rs:71-81: xorshift of index ^ 0x534d_4152_545f_534f, low 32 bits
    v = np.arange(count, dtype=np.uint64) ^ np.uint64(0x534D4152545F534F)
    v ^= v << np.uint64(13)
    v ^= v >> np.uint64(7)
    v ^= v << np.uint64(17)
    return v.astype(np.uint32)


def main():
    arrays, cases = {}, []

    def add(name, source, records, terms, expected, values=None, expected_values=None):
        arrays[f"{name}__records"] = np.asarray(records)
        arrays[f"{name}__expected"] = np.asarray(expected)
        if values is not None:
            arrays[f"{name}__values"] = np.asarray(values)
            arrays[f"{name}__expected_values"] = np.asarray(expected_values)
        cases.append(dict(name=name, source=source, terms=terms, has_values=values is not None))

    tp = "rccl-thrust/examples/sort.rs"
    up = np.array([79, 78, 62, 78, 94, 40, 86, 57, 40, 16, 28, 54, 77, 87, 93, 98], np.int32)
    add("C_upstream_descending", tp + ":28-35", up, [term(np.int32, descending=True)],
        np.array([98, 94, 93, 87, 86, 79, 78, 78, 77, 62, 57, 54, 40, 40, 28, 16], np.int32))
    # match ((l & 1) == 0, (r & 1) == 0): evens first, then l.cmp(r)
    add("C_upstream_evens_first", tp + ":37-50", up,
        [term(np.int32, projection="and", operand=1), term(np.int32)],
        np.array([16, 28, 40, 40, 54, 62, 78, 78, 86, 94, 98, 57, 77, 79, 87, 93], np.int32))
    small = np.array([1, 3, 6, 5, 2, 0, 4], np.int32)
    add("C_small_descending", tp + ":96-98", small, [term(np.int32, descending=True)],
        np.array([6, 5, 4, 3, 2, 1, 0], np.int32))
    add("C_parity_then_value", tp + ":100-104", np.array([5, 2, 9, 4, 7, 0, 3, 6], np.int32),
        [term(np.int32, projection="and", operand=1), term(np.int32)],
        np.array([0, 2, 4, 6, 3, 5, 7, 9], np.int32))
    stable_input = np.array([25, 14, 35, 16, 26, 34, 36, 24, 15], np.int32)
    stable_expected = np.array([14, 16, 15, 25, 26, 24, 35, 34, 36], np.int32)
    add("C_stable_div10", tp + ":106-114", stable_input,
        [term(np.int32, projection="div", operand=10)], stable_expected)
    add("C_pairs_descending", tp + ":129-139", small, [term(np.int32, descending=True)],
        np.array([6, 5, 4, 3, 2, 1, 0], np.int32), values=np.arange(7, dtype=np.int32),
        expected_values=np.array([2, 3, 6, 1, 4, 0, 5], np.int32))
    add("C_pairs_stable_div10", tp + ":150-165", stable_input,
        [term(np.int32, projection="div", operand=10)], stable_expected,
        values=np.arange(9, dtype=np.int32),
        expected_values=np.array([1, 3, 8, 0, 4, 7, 2, 5, 6], np.int32))

    # set_operations_tests.rs:133-152: KeyValue { key, value } (#[repr(C)]),
    # key = T::from_i32((i * 37 + 11) % 17), value = T::from_i32((i * 5 + 1) % 97),
    # first.sort_by(|l, r| l.key vs r.key) -- stable.
    sp = "rccl-thrust/examples/set_operations_tests.rs:133-152"
    idx = np.arange(4097)
    for dt in (np.int8, np.uint8, np.int16, np.uint16, np.int32, np.uint32, np.float32,
               np.float64):
        rec = np.stack([(idx * 37 + 11) % 17, (idx * 5 + 1) % 97], axis=1).astype(dt)
        order = np.argsort(rec[:, 0], kind="stable")
        add(f"C_keyvalue_{np.dtype(dt).name}", sp, rec, [term(dt, offset=0)], rec[order])

    # device_ordering_benchmark.rs:158-162, the first 12_289 of its 1_000_003
    # items (past the single-tile extent, so the onesweep passes run)
    keys = random_u32(12_289)
    order = np.argsort(keys & np.uint32(0x00FFFFFF), kind="stable")
    add("C_window_key", "rccl-cub/examples/device_ordering_benchmark.rs:71-81,158-162", keys,
        [term(np.uint32, projection="and", operand=0x00FFFFFF)], keys[order])

    np.savez_compressed(os.path.join(HERE, "compare_probes.npz"), **arrays)
    with open(os.path.join(HERE, "compare_probes.json"), "w") as fh:
        json.dump(cases, fh, indent=1)
    print(f"{len(cases)} cases")


if __name__ == "__main__":
    main()
