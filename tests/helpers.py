"""Shared test helpers: golden fixtures and numpy <-> torch transfer."""
from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

NP_OF = {"uint32": np.uint32, "int32": np.int32, "float32": np.float32, "uint64": np.uint64,
         "int64": np.int64, "float64": np.float64}


def load_cases():
    with open(os.path.join(GOLDEN, "probes.json")) as fh:
        meta = json.load(fh)
    arrays = np.load(os.path.join(GOLDEN, "probes.npz"))
    out = []
    for m in meta:
        name = m["name"]
        case = dict(m)
        case["keys"] = arrays[f"{name}__keys"]
        case["expected_keys"] = arrays[f"{name}__expected_keys"]
        if m["has_values"]:
            case["values"] = arrays[f"{name}__values"]
            case["expected_values"] = arrays[f"{name}__expected_values"]
        if m["has_second"]:
            case["second"] = arrays[f"{name}__second"]
        out.append(case)
    return out


def bits(a: np.ndarray) -> np.ndarray:
    """Raw bit patterns, so float comparisons are bit-exact (NaN payloads, -0.0)."""
    a = np.ascontiguousarray(a)
    if a.dtype.itemsize == 4:
        return a.view(np.uint32)
    if a.dtype.itemsize == 8:
        return a.view(np.uint64)
    if a.dtype.itemsize == 2:
        return a.view(np.uint16)
    return a.view(np.uint8)


def to_dev(a: np.ndarray, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def to_host(t) -> np.ndarray:
    return t.cpu().numpy()


def order_image(keys: np.ndarray, descending: bool = False) -> np.ndarray:
    """Unsigned image whose ascending order is the reference's sort order for
    full-width sorts (to_ordered + float zero fold, vectorized)."""
    w = keys.dtype.itemsize * 8
    ut = np.uint32 if w == 32 else np.uint64
    u = np.ascontiguousarray(keys).view(ut)
    sign = ut(1 << (w - 1))
    if keys.dtype.kind == "f":
        o = np.where((u & sign) != 0, ~u, u ^ sign)
    elif keys.dtype.kind == "i":
        o = u ^ sign
    else:
        o = u.copy()
    if descending:
        o = ~o
    if keys.dtype.kind == "f":
        o = np.where(o == sign - ut(1), sign, o)
    return o.astype(np.uint64)


def load_compare_cases():
    """The reference's comparator-sort golden cases (make_compare_golden.py)."""
    with open(os.path.join(GOLDEN, "compare_probes.json")) as fh:
        meta = json.load(fh)
    arrays = np.load(os.path.join(GOLDEN, "compare_probes.npz"))
    out = []
    for m in meta:
        name = m["name"]
        case = dict(m)
        case["records"] = arrays[f"{name}__records"]
        case["expected"] = arrays[f"{name}__expected"]
        if m["has_values"]:
            case["values"] = arrays[f"{name}__values"]
            case["expected_values"] = arrays[f"{name}__expected_values"]
        out.append(case)
    return out


def oracle_terms(terms):
    """Golden-case term dicts -> oracle.compare_oracle.Term."""
    from oracle.compare_oracle import Term
    return [Term(np.dtype(t["dtype"]), t["offset"], t["projection"], t["operand"],
                 t["descending"], t["total"]) for t in terms]


def program_of(terms):
    """Golden-case term dicts -> rccl_b200.compare.Comparator."""
    import torch
    from rccl_b200 import compare
    keys = []
    for t in terms:
        k = compare.Key(torch.from_numpy(np.zeros(0, np.dtype(t["dtype"]))).dtype, t["offset"])
        if t["projection"] != "identity":
            k = getattr(k, {"and": "and_"}.get(t["projection"], t["projection"]))(t["operand"])
        if t["descending"]:
            k = k.reverse()
        if t["total"]:
            k = k.total()
        keys.append(k)
    return compare.Comparator(tuple(keys))
