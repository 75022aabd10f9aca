"""Benchmark of the B200 DeviceRadixSort hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl rccl_b200|reference]

One step is one sort of the workload's whole input.  `value` is device-timed
sorted keys/s with the input resident in HBM (CUDA events around each sort on
the sort's stream; the untimed restore of the input happens between steps).
`e2e` is the same metric through the public rccl-thrust style API
(thrust.with_values(...).sort()) with the input copied from pinned host memory
and the sorted keys and values copied back inside the timed region.

With one GPU the headline line is config 2; its `configs` block carries
configs 1, 3, 4 and 5 timed the same way, each with its own roofline, clock
record and bit-exact output check.  With N > 1 GPUs (torchrun) the default is
config 5 as strong scaling: 2^32 pairs in total, rank r holding the contiguous
shard [r*n/N, (r+1)*n/N) of the global input, sorted by the sample sort.

Workloads are seeded synthetic inputs with the reference benchmark shapes.
Every item is a pure function of its global index (splitmix64 counters, Box-
Muller normals, inverse-CDF Zipf), so any shard or sample of a workload is
generated on its own, on the GPU or the CPU, identically:
  1: 2^20 u32 keys, uniform, ascending keys-only
  2: 2^28 u64 keys uniform over 64 bits + u32 values = index,
     stable ascending pairs (the headline)
  3: 2^28 f32 keys ~ N(0, 1e3) with 0.1% +-0, 0.01% +-inf and 0.01% quiet
     NaNs with random payloads, descending keys-only
  4: 2^30 u32 keys, 90% Zipf(1.1) over 2^20 values (mapped through a seeded
     bijection of u32) + 10% one constant, ascending keys-only
  5: config 2's distribution at n = 2^32 pairs (values = global index)
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "sorted keys/s (device-timed)"
UNIT = "keys/s"
FALLBACK_HBM_GBS = 6650.0
NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool
CHUNK = 1 << 26     # generation and check granularity (items)

# ---------------------------------------------------------------------------
# Counter-based generators (torch int64 arithmetic wraps like uint64)
# ---------------------------------------------------------------------------
_G = 0x9E3779B97F4A7C15
_M1 = 0xBF58476D1CE4E5B9
_M2 = 0x94D049BB133111EB


def _s64(c: int) -> int:
    return c - (1 << 64) if c >= 1 << 63 else c


def _lsr(x, k: int):
    """Logical right shift of an int64 tensor."""
    return (x >> k) & ((1 << (64 - k)) - 1)


def splitmix64(idx, seed: int):
    """splitmix64 finalizer of (index + seed) * golden ratio: uniform 64-bit
    words as int64 tensors."""
    z = (idx + seed) * _s64(_G)
    z = (z ^ _lsr(z, 30)) * _s64(_M1)
    z = (z ^ _lsr(z, 27)) * _s64(_M2)
    return z ^ _lsr(z, 31)


def multiset_hash(keys):
    """Order-independent hash of a key tensor: the wrapping int64 sum of a
    splitmix64 mix of each key's bits.  Equal for any permutation of the same
    keys, so a sort's output must reproduce its input's value (a checksum of
    checksums across ranks when summed over them)."""
    import torch
    w = keys.view(torch.int32 if keys.element_size() == 4 else torch.int64)
    total = torch.zeros((), dtype=torch.int64, device=keys.device)
    for a in range(0, w.numel(), CHUNK):
        bits = w[a:a + CHUNK].to(torch.int64)
        if keys.element_size() == 4:
            bits &= 0xFFFFFFFF
        total += splitmix64(bits, 0x5EED).sum()
    return total


def uniform01(h):
    """Uniform float64 in (0, 1] from a 64-bit word."""
    import torch
    return (_lsr(h, 11) + 1).to(torch.float64) * (2.0 ** -53)


def fmix32(x):
    """MurmurHash3's 32-bit finalizer: a bijection of u32 (int64 tensors
    holding values < 2^32)."""
    m = 0xFFFFFFFF
    x = x & m
    x = (x ^ (x >> 16)) & m
    x = (x * 0x85EBCA6B) & m
    x = (x ^ (x >> 13)) & m
    x = (x * 0xC2B2AE35) & m
    return (x ^ (x >> 16)) & m


def _to_i32(x):
    """int64 tensor of u32 bit patterns -> int32 tensor of the same bits."""
    import torch
    return torch.where(x >= 1 << 31, x - (1 << 32), x).to(torch.int32)


_ZIPF_CDF = {}


def zipf_cdf(device):
    import torch
    key = str(device)
    if key not in _ZIPF_CDF:
        ranks = torch.arange(1, (1 << 20) + 1, dtype=torch.float64, device=device)
        cdf = torch.cumsum(ranks ** -1.1, 0)
        _ZIPF_CDF[key] = cdf / cdf[-1]
    return _ZIPF_CDF[key]


class Workload:
    def __init__(self, config: int, n_override: int | None = None):
        self.config = config
        if config == 1:
            self.n, self.key, self.value, self.desc = 1 << 20, np.uint32, None, False
            self.name = "keys-only u32 ascending, uniform"
        elif config == 2:
            self.n, self.key, self.value, self.desc = 1 << 28, np.uint64, np.uint32, False
            self.name = "stable pairs u64 keys / u32 values ascending, uniform"
        elif config == 3:
            self.n, self.key, self.value, self.desc = 1 << 28, np.float32, None, True
            self.name = "keys-only f32 descending, N(0,1e3) with +-0/+-inf/NaN"
        elif config == 4:
            self.n, self.key, self.value, self.desc = 1 << 30, np.uint32, None, False
            self.name = "keys-only u32 ascending, 90% Zipf(1.1) over 2^20 + 10% constant"
        elif config == 5:
            self.n, self.key, self.value, self.desc = 1 << 32, np.uint64, np.uint32, False
            self.name = "stable pairs u64 keys / u32 values (global index) ascending, 2^32 pairs"
        else:
            raise SystemExit(f"unknown config {config}")
        if n_override:
            self.n = n_override
        self.kb = np.dtype(self.key).itemsize
        self.vb = np.dtype(self.value).itemsize if self.value is not None else 0
        self.passes = self.kb  # 8-bit digits over the full key width

    @property
    def bytes_per_sort(self) -> int:
        # one histogram read + per pass read and write of keys and values
        return self.n * self.kb + self.passes * 2 * self.n * (self.kb + self.vb)

    @property
    def bytes_per_pass(self) -> int:
        return 2 * self.n * (self.kb + self.vb)

    def torch_dtypes(self):
        import torch
        kd = {np.uint32: torch.uint32, np.uint64: torch.uint64, np.float32: torch.float32}[self.key]
        vd = torch.uint32 if self.value is not None else None
        return kd, vd

    def _keys_chunk(self, idx):
        """Key bit patterns of the global indices `idx` (int64 tensor): int64
        for 8-byte keys, int32 for 4-byte keys."""
        import torch
        c = self.config
        if c in (2, 5):
            return splitmix64(idx, 2)
        if c == 1:
            return _to_i32(splitmix64(idx, 1) & 0xFFFFFFFF)
        if c == 3:
            u1 = uniform01(splitmix64(2 * idx, 3))
            u2 = uniform01(splitmix64(2 * idx + 1, 3))
            x = (torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * np.pi * u2) * 1e3)
            bits = x.to(torch.float32).view(torch.int32).to(torch.int64) & 0xFFFFFFFF
            h = splitmix64(idx, 1003)
            sel = _lsr(h, 1) % 10000          # 10 of 10000: +-0; 1: +-inf; 1: NaN
            sign = (_lsr(h, 63) & 1) << 31
            payload = _lsr(h, 20) & ((1 << 22) - 1)
            payload = torch.where(payload == 0, torch.ones_like(payload), payload)
            bits = torch.where(sel < 10, sign, bits)
            bits = torch.where(sel == 10, sign | 0x7F800000, bits)
            bits = torch.where(sel == 11, sign | 0x7FC00000 | payload, bits)
            return _to_i32(bits)
        if c == 4:
            u = uniform01(splitmix64(idx, 4)).clamp_(max=1.0)
            r = torch.searchsorted(zipf_cdf(idx.device), u).clamp_(max=(1 << 20) - 1)
            const = _lsr(splitmix64(idx, 1004), 1) % 10 == 0
            vals = torch.where(const, torch.full_like(r, 1 << 20), r)
            return _to_i32(fmix32(vals + 0x5BD1E995))
        raise AssertionError(c)

    def fill(self, keys, values, start: int) -> None:
        """Write items [start, start + len) of the workload into the given
        (device or host) torch tensors, in chunks."""
        import torch
        m = keys.numel()
        kv = keys.view(torch.int64 if self.kb == 8 else torch.int32)
        vv = values.view(torch.int32) if values is not None else None
        for a in range(0, m, CHUNK):
            b = min(m, a + CHUNK)
            idx = torch.arange(start + a, start + b, dtype=torch.int64, device=keys.device)
            kv[a:b] = self._keys_chunk(idx)
            if vv is not None:
                vv[a:b] = _to_i32(idx & 0xFFFFFFFF)

    def generate(self, start: int, count: int, device):
        import torch
        kd, vd = self.torch_dtypes()
        keys = torch.empty(count, dtype=kd, device=device)
        values = torch.empty(count, dtype=vd, device=device) if vd is not None else None
        self.fill(keys, values, start)
        return keys, values

    def host_sample(self, count: int):
        """numpy arrays of the first `count` items (generated on the CPU)."""
        k, v = self.generate(0, min(count, self.n), "cpu")
        return k.numpy(), (v.numpy() if v is not None else None)


# ---------------------------------------------------------------------------
# Output checks (device-side, size-independent or against an independent
# stable sort of the input's order image)
# ---------------------------------------------------------------------------
def order_image(keys: np.ndarray, descending: bool) -> np.ndarray:
    """Unsigned image whose ascending order is the sort order (radix.rs:75-235
    transforms with the float zero fold)."""
    w = keys.dtype.itemsize * 8
    u = keys.view(np.uint32 if w == 32 else np.uint64)
    sign = (np.uint32 if w == 32 else np.uint64)(1 << (w - 1))
    if keys.dtype.kind == "f":
        neg = (u & sign) != 0
        o = np.where(neg, ~u, u ^ sign)
    elif keys.dtype.kind == "i":
        o = u ^ sign
    else:
        o = u.copy()
    if descending:
        o = ~o
    if keys.dtype.kind == "f":
        o = np.where(o == sign - 1, sign, o)
    return o


def image_i64(keys, kind: str, descending: bool):
    """Order image of a 32- or 64-bit key tensor as int64 whose signed order is
    the sort order (radix.rs:75-235 transforms with the float zero fold)."""
    import torch
    if keys.element_size() == 4:
        u = keys.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        if kind == "f":
            o = torch.where(u >= 1 << 31, u ^ 0xFFFFFFFF, u ^ (1 << 31))
        elif kind == "i":
            o = u ^ (1 << 31)
        else:
            o = u
        if descending:
            o = o ^ 0xFFFFFFFF
        if kind == "f":
            o = torch.where(o == (1 << 31) - 1, torch.full_like(o, 1 << 31), o)
        return o
    u = keys.view(torch.int64)
    top = -(1 << 63)
    if kind == "f":
        o = torch.where(u < 0, ~u, u ^ top)
    elif kind == "i":
        o = u ^ top
    else:
        o = u
    if descending:
        o = ~o
    if kind == "f":
        o = torch.where(o == (1 << 63) - 1, torch.full_like(o, top), o)
    return o ^ top  # unsigned order -> signed order


def check_keys_only(inp, out, kind: str, descending: bool) -> bool:
    """Bit-exact comparison with an independent stable sort (torch.sort,
    stable=True) of the input's order image."""
    import torch
    w = torch.int32 if inp.element_size() == 4 else torch.int64
    perm = torch.sort(image_i64(inp, kind, descending), stable=True).indices
    exp = inp.view(w)[perm]
    del perm
    return bool(torch.equal(exp, out.view(w)))


def check_pairs_index(workload: Workload, keys, values, mark=None) -> bool:
    """Stable pairs whose values are global input indices: every output key
    equals the key its value's index generates, the order image never
    decreases, equal keys keep ascending indices, and every index is marked
    in `mark` (a uint8 tensor over all indices; with the output count equal to
    the index count, an all-ones mark means every index appears once)."""
    import torch
    m = keys.numel()
    ok = True
    prev_img = prev_idx = None
    kd = torch.int64 if workload.kb == 8 else torch.int32
    for a in range(0, m, CHUNK):
        b = min(m, a + CHUNK)
        idx = values[a:b].view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        k = keys[a:b]
        ok &= bool(torch.equal(workload._keys_chunk(idx), k.view(kd)))
        img = image_i64(k, np.dtype(workload.key).kind, workload.desc)
        if prev_img is not None:
            img = torch.cat([prev_img, img])
            idx2 = torch.cat([prev_idx, idx])
        else:
            idx2 = idx
        ok &= bool(torch.all(img[1:] >= img[:-1]))
        ties = img[1:] == img[:-1]
        ok &= bool(torch.all(idx2[1:][ties] > idx2[:-1][ties]))
        prev_img, prev_idx = img[-1:], idx[-1:]
        if mark is not None:
            mark[idx] = 1
    return ok


# ---------------------------------------------------------------------------
# Helpers
# ---------------------------------------------------------------------------
def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(workload: Workload):
    """DRAM bytes per onesweep launch from the committed ncu summary, scaled
    from the captured size to this workload's size by the items processed."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    cfg = 2 if workload.config == 5 else workload.config
    for line in open(path):
        if line.startswith("#"):
            continue
        f = dict(kv.split("=", 1) for kv in line.split() if "=" in kv)
        if f.get("config") == str(cfg) and f.get("kernel") == "onesweep":
            return float(f["dram_bytes_per_launch"]) * workload.n / float(f["n"])
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self._first = threading.Event()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            # nvidia-smi takes a moment to start: wait for its first sample so
            # the timed region is covered from its start; only samples taken
            # after that point are kept.
            t0 = time.time()
            while not self._first.wait(0.05) and time.time() - t0 < 5:
                pass
            self.lines.clear()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())
            self._first.set()

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def read_profile(L, cap: int):
    kid = (ctypes.c_int32 * cap)()
    kms = (ctypes.c_float * cap)()
    nrec = L.rsort_profile_read(kid, kms, cap)
    from rccl_b200 import _lib
    per_kernel = {}
    for i in range(min(nrec, cap)):
        per_kernel.setdefault(_lib.KERNEL_NAMES.get(kid[i], str(kid[i])), []).append(kms[i])
    return per_kernel


def roofline_of(workload: Workload, per_kernel, sort_ms: float | None):
    """Roofline of the dominant kernel (the onesweep pass): algorithmic bytes
    per pass over the mean CUDA-event time of a pass, against the measured
    HBM peak; with `sort_ms`, also the whole sort's byte model over the sort
    time.  A pass after the first is two launches -- the uniform-step form
    (onesweep_runs), which sorts passes with runs of equal keys and exits at
    once elsewhere, then the onesweep kernel, which exits at once where the
    first sorted the pass -- so a pass's time is the sum of both."""
    peak, peak_kind = measured_peak()
    osw = per_kernel.get("onesweep", [])
    if not osw:
        return None
    avg_s = (sum(osw) + sum(per_kernel.get("onesweep_runs", []))) / len(osw) / 1e3
    achieved = workload.bytes_per_pass / avg_s / 1e9
    out = {"bound": "hbm", "kernel": "onesweep", "achieved": achieved, "peak": peak,
           "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
           "traffic": profiled_traffic(workload),
           "algorithmic_bytes_per_launch": workload.bytes_per_pass,
           "avg_launch_ms": avg_s * 1e3}
    if sort_ms:
        sort_gbs = workload.bytes_per_sort / (sort_ms / 1e3) / 1e9
        out.update(sort_achieved=sort_gbs, sort_frac=sort_gbs / peak)
    return out


def cpu_baseline(workload: Workload, budget_s: float = 10.0):
    """The oracle port (stable LSD radix restatement of the reference's
    ordering) on all host cores over a bounded sample of the workload, with
    the C++ comparison-sort stand-ins for Rust's sort_unstable (one core) and
    rayon's par_sort_unstable (all cores) beside it."""
    from oracle import pyoracle
    threads = os.cpu_count() or 1
    sample = min(workload.n, 1 << 24)
    keys, values = workload.host_sample(sample)

    def rate(fn, n, reps=3):
        rates = []
        t_end = time.perf_counter() + budget_s
        while len(rates) < reps and (len(rates) < 1 or time.perf_counter() < t_end):
            t0 = time.perf_counter()
            fn()
            rates.append(n / (time.perf_counter() - t0))
        return statistics.median(rates), len(rates)

    v, reps = rate(lambda: pyoracle.radix_sort(keys, values, workload.desc, threads=threads),
                   sample, 5)
    stable = values is not None
    small = min(sample, 1 << 22)
    ks, vs = keys[:small], (values[:small] if values is not None else None)
    one, _ = rate(lambda: pyoracle.cpu_sort(ks, vs, workload.desc, stable, 1), small)
    par, _ = rate(lambda: pyoracle.cpu_sort(keys, values, workload.desc, stable, threads), sample)
    algo = "std::stable_sort" if stable else "std::sort"
    return {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"first {sample} items of the workload, {reps} timed sorts, median; "
                      f"oracle stable LSD radix on {threads} host threads",
            "stand_ins": [
                {"value": one, "unit": UNIT, "cores": 1,
                 "what": f"{algo} (for Rust slice::sort_unstable), first {small} items"},
                {"value": par, "unit": UNIT, "cores": threads,
                 "what": f"{threads}-thread chunked {algo} + pairwise std::merge "
                         f"(for rayon par_sort_unstable), first {sample} items"}]}


def config_dict(args, workload: Workload, world: int = 1, per_gpu_n: int | None = None,
                scaling: str = "weak"):
    d = {"workload": f"config {workload.config}: {workload.name}", "n": workload.n,
         "key": np.dtype(workload.key).name,
         "value": np.dtype(workload.value).name if workload.value is not None else None,
         "order": "descending" if workload.desc else "ascending", "stable": True,
         "per_gpu_n": per_gpu_n or workload.n,
         "parallelism": f"sample sort over {world} GPUs ({scaling} scaling)" if world > 1
         else "single GPU",
         "l2": ("input (4 MB) is L2-resident: a 256 MB buffer is written between steps to "
                "flush L2; the number is launch-bound latency" if workload.config == 1 else
                "input larger than the 126 MB L2; untimed restore between steps")}
    return d


def dist_config(args, workload: Workload, world: int, mode: str | None = None):
    """config of a multi-GPU line: config 5 is strong scaling (n fixed, rank r
    holds the r-th of N contiguous shards); other configs weak scaling (every
    rank holds a workload-sized shard)."""
    strong = workload.config == 5
    m = workload.n // world if strong else workload.n
    d = config_dict(args, workload, world, m, "strong" if strong else "weak")
    d["n"] = m * world
    d["exchange"] = EXCHANGE_NAMES[mode or os.environ.get("RSORT_EXCHANGE", "peer")]
    return d


# ---------------------------------------------------------------------------
# Reference arm: the reference's CPU restatement (oracle port), rank 0 only
# ---------------------------------------------------------------------------
def run_reference(args, workload: Workload, rank: int, world: int):
    if rank != 0:
        return
    from oracle import pyoracle
    threads = os.cpu_count() or 1
    sample = min(workload.n, 1 << 24)
    keys, values = workload.host_sample(sample)
    for _ in range(args.warmup):
        pyoracle.radix_sort(keys, values, workload.desc, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        pyoracle.radix_sort(keys, values, workload.desc, threads=threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = sample * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": ("strong" if world > 1 and workload.config == 5 else "weak"),
        "vs_baseline": None, "dtype": np.dtype(workload.key).name,
        "data": "synthetic (counter-based, seeded)",
        "config": dist_config(args, workload, world) if world > 1 else config_dict(args, workload),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"each step sorts the first {sample} items of the workload "
                                   f"(a full {workload.n}-item sort takes minutes on the host)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Single GPU
# ---------------------------------------------------------------------------
class SingleRun:
    """One workload on one GPU: buffers, the timed steps and the output check."""

    def __init__(self, args, workload: Workload, dev, keep_source: bool = True):
        import torch
        from rccl_b200 import cub
        self.args, self.w, self.dev = args, workload, dev
        self.launch = cub.Program.load(dev).on()
        self.stream = self.launch.stream
        kd, vd = workload.torch_dtypes()
        self.keys = torch.empty(workload.n, dtype=kd, device=dev)
        self.values = torch.empty(workload.n, dtype=vd, device=dev) if vd is not None else None
        self.src_k = self.src_v = None
        if keep_source:
            self.src_k, self.src_v = workload.generate(0, workload.n, dev)
        if self.values is not None:
            self.ws = cub.device_radix_sort_pairs_workspace(self.launch, kd, vd, workload.n)
        else:
            self.ws = cub.device_radix_sort_workspace(self.launch, kd, workload.n)
        self.flush = (torch.empty(256 << 20, dtype=torch.uint8, device=dev)
                      if workload.config == 1 else None)

    def restore(self):
        if self.src_k is not None:
            self.keys.copy_(self.src_k)
            if self.values is not None:
                self.values.copy_(self.src_v)
        else:
            self.w.fill(self.keys, self.values, 0)
        if self.flush is not None:
            self.flush.zero_()

    def sort(self):
        from rccl_b200 import cub
        w = self.w
        if self.values is None:
            (cub.device_radix_sort_keys_descending if w.desc
             else cub.device_radix_sort_keys)(self.launch, self.keys, self.ws)
        else:
            (cub.device_radix_sort_pairs_descending if w.desc
             else cub.device_radix_sort_pairs)(self.launch, self.keys, self.values, self.ws)

    def timed(self, steps: int, warmup: int, sample_clocks: bool = True):
        """`steps` sorts with a CUDA event pair around every kernel launch (the
        per-kernel durations), then `steps` sorts without them: the step time
        and the launch count.  The events between launches add their own gaps,
        a visible share of a sort of 0.1 ms, so they stay out of the step
        time."""
        import contextlib

        import torch
        from rccl_b200 import _lib, cub
        for _ in range(warmup):
            self.restore()
            self.sort()
        cub.check_device_status(self.launch, self.ws.controls)
        torch.cuda.synchronize()
        L = _lib.lib()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        sampler = (ClockSampler(torch.cuda.current_device()) if sample_clocks
                   else contextlib.nullcontext())
        with sampler as clocks:  # both loops: the clocks cover the kernel times too
            L.rsort_profile_read(None, None, 0)
            L.rsort_profile_enable(1)
            for _ in range(steps):
                self.restore()
                self.sort()
            L.rsort_profile_enable(0)
            torch.cuda.synchronize()
            per_kernel = read_profile(L, 64 * steps)
            L.rsort_launch_count_reset()
            for i in range(steps):
                self.restore()
                starts[i].record(self.stream)
                self.sort()
                stops[i].record(self.stream)
            torch.cuda.synchronize()
        launches = int(L.rsort_launch_count())
        cub.check_device_status(self.launch, self.ws.controls)
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, stops)]
        return step_ms, per_kernel, launches, (clocks.summary() if sample_clocks else None)

    def check(self) -> tuple[bool, str]:
        import torch
        w = self.w
        if self.values is not None:
            mark = torch.zeros(w.n, dtype=torch.uint8, device=self.dev)
            ok = check_pairs_index(w, self.keys, self.values, mark)
            ok &= bool(torch.all(mark == 1))
            del mark
            return ok, ("bit-exact: every key equals its value's generated key, order image "
                        "non-decreasing, equal keys in ascending input index, values a "
                        "permutation of all indices")
        src = self.src_k
        if src is None:
            src = w.generate(0, w.n, self.dev)[0]
        ok = check_keys_only(src, self.keys, np.dtype(w.key).kind, w.desc)
        return ok, "bit-exact against torch.sort(stable=True) of the input's order image"

    def free(self):
        import torch
        self.keys = self.values = self.src_k = self.src_v = self.ws = self.flush = None
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def measure_config(args, workload: Workload, dev, keep_source=True, min_timed_ms=0.0):
    """Time one workload and check its output; returns (summary dict, run).
    With min_timed_ms, the step count grows (from args.steps) until the timed
    region lasts that long, so the clock sampler sees it."""
    run = SingleRun(args, workload, dev, keep_source=keep_source)
    steps = args.steps
    if min_timed_ms > 0:
        probe, _, _, _ = run.timed(1, max(args.warmup, 1), sample_clocks=False)
        steps = max(steps, min(2000, int(min_timed_ms / max(probe[0], 1e-3)) + 1))
    step_ms, per_kernel, launches, clocks = run.timed(steps, args.warmup)
    total_ms = sum(step_ms)
    ok, how = run.check()
    sort_ms = total_ms / steps
    out = {
        "workload": f"config {workload.config}: {workload.name}", "n": workload.n,
        "value": workload.n / (sort_ms / 1e3), "unit": UNIT, "ms_per_step": sort_ms,
        "steps": steps, "warmup": args.warmup, "dtype": np.dtype(workload.key).name,
        "roofline": roofline_of(workload, per_kernel, sort_ms), "gpu_launches": launches,
        "kernels": {k: {"launches": len(v), "total_ms": sum(v), "avg_ms": statistics.mean(v)}
                    for k, v in per_kernel.items()},
        "clocks": clocks, "output_checked": ok, "check": how,
        "l2": config_dict(args, workload)["l2"],
    }
    return out, run


def run_single(args, workload: Workload):
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    head, run = measure_config(args, workload, dev)
    host_k, host_v = None, None
    if not args.no_e2e:
        host_k = run.src_k.cpu().numpy()
        host_v = run.src_v.cpu().numpy() if run.src_v is not None else None
    run.free()
    thrust_call = None if args.no_e2e else thrust_call_cost(args, workload, host_k, host_v, dev,
                                                            head["ms_per_step"])
    e2e = None if args.no_e2e else run_e2e(args, workload, host_k, host_v, dev)
    del host_k, host_v
    torch.cuda.empty_cache()

    configs = []
    if not args.no_configs and args.n is None and workload.config == 2:
        for c in (1, 3, 4, 5):
            w = Workload(c)
            if c == 5 and torch.cuda.get_device_properties(dev).total_memory < (150 << 30):
                configs.append({"workload": f"config 5: {w.name}",
                                "unavailable": "needs about 110 GB of device memory"})
                continue
            summary, r = measure_config(args, w, dev, keep_source=(c != 5), min_timed_ms=200.0)
            r.free()
            configs.append(summary)

    line = {
        "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": head["dtype"], "data": "synthetic (counter-based, seeded; generated on the GPU)",
        "config": config_dict(args, workload), "roofline": head["roofline"], "e2e": e2e,
        "thrust_call": thrust_call, "gpu_launches": head["gpu_launches"],
        "kernels": head["kernels"], "clocks": head["clocks"],
        "output_checked": head["output_checked"], "check": head["check"],
    }
    if configs:
        line["configs"] = configs
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(workload)
    print(json.dumps(line), flush=True)


def thrust_sort(execution, dk, dv, descending: bool) -> None:
    """One call of the public Thrust-style API: sort() / with_values().sort(),
    or sort_by(DESCENDING) for descending workloads (rccl-thrust's
    comparator-free sort is ascending only)."""
    from rccl_b200 import cub, thrust
    if descending:
        if dv is None:
            thrust.sort_by(execution, dk, cub.Order.DESCENDING)
        else:
            thrust.with_values(dk, dv).sort_by(execution, cub.Order.DESCENDING)
    elif dv is None:
        thrust.sort(execution, dk)
    else:
        thrust.with_values(dk, dv).sort(execution)


def thrust_api_name(workload: Workload, keys_only: bool) -> str:
    name = {(True, True): "rccl_b200.thrust sort_by(Order.DESCENDING)",
            (True, False): "rccl_b200.thrust with_values().sort_by(Order.DESCENDING)",
            (False, True): "rccl_b200.thrust sort()",
            (False, False): "rccl_b200.thrust with_values().sort()"}[(bool(workload.desc), keys_only)]
    return name + " (temporary allocation + sync per call)"


def thrust_call_cost(args, workload: Workload, keys_h, values_h, dev, device_ms: float):
    """Host time of the synchronous Thrust-style call on device-resident data
    (temporary allocation from the caching allocator, the sort, the stream
    synchronization) beside the device-timed sort: the per-call cost the
    reference's Thrust path adds."""
    import torch
    from rccl_b200 import thrust
    execution = thrust.Program.load(dev).par()
    src_k = torch.from_numpy(keys_h).to(dev)
    src_v = torch.from_numpy(values_h).to(dev) if values_h is not None else None
    dk = torch.empty_like(src_k)
    dv = torch.empty_like(src_v) if src_v is not None else None
    times = []
    for i in range(2 + max(1, min(args.steps, 5))):
        dk.copy_(src_k)
        if dv is not None:
            dv.copy_(src_v)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        thrust_sort(execution, dk, dv, workload.desc)
        t1 = time.perf_counter()
        if i >= 2:
            times.append((t1 - t0) * 1e3)
    ms = statistics.mean(times)
    return {"ms": ms, "device_ms": device_ms, "overhead_ms": ms - device_ms,
            "api": thrust_api_name(workload, values_h is None),
            "timing": "host wall clock around the synchronous call, inputs resident"}


E2E_COPY_STREAMS = 4


def run_e2e(args, workload: Workload, keys_h, values_h, dev):
    """Public API end to end, as a streaming pipeline: every step copies its
    input from pinned host memory, sorts it through the public API and copies
    the result back to pinned host memory.  Three device input buffers let
    step i+1's upload overlap step i's sort and download (PCIe is full
    duplex) without waiting for step i-1's download.  Each copy is split into
    E2E_COPY_STREAMS chunks on as many streams, so several copy engines share
    it."""
    import torch
    from rccl_b200 import thrust

    execution = thrust.Program.load(dev).par()
    stream = execution.stream
    C = E2E_COPY_STREAMS
    in_s = [torch.cuda.Stream(dev) for _ in range(C)]
    out_s = [torch.cuda.Stream(dev) for _ in range(C)]
    hk = torch.from_numpy(keys_h).pin_memory()
    ok_ = torch.empty_like(hk).pin_memory()
    NB = 3
    dks = [torch.empty(hk.shape, dtype=hk.dtype, device=dev) for _ in range(NB)]
    hv = ov = None
    dvs = [None] * NB
    if values_h is not None:
        hv = torch.from_numpy(values_h).pin_memory()
        ov = torch.empty_like(hv).pin_memory()
        dvs = [torch.empty(hv.shape, dtype=hv.dtype, device=dev) for _ in range(NB)]
    h2d = hk.numel() * hk.element_size() + (hv.numel() * hv.element_size() if hv is not None else 0)
    n = hk.numel()
    bounds = [n * c // C for c in range(C + 1)]
    uploaded = [[torch.cuda.Event() for _ in range(C)] for _ in range(NB)]
    sorted_ = [torch.cuda.Event() for _ in range(NB)]
    downloaded = [[torch.cuda.Event() for _ in range(C)] for _ in range(NB)]

    def upload(i):
        b = i % NB
        for c in range(C):
            lo, hi = bounds[c], bounds[c + 1]
            for e in downloaded[b]:
                in_s[c].wait_event(e)  # the buffer's previous result is out
            with torch.cuda.stream(in_s[c]):
                dks[b][lo:hi].copy_(hk[lo:hi], non_blocking=True)
                if hv is not None:
                    dvs[b][lo:hi].copy_(hv[lo:hi], non_blocking=True)
            uploaded[b][c].record(in_s[c])

    def sort(i):
        b = i % NB
        dk, dv = dks[b], dvs[b]
        for e in uploaded[b]:
            stream.wait_event(e)
        thrust_sort(execution, dk, dv, workload.desc)
        sorted_[b].record(stream)

    def download(i):
        b = i % NB
        for c in range(C):
            lo, hi = bounds[c], bounds[c + 1]
            out_s[c].wait_event(sorted_[b])
            with torch.cuda.stream(out_s[c]):
                ok_[lo:hi].copy_(dks[b][lo:hi], non_blocking=True)
                if ov is not None:
                    ov[lo:hi].copy_(dvs[b][lo:hi], non_blocking=True)
            downloaded[b][c].record(out_s[c])

    def pipeline(steps, t0=None, t1=None):
        if t0 is not None:
            t0.record(in_s[0])
            for c in range(1, C):
                in_s[c].wait_event(t0)
        upload(0)
        for i in range(steps):
            if i + 1 < steps:
                upload(i + 1)
            sort(i)
            download(i)
        if t1 is not None:
            for c in range(1, C):
                out_s[0].wait_event(downloaded[(steps - 1) % NB][c])
            t1.record(out_s[0])
        torch.cuda.synchronize()

    # The timed pipeline starts with one upload and ends with one download
    # that nothing overlaps (about 60 ms each at 2^28 pairs over PCIe); the
    # bench's own step count (20 by default) spreads them the way a stream of
    # sorts does.  Every step still copies its input in and its result out.
    steps = max(3, min(args.steps, 20))
    pipeline(3)  # warm-up
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    pipeline(steps, t0, t1)
    ms = t0.elapsed_time(t1) / steps
    # every step's output went through the same host buffer: check the last
    img = order_image(ok_.numpy(), workload.desc)
    ok = bool(np.all(img[1:] >= img[:-1]))
    if ov is not None:
        ok = ok and bool(np.array_equal(keys_h[ov.numpy().astype(np.int64)], ok_.numpy()))
    return {"value": workload.n / (ms / 1e3), "unit": UNIT, "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": h2d, "steps": steps,
            "output_checked": ok,
            "pipelined": (f"step i+1's upload overlaps step i's sort and download; each copy "
                          f"split over {C} streams"),
            "api": thrust_api_name(workload, values_h is None)}


def run_cub_proxy(args, workload: Workload):
    """Comparator only: CUB DeviceRadixSort from the toolkit's CCCL headers
    (baseline/cub_proxy.cu, built here for sm_100a), which the reference's
    radix path ports, timed on the same inputs the same way as run_single."""
    import torch

    kind = {2: 0, 5: 0, 3: 1}.get(workload.config, 2)
    if (kind == 0 and (workload.key, workload.value) != (np.uint64, np.uint32)) or \
            (kind == 1 and workload.key != np.float32) or (kind == 2 and workload.key != np.uint32):
        print(json.dumps({"impl": "cub-proxy", "unavailable": "no CUB proxy for this workload"}))
        return
    src = os.path.join(ROOT, "baseline", "cub_proxy.cu")
    out_dir = os.path.join(ROOT, "baseline", "_cub")
    so = os.path.join(out_dir, "libcub_proxy.so")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        os.makedirs(out_dir, exist_ok=True)
        subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                        "-Xcompiler", "-fPIC", "-shared", src, "-o", so], check=True)
    L = ctypes.CDLL(so)
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    L.cub_proxy_temp_bytes.argtypes = [ctypes.c_int, sz, ctypes.POINTER(sz)]
    L.cub_proxy_sort.argtypes = [ctypes.c_int, vp, vp, vp, vp, sz, vp, sz,
                                 ctypes.POINTER(ctypes.c_int), vp]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    src_k, src_v = workload.generate(0, workload.n, dev)
    k0, k1 = torch.empty_like(src_k), torch.empty_like(src_k)
    v0 = v1 = None
    if src_v is not None:
        v0, v1 = torch.empty_like(src_v), torch.empty_like(src_v)
    nbytes = sz(0)
    assert L.cub_proxy_temp_bytes(kind, workload.n, ctypes.byref(nbytes)) == 0
    temp = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sel = ctypes.c_int(0)

    def restore():
        k0.copy_(src_k)
        if v0 is not None:
            v0.copy_(src_v)

    def sort():
        assert L.cub_proxy_sort(kind, k0.data_ptr(), k1.data_ptr(),
                                None if v0 is None else v0.data_ptr(),
                                None if v1 is None else v1.data_ptr(), workload.n,
                                temp.data_ptr(), nbytes.value, ctypes.byref(sel),
                                stream.cuda_stream) == 0

    for _ in range(args.warmup):
        restore()
        sort()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        restore()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        sort()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    out = k1 if sel.value else k0
    ms = statistics.mean(times)
    print(json.dumps({
        "impl": "cub-proxy", "metric": METRIC, "value": workload.n / (ms / 1e3), "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": np.dtype(workload.key).name,
        "config": config_dict(args, workload),
        "cub_version": "CCCL 2.8.2 headers from the CUDA 12.9 toolkit, nvcc -arch=sm_100a",
        "output_checked": check_keys_only(src_k, out, np.dtype(workload.key).kind, workload.desc)
        if src_v is None else None}), flush=True)


# ---------------------------------------------------------------------------
# N GPUs: distributed sample sort, one process per GPU
# ---------------------------------------------------------------------------
EXCHANGE_NAMES = {
    "peer": "first merge round reads the buckets from the peers' shards over NVLink (CUDA IPC)",
    "peer-copy": "copy kernel pulls the buckets over NVLink (CUDA IPC), then local merge",
    "nccl": "NCCL grouped send/recv, then local merge",
    "c-nccl": "whole sort in one C call per rank (rsort_dist_pairs_rank): NCCL all-gathers, "
              "grouped ncclSend/ncclRecv, local merge",
}


def host_memory_available() -> int:
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def run_dist(args, workload: Workload):
    import datetime

    import torch
    import torch.distributed as dist
    from rccl_b200 import _lib, cub
    from rccl_b200 import dist as D

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    strong = workload.config == 5
    m = workload.n // world if strong else workload.n
    n_total = m * world
    start = rank * m
    kd, vd = workload.torch_dtypes()
    keys = torch.empty(m, dtype=kd, device=dev)
    values = torch.empty(m, dtype=vd, device=dev) if vd is not None else None
    launch = cub.Program.load(dev).on()
    ops = D.CudaLocalOps(launch)
    L = _lib.lib()
    mode = os.environ.get("RSORT_EXCHANGE", "peer")
    comm = None
    if mode == "c-nccl":
        from rccl_b200 import nccl
        comm = nccl.comm_init_group()

    def global_sort(k, v, timings=None):
        if comm is not None:
            return D.sample_sort_c(k, v, workload.desc, comm, rank, world,
                                   stream=launch.stream.cuda_stream)
        return D.sample_sort(k, v, workload.desc, ops=ops, timings=timings)

    def restore():
        # Regenerate the shard (untimed): every item is a function of its
        # global index.
        workload.fill(keys, values, start)

    for _ in range(args.warmup):
        restore()
        out = global_sort(keys, values)
        del out
    in_hash = None
    if values is None:
        # keys-only: the multiset of all ranks' input keys, for the output check
        restore()
        in_hash = multiset_hash(keys)
        dist.all_reduce(in_hash)
    torch.cuda.synchronize()
    dist.barrier()

    step_ms, phases = [], {}
    L.rsort_launch_count_reset()
    L.rsort_profile_read(None, None, 0)
    out = None
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            out = None
            restore()
            torch.cuda.synchronize()
            dist.barrier()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            L.rsort_profile_enable(1)
            t0.record()
            out = global_sort(keys, values, timings=phases)
            t1.record()
            L.rsort_profile_enable(0)
            torch.cuda.synchronize()
            step_ms.append(t0.elapsed_time(t1))
    launches = int(L.rsort_launch_count())
    per_kernel = read_profile(L, 8192)

    # max over ranks of the per-step device time
    t = torch.tensor(step_ms, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_max = t.tolist()
    ph_names = ["local_sort", "partition", "exchange", "merge"]
    ph = torch.tensor([phases.get(k, 0.0) / args.steps for k in ph_names], dtype=torch.float64,
                      device=dev)
    dist.all_reduce(ph, op=dist.ReduceOp.MAX)

    # Output checks: this rank's part is bit-exact (keys regenerated from the
    # value indices, order, stability), every global index appears exactly
    # once over all ranks, and the parts are ordered across rank boundaries.
    ok_k, ok_v = out
    if ok_v is not None:
        mark = torch.zeros(n_total, dtype=torch.uint8, device=dev)
        ok = check_pairs_index(workload, ok_k, ok_v, mark)
        dist.all_reduce(mark, op=dist.ReduceOp.SUM)
        ok &= bool(torch.all(mark == 1))
        del mark
    else:
        img = image_i64(ok_k, np.dtype(workload.key).kind, workload.desc)
        ok = bool(torch.all(img[1:] >= img[:-1])) if img.numel() else True
        del img
        # the parts of all ranks together are a permutation of all inputs
        out_hash = multiset_hash(ok_k)
        dist.all_reduce(out_hash)
        ok &= bool(out_hash == in_hash)
    kind = np.dtype(workload.key).kind
    if ok_k.numel():
        img_ends = image_i64(torch.cat([ok_k[:1], ok_k[-1:]]), kind, workload.desc)
        edge = torch.tensor([float(img_ends[0].item()), float(img_ends[1].item()),
                             float(ok_k.numel())], dtype=torch.float64, device=dev)
        exact_edge = torch.stack([img_ends[0], img_ends[1]])
    else:
        edge = torch.tensor([0.0, 0.0, 0.0], dtype=torch.float64, device=dev)
        exact_edge = torch.zeros(2, dtype=torch.int64, device=dev)
    edges = [torch.empty_like(edge) for _ in range(world)]
    dist.all_gather(edges, edge)
    exact = [torch.empty_like(exact_edge) for _ in range(world)]
    dist.all_gather(exact, exact_edge)
    oks = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(oks, op=dist.ReduceOp.MIN)
    counts = [int(e[2].item()) for e in edges]
    total_out = sum(counts)
    nonempty = [exact[q] for q in range(world) if counts[q] > 0]
    bound_ok = all(int(a[1]) <= int(b[0]) for a, b in zip(nonempty, nonempty[1:]))
    sent = torch.tensor([float(m * (workload.kb + workload.vb) * (world - 1) / world)],
                        device=dev)
    del out, ok_k, ok_v

    # End to end through the public API: copy the pinned host shard to the
    # device, sample-sort it and copy this rank's sorted part back to pinned
    # host memory, every step.  Pinned buffers hold the whole shard in and
    # out, so this leg runs only where the host has room for them.
    e2e, h2d, d2h = None, 0, 0
    item = workload.kb + workload.vb
    need = torch.tensor([float(3 * m * item * world)], dtype=torch.float64)
    e2e_skip = None
    if args.no_e2e:
        e2e_skip = "skipped (--no-e2e)"
    elif host_memory_available() < need.item() * 1.2:
        e2e_skip = (f"skipped: the pinned host buffers of all ranks need {need.item() / 2**30:.0f}"
                    f" GiB, more than the host's available memory")
    skip = torch.tensor([1 if e2e_skip else 0], device=dev)
    dist.all_reduce(skip, op=dist.ReduceOp.MAX)
    if skip.item() == 0:
        hk = torch.empty(m, dtype=kd).pin_memory()
        hv = torch.empty(m, dtype=vd).pin_memory() if vd is not None else None
        workload.fill(hk, hv, start)
        h2d = m * item
        pinned = {}

        def host_out(t):
            buf = pinned.get(t.dtype)
            if buf is None or buf.numel() < t.numel():
                buf = torch.empty(max(t.numel(), 2 * m), dtype=t.dtype, pin_memory=True)
                pinned[t.dtype] = buf
            return buf[:t.shape[0]]

        host_out(torch.empty(0, dtype=kd))
        if vd is not None:
            host_out(torch.empty(0, dtype=vd))
        dk = torch.empty_like(keys)
        dv = torch.empty_like(values) if values is not None else None
        out_bytes = 0

        copy_streams = [torch.cuda.Stream(dev) for _ in range(E2E_COPY_STREAMS)]

        def chunked_copy(dst, src):
            """dst.copy_(src) split over the copy streams (several copy
            engines), ordered after and before the current stream's work."""
            main = torch.cuda.current_stream(dev)
            n_ = src.shape[0]
            C = len(copy_streams)
            for c, cs in enumerate(copy_streams):
                lo, hi = n_ * c // C, n_ * (c + 1) // C
                cs.wait_stream(main)
                with torch.cuda.stream(cs):
                    dst[lo:hi].copy_(src[lo:hi], non_blocking=True)
            for cs in copy_streams:
                main.wait_stream(cs)

        def e2e_step():
            nonlocal out_bytes
            chunked_copy(dk, hk)
            if dv is not None:
                chunked_copy(dv, hv)
            rk, rv = global_sort(dk, dv)
            chunked_copy(host_out(rk), rk)
            nb = rk.numel() * rk.element_size()
            if rv is not None:
                chunked_copy(host_out(rv), rv)
                nb += rv.numel() * rv.element_size()
            out_bytes = max(out_bytes, nb)

        e2e_step()
        torch.cuda.synchronize()
        dist.barrier()
        e_steps = 3
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(e_steps):
            e2e_step()
        a1.record()
        torch.cuda.synchronize()
        d2h = out_bytes
        tt = torch.tensor([a0.elapsed_time(a1) / e_steps], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e = {"value": n_total / (tt.item() / 1e3), "unit": UNIT, "ms_per_step": tt.item(),
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "rccl_b200.dist.sample_sort from pinned host shards (max over ranks; "
                      f"bytes per rank; copies split over {E2E_COPY_STREAMS} streams)"}
        del hk, hv, dk, dv, pinned
    dist.barrier()
    if rank == 0:
        total_ms = sum(step_max)
        value = n_total * args.steps / (total_ms / 1e3)
        roofline = roofline_of(Workload(workload.config, m), per_kernel, None)
        phase_ms = dict(zip(ph_names, ph.tolist()))
        # In the default mode the buckets cross NVLink inside the first merge
        # round, so the bytes are timed over exchange + merge.
        xfer_ms = phase_ms["exchange"] + (phase_ms["merge"] if mode == "peer" else 0.0)
        nvlink_gbs = sent.item() / (xfer_ms / 1e3) / 1e9 if xfer_ms > 0 else None
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None, "dtype": np.dtype(workload.key).name,
            "data": "synthetic (counter-based, seeded; each rank generates its shard on its GPU)",
            "config": dist_config(args, workload, world, mode),
            "roofline": roofline, "gpu_launches": launches,
            "phases_ms_max_over_ranks": phase_ms,
            "nvlink": {"bytes_per_rank": sent.item(), "achieved_gbs_per_rank": nvlink_gbs,
                       "peak_gbs": NVLINK_GBS, "frac": (nvlink_gbs / NVLINK_GBS
                                                        if nvlink_gbs else None),
                       "note": "uniform-key estimate of bytes leaving a rank"},
            "clocks": clocks.summary(),
            "output_checked": bool(oks.item() == 1 and bound_ok and total_out == n_total),
            "check": ("bit-exact per rank (keys regenerated from value indices, order, "
                      "stability), every global index exactly once over all ranks, rank "
                      "boundaries ordered" if vd is not None else
                      "keys-only: each rank's part in order, rank boundaries ordered, and the "
                      "multiset hash of all output parts equal to that of all inputs"),
            "out_per_rank": counts,
            "e2e": e2e if e2e is not None else {"unavailable": e2e_skip},
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    if comm is not None:
        torch.cuda.synchronize()
        from rccl_b200 import nccl
        nccl.comm_destroy(comm)
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=None,
                    help="workload (default: 2 on one GPU, 5 on several)")
    ap.add_argument("--n", type=int, default=None, help="override the workload size")
    ap.add_argument("--impl", default="rccl_b200", choices=["rccl_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end leg (used for profiler runs)")
    ap.add_argument("--no-configs", action="store_true",
                    help="headline workload only (no configs block)")
    ap.add_argument("--cub-proxy", action="store_true",
                    help="time CUB DeviceRadixSort (toolkit headers) on the same workload instead")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    multi = world > 1 or args.gpus > 1
    config = args.config or (5 if multi else 2)
    workload = Workload(config, args.n)
    if args.impl == "reference":
        run_reference(args, workload, rank, max(world, args.gpus))
        return
    if args.cub_proxy:
        run_cub_proxy(args, workload)
        return
    if multi:
        run_dist(args, workload)
        return
    run_single(args, workload)


if __name__ == "__main__":
    main()
