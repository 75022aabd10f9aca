"""Benchmark of the B200 DeviceRadixSort hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl rccl_b200|reference]

One step is one sort of the workload's whole input.  `value` is device-timed
sorted keys/s with the input resident in HBM (CUDA events around each sort on
the sort's stream; the untimed restore copy of the input happens between
steps).  `e2e` is the same metric through the public rccl-thrust style API
(thrust.with_values(...).sort()) with the input copied from pinned host memory
and the sorted keys and values copied back inside the timed region.

Workloads are seeded synthetic inputs with the reference benchmark shapes
(numpy PCG64):
  1: 2^20 u32 keys, uniform, ascending keys-only                (seed 1)
  2: 2^28 u64 keys uniform over 64 bits + u32 values = index,
     stable ascending pairs (default; the north-star pair config)  (seed 2)
  3: 2^28 f32 keys ~ N(0, 1e3) with +-0 / +-inf / NaN, descending (seed 3)
  4: 2^30 u32 keys, 90% Zipf(1.1) over 2^20 values + 10% constant (seeds 4, 5)
"""
from __future__ import annotations

import argparse
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


# ---------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------
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

    def generate(self, n: int | None = None, offset: int = 0):
        """Host arrays (keys, values) of this workload (`n` items from `offset`)."""
        n = self.n if n is None else n
        c = self.config
        if c == 1:
            keys = np.random.default_rng(1).integers(0, 2**32, self.n, dtype=np.uint64)
            keys = keys[offset:offset + n].astype(np.uint32)
        elif c == 2:
            bg = np.random.PCG64(2)
            bg.advance(offset)  # one 64-bit draw per full-range u64 key
            keys = np.random.Generator(bg).integers(0, 2**64, n, dtype=np.uint64)
        elif c == 3:
            keys = gen_f32_specials(np.random.default_rng(3 + offset), n)
        else:
            keys = gen_zipf(n, seed_offset=offset)
        values = None
        if self.value is not None:
            values = np.arange(offset, offset + n, dtype=np.uint64).astype(self.value)
        return keys, values


def gen_f32_specials(rng, n):
    x = rng.normal(0.0, 1e3, n).astype(np.float32)
    n_zero, n_inf, n_nan = n // 1000, n // 10000, n // 10000
    pos = rng.choice(n, n_zero + n_inf + n_nan, replace=False)
    z, i, q = pos[:n_zero], pos[n_zero:n_zero + n_inf], pos[n_zero + n_inf:]
    bits = x.view(np.uint32)
    sign = rng.integers(0, 2, pos.size).astype(np.uint32) << 31
    bits[z] = sign[:n_zero]
    bits[i] = 0x7F800000 | sign[n_zero:n_zero + n_inf]
    payload = rng.integers(1, 1 << 22, n_nan).astype(np.uint32)
    bits[q] = 0x7FC00000 | payload | sign[n_zero + n_inf:]
    return x


def gen_zipf(n, seed_offset=0):
    rng = np.random.default_rng(4 + seed_offset)
    ranks = np.arange(1, (1 << 20) + 1, dtype=np.float64)
    cdf = np.cumsum(ranks ** -1.1)
    cdf /= cdf[-1]
    mapping = np.random.default_rng(5).choice(2**32, 1 << 20, replace=False).astype(np.uint32)
    n_zipf = n * 9 // 10
    u = rng.random(n_zipf)
    keys = np.empty(n, np.uint32)
    keys[:n_zipf] = mapping[np.searchsorted(cdf, u)]
    keys[n_zipf:] = np.uint32(rng.integers(0, 2**32))
    rng.shuffle(keys)
    return keys


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
    from the captured size to this workload's size (traffic grows with n)."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        f = dict(kv.split("=", 1) for kv in line.split() if "=" in kv)
        if f.get("config") == str(workload.config) and f.get("kernel") == "onesweep":
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
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            # nvidia-smi takes a moment to start: wait for its first sample so
            # the timed region (often ~0.1 s) is covered from its start; only
            # samples taken after that point are kept.
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


def cpu_baseline(workload: Workload, budget_s: float = 12.0):
    """The oracle port (stable LSD radix restatement) on all host cores over a
    bounded sample of the workload."""
    from oracle import pyoracle
    threads = os.cpu_count() or 1
    sample = min(workload.n, 1 << 24)
    keys, values = workload.generate(sample)
    rates = []
    t_end = time.perf_counter() + budget_s
    while len(rates) < 5 and (len(rates) < 1 or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        pyoracle.radix_sort(keys, values, workload.desc, threads=threads)
        rates.append(sample / (time.perf_counter() - t0))
    return {"value": statistics.median(rates), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"first {sample} items of the workload, {len(rates)} timed sorts, "
                      f"median; oracle stable LSD radix on {threads} host threads"}


# ---------------------------------------------------------------------------
# Reference arm: the reference's CPU restatement (oracle port), rank 0 only
# ---------------------------------------------------------------------------
def run_reference(args, workload: Workload, rank: int):
    if rank != 0:
        return
    from oracle import pyoracle
    threads = os.cpu_count() or 1
    sample = min(workload.n, 1 << 24)
    keys, values = workload.generate(sample)
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
        "scaling": "weak", "vs_baseline": None, "dtype": np.dtype(workload.key).name,
        "data": "synthetic", "config": config_dict(args, workload, sample_n=sample),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"first {sample} items of the workload per step"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(args, workload: Workload, sample_n=None):
    d = {"workload": f"config {workload.config}: {workload.name}", "n": workload.n,
         "key": np.dtype(workload.key).name,
         "value": np.dtype(workload.value).name if workload.value is not None else None,
         "order": "descending" if workload.desc else "ascending", "stable": True,
         "per_gpu_n": workload.n, "parallelism": f"sample-sort x{args.gpus}" if args.gpus > 1
         else "single GPU",
         "l2": "input larger than the 126 MB L2; untimed restore copy between steps"}
    if sample_n is not None:
        d["sample_n"] = sample_n
    return d


# ---------------------------------------------------------------------------
# Single GPU
# ---------------------------------------------------------------------------
def run_single(args, workload: Workload):
    import torch
    from rccl_b200 import _lib, cub, thrust

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    launch = cub.Program.load(dev).on()
    stream = launch.stream
    keys_h, values_h = workload.generate()
    kd = torch.from_numpy(keys_h[:0]).dtype
    src_k = torch.from_numpy(keys_h).to(dev)
    keys = torch.empty_like(src_k)
    if values_h is not None:
        src_v = torch.from_numpy(values_h).to(dev)
        values = torch.empty_like(src_v)
        ws = cub.device_radix_sort_pairs_workspace(launch, kd, src_v.dtype, workload.n)
    else:
        src_v = values = None
        ws = cub.device_radix_sort_workspace(launch, kd, workload.n)
    controls = ws.controls

    def restore():
        keys.copy_(src_k)
        if values is not None:
            values.copy_(src_v)

    def sort():
        if values is None:
            (cub.device_radix_sort_keys_descending if workload.desc
             else cub.device_radix_sort_keys)(launch, keys, ws)
        else:
            (cub.device_radix_sort_pairs_descending if workload.desc
             else cub.device_radix_sort_pairs)(launch, keys, values, ws)

    for _ in range(args.warmup):
        restore()
        sort()
    cub.check_device_status(launch, controls)
    torch.cuda.synchronize()

    L = _lib.lib()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    L.rsort_launch_count_reset()
    L.rsort_profile_read(None, None, 0)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        torch.cuda.synchronize()
        for i in range(args.steps):
            restore()
            L.rsort_profile_enable(1)
            starts[i].record(stream)
            sort()
            stops[i].record(stream)
            L.rsort_profile_enable(0)
        torch.cuda.synchronize()
    launches = int(L.rsort_launch_count())
    cub.check_device_status(launch, controls)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, stops)]
    total_ms = sum(step_ms)

    import ctypes
    cap = 64 * args.steps
    kid = (ctypes.c_int32 * cap)()
    kms = (ctypes.c_float * cap)()
    nrec = L.rsort_profile_read(kid, kms, cap)
    per_kernel = {}
    for i in range(min(nrec, cap)):
        per_kernel.setdefault(_lib.KERNEL_NAMES.get(kid[i], str(kid[i])), []).append(kms[i])

    # Size-independent properties of the timed output: non-decreasing order
    # image, and for pairs the values (= input index) form the permutation
    # that maps the input onto the output, ascending within equal keys.
    out_k = keys.cpu().numpy()
    img = order_image(out_k, workload.desc)
    ok = bool(np.all(img[1:] >= img[:-1]))
    if values is not None:
        out_v = values.cpu().numpy().astype(np.int64)
        ok = ok and bool(np.array_equal(keys_h[out_v], out_k))
        ties = img[1:] == img[:-1]
        ok = ok and bool(np.all(out_v[1:][ties] > out_v[:-1][ties]))

    peak, peak_kind = measured_peak()
    osw = per_kernel.get("onesweep", [])
    roofline = None
    if osw:
        avg_s = statistics.mean(osw) / 1e3
        achieved = workload.bytes_per_pass / avg_s / 1e9
        traffic = profiled_traffic(workload)
        roofline = {"bound": "hbm", "kernel": "onesweep", "achieved": achieved, "peak": peak,
                    "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                    "traffic": traffic, "algorithmic_bytes_per_launch": workload.bytes_per_pass,
                    "avg_launch_ms": avg_s * 1e3,
                    "sort_achieved": workload.bytes_per_sort / (total_ms / args.steps / 1e3) / 1e9,
                    "sort_frac": workload.bytes_per_sort / (total_ms / args.steps / 1e3) / 1e9
                    / peak}
    kernel_ms = {k: {"launches": len(v), "total_ms": sum(v), "avg_ms": statistics.mean(v)}
                 for k, v in per_kernel.items()}

    del src_k, keys, src_v, values, ws
    torch.cuda.empty_cache()
    thrust_call = None if args.no_e2e else thrust_call_cost(args, workload, keys_h, values_h, dev,
                                                             total_ms / args.steps)
    e2e = None if args.no_e2e else run_e2e(args, workload, keys_h, values_h, dev)
    torch.cuda.empty_cache()

    value = workload.n * args.steps / (total_ms / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": np.dtype(workload.key).name,
        "data": "synthetic (numpy PCG64, seeded)", "config": config_dict(args, workload),
        "roofline": roofline, "e2e": e2e, "thrust_call": thrust_call, "gpu_launches": launches,
        "kernels": kernel_ms, "clocks": clocks.summary(), "output_checked": ok,
    }
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


def run_e2e(args, workload: Workload, keys_h, values_h, dev):
    """Public API end to end, as a streaming pipeline: every step copies its
    input from pinned host memory, sorts it through the public API and copies
    the result back to pinned host memory.  Three device input buffers let
    step i+1's upload overlap step i's sort and download (PCIe is full
    duplex) without waiting for step i-1's download."""
    import torch
    from rccl_b200 import thrust

    execution = thrust.Program.load(dev).par()
    stream = execution.stream
    in_s = torch.cuda.Stream(dev)
    out_s = torch.cuda.Stream(dev)
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
    uploaded = [torch.cuda.Event() for _ in range(NB)]
    sorted_ = [torch.cuda.Event() for _ in range(NB)]
    downloaded = [torch.cuda.Event() for _ in range(NB)]

    def upload(i):
        b = i % NB
        in_s.wait_event(downloaded[b])  # the buffer's previous result is out
        with torch.cuda.stream(in_s):
            dks[b].copy_(hk, non_blocking=True)
            if hv is not None:
                dvs[b].copy_(hv, non_blocking=True)
        uploaded[b].record(in_s)

    def sort(i):
        b = i % NB
        dk, dv = dks[b], dvs[b]
        stream.wait_event(uploaded[b])
        thrust_sort(execution, dk, dv, workload.desc)
        sorted_[b].record(stream)

    def download(i):
        b = i % NB
        out_s.wait_event(sorted_[b])
        with torch.cuda.stream(out_s):
            ok_.copy_(dks[b], non_blocking=True)
            if ov is not None:
                ov.copy_(dvs[b], non_blocking=True)
        downloaded[b].record(out_s)

    def pipeline(steps, t0=None, t1=None):
        if t0 is not None:
            t0.record(in_s)
        upload(0)
        for i in range(steps):
            if i + 1 < steps:
                upload(i + 1)
            sort(i)
            download(i)
        if t1 is not None:
            t1.record(out_s)
        torch.cuda.synchronize()

    steps = max(3, min(args.steps, 6))
    pipeline(3)  # warm-up
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    pipeline(steps, t0, t1)
    ms = t0.elapsed_time(t1) / steps
    # every step's output went through the same host buffer: check the last
    img = order_image(ok_.numpy(), workload.desc)
    ok = bool(np.all(img[1:] >= img[:-1]))
    return {"value": workload.n / (ms / 1e3), "unit": UNIT, "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": h2d, "steps": steps,
            "output_checked": ok,
            "pipelined": "step i+1's upload overlaps step i's sort and download",
            "api": thrust_api_name(workload, values_h is None)}


def run_cub_proxy(args, workload: Workload):
    """Comparator only: CUB DeviceRadixSort from the toolkit's CCCL headers
    (baseline/cub_proxy.cu, built here for sm_100a), which the reference's
    radix path ports, timed on the same inputs the same way as run_single."""
    import ctypes
    import torch

    kind = {2: 0, 3: 1}.get(workload.config, 2)
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
    keys_h, values_h = workload.generate()
    src_k = torch.from_numpy(keys_h).to(dev)
    k0, k1 = torch.empty_like(src_k), torch.empty_like(src_k)
    src_v = v0 = v1 = None
    if values_h is not None:
        src_v = torch.from_numpy(values_h).to(dev)
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
    out = (k1 if sel.value else k0).cpu().numpy()
    img = order_image(out, workload.desc)
    ms = statistics.mean(times)
    print(json.dumps({
        "impl": "cub-proxy", "metric": METRIC, "value": workload.n / (ms / 1e3), "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "dtype": np.dtype(workload.key).name,
        "config": config_dict(args, workload),
        "cub_version": "CCCL 2.8.2 headers from the CUDA 12.9 toolkit, nvcc -arch=sm_100a",
        "output_sorted": bool(np.all(img[1:] >= img[:-1]))}), flush=True)


# ---------------------------------------------------------------------------
# N GPUs: distributed sample sort, one process per GPU (weak scaling: every
# rank holds one workload-sized contiguous shard of the global input)
# ---------------------------------------------------------------------------
EXCHANGE_NAMES = {
    "peer": "first merge round reads the buckets from the peers' shards over NVLink (CUDA IPC)",
    "peer-copy": "copy kernel pulls the buckets over NVLink (CUDA IPC), then local merge",
    "nccl": "NCCL grouped send/recv, then local merge",
}


def run_dist(args, workload: Workload):
    import ctypes
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
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                            device_id=dev)
    m = workload.n
    keys_h, _ = workload.generate(m, offset=rank * m)
    src_k = torch.from_numpy(keys_h).to(dev)
    src_v = None
    if workload.value is not None:
        # values = global input index (fits u32 for W * 2^28 < 2^32)
        src_v = (torch.arange(m, dtype=torch.int64, device=dev) + rank * m).to(torch.int32).view(
            torch.uint32 if workload.vb == 4 else torch.int32)
    keys = torch.empty_like(src_k)
    values = torch.empty_like(src_v) if src_v is not None else None
    launch = cub.Program.load(dev).on()
    ops = D.CudaLocalOps(launch)
    L = _lib.lib()

    def restore():
        keys.copy_(src_k)
        if values is not None:
            values.copy_(src_v)

    for _ in range(args.warmup):
        restore()
        out = D.sample_sort(keys, values, workload.desc, ops=ops)
        del out
    torch.cuda.synchronize()
    dist.barrier()

    step_ms, phases = [], {}
    L.rsort_launch_count_reset()
    L.rsort_profile_read(None, None, 0)
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            restore()
            torch.cuda.synchronize()
            dist.barrier()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            L.rsort_profile_enable(1)
            t0.record()
            out = D.sample_sort(keys, values, workload.desc, ops=ops, timings=phases)
            t1.record()
            L.rsort_profile_enable(0)
            torch.cuda.synchronize()
            step_ms.append(t0.elapsed_time(t1))
            if i + 1 < args.steps:
                del out
    launches = int(L.rsort_launch_count())
    cap = 4096
    kid = (ctypes.c_int32 * cap)()
    kms = (ctypes.c_float * cap)()
    nrec = L.rsort_profile_read(kid, kms, cap)
    per_kernel = {}
    for i in range(min(nrec, cap)):
        per_kernel.setdefault(_lib.KERNEL_NAMES.get(kid[i], str(kid[i])), []).append(kms[i])

    # max over ranks of the per-step device time
    t = torch.tensor(step_ms, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_max = t.tolist()
    ph_names = ["local_sort", "partition", "exchange", "merge"]
    ph = torch.tensor([phases.get(k, 0.0) / args.steps for k in ph_names], dtype=torch.float64,
                      device=dev)
    dist.all_reduce(ph, op=dist.ReduceOp.MAX)

    # output checks: local order, rank boundaries, total count, stability
    ok_k, ok_v = out
    img = order_image(ok_k.cpu().numpy(), workload.desc)
    ok = bool(np.all(img[1:] >= img[:-1])) if img.size else True
    if ok_v is not None and img.size:
        v = ok_v.cpu().numpy().astype(np.int64)
        ties = img[1:] == img[:-1]
        ok = ok and bool(np.all(v[1:][ties] > v[:-1][ties]))
    edge = torch.tensor([int(img[0]) if img.size else -1, int(img[-1]) if img.size else -1,
                         img.size], dtype=torch.float64, device=dev)
    edges = [torch.empty_like(edge) for _ in range(world)]
    dist.all_gather(edges, edge)
    oks = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(oks, op=dist.ReduceOp.MIN)
    total_out = int(sum(e[2].item() for e in edges))
    nonempty = [e for e in edges if e[2].item() > 0]
    bound_ok = all(a[1].item() <= b[0].item() for a, b in zip(nonempty, nonempty[1:]))
    sent = torch.tensor([float(m * (workload.kb + workload.vb) * (world - 1) / world)],
                        device=dev)
    del out, ok_k, ok_v

    # End to end through the public API, as a streaming pipeline: every step
    # copies the pinned host shard to the device, sample-sorts it and copies
    # this rank's sorted part back to pinned host memory; three device input
    # buffers let step i+1's upload overlap step i's sort and download.
    e2e_ms, h2d, d2h = None, 0, 0
    if not args.no_e2e:
        hk = torch.from_numpy(keys_h).pin_memory()
        hv = src_v.cpu().pin_memory() if src_v is not None else None
        h2d = hk.numel() * hk.element_size() + (hv.numel() * hv.element_size() if hv is not None else 0)
        NB = 3
        in_s, out_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        dks = [torch.empty_like(hk, device=dev) for _ in range(NB)]
        dvs = [torch.empty_like(hv, device=dev) if hv is not None else None for _ in range(NB)]
        uploaded = [torch.cuda.Event() for _ in range(NB)]
        sorted_ = [torch.cuda.Event() for _ in range(NB)]
        downloaded = [torch.cuda.Event() for _ in range(NB)]
        pinned = {}
        out_bytes = [0]

        def host_out(t):
            # pinned result buffers, allocated once and grown only if a
            # partition comes out larger than any before
            buf = pinned.get(t.dtype)
            if buf is None or buf.numel() < t.numel():
                buf = torch.empty((max(t.numel(), 2 * m),) + tuple(t.shape[1:]), dtype=t.dtype,
                                  pin_memory=True)
                pinned[t.dtype] = buf
            return buf[:t.shape[0]]

        def upload(i):
            b = i % NB
            in_s.wait_event(downloaded[b])
            with torch.cuda.stream(in_s):
                dks[b].copy_(hk, non_blocking=True)
                if hv is not None:
                    dvs[b].copy_(hv, non_blocking=True)
            uploaded[b].record(in_s)

        def sort_and_download(i):
            b = i % NB
            torch.cuda.current_stream().wait_event(uploaded[b])
            rk, rv = D.sample_sort(dks[b], dvs[b], workload.desc, ops=ops)
            # the step's trailing all-reduce is on this stream: once this event
            # completes no peer reads the input buffer any more
            sorted_[b].record()
            out_s.wait_event(sorted_[b])
            nb = rk.numel() * rk.element_size()
            with torch.cuda.stream(out_s):
                host_out(rk).copy_(rk, non_blocking=True)
                rk.record_stream(out_s)
                if rv is not None:
                    host_out(rv).copy_(rv, non_blocking=True)
                    rv.record_stream(out_s)
                    nb += rv.numel() * rv.element_size()
            downloaded[b].record(out_s)
            out_bytes[0] = max(out_bytes[0], nb)

        def pipeline(steps, t0=None, t1=None):
            torch.cuda.synchronize()
            dist.barrier()
            if t0 is not None:
                t0.record(in_s)
            upload(0)
            for i in range(steps):
                if i + 1 < steps:
                    upload(i + 1)
                sort_and_download(i)
            if t1 is not None:
                t1.record(out_s)
            torch.cuda.synchronize()

        # warm the pinned buffers and the pipeline outside the timed steps
        host_out(torch.empty(m, dtype=src_k.dtype))
        if src_v is not None:
            host_out(torch.empty(m, dtype=src_v.dtype))
        e2e_steps = 3
        pipeline(2)
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        pipeline(e2e_steps, a0, a1)
        d2h = out_bytes[0]
        tt = torch.tensor([a0.elapsed_time(a1) / e2e_steps], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = tt.item()
        del dks, dvs
    dist.barrier()
    if rank == 0:
        total_ms = sum(step_max)
        value = world * m * args.steps / (total_ms / 1e3)
        peak, peak_kind = measured_peak()
        osw = per_kernel.get("onesweep", [])
        roofline = None
        if osw:
            avg_s = statistics.mean(osw) / 1e3
            achieved = workload.bytes_per_pass / avg_s / 1e9
            roofline = {"bound": "hbm", "kernel": "onesweep", "achieved": achieved,
                        "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "peak_source": peak_kind, "traffic": profiled_traffic(workload),
                        "algorithmic_bytes_per_launch": workload.bytes_per_pass,
                        "avg_launch_ms": avg_s * 1e3}
        phase_ms = dict(zip(ph_names, ph.tolist()))
        # In the default mode the buckets cross NVLink inside the first merge
        # round, so the bytes are timed over exchange + merge.
        xfer_ms = phase_ms["exchange"] + (phase_ms["merge"] if os.environ.get(
            "RSORT_EXCHANGE", "peer") == "peer" else 0.0)
        nvlink_gbs = sent.item() / (xfer_ms / 1e3) / 1e9 if xfer_ms > 0 else None
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": np.dtype(workload.key).name, "data": "synthetic (numpy PCG64, seeded)",
            "config": dict(config_dict(args, workload), n=world * m, per_gpu_n=m,
                           parallelism=f"sample sort over {world} GPUs",
                           exchange=EXCHANGE_NAMES[os.environ.get("RSORT_EXCHANGE", "peer")]),
            "roofline": roofline, "gpu_launches": launches,
            "phases_ms_max_over_ranks": phase_ms,
            "nvlink": {"bytes_per_rank": sent.item(), "achieved_gbs_per_rank": nvlink_gbs,
                       "peak_gbs": 770.0, "note": "uniform-key estimate of bytes leaving a rank"},
            "clocks": clocks.summary(),
            "output_checked": bool(oks.item() == 1 and bound_ok and total_out == world * m),
            "e2e": None if e2e_ms is None else {
                "value": world * m / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "pipelined": "step i+1's upload overlaps step i's sort and download",
                "api": "rccl_b200.dist.sample_sort from pinned host shards (max over ranks)"},
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--n", type=int, default=None, help="override the workload size")
    ap.add_argument("--impl", default="rccl_b200", choices=["rccl_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end leg (used for profiler runs)")
    ap.add_argument("--cub-proxy", action="store_true",
                    help="time CUB DeviceRadixSort (toolkit headers) on the same workload instead")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    workload = Workload(args.config, args.n)
    if args.impl == "reference":
        run_reference(args, workload, rank)
        return
    if args.cub_proxy:
        run_cub_proxy(args, workload)
        return
    if world > 1 or args.gpus > 1:
        run_dist(args, workload)
        return
    run_single(args, workload)


if __name__ == "__main__":
    main()
