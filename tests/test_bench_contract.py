"""bench.py's CPU-side contract: the reference arm (the oracle port timed on
host cores) prints one JSON line with the driver's keys, on every config, and
under torchrun only rank 0 prints; the byte models and the committed traffic
file parse.  The GPU arm's line is exercised by the GPU runs."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

REQUIRED = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
            "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
            "cpu_baseline", "e2e"}


def run(args, env=None):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, cwd=ROOT,
                         capture_output=True, text=True, timeout=600,
                         env=dict(os.environ, **(env or {})))
    assert out.returncode == 0, out.stderr[-2000:]
    return [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]


@pytest.mark.parametrize("config", [1, 2, 3])
def test_reference_arm_line(config):
    lines = run(["--impl", "reference", "--config", str(config), "--n", "65536", "--steps", "1",
                 "--warmup", "1"])
    assert len(lines) == 1
    line = lines[0]
    assert REQUIRED <= set(line)
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["config"]["workload"].startswith(f"config {config}")


def test_reference_arm_non_zero_rank_prints_nothing():
    lines = run(["--impl", "reference", "--n", "4096", "--steps", "1", "--warmup", "0"],
                env={"RANK": "1", "WORLD_SIZE": "2"})
    assert lines == []


def test_byte_models_and_traffic_file():
    w2 = bench.Workload(2)
    assert w2.bytes_per_pass == 2 * w2.n * 12
    assert w2.bytes_per_sort == w2.n * 8 + 8 * 2 * w2.n * 12  # 200 B per pair
    w3 = bench.Workload(3)
    assert w3.bytes_per_sort == w3.n * 36
    t2 = bench.profiled_traffic(w2)
    assert t2 is not None and 0.5 * w2.bytes_per_pass < t2 < 1.5 * w2.bytes_per_pass
    assert bench.profiled_traffic(w3) is not None


def test_reference_arm_under_torchrun_uses_the_strong_scaling_config():
    """With WORLD_SIZE > 1 the reference arm's line carries the same config as
    the GPU arm's multi-GPU line: config 5, strong scaling."""
    lines = run(["--impl", "reference", "--gpus", "2", "--n", "65536", "--steps", "1",
                 "--warmup", "0"], env={"RANK": "0", "WORLD_SIZE": "2"})
    assert len(lines) == 1
    line = lines[0]
    assert line["config"]["workload"].startswith("config 5")
    assert line["scaling"] == "strong" and line["n_gpus"] == 2
    assert line["config"]["per_gpu_n"] == 65536 // 2


def test_reference_arm_under_torchrun_uses_the_strong_scaling_config():
    """With WORLD_SIZE > 1 the reference arm's line carries the same config as
    the GPU arm's multi-GPU line: config 5, strong scaling."""
    lines = run(["--impl", "reference", "--gpus", "2", "--n", "65536", "--steps", "1",
                 "--warmup", "0"], env={"RANK": "0", "WORLD_SIZE": "2"})
    assert len(lines) == 1
    line = lines[0]
    assert line["config"]["workload"].startswith("config 5")
    assert line["scaling"] == "strong" and line["n_gpus"] == 2
    assert line["config"]["per_gpu_n"] == 65536 // 2
