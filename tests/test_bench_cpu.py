"""The benchmark's CPU-only legs: the reference arm (``bench.py --impl reference``)
prints one JSON line with the keys of the bench contract, and ranks other than 0
of a multi-rank launch exit without work."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(*args, env=None, timeout=600):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                          capture_output=True, text=True, timeout=timeout, env=e, cwd=ROOT)


def test_reference_arm_json_line():
    res = run_bench("--impl", "reference", "--steps", "2", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["steps"] == 2
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_reference_arm_other_ranks_do_nothing():
    res = run_bench("--impl", "reference", "--gpus", "2", "--steps", "2", "--warmup", "3",
                    env={"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"}, timeout=300)
    assert res.returncode == 0 and res.stdout.strip() == ""


def test_warmup_below_three_is_refused():
    res = run_bench("--steps", "2", "--warmup", "2", timeout=300)
    assert res.returncode != 0 and "warmup" in res.stderr


def test_reference_arm_prints_the_b200_arm_config():
    """Both arms describe the workload with the same ``config`` object."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    res = run_bench("--impl", "reference", "--steps", "2", "--warmup", "3")
    assert res.returncode == 0, res.stderr[-2000:]
    d = json.loads(res.stdout.strip().splitlines()[-1])
    assert d["config"] == bench.workload_config(1, bench.l2_size_bytes())
    for world in (1, 2, 4, 8):
        layers, per_gpu = bench.layer_count(world, bench.B200_L2_BYTES)
        assert layers * per_gpu >= 3 * bench.B200_L2_BYTES
