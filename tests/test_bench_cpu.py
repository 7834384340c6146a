"""bench.py's CPU-side contract: the reference arm (the reference's algorithm on
the host cores) prints one JSON line with the keys the benchmark driver reads,
ranks other than 0 print nothing, and the verify kernel's DRAM traffic comes
from the committed ncu summary of the benchmarked fragment."""
import json
import os
import subprocess
import sys

from conftest import ROOT

BENCH = os.path.join(ROOT, "bench.py")


def run_bench(args, env_extra=None):
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, BENCH] + args, capture_output=True, text=True, timeout=600, env=env,
                          cwd=ROOT)


def test_reference_arm_json_line():
    r = run_bench(["--impl", "reference", "--steps", "2", "--warmup", "3", "--tile", "512", "--K", "256",
                   "--iters", "4"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["unit"] == "TFLOP/s"
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["tile"] == [512, 512] and d["config"]["K"] == 256 and "workload" in d["config"]


def test_reference_arm_other_ranks_are_silent():
    r = run_bench(["--impl", "reference", "--steps", "1", "--warmup", "3", "--tile", "256", "--K", "128"],
                  {"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


def test_verify_traffic_comes_from_the_committed_summary():
    sys.path.insert(0, ROOT)
    import bench
    # the benchmarked 4096 x 1024 fragment has ncu summaries for both verify bodies
    for kernel in ("auto", "ldg", "tma"):
        t = bench.verify_traffic_per_launch(4096, 4, kernel)
        assert t is not None and 16.8e6 < t < 16.9e6, (kernel, t)
    assert bench.verify_traffic_per_launch(1234, 4, "auto") is None
