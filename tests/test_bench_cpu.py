"""bench.py's CPU-side contract: the reference arm (the reference's algorithm on
the host cores) prints one JSON line with the keys the benchmark driver reads,
ranks other than 0 print nothing, the arm never loads the product library,
the headline workload's strong-scaling geometry is the configuration's, and the
verify kernel's DRAM traffic comes from the committed ncu summary of the
benchmarked fragment."""
import json
import os
import subprocess
import sys
import types

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
    r = run_bench(["--impl", "reference", "--steps", "2", "--warmup", "3", "--workload", "tile4096", "--size", "512",
                   "--iters", "4"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["unit"] == "TFLOP/s" and d["scaling"] == "weak"
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["nproc"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["tile"] == [512, 512] and d["config"]["K"] == 512 and "workload" in d["config"]


def test_reference_arm_other_ranks_are_silent():
    r = run_bench(["--impl", "reference", "--steps", "1", "--warmup", "3", "--workload", "tile4096", "--size", "256"],
                  {"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_does_not_load_the_product():
    """The reference arm runs the oracle only: neither the product package nor
    its shared library may be loaded in that process."""
    code = (
        "import sys; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '3', "
        "'--size', '512', '--ref-rows', '64']\n"
        "import bench; bench.main()\n"
        "mods = [m for m in sys.modules if m.startswith(bench.PKG)]\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('PRODUCT', mods, 'libabft_b200.so' in maps, 'liboracle.so' in maps)\n")
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("PRODUCT")][0]
    assert line == "PRODUCT [] False True", line
    d = json.loads([l for l in r.stdout.splitlines() if l.startswith("{")][0])
    assert d["scaling"] == "strong" and d["config"]["M"] == d["config"]["N"] == d["config"]["K"] == 512


def test_headline_geometry_strong_scaling():
    """global16384 at 1, 2, 4, 8 ranks: choose_grid's 1x1, 1x2, 2x2, 2x4 grids,
    rank tiles 16384^2, 16384x8192, 8192^2, 8192x4096 with K = 16384 and F = 4;
    the oracle's helpers and the product's give the same geometry."""
    sys.path.insert(0, ROOT)
    import bench
    import oracle
    import importlib
    host = importlib.import_module(bench.PKG).host
    args = types.SimpleNamespace(kind="global", size=16384, frags=4)
    want = {1: ((1, 1), (16384, 16384)), 2: ((1, 2), (16384, 8192)), 4: ((2, 2), (8192, 8192)),
            8: ((2, 4), (8192, 4096))}
    for world, (grid, tile) in want.items():
        for rank in range(world):
            g = bench.Geometry(args, world, rank, oracle)
            h = bench.Geometry(args, world, rank, host)
            assert (g.Pr, g.Pc) == grid and (g.M_b, g.N_b) == tile and g.K == 16384 and g.F == 4
            assert list(g.counts) == [tile[1] // 4] * 4 and list(g.offsets) == [i * tile[1] // 4 for i in range(4)]
            assert (h.Pr, h.Pc, h.M_b, h.N_b, h.F) == (g.Pr, g.Pc, g.M_b, g.N_b, g.F)
            assert list(h.counts) == list(g.counts) and list(h.offsets) == list(g.offsets)
    # one step of the headline workload is one iteration, seeded as that iteration of one trial
    a1 = types.SimpleNamespace(iters=1)
    assert [bench.step_seed(a1, 10, j) for j in range(3)] == [10, 10 + 104729, 10 + 2 * 104729]
    a20 = types.SimpleNamespace(iters=20)
    assert bench.step_seed(a20, 10, 2) == 10 + 2 * 31337


def test_verify_traffic_comes_from_the_committed_summary():
    sys.path.insert(0, ROOT)
    import bench
    # the 4096 x 1024 fragment has ncu summaries for both verify bodies
    for kernel in ("auto", "ldg", "tma"):
        t = bench.verify_traffic_per_launch(4096, 1024, kernel)
        assert t is not None and 16.8e6 < t < 16.9e6, (kernel, t)
    assert bench.verify_traffic_per_launch(1234, 4, "auto") is None


def test_headline_fragments_have_committed_traffic():
    """Every fragment shape the headline workload runs at 1, 2, 4 and 8 GPUs
    has a committed ncu summary whose DRAM traffic is within 3 % of its
    algorithmic bytes (the excess is DRAM writes: lines that the buffer
    written to empty L2 left dirty, written back during the launch), so each
    N's bench line carries roofline.traffic."""
    sys.path.insert(0, ROOT)
    import bench
    for M_b, N_f in [(16384, 4096), (16384, 2048), (8192, 2048), (8192, 1024)]:
        t = bench.verify_traffic_per_launch(M_b, N_f, "auto")
        alg = 4.0 * M_b * N_f + 24.0 * N_f
        assert t is not None and alg <= t <= 1.03 * alg, (M_b, N_f, t, alg)
