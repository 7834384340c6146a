"""Generate tests/golden/host_golden.json from the reference's own host code.

Runs oracle/_ref/host_probe, which is the reference's core/, distribution/,
kernels/swifi.cuh and metrics/ host functions compiled from the reference
checkout (`make -C oracle ref`). Must run on a machine WITHOUT a GPU (the probe
refuses otherwise). The JSON it writes is committed; the tests read only that.

    make -C oracle ref && python tests/golden/make_golden.py
"""
import json
import os
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
PROBE = os.path.join(HERE, "..", "..", "oracle", "_ref", "host_probe")


def run(*args):
    r = subprocess.run([PROBE] + [str(a) for a in args], check=True, capture_output=True, text=True)
    return r.stdout


def main():
    g = {"source": "reference host functions via oracle/_ref/host_probe"}

    fills = []
    for seed, total, npr in [(123456, 4096, 64), (987654, 4096, 64), (0, 4096, 64), (1, 1000, 32),
                             (42, 1 << 20, 16), (18446744073709551557, 4096, 16), (123456 + 987654, 65536, 8)]:
        out = run("fill", seed, total, npr).split()
        assert out[0] == "hash"
        fills.append({"seed": seed, "total": total, "hash": int(out[1]), "first": out[2:]})
    g["fill_random"] = fills

    g["choose_grid"] = {str(w): list(map(int, run("grid", w).split())) for w in range(1, 17)}

    splits = []
    for total, parts in [(1024, 4), (1000, 3), (7, 4), (4096, 4), (1030, 3), (5, 5), (16384, 8), (17, 1)]:
        rows = [list(map(int, l.split())) for l in run("split", total, parts).strip().splitlines()]
        splits.append({"total": total, "parts": parts, "counts": [r[0] for r in rows],
                       "offsets": [r[1] for r in rows]})
    g["split_dim"] = splits

    g["swifi_zone_range"] = {z: list(map(int, run("zone", z).split()))
                             for z in ["any", "sign", "exponent", "sig_high", "sig_low", "bogus"]}

    forms = []
    for k, na, nb in [(1024, 520.25, 530.5), (4096, 2048.0, 2050.125), (8192, 4100.0, 2049.0), (1, 1.0, 1.0),
                      (16384, 8192.5, 8191.25)]:
        forms.append({"k": k, "nA": na, "nB": nb, "bits": run("formula", k, repr(na), repr(nb)).strip()})
    g["threshold_formula"] = forms

    ths = []
    for M, K, N, sa, sb, F, ovr in [(64, 80, 48, 123456, 987654, 4, -1), (1024, 1024, 1024, 123456, 987654, 4, -1),
                                    (1100, 300, 1030, 5, 7, 3, -1), (1024, 1024, 1024, 0, 0, 4, -1),
                                    (1024, 2048, 1024, 11, 12, 4, 0.5)]:
        lines = run("thresholds", M, K, N, sa, sb, F, ovr).strip().splitlines()
        Fr = int(lines[0].split()[1])
        ths.append({"M": M, "K": K, "N": N, "seed_a": sa, "seed_b": sb, "frags": F, "override": ovr, "F": Fr,
                    "normA": lines[1].split()[1], "tau": [l.split()[2] for l in lines[2:]]})
    g["thresholds"] = ths

    injs = []
    for base, rank, it, M_b, nfs in [(123456 + 987654, 0, 0, 1024, [256] * 4),
                                     (123456 + 987654 + 31337 * 2, 0, 7, 1024, [256] * 4),
                                     (1111110 + 31337 * 3, 5, 19, 4096, [512] * 4),
                                     (0, 0, 0, 64, [48]), (0, 3, 9, 1100, [344, 343, 343]),
                                     (12345, 1, 1, 16384, [4096] * 4), (1, 0, 0, 7, [2, 2, 1, 1])]:
        frag, row, col = map(int, run("inject", base, rank, it, M_b, *nfs).split())
        injs.append({"base_seed": base, "rank": rank, "it": it, "M_b": M_b, "nf": nfs, "frag": frag,
                     "row": row, "col": col})
    g["inject"] = injs

    stats = []
    for vals in [[3.0, 1.0, 2.0], [5.5, 1.25, 9.0, 2.0], [7.0], [0.1, 0.2, 0.3, 0.4, 0.5, 0.6]]:
        stats.append({"samples": vals, "bits": run("stats", *[repr(v) for v in vals]).split()})
    g["stats_of"] = stats

    metrics = []
    cases = [
        ["online", "add", "any", 0, 0, 1024, 1024, 1024, 1, 1, 4, 10, 0.01024, 40, 0, 0, 0, 0, 1.5, 1.75, 1.8, 2.5],
        ["online", "swifi", "exponent", 0, 0, 4096, 4096, 4096, 1, 1, 4, 20, 0.04096, 45, 300, 1, 54, 40, 3.25, 3.5,
         3.6, 4.0],
        ["baseline", "none", "any", 1, 0, 8192, 8192, 8192, 2, 4, 4, 20, 1148.25, 0, 640, 0, 0, 0, 20.0, 21.0, 21.5,
         23.0],
        ["calibrate", "none", "any", 0, 1, 2048, 1024, 512, 1, 2, 4, 5, 9.5, 0, 0, 0, 0, 0, 0.5, 0.625, 0.7, 0.9],
    ]
    with tempfile.TemporaryDirectory() as td:
        for i, c in enumerate(cases):
            path = os.path.join(td, f"m{i}.csv")
            out = run("metrics", path, *c)
            metrics.append({"args": c, "stdout": out, "csv": open(path).read()})
    g["metrics"] = metrics

    with open(os.path.join(HERE, "host_golden.json"), "w") as f:
        json.dump(g, f, indent=1)
    print("wrote", os.path.join(HERE, "host_golden.json"))


if __name__ == "__main__":
    main()
