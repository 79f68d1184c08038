"""Generate tests/golden/plan_ref_mi250.csv: plans from the reference planner itself.

Runs emugemm_plan of emugemm-cdna (src/emugemm.cpp:216-282), compiled from its own source into
oracle/_ref/libemuref.so by oracle/Makefile, over a fixed grid of shapes, targets, hints and forced
schemes, and writes one CSV row per case with predicted_err / predicted_speedup as exact hex floats.
tests/test_plan.py checks emugemm's planner (model "ref_mi250") against every row, bit for bit.

Usage: python tests/golden/make_plan_golden.py      (needs oracle/_ref/libemuref.so: make -C oracle ref)
"""
from __future__ import annotations

import csv
import itertools
import pathlib
import random
import sys

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "plan_ref_mi250.csv"


def cases():
    shapes = [(256, 256), (1024, 1024), (2048, 2048), (4096, 4096), (8192, 4096), (2048, 8192), (8192, 8192),
              (32768, 32768)]
    Ks = [64, 512, 1024, 4096, 8192, 16384, 65536, 262144, 1048576]
    tgts = [1e-3, 1e-4, 1e-5, 4.5e-6, 4e-6, 1e-6, 1e-7, 0.0]
    absm = [(1.0, 1.0), (4.19e6, 1.0), (1e-5, 1.0), (65504.0, 1.0), (-1.0, -1.0), (5.0, 5.0)]
    rhos = [-1.0, 0.0, 24.0, 192.0, 1e4, 1.1e6]
    grid = list(itertools.product(shapes, Ks, tgts, absm, rhos))
    rnd = random.Random(20260725)
    picked = rnd.sample(grid, 1200)
    # The plan-logic grid of bench/emugemm_test.cpp:38-59, then the benchmark shapes (1024^3 to 32768^3,
    # the long-K 256x256 cases, the 2048x2048x8192 cancellation cases and the 4096x4096x1048576 K-split).
    for K in (4096, 65536, 262144):
        for t in (1e-4, 1e-5, 4e-6, 1e-6, 1e-7):
            picked.append(((4096, 4096), K, t, (1.0, 1.0), 0.0))
    picked.append(((4096, 4096), 262144, 1e-6, (1e6, 1e6), 0.0))
    extra = [((1024, 1024), 1024, 1e-5, (1.0, 1.0), 24.0), ((8192, 8192), 8192, 1e-5, (4.19e6, 1.0), -1.0),
             ((16384, 16384), 16384, 1e-5, (4.19e6, 1.0), -1.0), ((256, 256), 65536, 1e-6, (1.0, 1.0), 192.0),
             ((256, 256), 65536, 1e-7, (1.0, 1.0), 192.0), ((256, 256), 262144, 1e-5, (1.0, 1.0), 384.0),
             ((256, 256), 262144, 1e-6, (1.0, 1.0), 384.0), ((2048, 2048), 8192, 1e-5, (4.0, 4.0), 1e4),
             ((2048, 2048), 8192, 1e-4, (4.0, 4.0), 1e4), ((2048, 2048), 8192, 1e-5, (1.0, 1.0), 3000.0),
             ((32768, 32768), 32768, 1e-5, (5.0, 5.0), -1.0), ((4096, 4096), 1048576, 1e-5, (5.0, 5.0), -1.0)]
    picked += extra
    for (MN, K, t, ab, rho) in picked:
        yield MN[0], MN[1], K, t, 0, ab[0], ab[1], rho, 1
    # forced schemes and NULL hints
    for force in (1, 2, 3, 4, 5):
        for K in (1024, 8192, 262144):
            for rho in (-1.0, 100.0):
                yield 1024, 1024, K, 1e-5, force, 1.0, 1.0, rho, 1
    for K in (1024, 65536):
        for t in (1e-5, 1e-7):
            yield 2048, 2048, K, t, 0, 0.0, 0.0, 0.0, 0


def main():
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libemuref.so is not built (make -C oracle ref)")
    rows = []
    for (M, N, K, t, force, a, b, rho, hints) in cases():
        p = oracle.ref_plan(M, N, K, t, force, a, b, rho, hints=bool(hints))
        rows.append([M, N, K, float(t).hex(), force, float(a).hex(), float(b).hex(), float(rho).hex(), hints,
                     p["chosen"], p["chunks"], p["predicted_err"].hex(), p["predicted_speedup"].hex(), p["reason"]])
    with OUT.open("w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["M", "N", "K", "tgt", "force", "a_absmax", "b_absmax", "rho", "hints", "chosen", "chunks",
                    "predicted_err", "predicted_speedup", "reason"])
        w.writerows(rows)
    print(f"wrote {len(rows)} plans to {OUT}")


if __name__ == "__main__":
    main()
