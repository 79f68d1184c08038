"""Per-shape kernel tuner: writes the tile table that emugemm_init loads (the B200 counterpart of emugemm-cdna's
bench/gen_tune_table.cpp: offline, resumable, shardable, header written once under an exclusive lock).

For every (M, N, K, dtype) of the grid it times the candidate kernels through the C ABI and appends one row
    arch,cuda_version,M,N,K,dtype,tile,best_ms,default_ms,gain
where `tile` is the winner (bf16/fp16: 1 = single-CTA, 2 = CTA pair, 3 = fused split, 4 = A split into TMEM (bf16);
fp32: SIMT tile 16 (16 x 32), 32, 64, 128 or 3264 (32 x 64)),
`default_ms` the built-in choice's time and `gain` = default_ms / best_ms. Rows already present for a key are
skipped, so an interrupted run resumes; --shard i/n takes every n-th shape starting at i (one process per GPU).
--dtypes restricts the grid; --replace first drops the table's rows of those dtypes, so that they are measured
again after a kernel change while the other rows stay.

    python emugemm-cdna_b200/tune_tiles.py tiles_b200.csv [--shard 0/8] [--quick] [--dtypes bf16,fp16 --replace]
"""
from __future__ import annotations

import argparse
import csv
import fcntl
import itertools
import os
import pathlib
import sys

import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import emugemm  # noqa: E402

HEADER = "arch,cuda_version,M,N,K,dtype,tile,best_ms,default_ms,gain\n"
DTYPES = {"bf16": emugemm.BF16X3, "fp16": emugemm.FP16X3, "fp32": emugemm.NATIVE_FP32}


def existing_keys(path: pathlib.Path) -> set:
    keys = set()
    if path.exists():
        with path.open() as f:
            for row in csv.reader(f):
                if len(row) == 10 and row[0] != "arch":
                    keys.add((int(row[2]), int(row[3]), int(row[4]), row[5]))
    return keys


def drop_rows(path: pathlib.Path, dtypes: set) -> None:
    """Rewrite the table without its rows of the given dtypes (the header and other rows stay, in order)."""
    if not path.exists():
        return
    with path.open("r+") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        keep = [ln for ln in f.read().splitlines(keepends=True)
                if not (len(ln.split(",")) == 10 and ln.split(",")[5] in dtypes)]
        f.seek(0)
        f.truncate()
        f.writelines(keep)
        f.flush()
        fcntl.flock(f, fcntl.LOCK_UN)


def append_row(path: pathlib.Path, row: str) -> None:
    with path.open("a") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        if f.tell() == 0:
            f.write(HEADER)
        f.write(row)
        f.flush()
        fcntl.flock(f, fcntl.LOCK_UN)


def time_call(h, fn, reps: int) -> float:
    fn()
    h.sync()
    h.profile_begin()
    for _ in range(reps):
        fn()
    p = h.profile_end()
    tot = sum(v[0] for v in p.values() if v[1])
    return tot / reps


def tune_shape(h, M, N, K, dtype, reps):
    A = torch.randn(M, K, device="cuda")
    B = torch.randn(K, N, device="cuda")
    C = torch.empty(M, N, device="cuda")
    scheme = DTYPES[dtype]
    hints = emugemm.EmuHints(1.0, 1.0, 0, 0.0, 0)
    res = {}

    def timed():
        return time_call(h, lambda: h.sgemm(M, N, K, A, B, C, force=scheme, hints=hints), reps)

    if dtype == "fp32":
        # time each SIMT tile by loading a one-row table per candidate
        for tile in (128, 64, 3264, 32, 16):
            tmp = pathlib.Path(f"/tmp/emugemm_tile_{os.getpid()}.csv")
            tmp.write_text(HEADER + f"{arch()},probe,{M},{N},{K},fp32,{tile},0,0,1\n")
            emugemm.lib().emugemm_init(str(tmp).encode())
            res[tile] = timed()
            tmp.unlink()
        emugemm.lib().emugemm_shutdown()
    else:
        kernels = (((1, "single"), (2, "pair"), (3, "fused"), (4, "fusea")) if dtype == "bf16"
                   else ((1, "single"), (2, "pair"), (3, "fused")))
        for tile, name in kernels:
            h.set_kernels(tc_kernel=name)
            res[tile] = timed()
        h.set_kernels(tc_kernel=0)
    default_ms = timed()   # the built-in choice: no table row, no override
    best = min(res, key=res.get)
    return best, res[best], default_ms


def arch() -> str:
    major, minor = torch.cuda.get_device_capability(0)
    return f"sm_{major}{minor}" + ("a" if (major, minor) == (10, 0) else "")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("table")
    ap.add_argument("--shard", default="0/1")
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--dtypes", default="bf16,fp16,fp32")
    ap.add_argument("--replace", action="store_true")
    args = ap.parse_args()
    dtypes = set(args.dtypes.split(","))
    i, n = (int(x) for x in args.shard.split("/"))
    torch.cuda.set_device(0)
    if args.quick:
        grid = list(itertools.product((2048, 8192), (2048, 8192), (2048, 8192), ("bf16", "fp16")))
    else:
        sizes = (1024, 2048, 4096, 8192, 16384)
        grid = list(itertools.product(sizes, sizes, (1024, 4096, 16384, 65536), ("bf16", "fp16", "fp32")))
        grid = [g for g in grid if g[0] * g[1] * g[2] <= 8192 ** 3 * 2]
    grid = [g for g in grid if g[3] in dtypes]
    path = pathlib.Path(args.table)
    if args.replace and i == 0:
        drop_rows(path, dtypes)
    done = existing_keys(path)
    with emugemm.Handle() as h:
        for j, (M, N, K, dt) in enumerate(grid):
            if j % n != i or (M, N, K, dt) in done:
                continue
            best, best_ms, def_ms = tune_shape(h, M, N, K, dt, args.reps)
            append_row(path, f"{arch()},{torch.version.cuda},{M},{N},{K},{dt},{best},{best_ms:.5f},{def_ms:.5f},"
                             f"{def_ms / best_ms:.4f}\n")
            print(M, N, K, dt, best, f"{best_ms:.4f}", f"{def_ms:.4f}", flush=True)


if __name__ == "__main__":
    main()
