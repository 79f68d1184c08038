"""Re-measure the constants of emugemm's error and speed model on the current GPU.

The B200 counterpart of emugemm-cdna's calibration studies (bench/flat_error.cpp: error vs K and chunk count;
bench/error_model.cpp: error per data distribution; bench/rho_sweep.cpp: error under cancellation). It runs the
library's own kernels through the C ABI against an FP64 ground truth and prints the fitted constants in the
order of the ModelConsts table in csrc/model.cpp, plus the raw measurements as JSON.

    python emugemm-cdna_b200/calibrate.py [--quick] [--out calib.json]

Fits (each with a safety margin, default 3%):
  a_fp32        max over measurements of err / sqrt(K/c)  (NATIVE_FP32 and FP32_CHUNKED, U[-1,1] and N(0,1))
  floor_bf16x3  max bf16x3 error at K <= 4096;  a_lowp = max sqrt(err^2 - floor^2) / sqrt(K)
  floor_fp16x3  max fp16x3 error at K <= 4096;  a_fp16x3 likewise
  spd_*         FP32 kernel time / scheme kernel time at S^3;  fp32_flops = 2 S^3 / FP32 kernel time
  hbm_bps       (4 + 4) bytes per input element / split time (the split reads FP32 and writes two slices)
  chunk costs   FP32_CHUNKED time at c / time at c = 1 (4096 x 4096 x 65536)
The rho factor is checked on the cancellation family of bench/emu_adversarial.cpp: measured error divided by
the iid-model error must stay below rho / (0.64 sqrt(K)) (or below 1 when that is smaller).
"""
from __future__ import annotations

import argparse
import json
import math
import pathlib
import sys

import torch

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import emugemm  # noqa: E402


def gen(kind: str, shape, g):
    if kind == "normal":
        return torch.randn(shape, device="cuda", generator=g)
    return torch.rand(shape, device="cuda", generator=g) * 2 - 1


def rel(C, R):
    return ((C.double() - R).norm() / R.norm()).item()


def accuracy(h, Ks, dists, M=256):
    rows = []
    for dist in dists:
        for K in Ks:
            g = torch.Generator(device="cuda").manual_seed(K)
            A, B = gen(dist, (M, K), g), gen(dist, (K, M), g)
            R = A.double() @ B.double()
            C = torch.empty(M, M, device="cuda")
            for name, s in (("native", emugemm.NATIVE_FP32), ("bf16x3", emugemm.BF16X3), ("fp16x3", emugemm.FP16X3)):
                h.sgemm(M, M, K, A, B, C, force=s, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
                h.sync()
                rows.append({"dist": dist, "K": K, "scheme": name, "c": 1, "err": rel(C, R)})
            for c in (4, 16, 64):
                P = torch.empty(M, M, dtype=torch.float64, device="cuda")
                h.partial_f64(M, M, K, A, K, B, M, P, emugemm.FP32_CHUNKED, c)
                h.reduce_f64(M, M, 1, P, C)
                h.sync()
                rows.append({"dist": dist, "K": K, "scheme": "chunked", "c": c, "err": rel(C, R)})
    return rows


def rho_check(h, K=8192, M=1024):
    sys.path.insert(0, str(HERE.parent / "tests"))
    import datagen

    out = []
    for rho in (1e2, 1e3, 1e4):
        A, B = datagen.family2(M, M, K, rho)
        dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
        R = dA.double() @ dB.double()
        rho_true = ((dA.double().abs() @ dB.double().abs()).norm() / R.norm()).item()
        C = torch.empty(M, M, device="cuda")
        for name, s in (("native", emugemm.NATIVE_FP32), ("bf16x3", emugemm.BF16X3)):
            h.sgemm(M, M, K, dA, dB, C, force=s, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
            h.sync()
            iid = emugemm.lib().emugemm_model_err(s, K, 1)
            out.append({"rho": rho_true, "scheme": name, "err": rel(C, R), "err_over_iid_model": rel(C, R) / iid,
                        "rho_over_rho_ref": rho_true / (0.64 * math.sqrt(K))})
    return out


def timing(h, S, reps):
    A = torch.randn(S, S, device="cuda")
    B = torch.randn(S, S, device="cuda")
    C = torch.empty(S, S, device="cuda")
    res = {}
    for name, s in (("native", emugemm.NATIVE_FP32), ("bf16x3", emugemm.BF16X3), ("fp16x3", emugemm.FP16X3)):
        for _ in range(2):
            h.sgemm(S, S, S, A, B, C, force=s, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        h.sync()
        h.profile_begin()
        for _ in range(reps if name != "native" else max(1, reps // 5)):
            h.sgemm(S, S, S, A, B, C, force=s, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        p = h.profile_end()
        res[name] = {k: (v[0] / v[1] if v[1] else None) for k, v in p.items()}
    return res


def chunk_costs(h, M=4096, K=65536):
    A = torch.rand(M, K, device="cuda")
    B = torch.rand(K, M, device="cuda")
    P = torch.empty(M, M, dtype=torch.float64, device="cuda")
    out = {}
    for c in (1, 4, 16, 64, 256):
        h.partial_f64(M, M, K, A, K, B, M, P, emugemm.FP32_CHUNKED, c)
        h.sync()
        h.profile_begin()
        h.partial_f64(M, M, K, A, K, B, M, P, emugemm.FP32_CHUNKED, c)
        p = h.profile_end()
        out[c] = p["fp32_gemm"][0]
    return {c: t / out[1] for c, t in out.items()}


def fit(acc, tim, margin):
    a32 = max(r["err"] / math.sqrt(r["K"] / r["c"]) for r in acc if r["scheme"] in ("native", "chunked"))
    fits = {"a_fp32": a32 * (1 + margin)}
    for scheme, key_floor, key_a in (("bf16x3", "floor_bf16x3", "a_lowp"), ("fp16x3", "floor_fp16x3", "a_fp16x3")):
        rs = [r for r in acc if r["scheme"] == scheme]
        floor = max(r["err"] for r in rs if r["K"] <= 4096) * (1 + margin)
        a = max(math.sqrt(max(0.0, r["err"] ** 2 - (floor / (1 + margin)) ** 2)) / math.sqrt(r["K"]) for r in rs)
        fits[key_floor] = floor
        fits[key_a] = a * (1 + margin)
    nat = tim["native"]["fp32_gemm"]
    fits["spd_bf16x3"] = nat / tim["bf16x3"]["tc_gemm"]
    fits["spd_fp16x3"] = nat / tim["fp16x3"]["tc_gemm"]
    return fits


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--margin", type=float, default=0.03)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    torch.cuda.set_device(0)
    Ks = (1024, 4096, 16384, 65536) if args.quick else (1024, 4096, 16384, 65536, 262144)
    with emugemm.Handle() as h:
        acc = accuracy(h, Ks, ("normal", "uniform"))
        tim = timing(h, args.size, 5 if args.quick else 20)
        rho = rho_check(h)
        cc = {} if args.quick else chunk_costs(h)
    fits = fit(acc, tim, args.margin)
    S = args.size
    fits["fp32_flops"] = 2.0 * S ** 3 / (tim["native"]["fp32_gemm"] * 1e-3)
    fits["hbm_bps"] = 2.0 * S * S * 8 / (tim["bf16x3"]["split"] * 1e-3)
    report = {"fits": fits, "accuracy": acc, "timing_ms": tim, "rho": rho, "chunk_cost": cc}
    print(json.dumps(report, indent=1))
    if args.out:
        pathlib.Path(args.out).write_text(json.dumps(report, indent=1))


if __name__ == "__main__":
    main()
