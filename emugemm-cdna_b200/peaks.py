"""Peak rates of one B200, measured with one instrument: the counterpart of emugemm-cdna bench/mfma_peak2.cpp.

That probe answers which precisions the emulation can stand on: it times each matrix-core instruction in a
register loop (all kernels interleaved, median of the repetitions) and prints the bf16:fp32 ratio R, from which a
3-product scheme is capped at R/3 of native FP32 (bench/mfma_peak2.cpp:120-131), and whether FP64 emulation could
pay (:133-139). Here the instruments (csrc/k_peak.cu, through emugemm_peak_probe) are tcgen05 MMAs of
kind::f16 (bf16, fp16) and kind::tf32 on operands resident in shared memory, FP32 and FP64 FMA chains, and a
device copy. Native FP32 on B200 is the FFMA pipe: the tensor cores take no FP32 inputs.

    python peaks.py [--reps 7] [--json]
"""
from __future__ import annotations

import argparse
import json
import sys

import emugemm


def ratios(r: dict) -> dict:
    """The economics of emulation on this GPU (bench/mfma_peak2.cpp:114-139 asks the same questions)."""
    ffma, dfma = r["ffma_tflops"], r["dfma_tflops"]
    R_bf16, R_fp16 = r["tc_bf16_tflops"] / ffma, r["tc_fp16_tflops"] / ffma
    return {
        "bf16_over_fp16": r["tc_bf16_tflops"] / r["tc_fp16_tflops"],
        "tf32_over_bf16": r["tc_tf32_tflops"] / r["tc_bf16_tflops"],
        "R_bf16": R_bf16,                       # bf16 tensor : native FP32
        "R_fp16": R_fp16,
        "bf16x3_ceiling": R_bf16 / 3.0,         # best case of 3 products against native FP32
        "fp16x3_ceiling": R_fp16 / 3.0,
        "bf16x6_ceiling": R_bf16 / 6.0,
        "fp32_over_fp64": ffma / dfma,
        "fp64_from_fp32_3_slices": ffma / dfma / 3.0,
        "fp64_from_bf16_7_slices": r["tc_bf16_tflops"] / dfma / 7.0,
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reps", type=int, default=7)
    ap.add_argument("--json", action="store_true", help="print one JSON object instead of the table")
    args = ap.parse_args(argv)
    h = emugemm.Handle()
    r = h.peak_probe(args.reps)
    q = ratios(r)
    if args.json:
        print(json.dumps({"rates": r, "ratios": q, "reps": args.reps}))
        return 0
    print(f"B200 peak rates ({args.reps} interleaved repetitions, median)\n")
    rows = [("tcgen05 kind::f16, bf16 in, FP32 acc", r["tc_bf16_tflops"], "TFLOP/s"),
            ("tcgen05 kind::f16, fp16 in, FP32 acc", r["tc_fp16_tflops"], "TFLOP/s"),
            ("tcgen05 kind::tf32, FP32 acc", r["tc_tf32_tflops"], "TFLOP/s"),
            ("FFMA (native FP32)", r["ffma_tflops"], "TFLOP/s"),
            ("DFMA (native FP64)", r["dfma_tflops"], "TFLOP/s"),
            ("device copy (read + write)", r["copy_gbs"], "GB/s")]
    for name, v, unit in rows:
        rel = f"{v / r['ffma_tflops']:7.2f}x FFMA" if unit == "TFLOP/s" else ""
        print(f"  {name:40s} {v:10.1f} {unit:8s} {rel}")
    print(f"\n  bf16 / fp16 = {q['bf16_over_fp16']:.3f}   tf32 / bf16 = {q['tf32_over_bf16']:.3f}")
    print(f"  R (bf16 : FP32) = {q['R_bf16']:.2f} -> bf16x3 ceiling {q['bf16x3_ceiling']:.2f}x native FP32, "
          f"bf16x6 {q['bf16x6_ceiling']:.2f}x")
    print(f"  R (fp16 : FP32) = {q['R_fp16']:.2f} -> fp16x3 ceiling {q['fp16x3_ceiling']:.2f}x")
    print(f"  FP64 emulation: fp32/fp64 = {q['fp32_over_fp64']:.2f} -> 3 FP32 slices "
          f"{q['fp64_from_fp32_3_slices']:.2f}x, 7 bf16 slices {q['fp64_from_bf16_7_slices']:.2f}x native FP64")
    return 0


if __name__ == "__main__":
    sys.exit(main())
