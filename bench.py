"""Benchmark of the emulated-FP32 GEMM hot path: bf16x3 emugemm_sgemm at M=N=K=8192 (the 8192^3 case of
the square sweep, inputs N(0,1) * 2^e with e uniform in [-20, 20]), one call per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--size S] [--scheme bf16x3]

ours:      value = emulated TFLOPS (2*M*N*K per step) with A, B resident in HBM, CUDA events on the handle's
           stream around the K timed steps, max over ranks; e2e = the same product through emugemm_sgemm_host
           with HOST inputs (pinned): H2D of A and B and D2H of C inside every timed step. Extra keys: roofline of the dominant kernel
           (tensor-core GEMM, timed with CUDA events on its own stream), cpu_baseline (the oracle's host FP64
           GEMM on a bounded row sample, all host threads), clocks sampled during the timed region,
           gpu_launches (kernels this library launched inside the timed region).
reference: the emugemm-cdna path has no CPU implementation of its GEMM (its slices go to rocBLAS on an AMD
           GPU), so this arm times the CPU restatement of that path (oracle: split + the three slice
           products, FP64 accumulation) on a bounded row sample with all host threads, rank 0 only.
With N > 1 (torchrun) each rank computes its own 8192-row block of a (8192*N) x 8192 x 8192 product through
emugemm_sgemm_rows: B travels from rank 0 inside every step, in column panels pulled by copy engines over NVLink
peer memory along a binary tree of the ranks, each panel's GEMM starting as it arrives (weak scaling). After the timed region the run checks sampled rows of every
rank's C against FP64 (`check`) and times the long-K sharded configuration, 4096 x 4096 x 1048576 with K split over
the ranks through emugemm_sgemm_ksplit, with its own check (`ksplit`).
Other workloads (--workload): `rows` = one S^3 product with the rows of A split over the ranks and B broadcast
from rank 0 in column panels (emugemm_sgemm_rows; strong scaling; S = 32768 is the sharded multi-GPU configuration,
iid N(0,1)); `ksplit` = S x S x --k with K split over the ranks, FP64 partial products summed by NCCL and rounded
once (emugemm_sgemm_ksplit; S = 4096, K = 1048576 is the long-K multi-GPU configuration, iid N(0,1)); `chunked` = FP32_CHUNKED at S x S x --k with --chunks
K-chunks (FP32 FMA chains, chunk sums in FP64; S = 256, K = 262144 is the long-K accumulation configuration),
U[-1,1] inputs, one partial + rounding per step; `rho` = the cancellation-ratio probe (--probes Hutchinson
vectors) on an S x S x S product, one emugemm_estimate_rho per step. `chunked` and `rho` run as independent
replicas under N > 1.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "emugemm-cdna_b200"))

SCHEMES = {"bf16x3": 3, "fp16x3": 4, "native": 1}

# DRAM bytes per launch of the tensor-core kernel from one ncu capture (read + write), by (scheme, size).
TRAFFIC = {("bf16x3", 8192): 3.564580e9 + 0.261143e9, ("fp16x3", 8192): 2.951390e9 + 0.266271e9}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--size", type=int, default=8192)
    ap.add_argument("--scheme", default="bf16x3", choices=list(SCHEMES))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--workload", default="square", choices=["square", "rows", "ksplit", "chunked", "longk", "rho"],
                    help="square: S^3 per GPU (weak); rows: one S^3 product, rows over GPUs; "
                         "ksplit: S x S x --k, K over GPUs; chunked: FP32_CHUNKED S x S x --k; "
                         "longk: --scheme at S x S x --k; rho: rho probe S^3")
    ap.add_argument("--k", type=int, default=1048576, help="K of the ksplit, chunked and longk workloads")
    ap.add_argument("--chunks", type=int, default=4, help="K-chunks of the chunked workload")
    ap.add_argument("--probes", type=int, default=64, help="probe vectors of the rho workload")
    ap.add_argument("--nccl-ctas", type=int, default=0, help="cap on NCCL CTAs per collective (0: NCCL's choice)")
    ap.add_argument("--no-ksplit", action="store_true", help="skip the K-split sub-record of the square workload")
    ap.add_argument("--no-check", action="store_true", help="skip the correctness check after the timed region")
    ap.add_argument("--no-sustained", action="store_true", help="skip the 2 s sustained-clock run after a short one")
    ap.add_argument("--no-clocks", action="store_true", help="no nvidia-smi clock sampling during the timed region")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), \
            float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def tc_kernel_name(M: int, N: int, K: int, scheme: str) -> str:
    """The tensor-core kernel the library picks for this shape: EMUGEMM_TC_KERNEL, else the tile table's code, else
    the built-in rule of the library (a copy of it); fp16x3 has no fused-A variant."""
    import emugemm

    fp16 = scheme == "fp16x3"
    env = os.environ.get("EMUGEMM_TC_KERNEL", "")
    code = {"single": 1, "pair": 2, "fused": 3, "fusea": 4}.get(env) or \
        emugemm.lib().emugemm_tune_lookup(M, N, K, 2 if fp16 else 1)
    if not code:
        pair_tiles, pairs = -(-M // 256) * -(-N // 256), 148 // 2
        if not fp16:
            code = 2 if (K > 1024 or pair_tiles >= pairs) else 1
            nck = -(-K // 128)
            if code == 2 and pair_tiles < 16 and min(pairs // pair_tiles, nck // 8) > 1:
                code = 3
        else:
            code = 2 if ((K > 1024 or pair_tiles >= 512) if pair_tiles >= pairs else K >= 16384) else 1
            nck = -(-K // 128)
            if code == 2 and pair_tiles < 16 and min(pairs // pair_tiles, nck // 8) > 1:
                code = 3
    if fp16 and code == 4:
        code = 2
    return {1: "k_tc_gemm", 2: "k_tc_gemm_pair", 3: "k_tc_fused",
            4: "k_tc_fused_a (+ k_split_cols of B)"}.get(code, "k_tc_gemm")


def ffma_peak() -> tuple[float, str]:
    """Nominal FP32 FMA throughput: 148 SMs x 128 FP32 lanes x 2 FLOP per clock at the maximum SM clock."""
    mhz = 1965.0
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        mhz = float(json.loads(p.read_text()).get("sm_max_mhz", mhz))
    return 148 * 128 * 2 * mhz * 1e6 / 1e12, f"nominal FFMA (148 SMs x 128 lanes x 2 FLOP x {mhz:.0f} MHz)"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of the job's GPUs sampled every 100 ms by one process and a reader
    thread (on rank 0 only; the other ranks pass enabled=False); only samples that arrive between mark_start() and
    mark_end() (the timed region) are summarised, over all the GPUs sampled."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, indices, enabled: bool = True):
        self.indices = list(indices)
        self.enabled = enabled
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def __enter__(self):
        import threading

        if not self.enabled:
            return self
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--id=" + ",".join(str(i) for i in self.indices),
                                          f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self

        def reader():
            for line in self.proc.stdout:
                self.lines.append((time.time(), line))

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        deadline = time.time() + 5.0
        while not self.lines and time.time() < deadline:   # wait for the first sample
            time.sleep(0.05)
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc:
            if self.t1 is not None:   # a timed region shorter than the interval: wait for the sample after it
                deadline = time.time() + 0.3
                while time.time() < deadline and not any(t > self.t1 for t, _ in self.lines[-2:]):
                    time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        """Median SM clock, max clock and active reasons over the samples taken inside the timed region; when the
        region is shorter than the sampling interval, over the samples nearest to it (the last one before it
        and the first one after it, each within 0.3 s), marked "window": "nearest"."""
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = self.lines
        window = "timed region"
        if self.t0 is not None:
            t1 = self.t1 or time.time()
            inside = [(t, l) for t, l in lines if self.t0 <= t <= t1]
            if not inside:
                before = [(t, l) for t, l in lines if self.t0 - 0.3 <= t < self.t0][-1:]
                after = [(t, l) for t, l in lines if t1 < t <= t1 + 0.3][:1]
                inside = before + after
                window = "nearest"
            lines = inside
        for t, line in lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm), "window": window}


def tensor_peak(ms_total: float, clocks: dict, burst: float, sustained: float) -> tuple[float, str]:
    """The bf16 peak a tensor-core kernel's rate is compared with. A timed loop of more than half a second, or one
    whose clock samples show the power cap holding the SM clock below 90 % of its maximum, runs under the power cap:
    the sustained peak. Otherwise (a sw_power_cap flag seen at the full clock included) the burst peak."""
    capped = ("sw_power_cap" in clocks.get("reasons", []) and clocks.get("sm_mhz") is not None
              and bool(clocks.get("sm_max_mhz")) and clocks["sm_mhz"] < 0.9 * clocks["sm_max_mhz"])
    if ms_total > 500.0 or capped:
        return sustained, "bf16_tflops_sustained"
    return burst, "bf16_tflops"


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_fp64_baseline(size: int, budget_s: float = 12.0) -> dict:
    """The oracle's blocked OpenMP FP64 GEMM (the host ground-truth GEMM) on a bounded sample of rows."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    oracle.set_num_threads(cpu_threads())
    rng = np.random.default_rng(1)
    K = N = size
    B = rng.standard_normal((K, N)).astype(np.float32)
    rows = 8
    while True:
        A = rng.standard_normal((rows, K)).astype(np.float32)
        t0 = time.perf_counter()
        oracle.gemm_f64(A, B)
        dt = time.perf_counter() - t0
        if dt > budget_s / 4 or rows >= size:
            break
        rows = min(size, max(rows * 2, int(rows * (budget_s / 4) / max(dt, 1e-3))))
    tflops = 2.0 * rows * N * K / dt / 1e12
    return {"value": tflops, "unit": "TFLOPS", "cores": oracle.num_threads(), "kind": "port",
            "sample": f"{rows} rows of the {size}^3 FP64 product (A[:{rows}] @ B), {dt:.2f} s"}


def _plan_err(M: int, N: int, K: int, scheme: int, chunks: int = 1) -> float:
    """The predicted normwise error of a forced scheme with absmax 1 and the iid model (the hints of the timed calls)."""
    import emugemm

    if chunks > 1:
        return float(emugemm.lib().emugemm_model_err(scheme, K, chunks))
    return float(emugemm.plan(M, N, K, 1e-5, force=scheme, a_absmax=1.0, b_absmax=1.0, rho=0.0).predicted_err)


def check_rows(torch, dist, A, B, C, M_glob: int, N: int, K: int, scheme: int, nrows: int = 64) -> dict:
    """Row-sharded product: nrows evenly spaced rows of this rank's C block against A[rows] @ B in FP64 (B complete
    on every rank); the largest error over the ranks."""
    m = A.shape[0]
    idx = torch.linspace(0, max(m - 1, 0), min(nrows, m), device="cuda").long()
    R = A[idx].double() @ B.double()
    err = ((C[idx].double() - R).norm() / R.norm()).item() if m > 0 else 0.0
    if dist is not None:
        t = torch.tensor([err], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        err = float(t.item())
    pred = _plan_err(M_glob, N, K, scheme)
    return {"max_rel_err": err, "predicted_err": pred, "ok": bool(err <= pred),
            "how": f"{min(nrows, m)} sampled rows of every rank's C block vs FP64 A[rows] @ B, max over ranks"}


def check_ksplit(torch, dist, h, A_loc, B_loc, C, M: int, N: int, K: int, world: int, rank: int, scheme: int,
                 nrows: int = 32) -> dict:
    """K-split product: nrows sampled rows of C (on rank 0) against the FP64 sum over ranks of A_loc[rows] @ B_loc."""
    idx = torch.linspace(0, M - 1, nrows, device="cuda").long()
    R = torch.zeros((nrows, N), dtype=torch.float64, device="cuda")
    kl = A_loc.shape[1]
    for k0 in range(0, kl, 65536):          # in K pieces, so no FP64 copy of all of B_loc is held
        k1 = min(kl, k0 + 65536)
        R += A_loc[idx, k0:k1].double() @ B_loc[k0:k1].double()
    if dist is not None:
        dist.all_reduce(R)
    err = ((C[idx].double() - R).norm() / R.norm()).item() if rank == 0 else 0.0
    if dist is not None:
        t = torch.tensor([err], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        err = float(t.item())
    pred = _plan_err(M, N, K, scheme, chunks=world)
    return {"max_rel_err": err, "predicted_err": pred, "ok": bool(err <= pred),
            "how": f"{nrows} sampled rows of C vs the FP64 product of those rows, model error with {world} FP64 chunks"}


def ksplit_record(torch, dist, h, args, world: int, rank: int, scheme: int, gen) -> dict:
    """The long-K sharded configuration in the same run: M = N = 4096, K = args.k (1048576) split over the ranks,
    iid N(0,1), emugemm_sgemm_ksplit (FP64 partials summed by NCCL, one rounding on rank 0), CUDA events on every
    rank, the max over ranks; then its correctness check."""
    M = N = 4096
    K = args.k
    k0, k1 = h.comm_krange(K)
    kl = k1 - k0
    A = torch.randn((M, kl), device="cuda", generator=gen)
    B = torch.randn((kl, N), device="cuda", generator=gen)
    C = torch.empty((M, N), device="cuda")
    stream = torch.cuda.current_stream()

    def step():
        h.sgemm_ksplit(M, N, K, A, kl, B, N, C, N, root=0, scheme=scheme)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    steps = 5
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if dist is not None:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    chk = check_ksplit(torch, dist, h, A, B, C, M, N, K, world, rank, scheme)
    del A, B, C
    torch.cuda.empty_cache()
    return {"workload": f"{M}x{N}x{K} bf16x3, K split over {world} GPU(s), FP64 partials summed by NCCL (strong)",
            "value": 2.0 * M * N * K / (ms * 1e-3) / 1e12, "unit": "TFLOPS", "ms_per_step": ms, "steps": steps,
            "warmup": 2, "data": "synthetic iid N(0,1)", "check": chk}


def reference_arm(args) -> None:
    import numpy as np

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    # a launcher such as torchrun sets OMP_NUM_THREADS=1 for every rank: use the cores this process may run on
    oracle.set_num_threads(cpu_threads())
    size = args.size
    rng = np.random.default_rng(2)
    K = N = size
    B = (rng.standard_normal((K, N)) * np.ldexp(1.0, rng.integers(-20, 21, (K, N)))).astype(np.float32)
    kind = 0 if args.scheme != "fp16x3" else 1
    # size the row sample so one step takes a few seconds
    rows = 4
    A = (rng.standard_normal((rows, K))).astype(np.float32)
    t0 = time.perf_counter()
    oracle.slice_product(A, B, kind)
    dt = time.perf_counter() - t0
    rows = int(max(4, min(size, rows * 3.0 / max(dt, 1e-3))))
    A = (rng.standard_normal((rows, K)) * np.ldexp(1.0, rng.integers(-20, 21, (rows, K)))).astype(np.float32)
    for _ in range(max(0, min(args.warmup, 1))):
        oracle.slice_product(A, B, kind)
    times = []
    for _ in range(args.steps if args.steps <= 5 else 5):
        t0 = time.perf_counter()
        oracle.slice_product(A, B, kind)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    tflops = 2.0 * rows * N * K / t / 1e12
    sample = f"{rows} rows of the {size}^3 {args.scheme} product per step, median of {len(times)}"
    line = {
        "metric": "emulated-FP32 TFLOPS", "value": tflops, "unit": "TFLOPS", "impl": "reference",
        "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1)*2^e, e~U{-20..20}",
        "config": {"workload": f"{args.scheme} emulated SGEMM {size}^3 (CPU restatement, row sample)",
                   "M": size, "N": size, "K": size, "scheme": args.scheme},
        "cpu_baseline": {"value": tflops, "unit": "TFLOPS", "cores": oracle.num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": tflops, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def ours(args) -> None:
    import torch

    import emugemm

    # the measured B200 tile table, loaded as the reference's harnesses load theirs (emugemm_init before any GEMM)
    emugemm.lib().emugemm_init(str(ROOT / "emugemm-cdna_b200" / "tiles_b200.csv").encode())

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    import multigpu

    S = args.size
    scheme = SCHEMES[args.scheme]
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)

    def wide(shape):
        x = torch.randn(shape, device="cuda", generator=gen)
        e = torch.randint(-20, 21, shape, device="cuda", generator=gen).float()
        return torch.ldexp(x, e)

    stream = torch.cuda.current_stream()
    h = emugemm.Handle(stream=stream.cuda_stream)
    hints = lambda: emugemm.EmuHints(1.0, 1.0, 0, 0.0, 0)  # noqa: E731  (forced scheme: no scans, no rho)
    wl = args.workload
    # the library's NCCL communicator (its row-sharded and K-split entry points); one rank without torchrun
    if dist is not None:
        multigpu.init_comm(h, max_ctas=args.nccl_ctas)
    elif wl == "ksplit" or (wl == "square" and not args.no_ksplit):
        h.comm_init(1, 0, emugemm.comm_unique_id(), args.nccl_ctas)

    if wl == "square":
        # M = N = K = S per GPU; with N GPUs each rank owns S rows of an (S*N) x S x S product (weak scaling)
        M, N, K = S, S, S
        m_loc, k_loc = M, K
        A = wide((M, K))
        B = wide((K, N)) if rank == 0 else torch.empty((K, N), device="cuda")
        C = torch.empty((M, N), device="cuda")
        total_flop = 2.0 * M * N * K * world
        scaling = "weak"
        desc = f"{args.scheme} emulated SGEMM {S}^3 per GPU" + (", B from rank 0 each step (emugemm_sgemm_rows: copy engines over NVLink)"
                                                                  if world > 1 else "")
        if dist is not None:
            def step():
                # this rank's row block (emugemm_sgemm_rows): B arrives from rank 0 in column panels, each panel's GEMM
                # starting on arrival
                h.sgemm_rows(M * world, N, K, A, K, B if rank == 0 else None, N, C, N, root=0, force=scheme,
                             hints=hints())
        else:
            def step():
                h.sgemm(M, N, K, A, B, C, force=scheme, hints=hints())
    elif wl == "rows":
        # one M = N = K = S product; rows of A split over the ranks, B broadcast from rank 0 (strong scaling)
        M, N, K = S, S, S
        r0, r1 = multigpu.row_range(M, rank, world)
        m_loc, k_loc = r1 - r0, K
        A = torch.randn((m_loc, K), device="cuda", generator=gen)          # the sharded configuration: iid N(0,1)
        B = torch.randn((K, N), device="cuda", generator=gen) if rank == 0 else torch.empty((K, N), device="cuda")
        C = torch.empty((m_loc, N), device="cuda")
        total_flop = 2.0 * M * N * K
        scaling = "strong"
        desc = f"{args.scheme} emulated SGEMM {S}^3, row blocks of A over {world} GPU(s), B broadcast in panels"

        def step():
            if dist is not None:
                h.sgemm_rows(M, N, K, A, K, B if rank == 0 else None, N, C, N, root=0, force=scheme, hints=hints())
            else:
                h.sgemm(m_loc, N, K, A, B, C, force=scheme, hints=hints())
    elif wl == "chunked":
        # FP32_CHUNKED: M = N = S, K = args.k in args.chunks chunks; FP32 FMA chains per chunk, chunk sums in FP64,
        # one rounding to FP32 (the partial + reduce pair that emugemm_sgemm runs for a chunked plan)
        M, N, K = S, S, args.k
        m_loc, k_loc = M, K
        A = torch.rand((M, K), device="cuda", generator=gen) * 2 - 1
        B = torch.rand((K, N), device="cuda", generator=gen) * 2 - 1
        C = torch.empty((M, N), device="cuda")
        P = torch.empty((M, N), dtype=torch.float64, device="cuda")
        total_flop = 2.0 * M * N * K * world
        scaling = "weak"
        desc = f"FP32_CHUNKED {M}x{N}x{K}, c={args.chunks}" + (f", {world} independent replicas" if world > 1 else "")

        def step():
            h.partial_f64(M, N, K, A, K, B, N, P, 2, args.chunks)
            h.reduce_f64(M, N, 1, P, C)
    elif wl == "longk":
        # the long-K comparison (M = N = S, K = args.k, U[-1,1]): the --scheme product forced, one emugemm_sgemm per
        # step; few output tiles, so the tensor-core kernel splits K over the SM pairs
        M, N, K = S, S, args.k
        m_loc, k_loc = M, K
        A = torch.rand((M, K), device="cuda", generator=gen) * 2 - 1
        B = torch.rand((K, N), device="cuda", generator=gen) * 2 - 1
        C = torch.empty((M, N), device="cuda")
        total_flop = 2.0 * M * N * K * world
        scaling = "weak"
        desc = f"{args.scheme} emulated SGEMM {M}x{N}x{K}" + (f", {world} independent replicas" if world > 1 else "")

        def step():
            h.sgemm(M, N, K, A, B, C, force=scheme, hints=hints())
    elif wl == "rho":
        # rho = ||(|A||B|)||_F / ||AB||_F estimated with args.probes Rademacher vectors (signed and |.| products)
        M, N, K = S, S, S
        m_loc, k_loc = M, K
        A = wide((M, K))
        B = wide((K, N))
        C = None
        total_flop = 4.0 * args.probes * K * (M + N) * world
        scaling = "weak"
        desc = f"rho probe, {args.probes} probes, {S}^3" + (f", {world} independent replicas" if world > 1 else "")
        rho_val = []

        def step():
            rho_val.append(h.estimate_rho(M, N, K, A, B, args.probes))
    else:
        # M = N = S, K = args.k split over the ranks; FP64 partials summed by NCCL, one rounding (strong scaling)
        M, N, K = S, S, args.k
        k0, k1 = multigpu.k_range(K, rank, world)
        m_loc, k_loc = M, k1 - k0
        A = torch.randn((M, k_loc), device="cuda", generator=gen)          # the sharded configuration: iid N(0,1)
        B = torch.randn((k_loc, N), device="cuda", generator=gen)
        C = torch.empty((M, N), device="cuda")
        total_flop = 2.0 * M * N * K
        scaling = "strong"
        desc = f"{args.scheme} emulated SGEMM {M}x{N}x{K}, K split over {world} GPU(s), FP64 partials reduced"

        def step():
            # emugemm_sgemm_ksplit: FP64 partials summed by NCCL, C rounded once on rank 0
            h.sgemm_ksplit(M, N, K, A, k_loc, B, N, C, N, root=0, scheme=scheme)

    for _ in range(args.warmup):
        step()
    # One sampler process, on rank 0, for every GPU of the job. It is started (and has delivered its first sample)
    # before the barrier, so that every rank leaves the barrier and starts its clock together: a rank that starts
    # timing while another still waits for its sampler measures that wait inside its first collective.
    with ClockSampler(range(world) if world > 1 else [local], enabled=(rank == 0 and not args.no_clocks)) as clk:
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = emugemm.launch_count()
        # Kernel times come from CUDA events the handle records around each launch. With N GPUs the row-sharded step
        # runs its panel GEMMs on two streams, where those events would stand between the panels: the kernel is then
        # timed in a separate pass of the same per-rank product after the timed region.
        prof_in_loop = dist is None or wl not in ("square", "rows")
        if prof_in_loop:
            h.profile_begin()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk.mark_start()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    prof = h.profile_end() if prof_in_loop else None
    prof_steps = args.steps
    launches = emugemm.launch_count() - launches0
    ms_total = ev0.elapsed_time(ev1)
    rank_ms = None
    if dist is not None:
        # every rank's timed-region length (stragglers show here), and the max over ranks as the job's time
        t = torch.zeros(world, device="cuda", dtype=torch.float64)
        t[rank] = ms_total
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        rank_ms = [round(float(x) / args.steps, 3) for x in t.cpu()]
        ms_total = float(t.max().item())
        dist.barrier()
    ms_step = ms_total / args.steps

    # Correctness of this run's C, outside the timed region: sampled rows of every rank's C against FP64 products of
    # the same rows, the largest normwise error over the ranks against the plan's predicted error.
    check = None
    if not args.no_check and wl in ("square", "rows", "ksplit"):
        if wl == "ksplit":
            check = check_ksplit(torch, dist, h, A, B, C, M, N, K, world, rank, scheme)
        else:
            if dist is not None:
                dist.broadcast(B, src=0)
            check = check_rows(torch, dist, A, B, C, M * (world if wl == "square" else 1), N, K, scheme)
    if prof is None:
        # this rank's product alone (B is complete on every rank after the check's broadcast), its kernels timed
        if dist is not None and (args.no_check or wl not in ("square", "rows", "ksplit")):
            dist.broadcast(B, src=0)
        h.sgemm(m_loc, N, K, A, B, C, force=scheme, hints=hints())
        h.profile_begin()
        prof_steps = 3
        for _ in range(prof_steps):
            h.sgemm(m_loc, N, K, A, B, C, force=scheme, hints=hints())
        prof = h.profile_end()
    # A short timed region runs at the burst clock; the same step held for about two seconds settles under the power
    # cap. Measured separately (not part of `value`) so that the two are never read as each other.
    sustained_rec = None
    if dist is None and wl == "square" and ms_total < 1500.0 and not args.no_sustained:
        n_sus = max(10, int(2000.0 / max(ms_step, 1e-3)))
        with ClockSampler([local], enabled=True) as clk2:
            torch.cuda.synchronize()
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            clk2.mark_start()
            s0.record(stream)
            for _ in range(n_sus):
                step()
            s1.record(stream)
            torch.cuda.synchronize()
            clk2.mark_end()
        sus_ms = s0.elapsed_time(s1) / n_sus
        sustained_rec = {"value": total_flop / (sus_ms * 1e-3) / 1e12, "unit": "TFLOPS", "ms_per_step": sus_ms,
                     "steps": n_sus, "seconds": sus_ms * n_sus / 1e3, "clocks": clk2.summary(),
                     "note": "the same step held for about 2 s after the timed region (power-capped clock); "
                             "value is the short timed region above"}
    ksplit_rec = None
    if wl == "square" and not args.no_ksplit:
        ksplit_rec = ksplit_record(torch, dist, h, args, world, rank, scheme, gen)
    value = total_flop / (ms_step * 1e-3) / 1e12

    # dominant kernel: the tensor-core 3-product GEMM (3 * 2 * m * n * k tensor FLOPs per rank and step), the FP32
    # SIMT GEMM (2 * m * n * k) for the chunked workload, the skinny probe products (4 * P * K * (M + N)) for rho
    if wl == "chunked" or (wl == "longk" and args.scheme == "native"):
        kern_key, kern_name, bound = "fp32_gemm", "k_fp32_gemm / k_fp32_gemm_cp / k_fp32_pipe / k_fp32_pipe_cp (+ k_reduce_f64)", "fp32"
        rank_tensor_flop = 2.0 * m_loc * N * k_loc
    elif wl == "rho":
        kern_key, kern_name, bound = "rho", "rho probe (k_omega, k_skinny_cp x2, k_combine[_sq], k_final)", "fp32"
        rank_tensor_flop = 4.0 * args.probes * K * (M + N)
    else:
        kern_key, kern_name, bound = "tc_gemm", tc_kernel_name(m_loc, N, k_loc, args.scheme), "tensor"
        rank_tensor_flop = 3 * 2.0 * m_loc * N * k_loc
    gemm_ms, gemm_n = prof[kern_key]
    gemm_avg = gemm_ms / max(gemm_n, 1)
    launches_per_step = max(1, gemm_n // max(1, prof_steps))
    tensor_tflops = (rank_tensor_flop / launches_per_step / (gemm_avg * 1e-3) / 1e12) if gemm_n else None
    burst, sustained, hbm, src = peaks()
    clocks = clk.summary()
    peak, peak_name = tensor_peak(ms_total, clocks, burst, sustained)
    peak_source = f"{peak_name} ({src})"
    peak_probe = None
    if bound == "fp32":
        # FP32 SIMT kernels: against the FFMA rate measured on this GPU by emugemm_peak_probe (run after the timed
        # region), else the nominal rate
        nominal, nominal_src = ffma_peak()
        try:
            peak_probe = h.peak_probe(5)
            burst = peak = peak_probe["ffma_tflops"]
            peak_source = f"measured FFMA (emugemm_peak_probe, median of 5; {nominal_src}: {nominal:.1f})"
        except Exception as exc:  # noqa: BLE001 - the nominal figure stands in, and the line says so
            burst = peak = nominal
            peak_source = f"{nominal_src} (peak probe failed: {exc})"
    extra = {}
    if wl == "rho":
        # the probe reads A and B once each; its GB/s against the HBM copy bandwidth, for reference
        rho_ms = prof["rho"][0] / max(1, args.steps)
        extra = {"rho_probe": {"rho": rho_val[-1] if rho_val else None, "ms": rho_ms,
                               "algorithmic_bytes": 4.0 * (M * K + K * N),
                               "gbs": 4.0 * (M * K + K * N) / (rho_ms * 1e-3) / 1e9,
                               "hbm_frac": 4.0 * (M * K + K * N) / (rho_ms * 1e-3) / 1e9 / hbm}}

    # end to end: host inputs (pinned) and the host result, the copies inside every timed step.
    # One GPU: emugemm_sgemm_host (B and C in column panels, overlapped with the panel GEMMs).
    # N GPUs: every rank's rows of A cross PCIe to its own GPU; B crosses PCIe once, as K-row slices spread over the
    # ranks, and reaches every GPU through an NCCL all-gather over NVLink (under the copy of A); each rank then runs
    # emugemm_sgemm on its rows and its C rows go back over PCIe. The job's time is the slowest rank's.
    e2e = None
    if not args.no_e2e and wl == "square" and (dist is None or K % world == 0):
        hA = A.cpu().pin_memory()
        hC = torch.empty((M, N), dtype=torch.float32).pin_memory()
        if dist is None:
            hB = B.cpu().pin_memory()
            h2d = hA.numel() * 4 + hB.numel() * 4

            def e2e_step():
                h.sgemm_host(M, N, K, hA, hB, hC, force=scheme, hints=hints())
            path = "emugemm_sgemm_host: pinned host A and B in, C out, inside every step"
        else:
            ks = K // world
            hBs = B[rank * ks:(rank + 1) * ks].cpu().pin_memory()      # B is complete on every rank after the check
            dA, dBs = torch.empty_like(A), torch.empty((ks, N), device="cuda")
            dB, dC = torch.empty((K, N), device="cuda"), torch.empty((M, N), device="cuda")
            h2d = (hA.numel() + hBs.numel()) * 4 * world

            def e2e_step():
                dBs.copy_(hBs, non_blocking=True)
                w = dist.all_gather_into_tensor(dB, dBs, async_op=True)
                dA.copy_(hA, non_blocking=True)
                w.wait()
                h.sgemm(M, N, K, dA, dB, dC, force=scheme, hints=hints())
                hC.copy_(dC, non_blocking=True)
            path = ("per rank: pinned host rows of A in, B in once as K-row slices over the ranks + NCCL all-gather, "
                    "emugemm_sgemm on the rows, C rows out; inside every step")

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        n_e2e = max(3, min(30, args.steps // 4))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / n_e2e
        if dist is not None:
            t = torch.tensor([e_ms], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": 2.0 * M * N * K * world / (e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(hC.numel() * 4) * world, "ms_per_step": e_ms,
               "path": path}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and wl == "square":
        cpu = cpu_fp64_baseline(S)

    # cuBLAS SGEMM on the same GPU and shape (strict FP32: no TF32), a comparison figure only
    cublas = None
    if world == 1 and not args.no_cublas and wl == "square":
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.set_float32_matmul_precision("highest")
        for _ in range(3):
            torch.matmul(A, B, out=C)
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_cb = 10
        c0.record(stream)
        for _ in range(n_cb):
            torch.matmul(A, B, out=C)
        c1.record(stream)
        torch.cuda.synchronize()
        cb_ms = c0.elapsed_time(c1) / n_cb
        cublas = {"sgemm_tflops": 2.0 * M * N * K / (cb_ms * 1e-3) / 1e12, "ms": cb_ms,
                  "note": "torch.matmul fp32, allow_tf32=False, same inputs"}

    if rank == 0:
        line = {
            "metric": ("rho-probe TFLOPS" if wl == "rho" else "emulated-FP32 TFLOPS"), "value": value,
            "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "f32",
            "data": ("synthetic U[-1,1] (torch generator)" if wl in ("chunked", "longk")
                     else "synthetic N(0,1)*2^e, e~U{-20..20} (torch generator)"),
            "config": {"workload": desc, "M": M * (world if wl == "square" else 1), "N": N, "K": K,
                       "scheme": ("fp32_chunked" if wl == "chunked" else "rho_probe" if wl == "rho" else args.scheme),
                       "force_scheme": (2 if wl == "chunked" else None if wl == "rho" else scheme),
                       "chunks": args.chunks if wl == "chunked" else None,
                       "hints": "absmax given, rho=0 (no scans)", "l2": "inputs larger than L2",
                       "parallelism": (f"{wl} x{world}" if world > 1 else "single GPU")},
            "roofline": {"bound": bound, "kernel": kern_name, "achieved": tensor_tflops,
                         "peak": peak, "peak_source": peak_source, "unit": "TFLOP/s",
                         "frac": (tensor_tflops / peak) if tensor_tflops else None,
                         "frac_of_burst": (tensor_tflops / burst) if tensor_tflops else None,
                         "flops_per_launch": rank_tensor_flop / launches_per_step, "kernel_ms": gemm_avg,
                         "traffic": TRAFFIC.get((args.scheme, S)) if wl == "square" else None,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch at this size"
                         if (wl == "square" and (args.scheme, S) in TRAFFIC) else None},
            "kernel_ms": {k: (v[0] / v[1] if v[1] else None) for k, v in prof.items()},
            **({"peak_probe": peak_probe} if peak_probe else {}),
            "cpu_baseline": cpu,
            "cublas_sgemm": cublas,
            "e2e": e2e,
            "clocks": clocks,
            "gpu_launches": launches,
        }
        if check is not None:
            line["check"] = check
        if ksplit_rec is not None:
            line["ksplit"] = ksplit_rec
        if sustained_rec is not None:
            line["sustained"] = sustained_rec
        if rank_ms is not None:
            line["ms_per_step_by_rank"] = rank_ms
        line.update(extra)
        print(json.dumps(line), flush=True)
    h.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
