"""ctypes binding of libemugemm.so (the C ABI declared in include/emugemm.h).

The library is the product; this module only loads it and mirrors its structs so that Python callers
(tests, bench.py, the multi-GPU driver) can call the same entry points a C caller would. Device buffers
are passed as raw pointers; torch tensors are accepted for convenience and must already live on the
device the handle was created on. Nothing here computes: if libemugemm.so is missing, loading fails.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import re

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libemugemm.so"
HEADER = HERE.parent / "include" / "emugemm.h"

# emu_scheme_t (src/emugemm.h:37-44 of emugemm-cdna)
AUTO, NATIVE_FP32, FP32_CHUNKED, BF16X3, FP16X3, BF16X6 = range(6)
SCHEME_NAMES = ["AUTO", "NATIVE_FP32", "FP32_CHUNKED", "BF16X3", "FP16X3", "BF16X6"]

# emugemm_attr_t: per-handle kernel choices
ATTR_TC_KERNEL, ATTR_TC_SPLITK, ATTR_FP32_TILE, ATTR_ROWS_PANELS, ATTR_COMM_SMS, ATTR_BCAST_NCCL = 0, 1, 2, 3, 4, 5
TC_KERNEL_CODES = {"auto": 0, "single": 1, "pair": 2, "fused": 3, "fusea": 4}

STATUS = {
    0: "SUCCESS", 1: "INVALID_HANDLE", 2: "NOT_IMPLEMENTED", 3: "INVALID_POINTER", 4: "INVALID_SIZE",
    5: "MEMORY_ERROR", 6: "INTERNAL_ERROR", 11: "INVALID_VALUE", 100: "ARCH_MISMATCH", 101: "TIMEOUT",
}


class EmuRequest(ctypes.Structure):
    _fields_ = [("max_rel_err", ctypes.c_double), ("force_scheme", ctypes.c_int)]


class EmuHints(ctypes.Structure):
    _fields_ = [
        ("a_absmax", ctypes.c_float),
        ("b_absmax", ctypes.c_float),
        ("a_is_reused", ctypes.c_int),
        ("rho", ctypes.c_float),
        ("rho_probes", ctypes.c_int),
    ]


class EmuPlan(ctypes.Structure):
    _fields_ = [
        ("chosen", ctypes.c_int),
        ("chunks", ctypes.c_int),
        ("predicted_err", ctypes.c_double),
        ("predicted_speedup", ctypes.c_double),
        ("reason", ctypes.c_char_p),
    ]

    def as_dict(self) -> dict:
        return {
            "chosen": SCHEME_NAMES[self.chosen] if 0 <= self.chosen < 6 else self.chosen,
            "chunks": self.chunks,
            "predicted_err": self.predicted_err,
            "predicted_speedup": self.predicted_speedup,
            "reason": self.reason.decode() if self.reason else None,
        }


class EmuGemmError(RuntimeError):
    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {STATUS.get(code, code)} ({code})")
        self.code = code


c_int, c_long, c_double, c_float, c_size_t, c_void_p = (
    ctypes.c_int, ctypes.c_long, ctypes.c_double, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p)
P = ctypes.POINTER

_SIGS = {
    "emugemm_create_handle": (c_int, [P(c_void_p)]),
    "emugemm_destroy_handle": (c_int, [c_void_p]),
    "emugemm_set_stream": (c_int, [c_void_p, c_void_p]),
    "emugemm_set_workspace_limit": (c_int, [c_void_p, c_size_t]),
    "emugemm_sync": (c_int, [c_void_p]),
    "emugemm_init": (c_int, [ctypes.c_char_p]),
    "emugemm_init_for_arch": (c_int, [ctypes.c_char_p, ctypes.c_char_p]),
    "emugemm_tune_rows": (c_int, []),
    "emugemm_tune_lookup": (c_int, [c_int, c_int, c_long, c_int]),
    "emugemm_shutdown": (None, []),
    "emugemm_plan": (EmuPlan, [c_int, c_int, c_long, P(EmuRequest), P(EmuHints)]),
    "emugemm_sgemm": (c_int, [c_void_p, c_int, c_int, c_long, c_void_p, c_void_p, c_void_p,
                              P(EmuRequest), P(EmuHints), P(EmuPlan)]),
    "emugemm_sgemm_ex": (c_int, [c_void_p, c_int, c_int, c_long, c_void_p, c_long, c_void_p, c_long,
                                 c_void_p, c_long, P(EmuRequest), P(EmuHints), P(EmuPlan)]),
    "emugemm_sgemm_host": (c_int, [c_void_p, c_int, c_int, c_long, c_void_p, c_void_p, c_void_p,
                                   P(EmuRequest), P(EmuHints), P(EmuPlan)]),
    "emugemm_sgemm_partial_f64": (c_int, [c_void_p, c_int, c_int, c_long, c_void_p, c_long, c_void_p,
                                          c_long, c_void_p, c_int, c_int]),
    "emugemm_reduce_f64": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "emugemm_model_err": (c_double, [c_int, c_long, c_int]),
    "emugemm_model_err_rho": (c_double, [c_int, c_long, c_int, c_double]),
    "emugemm_model_speed": (c_double, [c_int, c_int]),
    "emugemm_estimate_rho": (c_double, [c_void_p, c_int, c_int, c_long, c_void_p, c_void_p, c_int]),
    "emugemm_set_model": (c_int, [ctypes.c_char_p]),
    "emugemm_get_model": (ctypes.c_char_p, []),
    "emugemm_peak_probe": (c_int, [c_void_p, c_int, P(ctypes.c_double), c_int]),
    "emugemm_absmax": (c_int, [c_void_p, c_void_p, c_size_t, P(c_float)]),
    "emugemm_split_bf16": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "emugemm_split_f16": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "emugemm_fp32_groups": (c_int, [c_int, c_int, c_long, c_int, c_int]),
    "emugemm_fp32_groups_tile": (c_int, [c_int, c_int, c_long, c_int, c_int, c_int]),
    "emugemm_set_attr": (c_int, [c_void_p, c_int, c_long]),
    "emugemm_get_attr": (c_int, [c_void_p, c_int, P(c_long)]),
    "emugemm_test_stall_next_launches": (None, [c_int]),
    "emugemm_sgemm_bf16x3_noalloc": (c_int, [c_int, c_int, c_long, c_void_p, c_void_p, c_void_p, c_void_p]),
    "emugemm_noalloc_sync": (c_int, [c_void_p]),
    "emugemm_comm_unique_id": (c_int, [c_void_p]),
    "emugemm_comm_init": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int]),
    "emugemm_comm_destroy": (c_int, [c_void_p]),
    "emugemm_comm_rows": (c_int, [c_void_p, c_int, P(c_int), P(c_int)]),
    "emugemm_comm_krange": (c_int, [c_void_p, c_long, P(c_long), P(c_long)]),
    "emugemm_sgemm_rows": (c_int, [c_void_p, c_int, c_int, c_long, c_void_p, c_long, c_void_p, c_long, c_void_p,
                                   c_long, c_int, P(EmuRequest), P(EmuHints), P(EmuPlan)]),
    "emugemm_sgemm_ksplit": (c_int, [c_void_p, c_int, c_int, c_long, c_void_p, c_long, c_void_p, c_long, c_void_p,
                                     c_long, c_int, c_int, c_int]),
    "emugemm_rows_panels": (c_int, [c_int, c_int, c_int, c_long, c_int, c_int, c_void_p, c_void_p, c_int]),
    "emugemm_kernel_launch_count": (ctypes.c_ulonglong, []),
    "emugemm_profile_begin": (c_int, [c_void_p]),
    "emugemm_profile_end": (c_int, [c_void_p, P(c_double), P(c_int), c_int]),
    "emugemm_status_string": (ctypes.c_char_p, [c_int]),
}

_lib = None


def header_functions() -> list[str]:
    """Names of every function declared in include/emugemm.h."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(emugemm_[a-z0-9_]+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    """Load libemugemm.so (raises OSError if it has not been built)."""
    global _lib
    if _lib is None:
        path = os.environ.get("EMUGEMM_LIB", str(LIB_PATH))
        l = ctypes.CDLL(path)
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name, None)
            if f is None:
                continue
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def check(fn: str, code: int) -> None:
    if code != 0:
        raise EmuGemmError(fn, code)


def plan(M: int, N: int, K: int, max_rel_err: float = 1e-5, force: int = AUTO,
         a_absmax: float = -1.0, b_absmax: float = -1.0, rho: float = -1.0, probes: int = 0,
         hints: bool = True) -> EmuPlan:
    req = EmuRequest(max_rel_err, force)
    hn = EmuHints(a_absmax, b_absmax, 0, rho, probes)
    return lib().emugemm_plan(M, N, K, ctypes.byref(req), ctypes.byref(hn) if hints else None)


def set_model(name: str) -> None:
    check("emugemm_set_model", lib().emugemm_set_model(name.encode()))


def get_model() -> str:
    return lib().emugemm_get_model().decode()


class Handle:
    """An emugemm handle on the current CUDA device (context manager)."""

    def __init__(self, stream: int | None = None):
        h = c_void_p()
        check("emugemm_create_handle", lib().emugemm_create_handle(ctypes.byref(h)))
        self.h = h
        if stream is not None:
            self.set_stream(stream)
        # kernel choices as created (from the environment), restored by reset_kernels()
        self._kernel_defaults = tuple(self.get_attr(a) for a in (ATTR_TC_KERNEL, ATTR_TC_SPLITK, ATTR_FP32_TILE))

    def set_stream(self, stream) -> None:
        s = stream if isinstance(stream, int) else int(getattr(stream, "cuda_stream", 0))
        check("emugemm_set_stream", lib().emugemm_set_stream(self.h, c_void_p(s)))

    def set_workspace_limit(self, nbytes: int) -> None:
        check("emugemm_set_workspace_limit", lib().emugemm_set_workspace_limit(self.h, nbytes))

    def close(self) -> None:
        if self.h:
            lib().emugemm_destroy_handle(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self) -> None:
        check("emugemm_sync", lib().emugemm_sync(self.h))

    def sync_status(self) -> int:
        """emugemm_sync's status code (0 = SUCCESS, 101 = TIMEOUT, ...), without raising."""
        return int(lib().emugemm_sync(self.h))

    def set_attr(self, attr: int, value: int) -> None:
        check("emugemm_set_attr", lib().emugemm_set_attr(self.h, attr, value))

    def get_attr(self, attr: int) -> int:
        v = c_long()
        check("emugemm_get_attr", lib().emugemm_get_attr(self.h, attr, ctypes.byref(v)))
        return v.value

    def reset_kernels(self) -> None:
        """Restore the kernel choices the handle was created with."""
        for a, v in zip((ATTR_TC_KERNEL, ATTR_TC_SPLITK, ATTR_FP32_TILE), self._kernel_defaults):
            self.set_attr(a, v)

    def set_kernels(self, tc_kernel: str | int | None = None, splitk: int | None = None,
                    fp32_tile: int | None = None) -> None:
        """Per-handle kernel choices (emugemm_set_attr); a name of TC_KERNEL_CODES or a code; 0 = automatic."""
        if tc_kernel is not None:
            self.set_attr(ATTR_TC_KERNEL, TC_KERNEL_CODES[tc_kernel] if isinstance(tc_kernel, str) else tc_kernel)
        if splitk is not None:
            self.set_attr(ATTR_TC_SPLITK, splitk)
        if fp32_tile is not None:
            self.set_attr(ATTR_FP32_TILE, fp32_tile)

    def sgemm(self, M: int, N: int, K: int, A, B, C, max_rel_err: float = 1e-5, force: int = AUTO,
              hints: EmuHints | None = None, use_hints: bool = True) -> tuple[EmuPlan, EmuHints | None]:
        """C = A*B through emugemm_sgemm. hints=None -> measure absmax, do not estimate rho
        (the reference's invariant-suite convention, bench/emugemm_test.cpp:101); use_hints=False passes
        NULL (measure everything)."""
        req = EmuRequest(max_rel_err, force)
        if use_hints and hints is None:
            hints = EmuHints(-1.0, -1.0, 0, 0.0, 0)
        p = EmuPlan()
        code = lib().emugemm_sgemm(self.h, M, N, K, _ptr(A), _ptr(B), _ptr(C), ctypes.byref(req),
                                   ctypes.byref(hints) if use_hints else None, ctypes.byref(p))
        check("emugemm_sgemm", code)
        return p, hints

    def sgemm_host(self, M, N, K, A, B, C, max_rel_err=1e-5, force=AUTO, hints=None, use_hints=True):
        """C = A*B through emugemm_sgemm_host: A, B, C are HOST buffers (pinned tensors or addresses)."""
        req = EmuRequest(max_rel_err, force)
        if use_hints and hints is None:
            hints = EmuHints(-1.0, -1.0, 0, 0.0, 0)
        p = EmuPlan()
        check("emugemm_sgemm_host", lib().emugemm_sgemm_host(self.h, M, N, K, _ptr(A), _ptr(B), _ptr(C),
                                                             ctypes.byref(req),
                                                             ctypes.byref(hints) if use_hints else None,
                                                             ctypes.byref(p)))
        return p, hints

    def sgemm_ex(self, M, N, K, A, lda, B, ldb, C, ldc, max_rel_err=1e-5, force=AUTO, hints=None):
        req = EmuRequest(max_rel_err, force)
        if hints is None:
            hints = EmuHints(-1.0, -1.0, 0, 0.0, 0)
        p = EmuPlan()
        check("emugemm_sgemm_ex", lib().emugemm_sgemm_ex(self.h, M, N, K, _ptr(A), lda, _ptr(B), ldb, _ptr(C),
                                                         ldc, ctypes.byref(req), ctypes.byref(hints),
                                                         ctypes.byref(p)))
        return p, hints

    def partial_f64(self, M, N, K, A, lda, B, ldb, P64, scheme, chunks=1):
        check("emugemm_sgemm_partial_f64",
              lib().emugemm_sgemm_partial_f64(self.h, M, N, K, _ptr(A), lda, _ptr(B), ldb, _ptr(P64),
                                              scheme, chunks))

    def reduce_f64(self, M, N, G, P64, C):
        check("emugemm_reduce_f64", lib().emugemm_reduce_f64(self.h, M, N, G, _ptr(P64), _ptr(C)))

    def estimate_rho(self, M, N, K, A, B, probes=64) -> float:
        return lib().emugemm_estimate_rho(self.h, M, N, K, _ptr(A), _ptr(B), probes)

    # ---- several GPUs (one process and one handle per GPU; every call is collective) ----
    def comm_init(self, nranks: int, rank: int, uid: bytes, max_ctas: int = 0) -> None:
        """Join the library's NCCL communicator; uid = comm_unique_id() of one rank, shared by the caller."""
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        check("emugemm_comm_init", lib().emugemm_comm_init(self.h, nranks, rank, buf, max_ctas))

    def comm_destroy(self) -> None:
        check("emugemm_comm_destroy", lib().emugemm_comm_destroy(self.h))

    def comm_rows(self, M: int) -> tuple[int, int]:
        """This rank's rows [r0, r1) of an M-row emugemm_sgemm_rows product."""
        r0, n = c_int(), c_int()
        check("emugemm_comm_rows", lib().emugemm_comm_rows(self.h, M, ctypes.byref(r0), ctypes.byref(n)))
        return r0.value, r0.value + n.value

    def comm_krange(self, K: int) -> tuple[int, int]:
        """This rank's K range [k0, k1) of an emugemm_sgemm_ksplit product."""
        k0, n = c_long(), c_long()
        check("emugemm_comm_krange", lib().emugemm_comm_krange(self.h, K, ctypes.byref(k0), ctypes.byref(n)))
        return k0.value, k0.value + n.value

    def sgemm_rows(self, M, N, K, A_local, lda, B, ldb, C_local, ldc, root=0, max_rel_err=1e-5, force=AUTO,
                   hints=None):
        """emugemm_sgemm_rows: rows of A and C on the ranks, B (on `root`; None elsewhere) broadcast in panels."""
        req = EmuRequest(max_rel_err, force)
        if hints is None:
            hints = EmuHints(-1.0, -1.0, 0, 0.0, 0)
        p = EmuPlan()
        check("emugemm_sgemm_rows", lib().emugemm_sgemm_rows(self.h, M, N, K, _ptr(A_local), lda, _ptr(B), ldb,
                                                             _ptr(C_local), ldc, root, ctypes.byref(req),
                                                             ctypes.byref(hints), ctypes.byref(p)))
        return p, hints

    def sgemm_ksplit(self, M, N, K, A_local, lda, B_local, ldb, C, ldc, root=0, scheme=BF16X3, chunks=1) -> None:
        """emugemm_sgemm_ksplit: K split over the ranks, FP64 partials summed by NCCL, C on root (all ranks: -1)."""
        check("emugemm_sgemm_ksplit", lib().emugemm_sgemm_ksplit(self.h, M, N, K, _ptr(A_local), lda, _ptr(B_local),
                                                                 ldb, _ptr(C), ldc, root, scheme, chunks))

    PEAK_NAMES = ("tc_bf16_tflops", "tc_fp16_tflops", "tc_tf32_tflops", "ffma_tflops", "dfma_tflops", "copy_gbs")

    def peak_probe(self, reps: int = 7) -> dict:
        """Measured peak rates of this GPU (emugemm_peak_probe): tcgen05 bf16 / fp16 / tf32 and FFMA / DFMA in
        TFLOP/s, device copy in GB/s; medians of `reps` interleaved runs."""
        out = (ctypes.c_double * len(self.PEAK_NAMES))()
        check("emugemm_peak_probe", lib().emugemm_peak_probe(self.h, reps, out, len(self.PEAK_NAMES)))
        return dict(zip(self.PEAK_NAMES, list(out)))

    def absmax(self, X, n: int) -> float:
        out = c_float()
        check("emugemm_absmax", lib().emugemm_absmax(self.h, _ptr(X), n, ctypes.byref(out)))
        return out.value

    def split_bf16(self, X, n, hi, lo) -> None:
        check("emugemm_split_bf16", lib().emugemm_split_bf16(self.h, _ptr(X), n, _ptr(hi), _ptr(lo)))

    def split_f16(self, X, n, hi, lo) -> None:
        check("emugemm_split_f16", lib().emugemm_split_f16(self.h, _ptr(X), n, _ptr(hi), _ptr(lo)))

    PROF_KINDS = ["tc_gemm", "fp32_gemm", "split", "scan", "rho", "reduce"]

    def profile_begin(self) -> None:
        check("emugemm_profile_begin", lib().emugemm_profile_begin(self.h))

    def profile_end(self) -> dict:
        n = len(self.PROF_KINDS)
        ms = (c_double * n)()
        cnt = (c_int * n)()
        check("emugemm_profile_end", lib().emugemm_profile_end(self.h, ms, cnt, n))
        return {k: (ms[i], cnt[i]) for i, k in enumerate(self.PROF_KINDS)}


def launch_count() -> int:
    return int(lib().emugemm_kernel_launch_count())


def fp32_groups(M: int, N: int, K: int, chunks: int, num_sms: int, tile: int | None = None) -> int:
    """FP64 partial groups of the FP32_CHUNKED kernel; tile = the handle's EMUGEMM_ATTR_FP32_TILE (None: the
    environment default)."""
    if tile is None:
        return int(lib().emugemm_fp32_groups(M, N, K, chunks, num_sms))
    return int(lib().emugemm_fp32_groups_tile(M, N, K, chunks, num_sms, tile))


def comm_unique_id() -> bytes:
    """128 bytes identifying a new communicator (make on one rank, pass to every rank's Handle.comm_init)."""
    buf = ctypes.create_string_buffer(128)
    check("emugemm_comm_unique_id", lib().emugemm_comm_unique_id(buf))
    return buf.raw


def rows_panels(M: int, nranks: int, N: int, K: int, num_sms: int = 148, forced: int = 0) -> list[tuple[int, int]]:
    """The column panels [n0, n1) emugemm_sgemm_rows broadcasts B in (emugemm_rows_panels)."""
    n0, n1 = (c_int * 16)(), (c_int * 16)()
    n = lib().emugemm_rows_panels(M, nranks, N, K, num_sms, forced, n0, n1, 16)
    return [(n0[i], n1[i]) for i in range(n)]


def test_stall_next_launches(n: int) -> None:
    """Testing hook: the next n single-CTA tensor-core launches give up a 1 ms wait on a barrier nothing arrives
    on (emugemm_test_stall_next_launches)."""
    lib().emugemm_test_stall_next_launches(n)
