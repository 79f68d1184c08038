"""Test infrastructure: Python access to the CPU oracle (liboracle.so, from oracle.c) and to the
reference's own planner (_ref/libemuref.so, compiled from emugemm-cdna's src/emugemm.cpp by the Makefile
here). Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline leg use this module, to check
results and to time the CPU path; the library never does.

Parity status: the split rule, absmax, exponent rule, FP32 chunk chains and the Hutchinson estimate are
restated from the reference source; the planner is pinned against the reference planner itself (golden
fixtures in tests/golden/ generated from _ref/libemuref.so, and a live comparison when it is built).
"""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libemuref.so"

_c = ctypes
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")

_olib = None


def olib() -> ctypes.CDLL:
    global _olib
    if _olib is None:
        l = ctypes.CDLL(str(ORACLE_SO))
        l.orc_split_bf16.argtypes = [_f32p, _c.c_long, _u16p, _u16p]
        l.orc_split_f16.argtypes = [_f32p, _c.c_long, _u16p, _u16p]
        l.orc_split_f16_scaled.argtypes = [_f32p, _c.c_long, _c.c_int, _u16p, _u16p]
        l.orc_exponent_for_max.argtypes = [_c.c_float]
        l.orc_exponent_for_max.restype = _c.c_int
        l.orc_row_exponents.argtypes = [_f32p, _c.c_int, _c.c_long, _c.c_long, _i32p]
        l.orc_col_exponents.argtypes = [_f32p, _c.c_long, _c.c_int, _c.c_long, _i32p]
        l.orc_absmax.argtypes = [_f32p, _c.c_long]
        l.orc_absmax.restype = _c.c_float
        l.orc_gemm_f64.argtypes = [_f64p, _f64p, _f64p, _c.c_int, _c.c_int, _c.c_long, _c.c_long, _c.c_long,
                                   _c.c_long]
        l.orc_gemm_f32_in_f64.argtypes = [_f32p, _f32p, _f64p, _c.c_int, _c.c_int, _c.c_long, _c.c_long,
                                          _c.c_long, _c.c_long]
        l.orc_fp32_chunked.argtypes = [_f32p, _f32p, _c.c_void_p, _c.c_void_p, _c.c_int, _c.c_int, _c.c_long,
                                       _c.c_long, _c.c_long, _c.c_long, _c.c_int, _c.c_int]
        l.orc_slice_product.argtypes = [_f32p, _f32p, _f64p, _c.c_int, _c.c_int, _c.c_long, _c.c_long,
                                        _c.c_long, _c.c_int]
        l.orc_rho_hutchinson.argtypes = [_f32p, _f32p, _c.c_int, _c.c_int, _c.c_long, _c.c_long, _c.c_long,
                                         _c.c_int, _f64p]
        l.orc_rho_hutchinson.restype = _c.c_double
        l.orc_rho_true.argtypes = [_f32p, _f32p, _c.c_int, _c.c_int, _c.c_long, _c.c_long, _c.c_long]
        l.orc_rho_true.restype = _c.c_double
        l.orc_rel_err.argtypes = [_f32p, _f64p, _c.c_long]
        l.orc_rel_err.restype = _c.c_double
        l.orc_num_threads.restype = _c.c_int
        _olib = l
    return _olib


def _c32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def split_bf16(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = _c32(x).ravel()
    hi = np.empty(x.size, np.uint16)
    lo = np.empty(x.size, np.uint16)
    olib().orc_split_bf16(x, x.size, hi, lo)
    return hi, lo


def split_f16(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = _c32(x).ravel()
    hi = np.empty(x.size, np.uint16)
    lo = np.empty(x.size, np.uint16)
    olib().orc_split_f16(x, x.size, hi, lo)
    return hi, lo


def split_f16_scaled(x: np.ndarray, e: int) -> tuple[np.ndarray, np.ndarray]:
    x = _c32(x).ravel()
    hi = np.empty(x.size, np.uint16)
    lo = np.empty(x.size, np.uint16)
    olib().orc_split_f16_scaled(x, x.size, int(e), hi, lo)
    return hi, lo


def exponent_for_max(m: float) -> int:
    return int(olib().orc_exponent_for_max(float(m)))


def row_exponents(A: np.ndarray) -> np.ndarray:
    A = _c32(A)
    e = np.empty(A.shape[0], np.int32)
    olib().orc_row_exponents(A, A.shape[0], A.shape[1], A.shape[1], e)
    return e


def col_exponents(B: np.ndarray) -> np.ndarray:
    B = _c32(B)
    e = np.empty(B.shape[1], np.int32)
    olib().orc_col_exponents(B, B.shape[0], B.shape[1], B.shape[1], e)
    return e


def absmax(x: np.ndarray) -> float:
    x = _c32(x).ravel()
    return float(olib().orc_absmax(x, x.size))


def gemm_f64(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """FP64 ground truth of A*B from FP32 inputs."""
    A, B = _c32(A), _c32(B)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float64)
    olib().orc_gemm_f32_in_f64(A, B, C, M, N, K, K, N, N)
    return C


def fp32_chunked(A: np.ndarray, B: np.ndarray, chunks: int, cpg: int = 0, f64: bool = False) -> np.ndarray:
    """Bit-level replica of the FP32_CHUNKED / NATIVE_FP32 kernels (cpg = chunks per FP64 group)."""
    A, B = _c32(A), _c32(B)
    M, K = A.shape
    N = B.shape[1]
    if f64:
        out = np.empty((M, N), np.float64)
        olib().orc_fp32_chunked(A, B, None, out.ctypes.data, M, N, K, K, N, N, chunks, cpg)
    else:
        out = np.empty((M, N), np.float32)
        olib().orc_fp32_chunked(A, B, out.ctypes.data, None, M, N, K, K, N, N, chunks, cpg)
    return out


def group_size(K: int, chunks: int, G: int) -> int:
    """chunks per group for G groups (the library's grouping rule)."""
    c = max(1, chunks)
    kc = max(1, -(-K // c))
    ce = max(1, -(-K // kc))
    return -(-ce // max(1, G))


def slice_product(A: np.ndarray, B: np.ndarray, kind: int) -> np.ndarray:
    """Exact FP64 sum of the three slice products (kind 0 bf16x3, 1 scaled fp16x3, 2 unscaled fp16x3)."""
    A, B = _c32(A), _c32(B)
    M, K = A.shape
    N = B.shape[1]
    R = np.empty((M, N), np.float64)
    olib().orc_slice_product(A, B, R, M, N, K, K, N, kind)
    return R


def rho_hutchinson(A: np.ndarray, B: np.ndarray, P: int = 64) -> tuple[float, np.ndarray]:
    A, B = _c32(A), _c32(B)
    M, K = A.shape
    N = B.shape[1]
    out2 = np.zeros(2, np.float64)
    r = olib().orc_rho_hutchinson(A, B, M, N, K, K, N, P, out2)
    return float(r), out2


def rho_true(A: np.ndarray, B: np.ndarray) -> float:
    A, B = _c32(A), _c32(B)
    M, K = A.shape
    N = B.shape[1]
    return float(olib().orc_rho_true(A, B, M, N, K, K, N))


def rel_err(C: np.ndarray, R: np.ndarray) -> float:
    """Normwise ||C - R||_F / ||R||_F (bench/emugemm_test.cpp:96-99)."""
    C = _c32(C).ravel()
    R = np.ascontiguousarray(R, dtype=np.float64).ravel()
    return float(olib().orc_rel_err(C, R, C.size))


def num_threads() -> int:
    return int(olib().orc_num_threads())


def set_num_threads(n: int) -> None:
    """OpenMP threads of the oracle's later parallel loops, for the calling thread."""
    f = olib().orc_set_num_threads
    f.argtypes = [_c.c_int]
    f.restype = None
    f(int(n))


# ---- the reference planner (compiled from its own source) ---------------------------------------------
class RefRequest(ctypes.Structure):
    _fields_ = [("max_rel_err", ctypes.c_double), ("force_scheme", ctypes.c_int)]


class RefHints(ctypes.Structure):
    _fields_ = [("a_absmax", ctypes.c_float), ("b_absmax", ctypes.c_float), ("a_is_reused", ctypes.c_int),
                ("rho", ctypes.c_float), ("rho_probes", ctypes.c_int)]


class RefPlan(ctypes.Structure):
    _fields_ = [("chosen", ctypes.c_int), ("chunks", ctypes.c_int), ("predicted_err", ctypes.c_double),
                ("predicted_speedup", ctypes.c_double), ("reason", ctypes.c_char_p)]


_rlib = None


def ref_available() -> bool:
    return REF_SO.exists()


def rlib() -> ctypes.CDLL:
    global _rlib
    if _rlib is None:
        l = ctypes.CDLL(str(REF_SO))
        l.emugemm_plan.restype = RefPlan
        l.emugemm_plan.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_long, ctypes.POINTER(RefRequest),
                                   ctypes.POINTER(RefHints)]
        l.emugemm_model_err.restype = ctypes.c_double
        l.emugemm_model_err.argtypes = [ctypes.c_int, ctypes.c_long, ctypes.c_int]
        l.emugemm_model_err_rho.restype = ctypes.c_double
        l.emugemm_model_err_rho.argtypes = [ctypes.c_int, ctypes.c_long, ctypes.c_int, ctypes.c_double]
        l.emugemm_model_speed.restype = ctypes.c_double
        l.emugemm_model_speed.argtypes = [ctypes.c_int, ctypes.c_int]
        _rlib = l
    return _rlib


def ref_plan(M, N, K, tgt, force, a_absmax, b_absmax, rho, hints=True) -> dict:
    req = RefRequest(tgt, force)
    hn = RefHints(a_absmax, b_absmax, 0, rho, 0)
    p = rlib().emugemm_plan(M, N, K, ctypes.byref(req), ctypes.byref(hn) if hints else None)
    return {"chosen": p.chosen, "chunks": p.chunks, "predicted_err": p.predicted_err,
            "predicted_speedup": p.predicted_speedup, "reason": p.reason.decode()}
