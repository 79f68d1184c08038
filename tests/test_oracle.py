"""Pins of the CPU oracle before it is trusted to check the GPU kernels.

- split rule: known-answer bit patterns, and the identities hi + lo == x for every x whose residual fits
- bf16x3 representation floor: with exact FP64 slice products the normwise error of iid N(0,1) data is
  the reference's measured floor 4.4355e-6 (docs/RESULTS_ROUND9.md:33-49) to within a few percent
- fp16x3 (unscaled, the reference's rule) floor 3.6e-7 on in-range data (src/emugemm.cpp:19)
- FP32 chunk chains: exact on integer data, and the K/c law of docs/RESULTS_ROUND9.md:67-71
- Hutchinson estimate: equals the exact Frobenius ratio in expectation, and the FP64 restatement agrees
  with a direct numpy evaluation of the same formula and Rademacher hash
"""
from __future__ import annotations

import numpy as np
import pytest

import datagen
import oracle


def test_split_bf16_known_answers():
    x = np.array([1.0, 1.00390625, 1.0 + 2 ** -9, 1.0 + 3 * 2 ** -9, -3.14159265, 0.0, -0.0, 2 ** -130,
                  65504.0, 1e30], np.float32)
    hi, lo = oracle.split_bf16(x)
    assert hi[0] == 0x3F80 and lo[0] == 0
    assert hi[1] == 0x3F80 and lo[1] == 0x3B80          # 1+2^-8: tie to even keeps 1.0, lo = 2^-8
    assert hi[2] == 0x3F80 and lo[2] == 0x3B00          # 1+2^-9 rounds down to 1.0
    assert hi[3] == 0x3F81                               # 1+3*2^-9 rounds up
    assert hi[4] == 0xC049                               # -3.140625
    assert hi[5] == 0 and hi[6] == 0x8000


def test_split_bf16_reconstruction():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(100000) * 2.0 ** rng.integers(-20, 21, 100000)).astype(np.float32)
    hi, lo = oracle.split_bf16(x)
    h = (hi.astype(np.uint32) << 16).view(np.float32)
    l = (lo.astype(np.uint32) << 16).view(np.float32)
    # the residual x - hi is exact in FP32 and lo is its RNE bf16 rounding: |x - hi - lo| <= 2^-9 |x - hi|
    r = x.astype(np.float64) - h.astype(np.float64)
    assert np.all(np.abs(r - l.astype(np.float64)) <= np.abs(r) * 2.0 ** -8 + 1e-45)
    assert np.all(np.abs(r) <= np.abs(x.astype(np.float64)) * 2.0 ** -8)


def test_split_f16_known_answers():
    x = np.array([1.0, 1.0 + 2 ** -11, 1.0 + 3 * 2 ** -12, 65504.0, 1e-8], np.float32)
    hi, lo = oracle.split_f16(x)
    assert hi[0] == 0x3C00 and lo[0] == 0
    assert hi[1] == 0x3C00 and lo[1] == 0x3C00           # residual 2^-11 * 2048 = 1.0
    assert hi[3] == 0x7BFF
    assert hi[4] == 0x0000 or hi[4] < 0x0400             # subnormal or zero


def test_exponent_rule():
    for mx in (1.0, 0.75, 32767.0, 32768.0, 3.0e7, 2.0 ** -100):
        e = oracle.exponent_for_max(mx)
        assert mx * 2.0 ** -e < 2 ** 15
        assert mx * 2.0 ** -e >= 2 ** 14
    assert oracle.exponent_for_max(0.0) == 0


def test_bf16x3_floor_matches_reference_measurement():
    A = datagen.normal((256, 2048), 12345)
    B = datagen.normal((2048, 256), 67890)
    R = oracle.gemm_f64(A, B)
    Rh = oracle.slice_product(A, B, kind=0)
    err = np.linalg.norm(Rh - R) / np.linalg.norm(R)
    assert err == pytest.approx(4.4355e-6, rel=0.06)


def test_fp16x3_floor_matches_reference_constant():
    A = datagen.normal((256, 2048), 12345)
    B = datagen.normal((2048, 256), 67890)
    R = oracle.gemm_f64(A, B)
    err = np.linalg.norm(oracle.slice_product(A, B, kind=2) - R) / np.linalg.norm(R)
    assert err < 3.6e-7
    err_s = np.linalg.norm(oracle.slice_product(A, B, kind=1) - R) / np.linalg.norm(R)
    assert err_s < 3.6e-7


def test_scaled_fp16x3_survives_full_exponent_range():
    A = datagen.wide_range((128, 512), 1)
    B = datagen.wide_range((512, 96), 2)
    R = oracle.gemm_f64(A, B)
    err_s = np.linalg.norm(oracle.slice_product(A, B, kind=1) - R) / np.linalg.norm(R)
    assert err_s < 1e-6
    with np.errstate(all="ignore"):
        bad = oracle.slice_product(A, B, kind=2)
    assert not np.isfinite(bad).all() or np.linalg.norm(bad - R) / np.linalg.norm(R) > 1e-3


def test_fp32_chain_exact_on_integers():
    rng = np.random.default_rng(3)
    A = rng.integers(-8, 9, (37, 300)).astype(np.float32)
    B = rng.integers(-8, 9, (300, 29)).astype(np.float32)
    exact = A.astype(np.int64) @ B.astype(np.int64)
    for chunks in (1, 3, 7, 256):
        C = oracle.fp32_chunked(A, B, chunks)
        assert np.array_equal(C.astype(np.int64), exact)


def test_fp32_chunk_grouping_changes_only_fp64_order():
    A = datagen.uniform((16, 4096), 5)
    B = datagen.uniform((4096, 16), 6)
    c1 = oracle.fp32_chunked(A, B, 16, cpg=16, f64=True)
    c4 = oracle.fp32_chunked(A, B, 16, cpg=4, f64=True)
    assert np.max(np.abs(c1 - c4) / np.maximum(np.abs(c1), 1e-30)) < 1e-14


def test_k_over_c_law():
    """Error of FP32 with FP64 chunk sums depends on K/c only (docs/RESULTS_ROUND9.md:67-71)."""
    M = N = 64
    A1 = datagen.uniform((M, 16384), 11)
    B1 = datagen.uniform((16384, N), 12)
    A4 = datagen.uniform((M, 65536), 13)
    B4 = datagen.uniform((65536, N), 14)
    e1 = oracle.rel_err(oracle.fp32_chunked(A1, B1, 1), oracle.gemm_f64(A1, B1))
    e4 = oracle.rel_err(oracle.fp32_chunked(A4, B4, 4), oracle.gemm_f64(A4, B4))
    assert e4 == pytest.approx(e1, rel=0.25)
    e16 = oracle.rel_err(oracle.fp32_chunked(A4, B4, 16), oracle.gemm_f64(A4, B4))
    assert e16 < e4 * 0.7


def test_rho_hutchinson_restatement():
    A = datagen.normal((64, 256), 21)
    B = datagen.normal((256, 48), 22)
    r, sums = oracle.rho_hutchinson(A, B, 64)
    # the same formula with numpy, hash written independently
    n = np.arange(48, dtype=np.uint64)[:, None] * 64 + np.arange(64, dtype=np.uint64)[None, :]
    h = (n.astype(np.uint32) ^ np.uint32(0x5EED)).astype(np.uint64)
    h ^= h >> 16; h = (h * 0x7FEB352D) & 0xFFFFFFFF; h ^= h >> 15; h = (h * 0x846CA68B) & 0xFFFFFFFF; h ^= h >> 16
    Om = np.where(h & 1, 1.0, -1.0)
    A64, B64 = A.astype(np.float64), B.astype(np.float64)
    den = np.sum((A64 @ (B64 @ Om)) ** 2)
    num = np.sum((np.abs(A64) @ (np.abs(B64) @ Om)) ** 2)
    assert sums[1] == pytest.approx(den, rel=1e-12)
    assert sums[0] == pytest.approx(num, rel=1e-12)
    assert r == pytest.approx(np.sqrt(num / den), rel=1e-12)
    rt = oracle.rho_true(A, B)
    assert r == pytest.approx(rt, rel=0.35)


def test_family2_rho_is_tunable():
    M, K = 64, 2048
    for rho_t in (1e2, 1e4):
        A, B = datagen.family2(M, M, K, rho_t)
        rt = oracle.rho_true(A, B)
        assert rho_t / 3 < rt < rho_t * 3


def test_rescale_forms_equal_ldexpf():
    """The fp16x3 store tail undoes the 2^e row/column scaling in two forms: x * 2^e with 2^e a normal float (when
    -126 <= e <= 127), and float(double(x) * 2^e) otherwise. Both round once, so each equals ldexpf(x, e) bit for
    bit, subnormal, zero and overflowing results included (numpy's float32 ldexp as the reference)."""
    rng = np.random.default_rng(7)
    x = (rng.standard_normal(200000) * np.exp2(rng.integers(-40, 41, 200000))).astype(np.float32)
    x[:4] = [0.0, -0.0, np.float32(2.0 ** -149), np.float32(3.4e38)]
    e = rng.integers(-330, 231, x.size).astype(np.int32)
    normal = (e >= -126) & (e <= 127)
    with np.errstate(over="ignore"):   # overflowing results are part of the check
        want = np.ldexp(x, e).astype(np.float32)
        fast = (x[normal] * np.exp2(e[normal]).astype(np.float32)).astype(np.float32)
        exact = (x.astype(np.float64) * np.exp2(e.astype(np.float64))).astype(np.float32)
    assert np.array_equal(fast.view(np.uint32), want[normal].view(np.uint32))
    assert np.array_equal(exact.view(np.uint32), want.view(np.uint32))
    assert (~normal).sum() > 1000 and (np.abs(want) < 2.0 ** -126).sum() > 100 and np.isinf(want).sum() > 100


# The cancellation spans of the two C4 families at their benchmark size, 2048 x 2048 x 8192, in FP64 on the host
# (about 2 s per oscillatory case, 6 s per family-2 case): rho = || |A||B| ||_F / ||AB||_F.
C4_OSC_RHO = {1.3: (1.1, 1.35), 11.0: (25.0, 36.0), 1150.0: (2700.0, 3400.0)}       # measured 1.22, 30.2, 3022
C4_FAM2_RHO = {1e2: (90.0, 140.0), 1e4: (9.0e3, 1.1e4), 1.1e6: (1.0e6, 1.2e6)}     # measured 114, 1.0003e4, 1.1003e6


def _rho_f64(A, B):
    A64, B64 = A.astype(np.float64), B.astype(np.float64)
    return np.linalg.norm(np.abs(A64) @ np.abs(B64)) / np.linalg.norm(A64 @ B64)


def test_oscillatory_rho_spans_1_to_3000_at_c4_size():
    """The oscillatory family covers the cancellation span the benchmark configuration names (about 1.2 to 3000)
    at its own size, not only at the 512^2 size its docstring quotes."""
    rhos = {f0: _rho_f64(*datagen.oscillatory(2048, 2048, 8192, f0)) for f0 in C4_OSC_RHO}
    for f0, (lo, hi) in C4_OSC_RHO.items():
        assert lo < rhos[f0] < hi, (f0, rhos[f0])
    assert rhos[1.3] < rhos[11.0] < rhos[1150.0]


@pytest.mark.parametrize("rho", sorted(C4_FAM2_RHO))
def test_family2_rho_at_c4_size(rho):
    lo, hi = C4_FAM2_RHO[rho]
    r = _rho_f64(*datagen.family2(2048, 2048, 8192, rho))
    assert lo < r < hi, r
