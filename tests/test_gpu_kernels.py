"""GPU parity of every kernel on the hot path, called through the C ABI and checked against the CPU oracle.

Bars:
- slice split, absmax, exponent scans: bit-exact;
- NATIVE_FP32 / FP32_CHUNKED: bit-exact against the oracle's replica of the same FMA chains and FP64
  chunk sums (same group split);
- bf16x3 / fp16x3 tensor-core GEMM: against the exact FP64 value of the three slice products (the oracle's
  slice_product), within the FP32 accumulation bound stated per test; and against FP64 truth within the
  plan's predicted error;
- rho estimate: against the oracle's FP64 evaluation of the same Hutchinson estimate.
"""
from __future__ import annotations

import numpy as np
import pytest

import datagen
import emugemm
import oracle

pytestmark = pytest.mark.gpu


def dev(torch, x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def run_sgemm(torch, h, A, B, force=emugemm.AUTO, tgt=1e-5, hints=None, use_hints=True):
    M, K = A.shape
    N = B.shape[1]
    dA, dB = dev(torch, A), dev(torch, B)
    dC = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    p, hn = h.sgemm(M, N, K, dA, dB, dC, max_rel_err=tgt, force=force, hints=hints, use_hints=use_hints)
    h.sync()
    return dC.cpu().numpy(), p, hn


# ---------------------------------------------------------------------------------------------- split
@pytest.mark.parametrize("n", [1, 7, 4096, 1000003])
def test_split_bf16_bitexact(cuda, handle, n):
    torch = cuda
    x = datagen.wide_range((n,), 100 + n, emax=60)
    if n > 8:
        x[:8] = [0.0, -0.0, 1.0, 1.00390625, 2 ** -140, -3.4e38, 65504.0, 1.0 + 2 ** -9]
    dx = dev(torch, x)
    hi = torch.empty(n, dtype=torch.int16, device="cuda")
    lo = torch.empty(n, dtype=torch.int16, device="cuda")
    handle.split_bf16(dx, n, hi, lo)
    handle.sync()
    rh, rl = oracle.split_bf16(x)
    assert np.array_equal(hi.cpu().numpy().view(np.uint16), rh)
    assert np.array_equal(lo.cpu().numpy().view(np.uint16), rl)


@pytest.mark.parametrize("n", [5, 65536, 999999])
def test_split_f16_bitexact(cuda, handle, n):
    torch = cuda
    x = datagen.normal((n,), 7 + n, scale=100.0)
    dx = dev(torch, x)
    hi = torch.empty(n, dtype=torch.int16, device="cuda")
    lo = torch.empty(n, dtype=torch.int16, device="cuda")
    handle.split_f16(dx, n, hi, lo)
    handle.sync()
    rh, rl = oracle.split_f16(x)
    assert np.array_equal(hi.cpu().numpy().view(np.uint16), rh)
    assert np.array_equal(lo.cpu().numpy().view(np.uint16), rl)


@pytest.mark.parametrize("n", [1, 333, 1 << 22])
def test_absmax_exact(cuda, handle, n):
    torch = cuda
    x = datagen.wide_range((n,), 5 + n)
    assert handle.absmax(dev(torch, x), n) == oracle.absmax(x)


# ------------------------------------------------------------------------------------------- FP32 SIMT
FP32_SHAPES = [(64, 64, 64), (130, 70, 333), (1, 1, 1), (5, 3, 1), (256, 256, 4096), (300, 520, 1000),
               (1024, 1024, 256)]


@pytest.mark.parametrize("shape", FP32_SHAPES, ids=[str(s) for s in FP32_SHAPES])
def test_native_fp32_bitexact(cuda, handle, shape):
    torch = cuda
    M, N, K = shape
    A = datagen.uniform((M, K), 1 + M)
    B = datagen.uniform((K, N), 2 + N)
    C, p, _ = run_sgemm(torch, handle, A, B, force=emugemm.NATIVE_FP32)
    assert p.chosen == emugemm.NATIVE_FP32
    assert np.array_equal(C, oracle.fp32_chunked(A, B, 1))


@pytest.mark.parametrize("shape,chunks", [((256, 256, 8192), 4), ((256, 256, 8192), 16), ((64, 128, 5000), 7),
                                          ((256, 256, 4096), 256), ((512, 384, 3000), 2), ((33, 17, 100), 256)])
def test_chunked_fp32_bitexact(cuda, handle, shape, chunks):
    """FP32_CHUNKED through the partial (FP64 output) and reduce entry points, bit-exact in FP64."""
    torch = cuda
    M, N, K = shape
    A = datagen.uniform((M, K), 3 + K)
    B = datagen.uniform((K, N), 4 + K)
    dA, dB = dev(torch, A), dev(torch, B)
    P64 = torch.empty((M, N), dtype=torch.float64, device="cuda")
    handle.partial_f64(M, N, K, dA, K, dB, N, P64, emugemm.FP32_CHUNKED, chunks)
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    handle.reduce_f64(M, N, 1, P64, C)
    handle.sync()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    G = emugemm.fp32_groups(M, N, K, chunks, sms)
    cpg = oracle.group_size(K, chunks, G)
    want = oracle.fp32_chunked(A, B, chunks, cpg=cpg, f64=True)
    assert np.array_equal(P64.cpu().numpy(), want)
    assert np.array_equal(C.cpu().numpy(), want.astype(np.float32))


@pytest.mark.parametrize("tile", [16, 3264, 32, 64, 128])
@pytest.mark.parametrize("shape,chunks", [((256, 256, 8192), 1), ((256, 256, 8192), 4), ((100, 36, 1000), 3),
                                          ((33, 20, 260), 1), ((64, 130, 500), 2), ((64, 64, 1000), 2),
                                          ((48, 96, 4104), 3)])
def test_fp32_tiles_bitexact(cuda, handle, tile, shape, chunks):
    """Every FP32 SIMT tile (EMUGEMM_ATTR_FP32_TILE: 16 / 3264 = the 16 x 32 and 32 x 64 tiles of the register-pipelined
    kernel, fed by cp.async and by TMA; 32 / 64 / 128 square) runs the same chains and FP64 folds: bit-exact against the oracle
    with the group split the library reports. Ragged M, N not a multiple of 32, chunk lengths not a multiple of 64
    (chunks that end inside a k-block: the TMA-fed kernel must stop there although the block holds the next chunk's
    values); N = 130 is not a multiple of 4 and K = 1000 in 3 chunks gives chunk lengths that are not, so the kernels
    that copy 16-byte pieces fall back to the 32 tile there."""
    torch = cuda
    handle.set_kernels(fp32_tile=tile)
    M, N, K = shape
    A = datagen.uniform((M, K), 5 + K + tile)
    B = datagen.uniform((K, N), 6 + K + tile)
    dA, dB = dev(torch, A), dev(torch, B)
    P64 = torch.empty((M, N), dtype=torch.float64, device="cuda")
    handle.partial_f64(M, N, K, dA, K, dB, N, P64, emugemm.FP32_CHUNKED, chunks)
    handle.sync()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    G = emugemm.fp32_groups(M, N, K, chunks, sms, tile=tile)
    want = oracle.fp32_chunked(A, B, chunks, cpg=oracle.group_size(K, chunks, G), f64=True)
    assert np.array_equal(P64.cpu().numpy(), want)
    C, p, _ = run_sgemm(torch, handle, A, B, force=emugemm.NATIVE_FP32)
    assert np.array_equal(C, oracle.fp32_chunked(A, B, 1))


def test_auto_chunked_plan_runs_chunked(cuda, handle):
    """A target below what bf16x3 and fp16x3 can reach (2e-7 at K = 65536) routes to FP32_CHUNKED with c > 1;
    the result is the bit-exact chain."""
    torch = cuda
    M, N, K = 256, 256, 65536
    A = datagen.uniform((M, K), 31)
    B = datagen.uniform((K, N), 32)
    hints = emugemm.EmuHints(1.0, 1.0, 0, 0.0, 0)
    C, p, _ = run_sgemm(torch, handle, A, B, tgt=2e-7, hints=hints)
    assert p.chosen == emugemm.FP32_CHUNKED and p.chunks > 1
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    G = emugemm.fp32_groups(M, N, K, p.chunks, sms)
    want = oracle.fp32_chunked(A, B, p.chunks, cpg=oracle.group_size(K, p.chunks, G))
    assert np.array_equal(C, want)
    R = oracle.gemm_f64(A, B)
    assert oracle.rel_err(C, R) <= p.predicted_err


# ---------------------------------------------------------------------------------- tensor-core 3-product
# K above 16384 stores the slices in K panels of 8192 (3 and 5 panels below, the last one partly padding)
TC_SHAPES = [(128, 256, 64), (256, 512, 1024), (200, 300, 500), (1, 1, 1), (129, 257, 65), (1024, 1024, 1024),
             (384, 768, 4096), (130, 260, 20000), (64, 96, 40000)]


def _accum_bound(K):
    # Distance of C from the exact slice-product sum, relative to ||R||: truncation inside 128-long tensor-core
    # partial sums (three accumulations per k-step) plus the FP32 running sum and the output rounding,
    # measured at 5-8e-7. A wrong or missing slice product would show up at 1e-5 (a dropped lo) to 1e-3.
    return 1.0e-6 + 2.0e-9 * np.sqrt(K)


@pytest.mark.parametrize("shape", TC_SHAPES, ids=[str(s) for s in TC_SHAPES])
def test_bf16x3_matches_slice_products(cuda, handle, shape):
    torch = cuda
    M, N, K = shape
    A = datagen.normal((M, K), 12345)
    B = datagen.normal((K, N), 67890)
    C, p, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X3)
    assert p.chosen == emugemm.BF16X3 and p.reason == b"forced"
    Rh = oracle.slice_product(A, B, kind=0)
    R = oracle.gemm_f64(A, B)
    d = np.linalg.norm(C.astype(np.float64) - Rh) / np.linalg.norm(R)
    print(f"bf16x3 {shape}: |C-Rhat|/|R| = {d:.3e}  err vs fp64 = {oracle.rel_err(C, R):.3e}")
    assert np.isfinite(C).all()
    assert d <= _accum_bound(K)


@pytest.mark.parametrize("variant", ["single", "pair"])
@pytest.mark.parametrize("shape", [(128, 128, 64), (200, 300, 500), (512, 256, 2048), (1, 1, 1), (64, 128, 24000),
                                   (600, 520, 4100)])
def test_fp16x3_scaled_matches_slice_products(cuda, handle, variant, shape):
    """fp16x3 on N(0,1)*2^e data (the full exponent range, so every row and column is rescaled): both tensor-core
    kernels against the exact slice products. The pair kernel scales each stage's cross products by 2^-11 inside
    the accumulator (tcgen05 scale-input-d) before adding hi*hi; the single-CTA kernel keeps two accumulators."""
    torch = cuda
    M, N, K = shape
    handle.set_kernels(tc_kernel=variant)
    A = datagen.wide_range((M, K), 77)
    B = datagen.wide_range((K, N), 78)
    C, p, _ = run_sgemm(torch, handle, A, B, force=emugemm.FP16X3)
    assert p.chosen == emugemm.FP16X3
    Rh = oracle.slice_product(A, B, kind=1)
    R = oracle.gemm_f64(A, B)
    d = np.linalg.norm(C.astype(np.float64) - Rh) / np.linalg.norm(R)
    print(f"fp16x3 {shape}: |C-Rhat|/|R| = {d:.3e}  err vs fp64 = {oracle.rel_err(C, R):.3e}")
    assert np.isfinite(C).all()
    assert d <= _accum_bound(K)
    assert oracle.rel_err(C, R) < 2e-6


def test_bf16x6_forced_runs_bf16x3(cuda, handle):
    """Reference quirk (src/emugemm.cpp:331): a forced BF16X6 runs the bf16x3 kernel."""
    torch = cuda
    A = datagen.normal((256, 256), 1)
    B = datagen.normal((256, 256), 2)
    C6, p6, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X6)
    C3, _, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X3)
    assert p6.chosen == emugemm.BF16X6
    assert np.array_equal(C6, C3)


def test_bf16x3_deterministic(cuda, handle):
    torch = cuda
    A = datagen.normal((512, 1024), 3)
    B = datagen.normal((1024, 768), 4)
    C1, _, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X3)
    C2, _, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X3)
    assert np.array_equal(C1, C2)


# --------------------------------------------------------------------------------------------- rho
# (130,70,1000) and 30 probes take the synchronous-load kernel; the others the cp.async ring (16-aligned
# J), (130,96,1000) one of each, (128,64,4000) several K splits with a short last one.
@pytest.mark.parametrize("shape,probes", [((64, 48, 256), 64), ((256, 256, 2048), 64), ((130, 70, 1000), 64),
                                          ((130, 96, 1000), 64), ((128, 64, 4000), 64), ((256, 256, 2048), 30)])
def test_rho_estimate_matches_oracle(cuda, handle, shape, probes):
    torch = cuda
    M, N, K = shape
    A = datagen.normal((M, K), 5)
    B = datagen.normal((K, N), 6)
    r = handle.estimate_rho(M, N, K, dev(torch, A), dev(torch, B), probes)
    ro, _ = oracle.rho_hutchinson(A, B, probes)
    assert r == pytest.approx(ro, rel=1e-4)


def test_rho_estimate_adversarial(cuda, handle):
    torch = cuda
    M, K = 256, 4096
    A, B = datagen.family2(M, M, K, 1e4)
    r = handle.estimate_rho(M, M, K, dev(torch, A), dev(torch, B), 64)
    ro, _ = oracle.rho_hutchinson(A, B, 64)
    assert r == pytest.approx(ro, rel=2e-2)


def test_hints_written_back(cuda, handle):
    torch = cuda
    A = datagen.normal((256, 512), 8)
    B = datagen.normal((512, 128), 9)
    hn = emugemm.EmuHints(-1.0, -1.0, 0, -1.0, 32)
    C, p, hn = run_sgemm(torch, handle, A, B, tgt=1e-5, hints=hn)
    assert hn.a_absmax == oracle.absmax(A)
    assert hn.b_absmax == oracle.absmax(B)
    ro, _ = oracle.rho_hutchinson(A, B, 32)
    assert hn.rho == pytest.approx(ro, rel=1e-4)


def test_null_hints_measure_everything(cuda, handle):
    torch = cuda
    A = datagen.normal((128, 256), 10)
    B = datagen.normal((256, 128), 11)
    C, p, _ = run_sgemm(torch, handle, A, B, tgt=1e-5, use_hints=False)
    R = oracle.gemm_f64(A, B)
    assert oracle.rel_err(C, R) <= p.predicted_err


# ----------------------------------------------------------------------------------------- edge cases
def test_zero_sizes(cuda, handle):
    torch = cuda
    A = torch.zeros((4, 0), device="cuda")
    B = torch.zeros((0, 5), device="cuda")
    C = torch.full((4, 5), 7.0, device="cuda")
    for force in (emugemm.NATIVE_FP32, emugemm.BF16X3, emugemm.FP16X3):
        C.fill_(7.0)
        handle.sgemm(4, 5, 0, A, B, C, force=force)
        handle.sync()
        assert torch.count_nonzero(C).item() == 0
    handle.sgemm(0, 5, 3, torch.zeros(1, device="cuda"), torch.zeros(15, device="cuda"), C, force=emugemm.BF16X3)


def test_workspace_limit_reports_memory_error(cuda):
    torch = cuda
    h = emugemm.Handle()
    try:
        h.set_workspace_limit(1 << 20)
        A = torch.randn(1024, 1024, device="cuda")
        B = torch.randn(1024, 1024, device="cuda")
        C = torch.empty(1024, 1024, device="cuda")
        with pytest.raises(emugemm.EmuGemmError) as e:
            h.sgemm(1024, 1024, 1024, A, B, C, force=emugemm.BF16X3)
        assert e.value.code == 5
    finally:
        h.close()


def test_invalid_sizes(cuda, handle):
    torch = cuda
    A = torch.zeros(16, device="cuda")
    with pytest.raises(emugemm.EmuGemmError) as e:
        handle.sgemm(-1, 4, 4, A, A, A)
    assert e.value.code == 4


def test_strided_operands(cuda, handle):
    """emugemm_sgemm_ex on sub-blocks of larger arrays (leading dimensions > K, N)."""
    torch = cuda
    A = datagen.normal((300, 520), 40)
    B = datagen.normal((600, 410), 41)
    M, K, N = 200, 500, 400
    dA, dB = dev(torch, A), dev(torch, B)
    C = torch.zeros((250, 450), dtype=torch.float32, device="cuda")
    for force in (emugemm.NATIVE_FP32, emugemm.BF16X3, emugemm.FP16X3):
        C.zero_()
        handle.sgemm_ex(M, N, K, dA, 520, dB, 410, C, 450, force=force,
                        hints=emugemm.EmuHints(1.0, 1.0, 0, 0.0, 0))
        handle.sync()
        Cn = C.cpu().numpy()
        R = oracle.gemm_f64(A[:M, :K], B[:K, :N])
        assert oracle.rel_err(Cn[:M, :N], R) < 2e-5
        assert np.count_nonzero(Cn[M:, :]) == 0 and np.count_nonzero(Cn[:, N:]) == 0
        if force == emugemm.NATIVE_FP32:
            assert np.array_equal(Cn[:M, :N], oracle.fp32_chunked(A[:M, :K], B[:K, :N], 1))


def test_launch_counter_advances(cuda, handle):
    torch = cuda
    before = emugemm.launch_count()
    A = torch.randn(64, 64, device="cuda")
    C = torch.empty(64, 64, device="cuda")
    handle.sgemm(64, 64, 64, A, A, C, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    handle.sync()
    assert emugemm.launch_count() >= before + 3


def test_a_is_reused_reuses_the_split(cuda, handle):
    """hints.a_is_reused with an unchanged A: the second call skips A's split and gives the same bits."""
    torch = cuda
    A = datagen.normal((512, 768), 50)
    B1 = datagen.normal((768, 384), 51)
    B2 = datagen.normal((768, 384), 52)
    dA, dB1, dB2 = dev(torch, A), dev(torch, B1), dev(torch, B2)
    for force in (emugemm.BF16X3, emugemm.FP16X3):
        ref = torch.empty((512, 384), device="cuda")
        handle.sgemm(512, 384, 768, dA, dB2, ref, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        out = torch.empty((512, 384), device="cuda")
        handle.sgemm(512, 384, 768, dA, dB1, out, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        handle.profile_begin()
        handle.sgemm(512, 384, 768, dA, dB2, out, force=force, hints=emugemm.EmuHints(1, 1, 1, 0, 0))
        prof = handle.profile_end()
        assert torch.equal(out, ref)
        assert prof["split"][1] == 1          # only B was split


@pytest.mark.parametrize("force", [emugemm.BF16X3, emugemm.FP16X3])
@pytest.mark.parametrize("shape", [(256, 256, 128), (300, 520, 1000), (1024, 768, 2048), (1, 1, 1), (2048, 2048, 512),
                                   (256, 256, 20000)])
def test_pair_kernel_matches_single_cta_kernel(cuda, handle, force, shape):
    """bf16x3: the CTA-pair kernel (cta_group::2) computes every output from the same slices and k-steps as the
    single-CTA kernel: identical bits. fp16x3: the single-CTA kernel keeps hi*hi and the cross products in two
    accumulators; the pair kernel scales the cross products by 2^-11 inside one accumulator and promotes every 64
    of K. Their sums round differently, so both kernels must sit within the accumulation bound of the exact slice
    products. K is not split (the split-K form sums FP64 partials and is tested on its own)."""
    torch = cuda
    handle.set_kernels(splitk=1)
    M, N, K = shape
    A = datagen.normal((M, K), 60 + M)
    B = datagen.normal((K, N), 61 + N)
    out = {}
    for variant in ("single", "pair"):
        handle.set_kernels(tc_kernel=variant)
        C, p, _ = run_sgemm(torch, handle, A, B, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        out[variant] = C
    assert np.isfinite(out["pair"]).all()
    if force == emugemm.BF16X3:
        assert np.array_equal(out["pair"], out["single"])
    else:
        Rh = oracle.slice_product(A, B, kind=1)
        R = oracle.gemm_f64(A, B)
        for v in ("pair", "single"):
            d = np.linalg.norm(out[v].astype(np.float64) - Rh) / max(np.linalg.norm(R), 1e-300)
            assert d <= _accum_bound(K), (v, d)


@pytest.mark.parametrize("force", [emugemm.BF16X3, emugemm.FP16X3])
@pytest.mark.parametrize("shape,splits", [((256, 256, 20000), None), ((256, 256, 20000), 7), ((300, 260, 9000), None),
                                          ((200, 520, 4100), 3), ((64, 96, 40000), None)])
def test_pair_kernel_split_k(cuda, handle, force, shape, splits):
    """Few 256 x 256 pair tiles and a long K: each tile's K range is split over SM pairs (None: the built-in count;
    else EMUGEMM_ATTR_TC_SPLITK), every split writes an FP64 partial and the partials are summed in order. The result
    sits within the accumulation bound of the exact slice products, within 1e-6 of the unsplit kernel's (relative
    to ||AB||), and is deterministic; the FP64 partial entry point gives the same sum before its final rounding."""
    torch = cuda
    M, N, K = shape
    A = datagen.normal((M, K), 90 + M)
    B = datagen.normal((K, N), 91 + N)
    handle.set_kernels(tc_kernel="pair")
    handle.set_kernels(splitk=1)
    C1, _, _ = run_sgemm(torch, handle, A, B, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    if splits is None:
        handle.set_kernels(splitk=0)
    else:
        handle.set_kernels(splitk=splits)
    Cs, _, _ = run_sgemm(torch, handle, A, B, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    Cs2, _, _ = run_sgemm(torch, handle, A, B, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    dA, dB = dev(torch, A), dev(torch, B)
    P = torch.full((M, N), float("nan"), dtype=torch.float64, device="cuda")
    handle.partial_f64(M, N, K, dA, K, dB, N, P, force, 1)
    handle.sync()
    R = oracle.gemm_f64(A, B)
    nR = np.linalg.norm(R)
    Rh = oracle.slice_product(A, B, kind=0 if force == emugemm.BF16X3 else 1)
    assert np.isfinite(Cs).all()
    assert np.array_equal(Cs, Cs2)
    assert np.array_equal(P.cpu().numpy().astype(np.float32), Cs)
    assert np.linalg.norm(Cs.astype(np.float64) - Rh) / nR <= _accum_bound(K)
    assert np.linalg.norm(Cs.astype(np.float64) - C1) / nR <= 1e-6


@pytest.mark.parametrize("variant", ["fused", "fusea"])
@pytest.mark.parametrize("shape", [(256, 256, 128), (260, 516, 1004), (1024, 768, 2048), (2048, 2048, 512),
                                   (384, 264, 96), (1, 1, 1), (33, 65, 129), (260, 500, 20000)])
@pytest.mark.parametrize("gen", ["normal", "wide_range"])
def test_fused_split_kernel_matches_presplit(cuda, handle, variant, shape, gen):
    """bf16x3 with the split fused into the CTA-pair GEMM uses the same slices, k-steps and promotion points as
    the pre-split kernels: identical bits. `fused`: FP32 tiles of A and B by TMA, hi/lo made in shared memory;
    `fusea`: A's hi/lo made in the kernel and written into TMEM, B pre-split. Leading dimensions TMA cannot address
    (not a multiple of 4 floats) fall back to the pre-split path. The pair kernel runs without K splits."""
    torch = cuda
    handle.set_kernels(splitk=1)
    M, N, K = shape
    if gen == "normal":
        A = datagen.normal((M, K), 70 + M)
        B = datagen.normal((K, N), 71 + N)
    else:
        A = datagen.wide_range((M, K), 72 + M, emax=20)
        B = datagen.wide_range((K, N), 73 + N, emax=20)
    out, splits = {}, {}
    for v in ("pair", variant):
        handle.set_kernels(tc_kernel=v)
        handle.profile_begin()
        C, p, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        splits[v] = handle.profile_end()["split"][1]
        out[v] = C
    assert np.isfinite(out[variant]).all()
    assert np.array_equal(out[variant], out["pair"])
    if variant == "fused":
        fused_ran = K % 4 == 0 and N % 4 == 0
        assert splits["fused"] == (0 if fused_ran else 1)   # one profiled scope covers both splits
    else:
        assert splits["fusea"] == 1                           # B's split (or both, on the fallback)


@pytest.mark.parametrize("splits", [None, 5])
@pytest.mark.parametrize("shape", [(256, 256, 40000), (260, 500, 20000), (300, 264, 9000)])
def test_fused_split_k_matches_pair(cuda, handle, splits, shape):
    """Split-K in the fused kernel (FP32 tiles split in the kernel) and in the pre-split pair kernel: both split K on
    the same 128-K chunk boundaries and promote at the same points, so C is bit-identical; it also sits within the
    accumulation bound of the exact slice products (None: the built-in split count, else EMUGEMM_ATTR_TC_SPLITK)."""
    torch = cuda
    if splits is not None:
        handle.set_kernels(splitk=splits)
    M, N, K = shape
    A = datagen.normal((M, K), 95 + M)
    B = datagen.normal((K, N), 96 + N)
    out = {}
    for v in ("pair", "fused"):
        handle.set_kernels(tc_kernel=v)
        out[v], _, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    assert np.isfinite(out["fused"]).all()
    assert np.array_equal(out["fused"], out["pair"])
    R = oracle.gemm_f64(A, B)
    d = np.linalg.norm(out["fused"].astype(np.float64) - oracle.slice_product(A, B, kind=0)) / np.linalg.norm(R)
    assert d <= _accum_bound(K)


@pytest.mark.parametrize("variant", ["fused", "fusea"])
def test_fused_split_kernel_partial_f64(cuda, handle, variant):
    """The FP64 partial output of the fused kernels (K-split building block) equals the pre-split kernel's."""
    torch = cuda
    handle.set_kernels(splitk=1)
    M, N, K = 300, 260, 1536
    A = dev(torch, datagen.normal((M, K), 80))
    B = dev(torch, datagen.normal((K, N), 81))
    out = {}
    for variant_ in ("pair", variant):
        handle.set_kernels(tc_kernel=variant_)
        P = torch.full((M, N), float("nan"), dtype=torch.float64, device="cuda")
        handle.partial_f64(M, N, K, A, K, B, N, P, emugemm.BF16X3, 1)
        handle.sync()
        out[variant_] = P.cpu().numpy()
    assert np.isfinite(out[variant]).all()
    assert np.array_equal(out[variant], out["pair"])


@pytest.mark.parametrize("force", [emugemm.BF16X3, emugemm.FP16X3, emugemm.NATIVE_FP32])
@pytest.mark.parametrize("shape", [(1024, 2048, 512), (300, 520, 1000), (1, 1, 1), (257, 3000, 64)])
def test_sgemm_host_matches_device(cuda, handle, force, shape):
    """emugemm_sgemm_host (pinned host A, B, C; B first, A and C in row panels overlapped with the GEMMs) gives the bits
    of emugemm_sgemm on device copies of the same operands, with hints given (pipelined) and with NULL hints
    (copy everything, then the device path)."""
    torch = cuda
    M, N, K = shape
    A = datagen.wide_range((M, K), 90 + M, emax=10)
    B = datagen.wide_range((K, N), 91 + N, emax=10)
    want, _, _ = run_sgemm(torch, handle, A, B, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    hA = torch.from_numpy(A).pin_memory()
    hB = torch.from_numpy(B).pin_memory()
    for hints, use in ((emugemm.EmuHints(1, 1, 0, 0, 0), True), (None, False)):
        hC = torch.full((M, N), float("nan")).pin_memory()
        p, _ = handle.sgemm_host(M, N, K, hA, hB, hC, force=force, hints=hints, use_hints=use)
        handle.sync()
        assert p.chosen == force
        assert np.array_equal(hC.numpy(), want), (shape, use)


@pytest.mark.parametrize("force", [emugemm.BF16X3, emugemm.FP16X3])
def test_sgemm_host_long_k_matches_device(cuda, handle, force):
    """Few output tiles and a long K: the single call splits K over the SM pairs (bf16x3 in the fused kernel). The
    host-buffer entry point runs row panels with fewer tiles each, but with the kernel and split count of the
    whole product, so its C has the same bits."""
    torch = cuda
    M, N, K = 1024, 256, 24000
    A = datagen.normal((M, K), 93)
    B = datagen.normal((K, N), 94)
    want, _, _ = run_sgemm(torch, handle, A, B, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    hA = torch.from_numpy(A).pin_memory()
    hB = torch.from_numpy(B).pin_memory()
    hC = torch.full((M, N), float("nan")).pin_memory()
    handle.sgemm_host(M, N, K, hA, hB, hC, force=force, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    handle.sync()
    assert np.array_equal(hC.numpy(), want)


def test_log_lines(cuda):
    """EMUGEMM_LOG=1: one stderr line per GEMM with the plan (scheme, chunks, predicted error, reason) and one per
    tensor-core launch with the kernel chosen."""
    import subprocess
    import sys
    import textwrap

    code = textwrap.dedent("""
        import sys, torch
        sys.path.insert(0, "emugemm-cdna_b200")
        import emugemm
        A = torch.randn(256, 512, device="cuda"); B = torch.randn(512, 384, device="cuda")
        C = torch.empty(256, 384, device="cuda")
        with emugemm.Handle() as h:
            h.sgemm(256, 384, 512, A, B, C, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
            h.sync()
    """)
    import os
    import pathlib
    root = pathlib.Path(__file__).resolve().parent.parent
    env = dict(os.environ, EMUGEMM_LOG="1")
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stderr.splitlines() if l.startswith("emugemm: ")]
    assert any("sgemm M=256 N=384 K=512 scheme=BF16X3 chunks=1" in l and 'reason="forced"' in l for l in lines), lines
    assert any("tensor-core kernel=single (bf16x3) M=256 N=384 K=512" in l for l in lines), lines


def test_committed_tile_table_dispatch(cuda, handle):
    """With the measured B200 table loaded, a shape whose row names the fused-A kernel runs it (the log says so)
    and gives the pair kernel's bits; without the table the built-in choice runs."""
    import csv
    import pathlib

    torch = cuda
    lib = emugemm.lib()
    table = pathlib.Path(__file__).resolve().parent.parent / "emugemm-cdna_b200" / "tiles_b200.csv"
    rows = [r for r in csv.reader(table.open()) if r[0] != "arch" and r[5] == "bf16" and r[6] == "4"]
    assert rows, "the committed table names the fused-A kernel for no shape"
    M, N, K = (int(x) for x in rows[0][2:5])
    assert lib.emugemm_tune_lookup(M, N, K, 1) == 0          # no table yet
    A = datagen.normal((M, K), 97)
    B = datagen.normal((K, N), 98)
    handle.set_kernels(tc_kernel="pair")
    ref, _, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    handle.set_kernels(tc_kernel=0)
    try:
        assert lib.emugemm_init(str(table).encode()) == 0
        assert lib.emugemm_tune_lookup(M, N, K, 1) == 4
        n0 = emugemm.launch_count()
        C, p, _ = run_sgemm(torch, handle, A, B, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        launches = emugemm.launch_count() - n0
    finally:
        lib.emugemm_shutdown()
    assert launches == 2                   # B's split and the fused-A GEMM (the pre-split path launches 3)
    assert np.array_equal(C, ref)


# --------------------------------------------------------------------------------------------- peak probe
def test_peak_probe(cuda, handle):
    """emugemm_peak_probe (the counterpart of bench/mfma_peak2.cpp): every instrument ran and its rate is
    physically plausible for one B200: bf16 = fp16 on the tensor cores, tf32 at half their rate, FFMA near
    148 SMs x 128 lanes x 2 FLOP x clock, the copy below the HBM3e nominal 8 TB/s."""
    r = handle.peak_probe(3)
    assert 800 < r["tc_bf16_tflops"] < 2400
    assert 0.9 < r["tc_fp16_tflops"] / r["tc_bf16_tflops"] < 1.1
    assert 0.35 < r["tc_tf32_tflops"] / r["tc_bf16_tflops"] < 0.65
    assert 30 < r["ffma_tflops"] < 80
    assert 5 < r["dfma_tflops"] < r["ffma_tflops"]
    assert 2000 < r["copy_gbs"] < 8000
    # the handle stays usable after the probe
    assert handle.absmax(dev(cuda, np.ones(16, np.float32)), 16) == 1.0


@pytest.mark.parametrize("splits", [1, None, 5])
@pytest.mark.parametrize("shape", [(256, 256, 128), (260, 516, 1004), (1024, 768, 2048), (384, 264, 96), (1, 1, 1),
                                   (33, 68, 129), (256, 256, 40000), (260, 500, 20000), (300, 264, 9000)])
@pytest.mark.parametrize("gen", ["normal", "wide_range"])
def test_fused_fp16x3_matches_presplit_pair(cuda, handle, splits, shape, gen):
    """fp16x3 with the scaled split fused into the CTA-pair GEMM (FP32 tiles by TMA, x * 2^-e split into fp16 hi/lo in
    shared memory, the pair kernel's MMA order within each 64-K chunk, 2^e undone at the store) gives the bits of the
    pre-split fp16 pair kernel, with the same K splits (1, the built-in count, or 5); and within the accumulation bound
    of the exact scaled slice products."""
    torch = cuda
    M, N, K = shape
    if gen == "normal":
        A = datagen.normal((M, K), 170 + M)
        B = datagen.normal((K, N), 171 + N)
    else:
        A = datagen.wide_range((M, K), 172 + M, emax=20)
        B = datagen.wide_range((K, N), 173 + N, emax=20)
    if splits is not None:
        handle.set_kernels(splitk=splits)
    out = {}
    for v in ("pair", "fused"):
        handle.set_kernels(tc_kernel=v)
        handle.profile_begin()
        C, p, _ = run_sgemm(torch, handle, A, B, force=emugemm.FP16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        prof = handle.profile_end()
        assert p.chosen == emugemm.FP16X3
        out[v] = (C, prof["split"][1])
    assert np.isfinite(out["fused"][0]).all()
    assert np.array_equal(out["fused"][0], out["pair"][0])
    assert out["fused"][1] == (0 if (K % 4 == 0 and N % 4 == 0) else 1)   # no split pass when the fused kernel ran
    R = oracle.gemm_f64(A, B)
    d = np.linalg.norm(out["fused"][0].astype(np.float64) - oracle.slice_product(A, B, kind=1)) / np.linalg.norm(R)
    assert d <= _accum_bound(K)


def test_fused_fp16x3_is_the_builtin_choice_for_few_tiles_and_long_k(cuda, handle):
    """256 x 256 x 65536 fp16x3: one pair tile, K split over the SM pairs; the built-in choice is now the fused kernel
    (no split pass), with the bits of the pre-split pair kernel at the same split count."""
    torch = cuda
    M, N, K = 256, 256, 65536
    A = datagen.uniform((M, K), 181)
    B = datagen.uniform((K, N), 182)
    handle.profile_begin()
    C, _, _ = run_sgemm(torch, handle, A, B, force=emugemm.FP16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    prof = handle.profile_end()
    assert prof["split"][1] == 0
    handle.set_kernels(tc_kernel="pair")
    Cp, _, _ = run_sgemm(torch, handle, A, B, force=emugemm.FP16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    assert np.array_equal(C, Cp)
