"""The randomized-SVD application (emugemm-cdna bench/randsvd2.cpp) built on emugemm_sgemm.

CPU: the pipeline's products and argument order, run with an FP64 torch GEMM, against an independent numpy
evaluation of the same projection (Q from a Householder QR of A Omega, residual |A - Q Q^T A| / |A|).
GPU: the pipeline through emugemm_sgemm, native FP32 against AUTO at 1e-5, as the reference prints them."""
from __future__ import annotations

import numpy as np
import pytest

import randsvd


def test_pipeline_matches_numpy_projection():
    import torch

    m, n, l = 2048, 256, 48
    A, Om = randsvd.make_inputs(m, n, l, "cpu", seed=7)
    A, Om = A.double(), Om.double()

    def gemm(M, N, K, X, Y, Z):
        assert X.shape == (M, K) and Y.shape == (K, N) and Z.shape == (M, N)
        assert X.is_contiguous() and Y.is_contiguous()
        Z.copy_(X @ Y)
        return {"M": M, "N": N, "K": K, "scheme": "FP64", "chunks": 1, "predicted_err": 0.0}

    tags = []
    out = randsvd.pipeline(A, Om, gemm, tags.append)
    assert tags == ["start", "sketch", "qr", "end"]
    assert [(p["M"], p["N"], p["K"]) for p in out["plans"]] == [(m, l, n), (l, l, m), (l, l, m), (l, n, m)]
    An, On = A.numpy(), Om.numpy()
    Q, _ = np.linalg.qr(An @ On)
    resid = np.linalg.norm(An - Q @ (Q.T @ An)) / np.linalg.norm(An)
    assert out["residual"] == pytest.approx(resid, rel=1e-8)
    assert out["orthogonality"] < 1e-10
    assert 0.05 < resid < 0.9          # a meaningful rank-l approximation of the decaying spectrum

    inv = randsvd.pipeline(A, Om, gemm, solve="inverse")
    assert [(p["M"], p["N"], p["K"]) for p in inv["plans"]] == [(m, l, n), (l, l, m), (m, l, l), (l, l, m),
                                                               (m, l, l), (l, n, m)]
    assert inv["residual"] == pytest.approx(resid, rel=1e-8)
    assert inv["orthogonality"] < 1e-10


@pytest.mark.gpu
def test_randsvd_through_emugemm(cuda):
    res = randsvd.run(16384, 1024, 256, [1e-5], reps=1)
    native, emu = res["results"]
    assert native["schemes"] == ["NATIVE_FP32"] * 4
    assert len(emu["schemes"]) == 4
    assert emu["residual"] == pytest.approx(native["residual"], rel=1e-4)
    assert native["orthogonality"] < 1e-3 and emu["orthogonality"] < 1e-3
    assert emu["speedup_end_to_end"] > 0
    assert abs(emu["residual_vs_fp64"]) < 1e-3 and abs(native["residual_vs_fp64"]) < 1e-3
    inv = randsvd.run(16384, 1024, 256, [1e-5], reps=1, solve="inverse")
    assert len(inv["results"][1]["schemes"]) == 6
    assert inv["results"][1]["residual"] == pytest.approx(inv["fp64_residual"], rel=1e-3)
