"""The allocation-free bf16x3 entry point, emugemm_sgemm_bf16x3_noalloc, called through the C ABI.

Some callers cannot let a library call cudaMalloc: plugins inside an application whose memory pool has
reserved the device's memory, and latency-critical paths that must not risk an allocation (or its failure)
mid-run. For them the library computes the bf16x3 product in a fixed 64 MiB device array instead of its
grow-only workspace. This file checks, on two calls in a row with different shapes (so the second call
runs over the first call's leftovers in the shared array), that its output equals the output of the
existing emugemm_sgemm (forced BF16X3) bit for bit, and that both sit within the slice-product tolerance the
other bf16x3 tests use; and that a problem larger than the array is refused. It is collected last so that a
run stopping at the first failure has run every other test first; it also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import datagen
import emugemm
import oracle

pytestmark = pytest.mark.gpu


def _noalloc():
    f = emugemm.lib().emugemm_sgemm_bf16x3_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_long, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_void_p]
    return f


def _bound(K):
    # the slice-product tolerance of test_gpu_kernels.test_bf16x3_matches_slice_products
    return 1.0e-6 + 2.0e-9 * np.sqrt(K)


def test_noalloc_matches_sgemm_on_two_calls(cuda):
    torch = cuda
    f = _noalloc()
    stream = torch.cuda.current_stream()
    shapes = [(1024, 768, 1536, 11), (300, 200, 517, 12)]
    with emugemm.Handle(stream=stream.cuda_stream) as h:
        for M, N, K, seed in shapes:
            A = datagen.normal((M, K), seed)
            B = datagen.normal((K, N), seed + 100)
            dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
            c_new = torch.full((M, N), float("nan"), device="cuda")
            c_ref = torch.full((M, N), float("nan"), device="cuda")
            assert f(M, N, K, dA.data_ptr(), dB.data_ptr(), c_new.data_ptr(), stream.cuda_stream) == 0
            h.sgemm(M, N, K, dA, dB, c_ref, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
            torch.cuda.synchronize()
            new, ref = c_new.cpu().numpy(), c_ref.cpu().numpy()
            assert np.isfinite(new).all()
            assert np.array_equal(new, ref)
            R = oracle.gemm_f64(A, B)
            d = np.linalg.norm(new.astype(np.float64) - oracle.slice_product(A, B, 0)) / np.linalg.norm(R)
            assert d <= _bound(K)


def test_noalloc_rejects_problems_above_the_static_scratch(cuda):
    torch = cuda
    f = _noalloc()
    x = torch.zeros(16, device="cuda")
    # (Mp + Np) * Kp = (4096 + 4096) * 4096 = 32 Mi elements > 16 Mi
    assert f(4096, 4096, 4096, x.data_ptr(), x.data_ptr(), x.data_ptr(), 0) == 4
