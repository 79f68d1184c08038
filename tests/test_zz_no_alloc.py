"""The allocation-free bf16x3 entry point, emugemm_sgemm_bf16x3_noalloc, called through the C ABI.

Some callers cannot let a library call cudaMalloc: plugins inside an application whose memory pool has
reserved the device's memory, and latency-critical paths that must not risk an allocation (or its failure)
mid-run. For them the library computes the bf16x3 product in a fixed 64 MiB device array instead of its
grow-only workspace. This file checks, on two calls in a row with different shapes (so the second call
runs over the first call's leftovers in the shared array), that its output equals the output of the
existing emugemm_sgemm (forced BF16X3, single-CTA kernel) bit for bit, and that both sit within the
slice-product tolerance the other bf16x3 tests use; the same at the array's size limit, where K > 16384
stores the slices in K panels; that a problem one row above the limit is refused; and that a bounded wait
that gives up inside its kernel is reported by emugemm_noalloc_sync instead of passing as a success. It is
collected last so that a run stopping at the first failure has run every other test first; it also passes
alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

import datagen
import emugemm
import oracle

pytestmark = pytest.mark.gpu

TIMEOUT = 101   # EMUGEMM_STATUS_TIMEOUT


def _bound(K):
    # the slice-product tolerance of test_gpu_kernels.test_bf16x3_matches_slice_products
    return 1.0e-6 + 2.0e-9 * np.sqrt(K)


def _check_against_sgemm(torch, h, stream, M, N, K, seed):
    lib = emugemm.lib()
    A = datagen.normal((M, K), seed)
    B = datagen.normal((K, N), seed + 100)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    c_new = torch.full((M, N), float("nan"), device="cuda")
    c_ref = torch.full((M, N), float("nan"), device="cuda")
    assert lib.emugemm_sgemm_bf16x3_noalloc(M, N, K, dA.data_ptr(), dB.data_ptr(), c_new.data_ptr(),
                                            stream.cuda_stream) == 0
    assert lib.emugemm_noalloc_sync(stream.cuda_stream) == 0   # no bounded wait gave up
    h.sgemm(M, N, K, dA, dB, c_ref, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
    h.sync()
    new, ref = c_new.cpu().numpy(), c_ref.cpu().numpy()
    assert np.isfinite(new).all()
    assert np.array_equal(new, ref)
    R = oracle.gemm_f64(A, B)
    d = np.linalg.norm(new.astype(np.float64) - oracle.slice_product(A, B, 0)) / np.linalg.norm(R)
    assert d <= _bound(K)


def test_noalloc_matches_sgemm_on_two_calls(cuda):
    torch = cuda
    stream = torch.cuda.current_stream()
    with emugemm.Handle(stream=stream.cuda_stream) as h:
        h.set_kernels(tc_kernel="single")   # the kernel the allocation-free entry point runs
        for M, N, K, seed in [(1024, 768, 1536, 11), (300, 200, 517, 12)]:
            _check_against_sgemm(torch, h, stream, M, N, K, seed)


def test_noalloc_at_the_size_limit(cuda):
    """(256 + 256) * 32768 = 16 Mi slice elements, exactly the array; K = 32768 is stored in four K panels."""
    torch = cuda
    stream = torch.cuda.current_stream()
    with emugemm.Handle(stream=stream.cuda_stream) as h:
        h.set_kernels(tc_kernel="single")
        _check_against_sgemm(torch, h, stream, 256, 256, 32768, 21)


def test_noalloc_rejects_problems_above_the_static_scratch(cuda):
    torch = cuda
    lib = emugemm.lib()
    x = torch.zeros(16, device="cuda")
    # (Mp + Np) * Kp = (4096 + 4096) * 4096 = 32 Mi elements > 16 Mi
    assert lib.emugemm_sgemm_bf16x3_noalloc(4096, 4096, 4096, x.data_ptr(), x.data_ptr(), x.data_ptr(), 0) == 4
    # one row above the limit: Mp = 384, (384 + 256) * 32768 > 16 Mi
    assert lib.emugemm_sgemm_bf16x3_noalloc(257, 256, 32768, x.data_ptr(), x.data_ptr(), x.data_ptr(), 0) == 4


def test_noalloc_reports_a_timed_out_wait(cuda):
    """The testing hook makes the kernel's MMA issuer give up a 1 ms wait on a barrier nothing arrives on; the
    kernel unwinds and stores nothing. The call itself has already returned SUCCESS (it only enqueues), so the
    timeout must come back from emugemm_noalloc_sync; the next call computes the right product again."""
    torch = cuda
    lib = emugemm.lib()
    stream = torch.cuda.current_stream()
    M, N, K = 256, 512, 1024   # 8 chunks of 128 K: the stall comes before the second
    A = torch.from_numpy(datagen.normal((M, K), 31)).cuda()
    B = torch.from_numpy(datagen.normal((K, N), 32)).cuda()
    good = torch.full((M, N), float("nan"), device="cuda")
    assert lib.emugemm_sgemm_bf16x3_noalloc(M, N, K, A.data_ptr(), B.data_ptr(), good.data_ptr(),
                                            stream.cuda_stream) == 0
    assert lib.emugemm_noalloc_sync(stream.cuda_stream) == 0
    C = torch.full((M, N), float("nan"), device="cuda")
    emugemm.test_stall_next_launches(1)
    try:
        assert lib.emugemm_sgemm_bf16x3_noalloc(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(),
                                                stream.cuda_stream) == 0
        assert lib.emugemm_noalloc_sync(stream.cuda_stream) == TIMEOUT
    finally:
        emugemm.test_stall_next_launches(0)
    assert torch.isnan(C).all()                                    # the unwound launch stored nothing
    assert lib.emugemm_noalloc_sync(stream.cuda_stream) == 0       # the query cleared the word
    assert lib.emugemm_sgemm_bf16x3_noalloc(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr(),
                                            stream.cuda_stream) == 0
    assert lib.emugemm_noalloc_sync(stream.cuda_stream) == 0
    assert torch.equal(C, good)
