"""Failure reporting on the GPU without a fault: a bounded device-side wait that gives up.

The reference maps a failed device operation to a status code (src/emugemm.cpp:13, HC). Here every mbarrier
wait of the tensor-core kernels is bounded; a wait that gives up sets a bit in the handle's mapped error word,
the kernel drains its loads and MMAs in flight, frees TMEM and returns, and emugemm_sync reports
EMUGEMM_STATUS_TIMEOUT. The testing hook emugemm_test_stall_next_launches makes that happen on purpose: the
single-CTA kernel's MMA issuer waits before its second 128-K chunk on a barrier nothing arrives on, with a
1 ms limit (and the TMA-fed FP32 kernel's threads before its second k-block). Nothing faults, traps or hangs, and
the context stays usable.
"""
from __future__ import annotations

import numpy as np
import pytest

import datagen
import emugemm
import oracle

pytestmark = pytest.mark.gpu

TIMEOUT = 101   # EMUGEMM_STATUS_TIMEOUT


@pytest.mark.parametrize("shape", [(256, 512, 1024), (300, 260, 4100)])
def test_timed_out_wait_is_reported_and_the_handle_recovers(cuda, handle, shape):
    torch = cuda
    M, N, K = shape
    handle.set_kernels(tc_kernel="single")
    A = torch.from_numpy(datagen.normal((M, K), 41 + M)).cuda()
    B = torch.from_numpy(datagen.normal((K, N), 42 + N)).cuda()
    hints = emugemm.EmuHints(1, 1, 0, 0, 0)
    good = torch.full((M, N), float("nan"), device="cuda")
    handle.sgemm(M, N, K, A, B, good, force=emugemm.BF16X3, hints=hints)
    handle.sync()

    C = torch.full((M, N), float("nan"), device="cuda")
    n0 = emugemm.launch_count()
    emugemm.test_stall_next_launches(1)
    try:
        handle.sgemm(M, N, K, A, B, C, force=emugemm.BF16X3, hints=hints)   # enqueues: SUCCESS
        assert handle.sync_status() == TIMEOUT
    finally:
        emugemm.test_stall_next_launches(0)
    assert emugemm.launch_count() - n0 == 3          # both splits and the GEMM ran; the GEMM gave up
    assert torch.isnan(C).all()                      # every CTA unwound before its first store
    assert handle.sync_status() == 0                 # the error word was read and cleared

    handle.sgemm(M, N, K, A, B, C, force=emugemm.BF16X3, hints=hints)
    handle.sync()
    assert torch.equal(C, good)                      # same handle, same workspace: the right product again
    assert np.isfinite(C.cpu().numpy()).all()


def test_stall_hook_is_consumed_by_one_launch(cuda, handle):
    """The hook counts launches: after the stalled one, the next launch runs normally."""
    torch = cuda
    M, N, K = 128, 256, 512
    handle.set_kernels(tc_kernel="single")
    A = torch.from_numpy(datagen.normal((M, K), 51)).cuda()
    B = torch.from_numpy(datagen.normal((K, N), 52)).cuda()
    C = torch.empty((M, N), device="cuda")
    hints = emugemm.EmuHints(1, 1, 0, 0, 0)
    emugemm.test_stall_next_launches(1)
    try:
        handle.sgemm(M, N, K, A, B, C, force=emugemm.BF16X3, hints=hints)
        handle.sgemm(M, N, K, A, B, C, force=emugemm.BF16X3, hints=hints)
        assert handle.sync_status() == TIMEOUT     # the first launch timed out, the word is sticky until read
    finally:
        emugemm.test_stall_next_launches(0)
    assert np.isfinite(C.cpu().numpy()).all()      # the second launch wrote all of C


def test_fp32_tma_kernel_timed_out_wait_is_reported(cuda, handle):
    """The TMA-fed FP32 kernel (32 x 64 tiles) under the same hook: every thread gives up a 1 ms wait once its first
    k-blocks are issued, thread 0 issues no further k-block, the loads already in flight land before the CTAs exit,
    and emugemm_sync reports TIMEOUT; the next call gives the right FP64 sums again (bit-exact against the oracle)."""
    torch = cuda
    M, N, K, chunks = 256, 256, 4096, 4
    handle.set_kernels(fp32_tile=3264)
    A = datagen.uniform((M, K), 61)
    B = datagen.uniform((K, N), 62)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    G = emugemm.fp32_groups(M, N, K, chunks, sms, tile=3264)
    want = oracle.fp32_chunked(A, B, chunks, cpg=oracle.group_size(K, chunks, G), f64=True)
    P64 = torch.empty((M, N), dtype=torch.float64, device="cuda")
    n0 = emugemm.launch_count()
    emugemm.test_stall_next_launches(1)
    try:
        handle.partial_f64(M, N, K, dA, K, dB, N, P64, emugemm.FP32_CHUNKED, chunks)
        assert handle.sync_status() == TIMEOUT
    finally:
        emugemm.test_stall_next_launches(0)
    assert emugemm.launch_count() > n0
    assert handle.sync_status() == 0
    P64.fill_(float("nan"))
    handle.partial_f64(M, N, K, dA, K, dB, N, P64, emugemm.FP32_CHUNKED, chunks)
    handle.sync()
    assert np.array_equal(P64.cpu().numpy(), want)
