"""The multi-GPU entry points of the C ABI on real GPUs with NCCL (the library's own communicator).

- One rank (runs on any single B200): emugemm_sgemm_rows with the modelled and with forced panel schedules, and
  emugemm_sgemm_ksplit, on a one-rank communicator; rows: identical bits to emugemm_sgemm; K-split: the FP64 partial
  rounded once, identical to emugemm_sgemm_partial_f64 + emugemm_reduce_f64.
- Two ranks (one process per GPU; skipped unless two sm_100 GPUs are visible): each rank's C rows equal a
  single-GPU emugemm_sgemm of the whole product bit for bit, for bf16x3 and fp16x3 and for ragged shapes whose row
  blocks differ by one row, with B moved by copy engines over peer memory and by NCCL, from either root, over
  several calls in a row (the received B equals the root's); a measured rho (hint -1) agrees with the single-GPU estimate; the K-split sits within
  the bf16x3 model error against FP64. NVLS stays off (NCCL_NVLS_ENABLE=0).
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import emugemm

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_one_rank_comm(cuda):
    torch = cuda
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    g = torch.Generator(device="cuda").manual_seed(7)
    M, N, K = 600, 1300, 2100
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(K, N, device="cuda", generator=g)
    hints = lambda: emugemm.EmuHints(1.0, 1.0, 0, 0.0, 0)  # noqa: E731
    with emugemm.Handle() as h:
        h.comm_init(1, 0, emugemm.comm_unique_id())
        assert h.comm_rows(M) == (0, M) and h.comm_krange(K) == (0, K)
        for force in (emugemm.BF16X3, emugemm.FP16X3, emugemm.NATIVE_FP32):
            ref = torch.full((M, N), float("nan"), device="cuda")
            h.sgemm(M, N, K, A, B, ref, force=force, hints=hints())
            for panels in (0, 3, 16):
                h.set_attr(emugemm.ATTR_ROWS_PANELS, panels)
                C = torch.full((M, N), float("nan"), device="cuda")
                p, _ = h.sgemm_rows(M, N, K, A, K, B, N, C, N, root=0, force=force, hints=hints())
                h.sync()
                assert p.chosen == force
                assert torch.equal(C, ref), (force, panels)
        h.set_attr(emugemm.ATTR_ROWS_PANELS, 0)
        # measured hints through the rows path: the same absmax and (one rank) the same rho as emugemm_sgemm
        C = torch.empty((M, N), device="cuda")
        p1, hn1 = h.sgemm_rows(M, N, K, A, K, B, N, C, N, hints=emugemm.EmuHints(-1, -1, 0, -1.0, 64))
        p2, hn2 = h.sgemm(M, N, K, A, B, C, hints=emugemm.EmuHints(-1, -1, 0, -1.0, 64))
        h.sync()
        assert hn1.a_absmax == hn2.a_absmax and hn1.b_absmax == hn2.b_absmax
        assert abs(hn1.rho - hn2.rho) <= 1e-5 * hn2.rho
        assert p1.chosen == p2.chosen
        # K-split with one rank: the FP64 partial rounded once
        P = torch.empty((M, N), dtype=torch.float64, device="cuda")
        h.partial_f64(M, N, K, A, K, B, N, P, emugemm.BF16X3, 1)
        want = torch.empty((M, N), device="cuda")
        h.reduce_f64(M, N, 1, P, want)
        C = torch.full((M, N), float("nan"), device="cuda")
        h.sgemm_ksplit(M, N, K, A, K, B, N, C, N, root=0, scheme=emugemm.BF16X3)
        h.sync()
        assert torch.equal(C, want)
        h.comm_destroy()


def _worker(rank, world, port, q):
    try:
        _work(rank, world, port, q)
    except BaseException as exc:  # noqa: BLE001 - reported to the parent instead of leaving it waiting
        q.put((rank, {"error": repr(exc)}))
        raise


def _work(rank, world, port, q):
    import datetime
    import sys

    sys.path.insert(0, os.path.join(ROOT, "emugemm-cdna_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import torch.distributed as dist

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    import emugemm
    import multigpu

    res = {}
    hints = lambda: emugemm.EmuHints(1.0, 1.0, 0, 0.0, 0)  # noqa: E731
    with emugemm.Handle() as h:
        multigpu.init_comm(h)
        for case, (M, N, K, force) in enumerate([(1024, 1536, 2048, emugemm.BF16X3), (1001, 1300, 4100,
                                                                                     emugemm.BF16X3),
                                                (777, 2048, 3000, emugemm.FP16X3)]):
            g = torch.Generator(device="cuda").manual_seed(3 + case)
            A = torch.randn(M, K, device="cuda", generator=g)
            B = torch.randn(K, N, device="cuda", generator=g)
            ref = torch.empty(M, N, device="cuda")
            h.sgemm(M, N, K, A, B, ref, force=force, hints=hints())
            r0, r1 = h.comm_rows(M)
            assert (r0, r1) == multigpu.row_range(M, rank, world)
            C_local = torch.full((r1 - r0, N), float("nan"), device="cuda")
            # B by copy engines over peer memory (default) and by NCCL broadcast; several calls in a row, so the
            # double-buffered staging and its release flags cycle; root 1 as well as root 0
            for panels, comm_sms, nccl, root in ((0, 0, 0, 0), (5, 0, 0, 0), (3, 0, 0, 1), (0, 0, 0, 0),
                                                 (0, 8, 1, 0), (5, 0, 1, 1), (7, 0, 0, 0)):
                h.set_attr(emugemm.ATTR_ROWS_PANELS, panels)
                h.set_attr(emugemm.ATTR_COMM_SMS, comm_sms)    # a smaller GEMM grid: the same bits
                h.set_attr(emugemm.ATTR_BCAST_NCCL, nccl)
                Bb = B.clone() if rank == root else torch.full_like(B, float("nan"))
                C_local.fill_(float("nan"))
                h.sgemm_rows(M, N, K, A[r0:r1].contiguous(), K, Bb, N, C_local, N, root=root, force=force,
                             hints=hints())
                assert h.sync_status() == 0
                res[f"rows_equal_{case}_{panels}_{comm_sms}_{nccl}_{root}"] = bool(torch.equal(C_local, ref[r0:r1]))
                res[f"b_received_{case}_{panels}_{nccl}_{root}"] = bool(torch.equal(Bb, B))
        h.set_attr(emugemm.ATTR_ROWS_PANELS, 0)
        h.set_attr(emugemm.ATTR_COMM_SMS, 0)
        h.set_attr(emugemm.ATTR_BCAST_NCCL, 0)
        # rho measured over both row blocks against the single-GPU estimate
        M, N, K = 1024, 1024, 2048
        g = torch.Generator(device="cuda").manual_seed(11)
        A = torch.randn(M, K, device="cuda", generator=g)
        B = torch.randn(K, N, device="cuda", generator=g)
        rho1 = h.estimate_rho(M, N, K, A, B, 64)
        r0, r1 = h.comm_rows(M)
        C_local = torch.empty((r1 - r0, N), device="cuda")
        _, hn = h.sgemm_rows(M, N, K, A[r0:r1].contiguous(), K, B if rank == 0 else None, N, C_local, N,
                             hints=emugemm.EmuHints(-1, -1, 0, -1.0, 64))
        torch.cuda.synchronize()
        res["rho_rel"] = abs(hn.rho - rho1) / rho1
        # K split, C on every rank
        M, N, K = 1024, 1536, 6000
        g = torch.Generator(device="cuda").manual_seed(13)
        A = torch.randn(M, K, device="cuda", generator=g)
        B = torch.randn(K, N, device="cuda", generator=g)
        k0, k1 = h.comm_krange(K)
        assert (k0, k1) == multigpu.k_range(K, rank, world)
        C = torch.full((M, N), float("nan"), device="cuda")
        h.sgemm_ksplit(M, N, K, A[:, k0:k1].contiguous(), k1 - k0, B[k0:k1].contiguous(), N, C, N, root=-1,
                       scheme=emugemm.BF16X3)
        torch.cuda.synchronize()
        R = A.double() @ B.double()
        res["ksplit_err"] = ((C.double() - R).norm() / R.norm()).item()
        res["pred"] = emugemm.lib().emugemm_model_err(emugemm.BF16X3, K, world)
        h.comm_destroy()
    q.put((rank, res))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_entry_points():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive
    out = dict(q.get(timeout=30) for _ in range(2))
    assert not any("error" in v for v in out.values()), out
    for r in (0, 1):
        for k, v in out[r].items():
            if k.startswith(("rows_equal", "b_received")):
                assert v, (r, k, out)
        assert out[r]["rho_rel"] < 1e-4, out
        assert out[r]["ksplit_err"] <= out[r]["pred"], out
