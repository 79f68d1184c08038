"""The multi-GPU drivers on real GPUs with NCCL: two ranks (one process per GPU), row blocks of A with B
broadcast from rank 0 in column panels, and the K-split with FP64 partials summed by NCCL. Checked against
a single-GPU emugemm_sgemm of the same product (row blocks: identical bits; K-split: within the bf16x3
model error against FP64). Skipped unless two sm_100 GPUs are visible. NVLS stays off (NCCL_NVLS_ENABLE=0)."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
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
    g = torch.Generator(device="cuda").manual_seed(3)
    M, N, K = 1024, 1536, 2048
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(K, N, device="cuda", generator=g)
    with emugemm.Handle() as h:
        ref = torch.empty(M, N, device="cuda")
        h.sgemm(M, N, K, A, B, ref, force=emugemm.BF16X3, hints=emugemm.EmuHints(1, 1, 0, 0, 0))
        r0, r1 = multigpu.row_range(M, rank, world)
        Bb = B.clone() if rank == 0 else torch.empty_like(B)
        C_local = torch.empty(r1 - r0, N, device="cuda")
        multigpu.row_sharded(A[r0:r1].contiguous(), Bb, C_local, src=0, panel=512, handle=h,
                             scheme=emugemm.BF16X3)
        torch.cuda.synchronize()
        # the panel GEMMs are column blocks of the same tensor-core kernel: identical bits
        res["rows_equal"] = bool(torch.equal(C_local, ref[r0:r1]))
        k0, k1 = multigpu.k_range(K, rank, world)
        C = torch.empty(M, N, device="cuda")
        multigpu.k_split(A[:, k0:k1].contiguous(), B[k0:k1].contiguous(), C, M=M, N=N, handle=h,
                         scheme=emugemm.BF16X3, all_ranks=True)
        torch.cuda.synchronize()
        R = A.double() @ B.double()
        res["ksplit_err"] = ((C.double() - R).norm() / R.norm()).item()
        res["pred"] = emugemm.lib().emugemm_model_err(emugemm.BF16X3, K, world)
    q.put((rank, res))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_drivers():
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
    out = dict(q.get() for _ in range(2))
    for r in (0, 1):
        assert out[r]["rows_equal"], out
        assert out[r]["ksplit_err"] <= out[r]["pred"], out
