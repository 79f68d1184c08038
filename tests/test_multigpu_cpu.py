"""Multi-GPU driver logic on CPU: two gloo ranks as spawned processes, with the per-rank GEMM injected as an
FP64 matmul, so the partitioning, panel packing, broadcast order and FP64 reduction are checked without a GPU.
A rank that leaves before the collective must make the other rank fail with an error, not hang."""
from __future__ import annotations

import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=30):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, os.path.join(ROOT, "emugemm-cdna_b200"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _row_worker(rank, world, port, M, N, K, panel, q):
    dist = _init(rank, world, port)
    import multigpu

    g = torch.Generator().manual_seed(5)
    A = torch.randn(M, K, generator=g)
    Bfull = torch.randn(K, N, generator=g)
    r0, r1 = multigpu.row_range(M, rank, world)
    A_local = A[r0:r1].contiguous()
    B = Bfull.clone() if rank == 0 else torch.full((K, N), float("nan"))
    C_local = torch.full((r1 - r0, N), float("nan"))

    def gemm(m, n, k, A_, lda, B_, ldb, C_, ldc):
        assert B_.is_contiguous() and B_.shape == (k, n) and ldb == n and ldc == N
        C_.copy_((A_.double() @ B_.double()).float())

    st = multigpu.row_sharded(A_local, B, C_local, src=0, panel=panel, gemm=gemm, keep_b=True)
    ref = (A[r0:r1].double() @ Bfull.double()).float()
    ok = torch.equal(C_local, ref) and torch.equal(B, Bfull)
    q.put((rank, ok, st.n_panels))
    dist.destroy_process_group()


def _ksplit_worker(rank, world, port, M, N, K, q):
    dist = _init(rank, world, port)
    import multigpu

    g = torch.Generator().manual_seed(9)
    A = torch.randn(M, K, generator=g)
    B = torch.randn(K, N, generator=g)
    k0, k1 = multigpu.k_range(K, rank, world)

    def partial(M_, N_, K_, A_, B_, P_):
        P_.copy_(A_.double() @ B_.double())

    def reduce(M_, N_, P_, C_):
        C_.copy_(P_.float())

    C = torch.empty(M, N)
    P = multigpu.k_split(A[:, k0:k1].contiguous(), B[k0:k1].contiguous(), C, M=M, N=N, partial=partial,
                         reduce=reduce, all_ranks=True)
    full = A.double() @ B.double()
    ok = bool(torch.allclose(P, full, rtol=1e-12, atol=1e-9)) and torch.equal(C, P.float())
    q.put((rank, ok, (k0, k1)))
    dist.destroy_process_group()


def _dead_peer_worker(rank, world, port, q):
    dist = _init(rank, world, port, timeout_s=5)
    import multigpu

    if rank == 1:
        dist.barrier()
        os._exit(0)          # leaves between steps, before the next collective
    dist.barrier()
    try:
        A = torch.randn(4, 8)
        B = torch.randn(8, 6)
        C = torch.empty(4, 6)
        multigpu.row_sharded(A, B, C, src=0, panel=3, gemm=lambda *a: None)
        multigpu.k_split(A, B, C, M=4, N=6, partial=lambda *a: None, reduce=lambda *a: None)
        q.put((rank, "no error"))
    except Exception as e:   # noqa: BLE001 - any collective error is the expected outcome
        q.put((rank, "error: " + type(e).__name__))


def _run(target, args, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    out = []
    while not q.empty():
        out.append(q.get())
    return out, alive


def test_partitions():
    sys.path.insert(0, os.path.join(ROOT, "emugemm-cdna_b200"))
    import multigpu

    for M, world in ((10, 3), (32768, 8), (5, 8)):
        rs = [multigpu.row_range(M, r, world) for r in range(world)]
        assert rs[0][0] == 0 and rs[-1][1] == M
        assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
    for K, world in ((1048576, 8), (1000, 3), (64, 4)):
        ks = [multigpu.k_range(K, r, world) for r in range(world)]
        assert ks[0][0] == 0 and ks[-1][1] == K
        assert all(k[0] % 64 == 0 for k in ks)
    assert multigpu.panels(10, 4) == [(0, 4), (4, 8), (8, 10)]


@pytest.mark.parametrize("shape", [(37, 29, 41, 8), (64, 256, 32, 256), (5, 7, 3, 2)])
def test_row_sharded_gloo(shape):
    out, alive = _run(_row_worker, shape)
    assert not alive
    assert len(out) == 2 and all(o[1] for o in out), out


def test_k_split_gloo():
    out, alive = _run(_ksplit_worker, (24, 20, 300))
    assert not alive
    assert len(out) == 2 and all(o[1] for o in out), out


def test_rank_leaving_makes_peer_fail_not_hang():
    out, alive = _run(_dead_peer_worker, (), timeout=90)
    assert not alive, "a rank hung after its peer left"
    res = dict(out)
    assert res.get(0, "").startswith("error"), out


@pytest.mark.parametrize("M,world,N,K", [(16384, 2, 8192, 8192), (65536, 8, 8192, 8192), (32768, 8, 32768, 32768),
                                         (1000, 3, 1300, 2100), (5, 2, 100, 64), (32768, 4, 32768, 8192)])
def test_rows_panel_schedule(M, world, N, K):
    """emugemm_rows_panels (the column panels of emugemm_sgemm_rows, computed alike on every rank): contiguous,
    covering [0, N), whole 256-column tiles except the last, at most 16; a forced count gives equal panels."""
    import emugemm

    for forced in (0, 1, 3, 16):
        p = emugemm.rows_panels(M, world, N, K, 148, forced)
        assert 1 <= len(p) <= 16
        assert p[0][0] == 0 and p[-1][1] == N
        assert all(a[1] == b[0] for a, b in zip(p, p[1:]))
        assert all(n0 % 256 == 0 and n1 > n0 for n0, n1 in p)
        if forced:
            assert len(p) == min(forced, -(-N // 256))
    # the schedule is a function of the whole product, so every rank computes the same one
    assert emugemm.rows_panels(M, world, N, K) == emugemm.rows_panels(M, world, N, K)
