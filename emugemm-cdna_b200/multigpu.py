"""Multi-GPU drivers of the emulated SGEMM: one process per GPU.

The product path is the library's own C ABI (emugemm_sgemm_rows / emugemm_sgemm_ksplit over its NCCL communicator);
init_comm() joins a handle to it, sharing the communicator id over an existing torch.distributed group.

The functions below restate the same partitioning on torch.distributed with an injectable GEMM, so that the
partitioning, panel order and FP64 reduction run on CPU (gloo) in tests:

row_sharded   C = A*B with the rows of A (and C) split across ranks and B held by one rank. B travels in
              column panels: rank `src` packs B[:, n0:n1] into a contiguous panel and NCCL broadcasts it; each
              rank's GEMM of panel j (emugemm_sgemm_ex on the panel, writing C[:, n0:n1] in place) starts as
              soon as that panel has arrived, so the broadcast of later panels overlaps the GEMMs of earlier
              ones. No data-path collective besides the broadcast.
k_split       C = A*B with K split across ranks: rank g holds A[:, Kg] and B[Kg, :], computes its partial product
              in FP64 (emugemm_sgemm_partial_f64), the partials are summed with NCCL in FP64, and one final
              rounding gives C (emugemm_reduce_f64). With bf16x3 per rank the error model sees G = world size
              chunks summed in FP64.
The GEMM callables are injectable so the partitioning and collective logic runs on CPU (gloo) in tests.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


def init_comm(handle, group=None, max_ctas: int = 0) -> None:
    """Join `handle` to the library's NCCL communicator over the ranks of `group` (rank 0 makes the id, a
    torch.distributed broadcast shares it)."""
    import emugemm

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    obj = [emugemm.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    handle.comm_init(world, rank, obj[0], max_ctas)


def row_range(M: int, rank: int, world: int) -> tuple[int, int]:
    """Rows of A owned by `rank`: contiguous blocks, the first M % world ranks one row longer."""
    base, extra = divmod(M, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def k_range(K: int, rank: int, world: int, align: int = 64) -> tuple[int, int]:
    """K range of `rank` for the K-split: blocks aligned to `align` so every rank's slices are whole k-blocks."""
    blocks = -(-K // align)
    b0, b1 = row_range(blocks, rank, world)
    return min(K, b0 * align), min(K, b1 * align)


def panels(N: int, panel: int) -> list[tuple[int, int]]:
    return [(n0, min(N, n0 + panel)) for n0 in range(0, N, panel)]


@dataclass
class PanelStats:
    n_panels: int
    bytes_broadcast: int


def _emugemm_ex(handle, scheme: int):
    """Panel GEMM through emugemm_sgemm_ex. The first panel splits A; later panels pass a_is_reused so the
    library keeps A's slices instead of splitting the same rows again."""
    import emugemm

    calls = [0]

    def gemm(M, N, K, A, lda, B, ldb, C, ldc):
        reused = 1 if calls[0] > 0 else 0
        calls[0] += 1
        handle.sgemm_ex(M, N, K, A, lda, B, ldb, C, ldc, force=scheme,
                        hints=emugemm.EmuHints(1.0, 1.0, reused, 0.0, 0))
    return gemm


def row_sharded(A_local: torch.Tensor, B: torch.Tensor, C_local: torch.Tensor, *, src: int = 0,
                panel: int = 2048, gemm: Callable | None = None, handle=None, scheme: int = 3,
                keep_b: bool = False, group=None) -> PanelStats:
    """C_local = A_local * B with B broadcast from `src` in column panels.

    A_local: (m x K) rows of A owned by this rank; B: (K x N), valid on `src` (on other ranks it is only written
    when keep_b is set); C_local: (m x N). `gemm(M, N, K, A, lda, B, ldb, C, ldc)` computes one panel into the
    column block of C_local (default: emugemm_sgemm_ex with `scheme` on `handle`)."""
    if gemm is None:
        gemm = _emugemm_ex(handle, scheme)
    rank = dist.get_rank(group)
    m, K = A_local.shape
    N = B.shape[1]
    plist = panels(N, panel)
    bufs = []
    works = []
    for (n0, n1) in plist:
        buf = B[:, n0:n1].contiguous() if rank == src else torch.empty((K, n1 - n0), dtype=B.dtype,
                                                                       device=B.device)
        bufs.append(buf)
        works.append(dist.broadcast(buf, src=src, group=group, async_op=True))
    for (n0, n1), buf, w in zip(plist, bufs, works):
        w.wait()      # the compute stream waits for this panel; later broadcasts keep going
        if m > 0:
            gemm(m, n1 - n0, K, A_local, K, buf, n1 - n0, C_local[:, n0:n1], N)
        if keep_b and rank != src:
            B[:, n0:n1].copy_(buf)
    return PanelStats(len(plist), sum(b.numel() * b.element_size() for b in bufs))


def k_split(A_local: torch.Tensor, B_local: torch.Tensor, C: torch.Tensor | None, *, M: int, N: int,
            partial: Callable | None = None, reduce: Callable | None = None, handle=None, scheme: int = 3,
            chunks: int = 1, all_ranks: bool = False, group=None, P: torch.Tensor | None = None) -> torch.Tensor:
    """C = sum over ranks of A_local * B_local, partials in FP64 summed by NCCL, one rounding to FP32.

    A_local: (M x Kg), B_local: (Kg x N). Returns the FP64 sum (valid on rank 0, or on all ranks with
    all_ranks=True); C (M x N, FP32) is written on the ranks where the sum is valid. P: optional (M x N) FP64
    buffer for the partial and the sum, reused across calls (the partial overwrites all of it)."""
    if partial is None:
        def partial(M_, N_, K_, A_, B_, P_):
            handle.partial_f64(M_, N_, K_, A_, K_, B_, N_, P_, scheme, chunks)
    if reduce is None:
        def reduce(M_, N_, P_, C_):
            handle.reduce_f64(M_, N_, 1, P_, C_)
    Kg = A_local.shape[1]
    if P is None:
        P = torch.zeros((M, N), dtype=torch.float64, device=A_local.device)
    if Kg > 0:
        partial(M, N, Kg, A_local, B_local, P)
    else:
        P.zero_()
    if all_ranks:
        dist.all_reduce(P, op=dist.ReduceOp.SUM, group=group)
    else:
        dist.reduce(P, dst=0, op=dist.ReduceOp.SUM, group=group)
    if (all_ranks or dist.get_rank(group) == 0) and C is not None:
        reduce(M, N, P, C)
    return P
