"""Row-sharded tropical GEMM across the GPUs of one node.

C = A (x) B where the rows of A (and of C / argmax) are split into contiguous
blocks, one per rank, and B is needed whole by every rank.  The only exchange
is one broadcast of B from its owner over NCCL (NVLink / NVSwitch on a B200
node); C and argmax stay sharded, so no reduction is needed.  This is the
multi-GPU layout of the engine; the reference itself has no multi-GPU path
(its sources make no collective calls).  Strided-batched GEMMs shard by
batch index instead and need no collective at all.

One process per GPU, plumbing by torch.distributed.  Nothing here waits on a
peer without a timeout: process groups are created with a finite timeout so a
rank that never joins, or dies between steps, surfaces as an exception on the
others instead of a hang.
"""
from datetime import timedelta
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _native as N

ROW_ALIGN = 128  # rows per CTA tile of the fast kernel


def shard_rows(m: int, world: int, rank: int, align: int = ROW_ALIGN) -> Tuple[int, int]:
    """[start, stop) of the rows of an m-row A owned by `rank`.

    Blocks are contiguous, ascending in rank, multiples of `align` except the
    last non-empty one, and as even as the alignment allows.
    """
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    units = (m + align - 1) // align
    base, extra = divmod(units, world)
    start_u = rank * base + min(rank, extra)
    stop_u = start_u + base + (1 if rank < extra else 0)
    return min(m, start_u * align), min(m, stop_u * align)


def init(backend: str = "nccl", timeout_s: float = 60.0, **kw) -> None:
    """init_process_group with a finite timeout (env:// rendezvous)."""
    if not dist.is_initialized():
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kw)


def broadcast_b(b: torch.Tensor, src: int = 0, group=None) -> torch.Tensor:
    """Make every rank's `b` equal to the src rank's (in place)."""
    dist.broadcast(b, src=src, group=group)
    return b


def sharded_matmul(semiring: str, a_local: torch.Tensor, b: torch.Tensor, src: int = 0, group=None,
                   with_argmax: bool = True,
                   compute: Optional[Callable] = None):
    """Broadcast B from `src`, then C_local = A_local (x) B on this rank.

    `a_local` is this rank's row block of A; `b` is a (K, N) buffer on every
    rank (its contents matter only on `src`).  Returns (C_local, argmax_local).
    `compute(semiring, a, b, with_argmax)` defaults to the engine's GEMM.
    """
    broadcast_b(b, src=src, group=group)
    fn = compute or N.gemm
    return fn(semiring, a_local, b, with_argmax)


def k_slices(k: int, chunks: int, align: int = 64):
    """[start, stop) bounds of `chunks` ascending K slices (multiples of
    `align` except the last), as even as the alignment allows."""
    if chunks < 1:
        raise ValueError("chunks must be >= 1")
    units = (k + align - 1) // align
    chunks = max(1, min(chunks, units))
    base, extra = divmod(units, chunks)
    bounds, u = [0], 0
    for i in range(chunks):
        u += base + (1 if i < extra else 0)
        bounds.append(min(k, u * align))
    return [(a, b) for a, b in zip(bounds, bounds[1:]) if b > a]


def pipelined_sharded_matmul(semiring: str, a_local: torch.Tensor, b: torch.Tensor, src: int = 0, group=None,
                             with_argmax: bool = True, chunks: int = 4,
                             first: Optional[Callable] = None, accumulate: Optional[Callable] = None):
    """sharded_matmul with the broadcast of B pipelined along K: B's K slices
    (contiguous row blocks of the row-major K x N buffer) go out as
    asynchronous broadcasts, and slice i is multiplied while slice i+1 is on
    the wire.  Slice 0 is an ordinary GEMM; each later slice updates C and
    argmax in place where one of its products strictly beats them, with the
    global k as index, so the result is bit-identical to one pass over the
    whole K (the reference's strict, first-k-wins rule).

    `first(semiring, a, b, with_argmax)` and
    `accumulate(semiring, a, b, c, argmax, k_offset)` default to the engine's
    gemm and gemm_accumulate (f32)."""
    first = first or N.gemm
    accumulate = accumulate or N.gemm_accumulate
    k = b.shape[0]
    if k == 0 or a_local.shape[1] != k:
        broadcast_b(b, src=src, group=group)
        return first(semiring, a_local, b, with_argmax)
    spans = k_slices(k, chunks)
    works = [dist.broadcast(b[spans[0][0]:spans[0][1]], src=src, group=group, async_op=True)]
    c = am = None
    for i, (s0, s1) in enumerate(spans):
        if i + 1 < len(spans):   # next slice on the wire while this one computes
            n0, n1 = spans[i + 1]
            works.append(dist.broadcast(b[n0:n1], src=src, group=group, async_op=True))
        works[i].wait()
        if i == 0:
            c, am = first(semiring, a_local[:, s0:s1], b[s0:s1], with_argmax)
        else:
            accumulate(semiring, a_local[:, s0:s1], b[s0:s1], c, am, s0)
    return c, am


def gather_rows(x_local: torch.Tensor, m: int, group=None) -> torch.Tensor:
    """All-gather row blocks (as produced by shard_rows) into the full matrix."""
    world = dist.get_world_size(group)
    rows = [shard_rows(m, world, r) for r in range(world)]
    maxr = max(stop - start for start, stop in rows)
    pad = torch.zeros((maxr,) + tuple(x_local.shape[1:]), dtype=x_local.dtype, device=x_local.device)
    pad[: x_local.shape[0]] = x_local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[: stop - start] for p, (start, stop) in zip(parts, rows)], dim=0)


def shard_batch(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of the batch indices of a strided-batched GEMM owned by
    `rank`: contiguous, ascending in rank, sizes differing by at most one."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def sharded_batched_matmul(semiring: str, a_local: torch.Tensor, b_local: torch.Tensor, with_argmax: bool = True,
                           compute: Optional[Callable] = None):
    """C[p] = A[p] (x) B[p] for this rank's batch slice (as given by
    shard_batch): every batch item is independent, so there is no exchange.
    `compute(semiring, a, b, with_argmax)` defaults to the engine's batched GEMM."""
    fn = compute or N.gemm_batched
    return fn(semiring, a_local, b_local, with_argmax)


def gather_batches(x_local: torch.Tensor, batch: int, group=None) -> torch.Tensor:
    """All-gather batch slices (as produced by shard_batch) into the full batch."""
    world = dist.get_world_size(group)
    spans = [shard_batch(batch, world, r) for r in range(world)]
    maxb = max(stop - start for start, stop in spans)
    pad = torch.zeros((maxb,) + tuple(x_local.shape[1:]), dtype=x_local.dtype, device=x_local.device)
    pad[: x_local.shape[0]] = x_local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([q[: stop - start] for q, (start, stop) in zip(parts, spans)], dim=0)
