"""All-pairs shortest paths by repeated tropical squaring on the GPU.

The reference demonstrates APSP as D^2 = D (x) D, D^4 = D^2 (x) D^2 over
MinPlus, with argmax giving the intermediate node of each squaring
(crates/tropical-gemm/examples/shortest_path.rs:33-74); on its GPU path every
step is a separate allocating, synchronising call
(tropical_matmul_gpu_with_ctx_and_argmax, crates/tropical-gemm-cuda/src/lib.rs:425-445).
Here the squarings run back to back on the current stream in ping-pong
buffers, keeping each step's argmax (int32) for path reconstruction.

Integer graphs use the reference's GPU convention: a missing edge is the
MinPlus sentinel 46340 and results never exceed it (a path is either shorter
than 46340 or reported as missing).  Float graphs use +inf.
"""
import math
from typing import List, Optional, Tuple

import torch

from . import _native as N

I32_INF = 46340


def squarings_needed(n: int) -> int:
    """ceil(log2(n - 1)) squarings cover every simple path of an n-node graph."""
    return max(0, math.ceil(math.log2(max(1, n - 1))))


def all_pairs_shortest_paths(d: torch.Tensor, squarings: Optional[int] = None, with_argmax: bool = True,
                             stop_when_stable: bool = False) -> Tuple[torch.Tensor, List[torch.Tensor]]:
    """Repeated MinPlus squaring of the (n x n) distance matrix `d` (CUDA, f32/f64/i32/i64).

    Returns (D^(2^s), [argmax of step 1, ..., argmax of step s]); argmax[t][i, j]
    is the intermediate node k of the winning D_t[i, k] + D_t[k, j] (lowest k
    among ties, 0 when no path -- the reference's rule).  With
    stop_when_stable the loop ends early once a squaring changes nothing
    (one device-to-host flag read per step).
    """
    if d.dim() != 2 or d.shape[0] != d.shape[1]:
        raise ValueError(f"expected a square distance matrix, got shape {tuple(d.shape)}")
    if not d.is_cuda:
        raise RuntimeError("all_pairs_shortest_paths needs a CUDA tensor")
    n = d.shape[0]
    s = squarings_needed(n) if squarings is None else int(squarings)
    cur = d.contiguous().clone()
    nxt = torch.empty_like(cur)
    argmaxes: List[torch.Tensor] = []
    lib = N.lib()
    stream = torch.cuda.current_stream(d.device).cuda_stream
    for _ in range(s):
        am = torch.empty((n, n), dtype=torch.int32, device=d.device) if with_argmax else None
        with torch.cuda.device(d.device):
            N.check(lib.tg_gemm(N.SEMIRINGS["minplus"], N.DTYPES[cur.dtype], N.ROW_MAJOR, n, n, n,
                                cur.data_ptr(), n, cur.data_ptr(), n, nxt.data_ptr(), n,
                                am.data_ptr() if am is not None else None, stream))
        if am is not None:
            argmaxes.append(am)
        cur, nxt = nxt, cur
        if stop_when_stable and torch.equal(cur, nxt):
            break
    return cur, argmaxes


def reconstruct_path(i: int, j: int, argmaxes: List[torch.Tensor], dists: Optional[List[torch.Tensor]] = None
                     ) -> List[int]:
    """Node sequence of the path i -> j encoded by the per-squaring argmaxes.

    Step t splits a path of D_t into halves through argmax[t-1][i, j]; the
    recursion bottoms out at the input matrix (a direct edge, or i == j).
    Consecutive duplicates (a zero-length self-step) are removed.
    """
    ams = [a.cpu() for a in argmaxes]

    def rec(a: int, b: int, level: int) -> List[int]:
        if level == 0:
            return [a, b]
        k = int(ams[level - 1][a, b])
        left = rec(a, k, level - 1)
        right = rec(k, b, level - 1)
        return left + right[1:]

    path = rec(i, j, len(ams))
    out = [path[0]]
    for v in path[1:]:
        if v != out[-1]:
            out.append(v)
    return out
