"""tg_sharded_gemm: one rank's part of the row-sharded GEMM, with the
broadcast of B supplied by the caller.  Two ranks are emulated on one GPU,
one after the other (their kernels never wait on each other): rank 1's
callback copies rank 0's B into its own buffer, as ncclBroadcast would.
The stacked row blocks must equal the unsharded GEMM bit for bit."""
import ctypes

import pytest
import torch

from tropical_gemm import _native as N
from tropical_gemm.distributed import shard_rows
from test_abi import BCAST, _sharded_lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.int32])
@pytest.mark.parametrize("semi", ["maxplus", "minplus"])
def test_two_ranks_on_one_gpu_match_unsharded(semi, dtype):
    L = _sharded_lib()
    g = torch.Generator(device="cuda").manual_seed(5)
    m, k, n, world = 300, 700, 260, 2
    if dtype.is_floating_point:
        a = torch.randn((m, k), generator=g, device="cuda", dtype=dtype)
        b_root = torch.randn((k, n), generator=g, device="cuda", dtype=dtype)
    else:
        a = torch.randint(-500, 500, (m, k), generator=g, device="cuda", dtype=dtype)
        b_root = torch.randint(-500, 500, (k, n), generator=g, device="cuda", dtype=dtype)
    c_ref, am_ref = N.gemm(semi, a, b_root, True)
    st = torch.cuda.current_stream().cuda_stream
    cs, ams = [], []
    for rank in range(world):
        s, e = shard_rows(m, world, rank)
        b = b_root.clone() if rank == 0 else torch.zeros_like(b_root)

        def cb(buf, nbytes, root, stream, ctx, b=b):
            assert root == 0 and buf == b.data_ptr() and nbytes == b.numel() * b.element_size()
            if rank != root:
                b.copy_(b_root)   # stands in for ncclBroadcast on `stream` (torch's current stream)
            return 0

        f = BCAST(cb)
        c = torch.empty((e - s, n), device="cuda", dtype=dtype)
        am = torch.empty((e - s, n), device="cuda", dtype=torch.int32)
        a_loc = a[s:e].contiguous()
        N.check(L.tg_sharded_gemm(N.SEMIRINGS[semi], N.DTYPES[dtype], e - s, n, k, a_loc.data_ptr(), k,
                                  b.data_ptr(), n, c.data_ptr(), n, am.data_ptr(), 0, f, None, st))
        cs.append(c)
        ams.append(am)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(cs), c_ref) and torch.equal(torch.cat(ams), am_ref)
