"""tg_sharded_gemm with a real NCCL communicator: two processes, one GPU
each, the broadcast callback calling torch.distributed.broadcast (NCCL) on
the rank's B.  Each rank checks its row block against the unsharded GEMM
computed on its own GPU from the same seeded inputs, bit for bit.  Needs two
GPUs (skipped otherwise)."""
import ctypes
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, semi, dtype_name):
    import torch.distributed as dist
    from tropical_gemm import _native as N
    from tropical_gemm.distributed import init, shard_rows
    from test_abi import BCAST, _sharded_lib

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    init("nccl", timeout_s=60, device_id=dev)
    try:
        dtype = getattr(torch, dtype_name)
        g = torch.Generator(device=dev).manual_seed(7)
        m, k, n = 1000, 1300, 700
        if dtype.is_floating_point:
            a = torch.randn((m, k), generator=g, device=dev, dtype=dtype)
            b_full = torch.randn((k, n), generator=g, device=dev, dtype=dtype)
        else:
            a = torch.randint(-500, 500, (m, k), generator=g, device=dev, dtype=dtype)
            b_full = torch.randint(-500, 500, (k, n), generator=g, device=dev, dtype=dtype)
        c_ref, am_ref = N.gemm(semi, a, b_full, True)
        s, e = shard_rows(m, world, rank)
        b = b_full.clone() if rank == 0 else torch.zeros_like(b_full)   # only the root's B is meaningful

        def cb(buf, nbytes, root, stream, ctx):
            if buf != b.data_ptr() or nbytes != b.numel() * b.element_size():
                return 1
            dist.broadcast(b, src=root)   # NCCL; the current stream waits for it
            return 0

        f = BCAST(cb)
        L = _sharded_lib()
        a_loc = a[s:e].contiguous()
        c = torch.empty((e - s, n), device=dev, dtype=dtype)
        am = torch.empty((e - s, n), device=dev, dtype=torch.int32)
        st = torch.cuda.current_stream(dev).cuda_stream
        N.check(L.tg_sharded_gemm(N.SEMIRINGS[semi], N.DTYPES[dtype], e - s, n, k, a_loc.data_ptr(), k,
                                  b.data_ptr(), n, c.data_ptr(), n, am.data_ptr(), 0, f, None, st))
        torch.cuda.synchronize(dev)
        assert torch.equal(b, b_full), f"rank {rank}: B not broadcast"
        assert torch.equal(c, c_ref[s:e]) and torch.equal(am, am_ref[s:e]), f"rank {rank}: row block differs"
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("semi,dtype_name", [("maxplus", "float32"), ("minplus", "int32"), ("maxmul", "float64")])
def test_sharded_gemm_over_nccl_two_ranks(semi, dtype_name):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port(), semi, dtype_name), nprocs=2, join=True)
