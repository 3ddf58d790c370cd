"""Multi-rank host logic of the row-sharded GEMM on CPU (gloo, world size 2).

The GPU compute is replaced by the oracle here (passed as `compute`), so what
is tested is the sharding, the broadcast of B and the gather; the GPU kernel
is covered by the -m gpu tests.  Also: a rank that never joins makes the
others fail with a timeout instead of hanging."""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from tropical_gemm.distributed import shard_batch, shard_rows

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("m,world", [(1, 2), (100, 2), (256, 2), (1000, 3), (8192 * 4, 4), (129, 8)])
def test_shard_rows_partition(m, world):
    spans = [shard_rows(m, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == m
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c and a <= b
    nonempty = [(a, b) for a, b in spans if b > a]
    for a, b in nonempty:
        assert a % 128 == 0
    for a, b in nonempty[:-1]:
        assert (b - a) % 128 == 0


@pytest.mark.parametrize("batch,world", [(1, 2), (5, 2), (64, 8), (7, 3), (3, 4)])
def test_shard_batch_partition(batch, world):
    spans = [shard_batch(batch, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == batch
    sizes = [b - a for a, b in spans]
    assert all(b == c for (_, b), (c, _) in zip(spans, spans[1:]))
    assert max(sizes) - min(sizes) <= 1


WORKER = textwrap.dedent('''
    import os, sys
    sys.path.insert(0, os.path.join(sys.argv[1], "tropical-gemm_b200")); sys.path.insert(0, sys.argv[1])
    import numpy as np, torch
    import torch.distributed as dist
    from tropical_gemm import distributed as D
    from oracle import tg_oracle as O
    D.init("gloo", timeout_s=30)
    rank, world = dist.get_rank(), dist.get_world_size()
    rng = np.random.default_rng(0)
    m, k, n = 300, 70, 50
    a = rng.standard_normal((m, k)).astype(np.float32)
    b_full = rng.standard_normal((k, n)).astype(np.float32)
    s, e = D.shard_rows(m, world, rank)
    b = torch.from_numpy(b_full.copy()) if rank == 0 else torch.zeros((k, n))
    def compute(semi, aa, bb, wa):
        c, am = O.gemm(semi, aa.numpy(), bb.numpy(), wa)
        return torch.from_numpy(c), torch.from_numpy(am)
    c, am = D.sharded_matmul("maxplus", torch.from_numpy(a[s:e]), b, compute=compute)
    assert torch.equal(b, torch.from_numpy(b_full))
    C = D.gather_rows(c, m); AM = D.gather_rows(am, m)
    c0, am0 = O.gemm("maxplus", a, b_full)
    assert np.array_equal(C.numpy(), c0) and np.array_equal(AM.numpy(), am0)
    # strided-batched: shard by batch index, no exchange, gather the slices
    bs = 5
    ab = rng.standard_normal((bs, 20, 9)).astype(np.float32)
    bb = rng.standard_normal((bs, 9, 11)).astype(np.float32)
    s, e = D.shard_batch(bs, world, rank)
    def compute_b(semi, aa, bbb, wa):
        c, am = O.gemm_batched(semi, aa.numpy(), bbb.numpy(), wa)
        return torch.from_numpy(c), torch.from_numpy(am)
    cb, amb = D.sharded_batched_matmul("minplus", torch.from_numpy(ab[s:e]), torch.from_numpy(bb[s:e]),
                                       compute=compute_b)
    CB = D.gather_batches(cb, bs); AMB = D.gather_batches(amb, bs)
    cb0, amb0 = O.gemm_batched("minplus", ab, bb)
    assert np.array_equal(CB.numpy(), cb0) and np.array_equal(AMB.numpy(), amb0)
    # the K-pipelined broadcast: slice 0 by an ordinary GEMM, later slices
    # merged in place with the strict first-k-wins rule and global indices;
    # small integers make ties across slice boundaries frequent
    ai = rng.integers(-4, 5, (m, 200)).astype(np.float32)
    bi_full = rng.integers(-4, 5, (200, n)).astype(np.float32)
    b2 = torch.from_numpy(bi_full.copy()) if rank == 0 else torch.zeros((200, n))
    def acc(semi, aa, bb, c, am, off):
        v, i = O.gemm(semi, np.ascontiguousarray(aa.numpy()), np.ascontiguousarray(bb.numpy()), True)
        v, i = torch.from_numpy(v), torch.from_numpy(i)
        win = v > c if semi != "minplus" else v < c
        c[win] = v[win]
        am[win] = i[win] + off
    def first(semi, aa, bb, wa):
        c, am = O.gemm(semi, np.ascontiguousarray(aa.numpy()), np.ascontiguousarray(bb.numpy()), wa)
        return torch.from_numpy(c), torch.from_numpy(am)
    s, e = D.shard_rows(m, world, rank)
    for semi in ("maxplus", "minplus"):
        c, am = D.pipelined_sharded_matmul(semi, torch.from_numpy(ai[s:e]), b2, chunks=3, first=first, accumulate=acc)
        assert torch.equal(b2, torch.from_numpy(bi_full))
        C = D.gather_rows(c, m); AM = D.gather_rows(am, m)
        c0, am0 = O.gemm(semi, ai, bi_full)
        assert np.array_equal(C.numpy(), c0) and np.array_equal(AM.numpy(), am0), semi
    assert D.k_slices(200, 3) == [(0, 128), (128, 192), (192, 200)]
    dist.destroy_process_group()
    print("rank", rank, "ok")
''')


def test_gloo_world2_sharded_matmul(tmp_path):
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    port = _free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                   CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, str(script), ROOT], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = [p.communicate(timeout=180)[0] for p in procs]
    for p, o in zip(procs, outs):
        assert p.returncode == 0, o
        assert "ok" in o


def test_rank_that_never_joins_times_out(tmp_path):
    script = tmp_path / "lonely.py"
    script.write_text(textwrap.dedent('''
        import os, sys, time
        sys.path.insert(0, os.path.join(sys.argv[1], "tropical-gemm_b200"))
        from tropical_gemm import distributed as D
        t0 = time.time()
        try:
            D.init("gloo", timeout_s=3)
            print("joined?!")
        except Exception as e:
            print("timeout after %.1f s: %s" % (time.time() - t0, type(e).__name__))
    '''))
    env = dict(os.environ, RANK="0", WORLD_SIZE="2", MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()),
               CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(script), ROOT], env=env, capture_output=True, text=True, timeout=120)
    assert "timeout after" in out.stdout, out.stdout + out.stderr
