"""tg_gemm_i32_noalloc: the i32 GEMM for callers that cannot allocate device
memory at call time (a framework that owns the GPU's memory pool, a serving
loop that forbids allocation after start-up).  It must give exactly what
tg_gemm gives for the same i32 inputs, on repeated calls that reuse its fixed
scratch array, and refuse problems that do not fit that array.

This file is collected last on purpose: a failure here leaves every other
test already run in a stop-at-first-failure session."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import tg_oracle
from tropical_gemm import _native as N

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 64 << 20


def _lib():
    L = N.lib()
    i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
    L.tg_gemm_i32_noalloc.argtypes = [i32, i32, i64, i64, i64, vp, i64, vp, i64, vp, i64, vp, vp]
    L.tg_gemm_i32_noalloc.restype = i32
    return L


def _inputs(seed, m, k, n, semi):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randint(-50, 50, (m, k), generator=g, device="cuda", dtype=torch.int32)
    b = torch.randint(-50, 50, (k, n), generator=g, device="cuda", dtype=torch.int32)
    if semi == "minplus":   # sprinkle the reference's "infinity" sentinel
        a[torch.rand((m, k), generator=g, device="cuda") < 0.3] = 46340
    return a, b


@pytest.mark.parametrize("semi", ["maxplus", "minplus", "maxmul"])
def test_noalloc_matches_tg_gemm_twice(semi):
    L = _lib()
    st = torch.cuda.current_stream().cuda_stream
    for call, (m, k, n) in enumerate([(300, 257, 200), (129, 64, 301)]):   # two calls in a row, reusing scratch
        a, b = _inputs(call, m, k, n, semi)
        c_ref = torch.empty((m, n), dtype=torch.int32, device="cuda")
        i_ref = torch.empty((m, n), dtype=torch.int32, device="cuda")
        N.check(L.tg_gemm(N.SEMIRINGS[semi], 2, 0, m, n, k, a.data_ptr(), k, b.data_ptr(), n,
                          c_ref.data_ptr(), n, i_ref.data_ptr(), st))
        c = torch.full((m, n), -7, dtype=torch.int32, device="cuda")
        i = torch.full((m, n), -7, dtype=torch.int32, device="cuda")
        N.check(L.tg_gemm_i32_noalloc(N.SEMIRINGS[semi], 0, m, n, k, a.data_ptr(), k, b.data_ptr(), n,
                                      c.data_ptr(), n, i.data_ptr(), st))
        torch.cuda.synchronize()
        assert torch.equal(c, c_ref) and torch.equal(i, i_ref)   # integer results: exact
        # and the CPU oracle (the reference's GPU integer semantics, restated)
        c_or, i_or = tg_oracle.gemm(semi, a.cpu().numpy(), b.cpu().numpy())
        assert np.array_equal(c.cpu().numpy(), c_or) and np.array_equal(i.cpu().numpy(), i_or)


def test_noalloc_takes_no_device_memory():
    """Warm calls leave the device's free memory unchanged (no allocation,
    not even a stream-ordered one), while the results stay exact."""
    L = _lib()
    st = torch.cuda.current_stream().cuda_stream
    m, k, n = 512, 700, 384
    a, b = _inputs(5, m, k, n, "minplus")
    c = torch.empty((m, n), dtype=torch.int32, device="cuda")
    i = torch.empty((m, n), dtype=torch.int32, device="cuda")

    def call():
        N.check(L.tg_gemm_i32_noalloc(N.SEMIRINGS["minplus"], 0, m, n, k, a.data_ptr(), k, b.data_ptr(), n,
                                      c.data_ptr(), n, i.data_ptr(), st))

    call()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    alloc0 = torch.cuda.memory_allocated()
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0 and torch.cuda.memory_allocated() == alloc0
    c_or, i_or = tg_oracle.gemm("minplus", a.cpu().numpy(), b.cpu().numpy())
    assert np.array_equal(c.cpu().numpy(), c_or) and np.array_equal(i.cpu().numpy(), i_or)


def test_noalloc_out_of_range_values_and_colmajor():
    L = _lib()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(9)
    m, k, n = 200, 100, 150
    a = torch.randint(-2**30, 2**30, (k, m), generator=g, device="cuda", dtype=torch.int32)  # column-major A
    b = torch.randint(-2**30, 2**30, (n, k), generator=g, device="cuda", dtype=torch.int32)  # column-major B
    for _ in range(2):
        c_ref = torch.empty((n, m), dtype=torch.int32, device="cuda")
        i_ref = torch.empty((n, m), dtype=torch.int32, device="cuda")
        N.check(L.tg_gemm(0, 2, 1, m, n, k, a.data_ptr(), m, b.data_ptr(), k, c_ref.data_ptr(), m,
                          i_ref.data_ptr(), st))
        c = torch.empty_like(c_ref)
        i = torch.empty_like(i_ref)
        N.check(L.tg_gemm_i32_noalloc(0, 1, m, n, k, a.data_ptr(), m, b.data_ptr(), k, c.data_ptr(), m,
                                      i.data_ptr(), st))
        torch.cuda.synchronize()
        assert torch.equal(c, c_ref) and torch.equal(i, i_ref)


def test_noalloc_rejects_problems_beyond_its_scratch():
    L = _lib()
    m = n = k = 4096   # A and B as f32: 128 MiB > 64 MiB
    a = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = L.tg_gemm_i32_noalloc(0, 0, m, n, k, a.data_ptr(), k, a.data_ptr(), n, a.data_ptr(), n, None,
                               torch.cuda.current_stream().cuda_stream)
    assert rc == N.TG_ERR_UNSUPPORTED
    assert b"scratch" in L.tg_last_error()
