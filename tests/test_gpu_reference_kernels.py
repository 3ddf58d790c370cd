"""Bit-exact parity with the reference's own CUDA kernels at full BASELINE sizes.

oracle/_ref/libref_gpu.so is the unmodified reference kernel file
(crates/tropical-gemm-cuda/kernels/tropical_gemm.cu) compiled from source by
oracle/Makefile and launched with the reference's geometry and swap convention.
It lets the large configurations (8192^3, the 90%-inf MinPlus graph, batched
64 x 512x256x512) be checked exactly where the CPU oracle would take minutes."""
import numpy as np
import pytest
import torch

from helpers import SEMIS, ref_lib, ref_rowmajor, dev
from tropical_gemm import _native as N

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(ref_lib() is None, reason="reference kernels not built")]


def _eq(x: torch.Tensor, y: torch.Tensor) -> bool:
    if x.dtype in (torch.float32, torch.int32):
        return torch.equal(x.view(torch.int32), y.view(torch.int32))
    return torch.equal(x.view(torch.int64), y.view(torch.int64))


@pytest.mark.parametrize("semi", SEMIS)
def test_f32_8192_cubed_matches_reference_kernel(semi):
    g = torch.Generator(device=dev()).manual_seed(1)
    a = torch.randn((8192, 8192), generator=g, device=dev())
    b = torch.randn((8192, 8192), generator=g, device=dev())
    c, am = N.gemm(semi, a, b, True)
    cr, amr = ref_rowmajor(semi, a, b, True)
    torch.cuda.synchronize()
    assert _eq(c, cr) and torch.equal(am, amr)
    c2, _ = N.gemm(semi, a, b, False)
    cr2, _ = ref_rowmajor(semi, a, b, False)
    assert _eq(c2, cr2)


def test_minplus_sparse_graph_8192():
    g = torch.Generator(device=dev()).manual_seed(1)
    mats = []
    for _ in range(2):
        v = 100 * torch.rand((8192, 8192), generator=g, device=dev())
        v[torch.rand((8192, 8192), generator=g, device=dev()) < 0.9] = float("inf")
        mats.append(v)
    c, am = N.gemm("minplus", *mats, True)
    cr, amr = ref_rowmajor("minplus", *mats, True)
    assert _eq(c, cr) and torch.equal(am, amr)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("dtype", [torch.float64, torch.int32, torch.int64])
def test_other_dtypes_match_reference_kernel(semi, dtype):
    g = torch.Generator(device=dev()).manual_seed(2)
    if dtype == torch.float64:
        a = torch.randn((700, 513), generator=g, device=dev(), dtype=dtype)
        b = torch.randn((513, 650), generator=g, device=dev(), dtype=dtype)
    else:
        a = torch.randint(-20, 20, (700, 513), generator=g, device=dev(), dtype=dtype)
        b = torch.randint(-20, 20, (513, 650), generator=g, device=dev(), dtype=dtype)
    for wa in (True, False):
        c, am = N.gemm(semi, a, b, wa)
        cr, amr = ref_rowmajor(semi, a, b, wa)
        assert _eq(c, cr)
        if wa:
            assert torch.equal(am, amr)


@pytest.mark.parametrize("semi", SEMIS)
def test_batched_config3_matches_reference_kernel(semi):
    g = torch.Generator(device=dev()).manual_seed(0)
    a = torch.randn((64, 512, 256), generator=g, device=dev())
    b = torch.randn((64, 256, 512), generator=g, device=dev())
    c, am = N.gemm_batched(semi, a, b, True)
    cr = torch.empty_like(c)
    amr = torch.empty_like(am)
    # reference batched launcher with its swap: (B, A, N, M, K, strideB, strideA, strideC)
    rc = ref_lib().ref_gemm_batched_argmax_f32(N.SEMIRINGS[semi], 64, 512, 512, 256, b.data_ptr(), a.data_ptr(),
                                               cr.data_ptr(), amr.data_ptr(), 256 * 512, 512 * 256, 512 * 512,
                                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert _eq(c, cr) and torch.equal(am, amr)


def test_backward_matches_reference_kernels():
    g = torch.Generator(device=dev()).manual_seed(3)
    m, n, k = 1024, 768, 512
    am = torch.randint(0, k, (m, n), generator=g, device=dev(), dtype=torch.int32)
    gc = torch.randn((m, n), generator=g, device=dev())
    ga = N.backward("maxplus", True, gc, am, k)
    gb = N.backward("maxplus", False, gc, am, k)
    # reference kernels are column-major: pass the transposed problem (C^T is n x m)
    ga_r = torch.zeros((m, k), device=dev())   # == grad_B of the transposed problem, col-major k x m
    gb_r = torch.zeros((k, n), device=dev())
    st = torch.cuda.current_stream().cuda_stream
    assert ref_lib().ref_backward(0, 0, gc.data_ptr(), am.data_ptr(), ga_r.data_ptr(), n, m, k, st) == 0
    assert ref_lib().ref_backward(1, 0, gc.data_ptr(), am.data_ptr(), gb_r.data_ptr(), n, m, k, st) == 0
    torch.cuda.synchronize()
    assert torch.allclose(ga, ga_r, rtol=1e-6, atol=1e-5)
    assert torch.allclose(gb, gb_r, rtol=1e-6, atol=1e-5)


def _apsp_matrix(n, seed):
    """BASELINE config 4 input: 5 % density, weights 1..1000, missing edges =
    the reference's i32 infinity (46340), zero diagonal."""
    g = torch.Generator(device=dev()).manual_seed(seed)
    w = torch.randint(1, 1001, (n, n), generator=g, device=dev(), dtype=torch.int32)
    d = torch.where(torch.rand((n, n), generator=g, device=dev()) < 0.05, w,
                    torch.full_like(w, 46340))
    d.fill_diagonal_(0)
    return d


def test_config4_apsp_squaring_16384_matches_reference_kernel():
    """One full-size APSP squaring (MinPlus i32 + argmax, n = 16384): ties are
    frequent, so the index tie-break is exercised at scale."""
    d = _apsp_matrix(16384, 4)
    c, am = N.gemm("minplus", d, d, True)
    cr, amr = ref_rowmajor("minplus", d, d, True)
    torch.cuda.synchronize()
    assert torch.equal(c, cr) and torch.equal(am, amr)
    del c, am, cr, amr
    # the second squaring starts from distances, not edge weights
    d2, _ = N.gemm("minplus", d, d, False)
    c, am = N.gemm("minplus", d2, d2, True)
    cr, amr = ref_rowmajor("minplus", d2, d2, True)
    assert torch.equal(c, cr) and torch.equal(am, amr)


@pytest.mark.parametrize("case", ["maxplus_f32_argmax", "maxmul_f64_values"])
def test_config5_row_block_matches_reference_kernel(case):
    """One rank's row block of BASELINE config 5 (4096 of M = 32768 rows,
    N = 32768, K = 8192): MaxPlus f32 + argmax on N(0,1) and MaxMul f64
    values on U[0,1)."""
    g = torch.Generator(device=dev()).manual_seed(2)
    if case == "maxplus_f32_argmax":
        a = torch.randn((4096, 8192), generator=g, device=dev())
        b = torch.randn((8192, 32768), generator=g, device=dev())
        c, am = N.gemm("maxplus", a, b, True)
        cr, amr = ref_rowmajor("maxplus", a, b, True)
        assert _eq(c, cr) and torch.equal(am, amr)
    else:
        a = torch.rand((4096, 8192), generator=g, device=dev(), dtype=torch.float64)
        b = torch.rand((8192, 32768), generator=g, device=dev(), dtype=torch.float64)
        c, _ = N.gemm("maxmul", a, b, False)
        cr, _ = ref_rowmajor("maxmul", a, b, False)
        assert _eq(c, cr)
