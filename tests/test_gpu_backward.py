"""GPU parity of the argmax-scatter backward and the autograd classes.

Gradients are float sums whose order inside a bin is not fixed, so they are
compared with the ordered oracle at rtol 1e-6 (the reference's stated
tolerance for gradients); everything else is exact."""
import numpy as np
import pytest
import torch

from helpers import engine, dev
from oracle import tg_oracle as O
from tropical_gemm import _native as N
import tropical_gemm
import tropical_gemm.pytorch as tp

pytestmark = pytest.mark.gpu
RTOL = 1e-6


def _close(x, y, rtol=RTOL):
    return np.allclose(x, y, rtol=rtol, atol=rtol * max(1.0, float(np.abs(y).max(initial=0.0))))


@pytest.mark.parametrize("semi", ["maxplus", "minplus", "maxmul"])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("shape", [(5, 7, 3), (64, 300, 129), (300, 40, 257), (33, 2000, 65), (96, 256, 128), (40, 3000, 64)])
def test_backward_matches_oracle(semi, dtype, shape):
    m, k, n = shape
    rng = np.random.default_rng(m * k + n)
    a = rng.standard_normal((m, k)).astype(dtype)
    b = rng.standard_normal((k, n)).astype(dtype)
    _, am = engine(semi, a, b)
    g = rng.standard_normal((m, n)).astype(dtype)
    tg, tam = torch.from_numpy(g).to(dev()), torch.from_numpy(am).to(dev())
    pa = torch.from_numpy(b).to(dev()) if semi == "maxmul" else None
    pb = torch.from_numpy(a).to(dev()) if semi == "maxmul" else None
    ga = N.backward(semi, True, tg, tam, k, pa).cpu().numpy()
    gb = N.backward(semi, False, tg, tam, k, pb).cpu().numpy()
    assert _close(ga, O.backward(semi, True, g, am, k, b if semi == "maxmul" else None))
    assert _close(gb, O.backward(semi, False, g, am, k, a if semi == "maxmul" else None))


@pytest.mark.parametrize("k", [20000, 70000])
def test_backward_large_k_fallback(k):
    """K beyond the shared-memory bins -> global-atomic path."""
    rng = np.random.default_rng(k)
    m, n = 40, 50
    am = rng.integers(0, k, (m, n)).astype(np.int32)
    am[0, 0] = k + 5  # out of range: skipped
    g = rng.standard_normal((m, n)).astype(np.float32)
    tg, tam = torch.from_numpy(g).to(dev()), torch.from_numpy(am).to(dev())
    assert _close(N.backward("maxplus", True, tg, tam, k).cpu().numpy(), O.backward("maxplus", True, g, am, k))
    assert _close(N.backward("maxplus", False, tg, tam, k).cpu().numpy(), O.backward("maxplus", False, g, am, k))


def test_backward_batched_and_accumulate():
    rng = np.random.default_rng(2)
    bs, m, k, n = 4, 64, 256, 96
    am = rng.integers(0, k, (bs, m, n)).astype(np.int32)
    g = rng.standard_normal((bs, m, n)).astype(np.float32)
    tg, tam = torch.from_numpy(g).to(dev()), torch.from_numpy(am).to(dev())
    ga = N.backward("maxplus", True, tg, tam, k).cpu().numpy()
    gb = N.backward("maxplus", False, tg, tam, k).cpu().numpy()
    for i in range(bs):
        assert _close(ga[i], O.backward("maxplus", True, g[i], am[i], k))
        assert _close(gb[i], O.backward("maxplus", False, g[i], am[i], k))
    # accumulate=1 adds into an existing buffer
    out = torch.ones((m, k), device=dev())
    N.check(N.lib().tg_backward_a(0, 0, 0, 1, m, n, k, tg[0].data_ptr(), n, m * n, tam[0].data_ptr(), None, n,
                                  0, out.data_ptr(), k, m * k, 1, torch.cuda.current_stream().cuda_stream))
    assert _close(out.cpu().numpy(), 1.0 + O.backward("maxplus", True, g[0], am[0], k))


def test_backward_colmajor_layout():
    rng = np.random.default_rng(8)
    m, k, n = 37, 50, 41
    am = rng.integers(0, k, (m, n)).astype(np.int32)
    g = rng.standard_normal((m, n)).astype(np.float32)
    tg = torch.from_numpy(np.asfortranarray(g).ravel(order="K").copy()).to(dev())
    tam = torch.from_numpy(np.asfortranarray(am).ravel(order="K").copy()).to(dev())
    ga = torch.empty(m * k, device=dev())
    gb = torch.empty(k * n, device=dev())
    st = torch.cuda.current_stream().cuda_stream
    N.check(N.lib().tg_backward_a(0, 0, 1, 1, m, n, k, tg.data_ptr(), m, 0, tam.data_ptr(), None, k, 0,
                                  ga.data_ptr(), m, 0, 0, st))
    N.check(N.lib().tg_backward_b(0, 0, 1, 1, m, n, k, tg.data_ptr(), m, 0, tam.data_ptr(), None, m, 0,
                                  gb.data_ptr(), k, 0, 0, st))
    assert _close(ga.cpu().numpy().reshape(k, m).T, O.backward("maxplus", True, g, am, k))
    assert _close(gb.cpu().numpy().reshape(n, k).T, O.backward("maxplus", False, g, am, k))


@pytest.mark.parametrize("fn_name,semi", [("tropical_maxplus_matmul_gpu", "maxplus"),
                                          ("tropical_minplus_matmul_gpu", "minplus"),
                                          ("tropical_maxmul_matmul_gpu", "maxmul")])
def test_autograd_gpu_classes(fn_name, semi):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((50, 30)).astype(np.float32)
    b = rng.standard_normal((30, 40)).astype(np.float32)
    ta = torch.from_numpy(a).to(dev()).requires_grad_(True)
    tb = torch.from_numpy(b).to(dev()).requires_grad_(True)
    c = getattr(tp, fn_name)(ta, tb)
    g = torch.randn_like(c)
    c.backward(g)
    c0, am0 = O.gemm(semi, a, b)
    assert np.array_equal(c.detach().cpu().numpy(), c0)
    gn = g.cpu().numpy()
    assert _close(ta.grad.cpu().numpy(), O.backward(semi, True, gn, am0, 30, b if semi == "maxmul" else None))
    assert _close(tb.grad.cpu().numpy(), O.backward(semi, False, gn, am0, 30, a if semi == "maxmul" else None))


def test_autograd_cpu_tensors_roundtrip():
    """The reference's CPU classes: CPU tensors in, CPU tensors and grads out."""
    rng = np.random.default_rng(1)
    a = torch.from_numpy(rng.standard_normal((20, 10)).astype(np.float32)).requires_grad_(True)
    b = torch.from_numpy(rng.standard_normal((10, 15)).astype(np.float32)).requires_grad_(True)
    c = tp.tropical_maxplus_matmul(a, b)
    assert c.device.type == "cpu"
    c.sum().backward()
    assert a.grad.device.type == "cpu"
    # each output routes a gradient of 1 to exactly one A entry in its row
    assert np.allclose(a.grad.sum(1).numpy(), 15.0)
    assert np.allclose(b.grad.sum().item(), 20 * 15)


def test_gpu_class_rejects_cpu_tensors():
    with pytest.raises(RuntimeError, match="requires CUDA"):
        tp.tropical_maxplus_matmul_gpu(torch.zeros(2, 2), torch.zeros(2, 2))


@pytest.mark.parametrize("semi", ["maxplus", "minplus", "maxmul"])
def test_autograd_batched(semi):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((4, 33, 20)).astype(np.float32)
    b = rng.standard_normal((4, 20, 17)).astype(np.float32)
    ta = torch.from_numpy(a).to(dev()).requires_grad_(True)
    tb = torch.from_numpy(b).to(dev()).requires_grad_(True)
    fn = getattr(tp, f"tropical_{semi}_matmul_batched")
    c = fn(ta, tb)
    c.sum().backward()
    for i in range(4):
        c0, am0 = O.gemm(semi, a[i], b[i])
        assert np.array_equal(c[i].detach().cpu().numpy(), c0)
        ones = np.ones_like(c0)
        assert _close(ta.grad[i].cpu().numpy(), O.backward(semi, True, ones, am0, 20, b[i] if semi == "maxmul" else None))
        assert _close(tb.grad[i].cpu().numpy(), O.backward(semi, False, ones, am0, 20, a[i] if semi == "maxmul" else None))


def test_finite_difference_maxplus():
    """Argmax-as-gradient against central differences (cu/src/lib.rs:1266-1483, eps 1e-3, tol 0.05)."""
    rng = np.random.default_rng(4)
    a = torch.from_numpy(rng.standard_normal((6, 5))).to(dev()).requires_grad_(True)
    b = torch.from_numpy(rng.standard_normal((5, 4))).to(dev()).requires_grad_(True)
    c = tp.tropical_maxplus_matmul_gpu(a, b)
    c.sum().backward()
    eps = 1e-3
    for i in range(6):
        for k in range(5):
            ap = a.detach().clone(); ap[i, k] += eps
            am_ = a.detach().clone(); am_[i, k] -= eps
            num = (N.gemm("maxplus", ap, b.detach(), False)[0].sum() - N.gemm("maxplus", am_, b.detach(), False)[0].sum()) / (2 * eps)
            assert abs(num.item() - a.grad[i, k].item()) < 0.05


def test_numpy_functions_on_gpu():
    rng = np.random.default_rng(6)
    a = rng.standard_normal((16, 16)).astype(np.float32)
    b = rng.standard_normal((16, 16)).astype(np.float32)
    c0, am0 = O.gemm("maxplus", a, b)
    assert np.array_equal(tropical_gemm.maxplus_matmul(a, b), c0.ravel())
    c, am = tropical_gemm.maxplus_matmul_with_argmax(a, b)
    assert np.array_equal(c, c0.ravel()) and np.array_equal(am, am0.ravel())
    assert np.array_equal(tropical_gemm.maxplus_matmul_2d(a, b), c0)
    ga = tropical_gemm.backward_a(np.ones((16, 16), np.float32), am0, 16)
    assert np.allclose(ga, O.backward("maxplus", True, np.ones((16, 16), np.float32), am0, 16).ravel())
    ai = rng.integers(-9, 9, (8, 5)).astype(np.int32)
    bi = rng.integers(-9, 9, (5, 7)).astype(np.int32)
    assert np.array_equal(tropical_gemm.minplus_matmul_2d_i32(ai, bi), O.gemm("minplus", ai, bi, False)[0])
    # literal reference convention of *_matmul_gpu: buffers read column-major
    cg = tropical_gemm.maxplus_matmul_gpu(a, b)
    af = a.ravel().reshape(16, 16, order="F")
    bf = b.ravel().reshape(16, 16, order="F")
    assert np.array_equal(cg, O.gemm("maxplus", af, bf, False)[0].ravel(order="F"))
    # dlpack-style tensors
    c_t, am_t = tropical_gemm.maxplus_matmul_dlpack(torch.from_numpy(a).to(dev()), torch.from_numpy(b).to(dev()))
    assert np.array_equal(c_t.cpu().numpy(), c0.ravel()) and np.array_equal(am_t.cpu().numpy(), am0.ravel())
    with pytest.raises(ValueError, match="Only f32"):
        tropical_gemm.maxplus_matmul_dlpack(torch.zeros(2, 2, dtype=torch.float64, device=dev()),
                                            torch.zeros(2, 2, dtype=torch.float64, device=dev()))
    with pytest.raises(ValueError, match="contiguous"):
        tropical_gemm.maxplus_matmul_dlpack(torch.zeros(4, 2, device=dev()).t(), torch.zeros(4, 2, device=dev()))


@pytest.mark.parametrize("want_a", [True, False])
def test_backward_empty_c_zeroes_every_batch(want_a):
    """M = 0: nothing scatters, and an overwrite must zero the gradient of
    every batch item, past the 65535 items of one grid dimension."""
    batch, m, n, k = 65537, 0, 2, 3
    L = N.lib()
    st = torch.cuda.current_stream().cuda_stream
    if want_a:   # grad_A is M x K = 0 x 3: nothing to write, must still succeed
        g = torch.full((batch, 1, k), float("nan"), device=dev())
        N.check(L.tg_backward_a(0, 0, 0, batch, m, n, k, None, n, 0, None, None, n, 0, g.data_ptr(), k, k, 0, st))
        torch.cuda.synchronize()
        assert torch.isnan(g).all()
    else:        # grad_B is K x N per item
        g = torch.full((batch, k, n), float("nan"), device=dev())
        N.check(L.tg_backward_b(0, 0, 0, batch, m, n, k, None, n, 0, None, None, k, 0, g.data_ptr(), n, k * n, 0, st))
        torch.cuda.synchronize()
        assert torch.count_nonzero(g).item() == 0
