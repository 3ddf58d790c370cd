"""GPU parity: the engine's forward kernels against the CPU oracle, bit-exact
(values and argmax), for every semiring x dtype, both layouts, odd shapes,
ties, special values, batching and edge cases the reference tests."""
import os

import numpy as np
import pytest
import torch

from helpers import SEMIS, engine, engine_colmajor, oracle, same_bits, dev
from tropical_gemm import _native as N

pytestmark = pytest.mark.gpu

FIX = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_fixtures.npz"))
NAMES = [str(n) for n in FIX["__names__"]]


@pytest.mark.parametrize("name", NAMES)
def test_reference_fixtures_on_gpu(name):
    a, b = FIX[name + "__a"], FIX[name + "__b"]
    c, am = engine(name.split("_")[0], a, b)
    assert same_bits(c, FIX[name + "__c"])
    assert np.array_equal(am, FIX[name + "__argmax"])


@pytest.mark.parametrize("name", [n for n in NAMES if "batched" not in n])
def test_reference_fixtures_colmajor(name):
    a, b = FIX[name + "__a"], FIX[name + "__b"]
    c, am = engine_colmajor(name.split("_")[0], a, b)
    assert same_bits(c, FIX[name + "__c"])
    assert np.array_equal(am, FIX[name + "__argmax"])


def _data(rng, dtype, shape, kind):
    if kind == "normal":
        if np.issubdtype(dtype, np.floating):
            return rng.standard_normal(shape).astype(dtype)
        return rng.integers(-1000, 1000, shape).astype(dtype)
    if kind == "ties":  # few distinct values -> many exact ties
        return rng.integers(-3, 4, shape).astype(dtype)
    raise ValueError(kind)


SHAPES = [(1, 1, 1), (7, 13, 5), (63, 65, 127), (129, 130, 257), (200, 3, 70), (128, 128, 32), (1, 300, 1000)]


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int32, np.int64])
@pytest.mark.parametrize("kind", ["normal", "ties"])
@pytest.mark.parametrize("with_argmax", [True, False])
def test_random_shapes(semi, dtype, kind, with_argmax):
    rng = np.random.default_rng(hash((semi, str(dtype), kind)) % 2**32)
    for (m, k, n) in SHAPES:
        a = _data(rng, dtype, (m, k), kind)
        b = _data(rng, dtype, (k, n), kind)
        c, am = engine(semi, a, b, with_argmax)
        c0, am0 = oracle(semi, a, b, with_argmax)
        assert same_bits(c, c0), f"values differ at {(m, k, n)}"
        if with_argmax:
            assert np.array_equal(am, am0), f"argmax differs at {(m, k, n)}"


@pytest.mark.parametrize("semi", SEMIS)
def test_colmajor_random(semi):
    rng = np.random.default_rng(5)
    for dtype in (np.float32, np.float64, np.int32):
        a = _data(rng, dtype, (77, 45), "ties")
        b = _data(rng, dtype, (45, 91), "ties")
        c, am = engine_colmajor(semi, a, b)
        c0, am0 = oracle(semi, a, b)
        assert same_bits(c, c0) and np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("k", [1, 2, 3, 4, 31, 32, 33, 63, 64, 65, 100, 511, 1000, 1024, 1025, 1537])
def test_fast_path_k_tails(semi, k):
    rng = np.random.default_rng(k)
    a = rng.standard_normal((130, k)).astype(np.float32)
    b = rng.standard_normal((k, 140)).astype(np.float32)
    for wa in (True, False):
        c, am = engine(semi, a, b, wa)
        c0, am0 = oracle(semi, a, b, wa)
        assert same_bits(c, c0)
        if wa:
            assert np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
def test_fast_path_many_chunks(semi):
    """K large enough that the chunk length grows (more than 1024 chunks of 64)."""
    rng = np.random.default_rng(11)
    k = 70000
    a = rng.integers(-50, 50, (20, k)).astype(np.float32)
    b = rng.integers(-50, 50, (k, 24)).astype(np.float32)
    c, am = engine(semi, a, b)
    c0, am0 = oracle(semi, a, b)
    assert same_bits(c, c0) and np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
def test_special_values_fast_and_generic(semi):
    rng = np.random.default_rng(3)
    for dtype in (np.float32, np.float64):
        a = rng.standard_normal((150, 97)).astype(dtype)
        b = rng.standard_normal((97, 133)).astype(dtype)
        for arr in (a, b):
            mask = rng.random(arr.shape)
            arr[mask < 0.05] = np.inf
            arr[(mask >= 0.05) & (mask < 0.10)] = -np.inf
            arr[(mask >= 0.10) & (mask < 0.13)] = np.nan
            arr[(mask >= 0.13) & (mask < 0.18)] = 0.0
            arr[(mask >= 0.18) & (mask < 0.23)] = -0.0
        for wa in (True, False):
            c, am = engine(semi, a, b, wa)
            c0, am0 = oracle(semi, a, b, wa)
            assert same_bits(c, c0)
            if wa:
                assert np.array_equal(am, am0)


def test_minplus_sparse_graph_distances():
    """BASELINE config 2b shape at reduced size: 90% +inf, values in [0,100)."""
    rng = np.random.default_rng(1)
    mats = []
    for _ in range(2):
        v = (100 * rng.random((300, 300))).astype(np.float32)
        v[rng.random((300, 300)) < 0.9] = np.inf
        mats.append(v)
    c, am = engine("minplus", *mats)
    c0, am0 = oracle("minplus", *mats)
    assert same_bits(c, c0) and np.array_equal(am, am0)


@pytest.mark.parametrize("semi", ["minplus", "maxplus"])
def test_integer_sentinels_on_gpu(semi):
    rng = np.random.default_rng(7)
    for dtype, inf in ((np.int32, 46340), (np.int64, 3037000499)):
        a = rng.integers(0, 1000, (90, 70)).astype(dtype)
        b = rng.integers(0, 1000, (70, 80)).astype(dtype)
        s = inf if semi == "minplus" else -inf
        a[rng.random(a.shape) < 0.5] = s
        b[rng.random(b.shape) < 0.5] = s
        if semi == "maxplus":
            a, b = np.where(a == s, a, -a), np.where(b == s, b, -b)
        c, am = engine(semi, a, b)
        c0, am0 = oracle(semi, a, b)
        assert same_bits(c, c0) and np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int32])
def test_batched(semi, dtype):
    rng = np.random.default_rng(9)
    for (bs, m, k, n) in [(3, 8, 8, 8), (5, 65, 33, 70), (2, 130, 300, 129)]:
        a = _data(rng, dtype, (bs, m, k), "ties")
        b = _data(rng, dtype, (bs, k, n), "ties")
        c, am = engine(semi, a, b)
        c0, am0 = oracle(semi, a, b)
        assert same_bits(c, c0) and np.array_equal(am, am0)


def test_k_zero_gives_semiring_zero_and_index_zero():
    for semi, z in (("maxplus", -np.inf), ("minplus", np.inf), ("maxmul", 0.0)):
        a = torch.empty((5, 0), device=dev())
        b = torch.empty((0, 6), device=dev())
        c, am = N.gemm(semi, a, b, True)
        assert (c.cpu().numpy() == z).all() and (am.cpu().numpy() == 0).all()


def test_empty_m_or_n():
    a = torch.zeros((0, 4), device=dev())
    b = torch.zeros((4, 3), device=dev())
    c, am = N.gemm("maxplus", a, b, True)
    assert c.shape == (0, 3)


def test_unaligned_leading_dimension():
    """lda not a multiple of 4 (a padded buffer): 4-byte staging of A, same bits."""
    rng = np.random.default_rng(4)
    m, k, n = 70, 37, 50
    buf = rng.standard_normal((m, k + 1)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    ta = torch.from_numpy(buf).to(dev())
    tb = torch.from_numpy(b).to(dev())
    c = torch.empty((m, n), device=dev())
    am = torch.empty((m, n), dtype=torch.int32, device=dev())
    N.check(N.lib().tg_gemm(0, 0, 0, m, n, k, ta.data_ptr(), k + 1, tb.data_ptr(), n, c.data_ptr(), n,
                            am.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    c0, am0 = oracle("maxplus", np.ascontiguousarray(buf[:, :k]), b)
    assert same_bits(c.cpu().numpy(), c0) and np.array_equal(am.cpu().numpy(), am0)


def test_large_square_vs_oracle_sampled_rows():
    """2048^2 x 1024 on the fast path, checked on a sample of rows (full rows, all k)."""
    rng = np.random.default_rng(1)
    m, k, n = 2048, 1024, 2048
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    c, am = engine("maxplus", a, b)
    rows = rng.choice(m, 64, replace=False)
    c0, am0 = oracle("maxplus", a[rows], b)
    assert same_bits(c[rows], c0) and np.array_equal(am[rows], am0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("pattern", ["increasing", "decreasing", "plateau"])
@pytest.mark.parametrize("k", [200, 900, 1500])
def test_argmax_improvement_patterns(semi, pattern, k):
    """Running values that improve in every k-chunk, only in the first one,
    or tie on a long plateau: the pair (K <= 1024) and chunk bookkeeping must
    give the reference's first-k winner in all of them."""
    m, n = 256, 256
    kk = np.arange(k, dtype=np.float32) * 0.01
    if semi == "minplus":
        kk = -kk
    if pattern == "increasing":
        a = np.tile(kk, (m, 1)) + 1.0
    elif pattern == "decreasing":
        a = np.tile(-kk, (m, 1)) + 1.0
    else:
        a = np.ones((m, k), np.float32)
        a[:, 500:800] = 2.0 if semi != "minplus" else 0.5
    a = a.astype(np.float32)
    b = np.ones((k, n), np.float32)
    c, am = engine(semi, a, b)
    c0, am0 = oracle(semi, a, b)
    assert same_bits(c, c0) and np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("dtype,lim", [(np.int64, 1000), (np.int64, 2**62), (np.int32, 2**30)])
def test_batched_integers_in_and_out_of_range(semi, dtype, lim):
    """Batched i64 (through the f64 kernel when exact, else the integer kernel)
    and batched i32 beyond the exact-in-f32 range (exact integer kernel, with
    wrap-around), values and argmax, with and without argmax."""
    rng = np.random.default_rng(21)
    for (bs, m, k, n) in [(3, 40, 70, 33), (2, 129, 260, 131)]:
        a = rng.integers(-lim, lim, (bs, m, k)).astype(dtype)
        b = rng.integers(-lim, lim, (bs, k, n)).astype(dtype)
        for wa in (True, False):
            c, am = engine(semi, a, b, wa)
            c0, am0 = oracle(semi, a, b, wa)
            assert same_bits(c, c0)
            if wa:
                assert np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
def test_i32_out_of_range_falls_back_exactly(semi):
    """Operands beyond the exact-in-f32 range (|x| > 2^23; MaxMul |x| > 4096)
    take the exact integer kernel, including wrap-around on overflow."""
    rng = np.random.default_rng(12)
    a = rng.integers(-2**30, 2**30, (150, 90)).astype(np.int32)
    b = rng.integers(-2**30, 2**30, (90, 140)).astype(np.int32)
    for wa in (True, False):
        c, am = engine(semi, a, b, wa)
        c0, am0 = oracle(semi, a, b, wa)
        assert same_bits(c, c0)
        if wa:
            assert np.array_equal(am, am0)


def test_i32_apsp_step_with_sentinels():
    """One APSP squaring step (BASELINE config 4 shape, reduced): 5% density,
    weights 1..1000, missing = 46340, diagonal 0; ties are frequent."""
    rng = np.random.default_rng(4)
    n = 600
    mask = rng.random((n, n)) < 0.05
    w = rng.integers(1, 1001, (n, n)).astype(np.int32)
    d = np.where(mask, w, 46340).astype(np.int32)
    np.fill_diagonal(d, 0)
    c, am = engine("minplus", d, d)
    c0, am0 = oracle("minplus", d, d)
    assert same_bits(c, c0) and np.array_equal(am, am0)
    c2, am2 = engine("minplus", c, c)
    c20, am20 = oracle("minplus", c0, c0)
    assert same_bits(c2, c20) and np.array_equal(am2, am20)


@pytest.mark.parametrize("semi", SEMIS)
def test_i64_out_of_range_falls_back_exactly(semi):
    """i64 operands beyond the exact-in-f64 range take the exact integer kernel."""
    rng = np.random.default_rng(13)
    a = rng.integers(-2**62, 2**62, (140, 70)).astype(np.int64)
    b = rng.integers(-2**62, 2**62, (70, 150)).astype(np.int64)
    for wa in (True, False):
        c, am = engine(semi, a, b, wa)
        c0, am0 = oracle(semi, a, b, wa)
        assert same_bits(c, c0)
        if wa:
            assert np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("k", [37, 300, 1001, 1100])
def test_misaligned_base_and_odd_batch_stride(semi, k):
    """A starting 4 bytes past a 16-byte boundary and odd batch strides."""
    rng = np.random.default_rng(k)
    bs, m, n = 3, 150, 140
    buf = rng.standard_normal(bs * m * k + 1).astype(np.float32)
    a = buf[1:].reshape(bs, m, k)
    b = rng.standard_normal((bs, k, n)).astype(np.float32)
    ta = torch.from_numpy(buf).to(dev())[1:]
    tb = torch.from_numpy(b).to(dev())
    c = torch.empty((bs, m, n), device=dev())
    am = torch.empty((bs, m, n), dtype=torch.int32, device=dev())
    N.check(N.lib().tg_gemm_strided_batched(N.SEMIRINGS[semi], 0, 0, bs, m, n, k, ta.data_ptr(), k, m * k,
                                            tb.data_ptr(), n, k * n, c.data_ptr(), n, m * n, am.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    c0, am0 = oracle(semi, np.ascontiguousarray(a), b)
    assert same_bits(c.cpu().numpy(), c0) and np.array_equal(am.cpu().numpy(), am0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_zero_sign_of_value_only_results(semi, dtype):
    """Results that are a signed zero: the value-only fold must give fmax/fmin's
    sign (max(+0,-0) = +0 and min(+0,-0) = -0 in either order), on tiles where
    only some outputs are zero and on tiles where none are."""
    rng = np.random.default_rng(11)
    m, k, n = 300, 260, 200
    a = np.abs(rng.standard_normal((m, k))).astype(dtype)
    b = np.abs(rng.standard_normal((k, n))).astype(dtype)
    if semi == "maxplus":
        a, b = -a, -b
    elif semi == "maxmul":
        a = -a
    for arr in (a, b):
        arr[:150][rng.random(arr[:150].shape) < 0.3] = 0.0
        arr[:150][rng.random(arr[:150].shape) < 0.3] = -0.0
    for wa in (False, True):
        c, am = engine(semi, a, b, wa)
        c0, am0 = oracle(semi, a, b, wa)
        assert same_bits(c, c0)
        assert np.count_nonzero(c0 == 0) > 0
        if wa:
            assert np.array_equal(am, am0)


def test_i32_argmax_beyond_the_chunk_limit():
    """i32 with argmax and K past the fast kernel's chunk table (4 x 1024 tiles
    of 32): both the allocating entry point and tg_gemm_i32_noalloc must fall
    back to the exact kernel, not run the fast kernel with oversized chunks."""
    import ctypes
    rng = np.random.default_rng(12)
    k = 4 * 1024 * 32 + 5000
    for m, n, noalloc in ((128, 128, False), (40, 48, True)):
        a = rng.integers(-50, 50, (m, k)).astype(np.int32)
        b = rng.integers(-50, 50, (k, n)).astype(np.int32)
        c0, am0 = oracle("maxplus", a, b)
        if not noalloc:
            c, am = engine("maxplus", a, b)
        else:
            L = N.lib()
            i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
            L.tg_gemm_i32_noalloc.argtypes = [i32, i32, i64, i64, i64, vp, i64, vp, i64, vp, i64, vp, vp]
            L.tg_gemm_i32_noalloc.restype = i32
            ta, tb = torch.from_numpy(a).to(dev()), torch.from_numpy(b).to(dev())
            tc = torch.empty((m, n), dtype=torch.int32, device=dev())
            ti = torch.empty((m, n), dtype=torch.int32, device=dev())
            N.check(L.tg_gemm_i32_noalloc(0, 0, m, n, k, ta.data_ptr(), k, tb.data_ptr(), n, tc.data_ptr(), n,
                                          ti.data_ptr(), torch.cuda.current_stream().cuda_stream))
            c, am = tc.cpu().numpy(), ti.cpu().numpy()
        assert np.array_equal(c, c0) and np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("k,cuts,with_argmax", [(2000, (700, 1600), True), (900, (300,), True),
                                                (1500, (512, 1000), False), (3000, (64, 2900), True)])
def test_accumulate_over_k_slices_equals_one_pass(semi, k, cuts, with_argmax):
    """K sliced at `cuts`: tg_gemm on the first slice, tg_gemm_accumulate on
    the rest (A's column slices passed with its full leading dimension) gives
    the one-pass result bit for bit.  Small-integer values make ties across
    slice boundaries frequent: the earlier slice must keep them."""
    g = torch.Generator(device=dev()).manual_seed(k)
    m, n = 300, 260
    a = torch.randint(-6, 7, (m, k), generator=g, device=dev()).float()
    b = torch.randint(-6, 7, (k, n), generator=g, device=dev()).float()
    if semi == "maxmul":
        a, b = a.abs(), b.abs()
    c_ref, am_ref = N.gemm(semi, a, b, with_argmax)
    bounds = [0, *cuts, k]
    c, am = N.gemm(semi, a[:, : bounds[1]], b[: bounds[1]].contiguous(), with_argmax)
    for s0, s1 in zip(bounds[1:-1], bounds[2:]):
        N.gemm_accumulate(semi, a[:, s0:s1], b[s0:s1].contiguous(), c, am, s0)
    torch.cuda.synchronize()
    assert torch.equal(c.view(torch.int32), c_ref.view(torch.int32))
    if with_argmax:
        assert torch.equal(am, am_ref)
        _, am_or = oracle(semi, a.cpu().numpy(), b.cpu().numpy())
        assert np.array_equal(am.cpu().numpy(), am_or)


def test_accumulate_rejects_other_dtypes():
    a = torch.zeros((4, 4), dtype=torch.float64, device=dev())
    c = torch.zeros((4, 4), dtype=torch.float64, device=dev())
    with pytest.raises(ValueError):
        N.gemm_accumulate("maxplus", a, a, c, None, 0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("k", [1, 3, 4, 5, 130, 199, 256])
def test_short_k_group_tracking_ties(semi, k):
    """K <= 256 runs the resident-B-panel kernel that tracks the argmax per
    4-k group: small integers make ties inside a group and across groups
    frequent, and K not a multiple of 4 leaves a partial last group."""
    rng = np.random.default_rng(k)
    a = rng.integers(0 if semi == "maxmul" else -3, 4, (300, k)).astype(np.float32)
    b = rng.integers(0 if semi == "maxmul" else -3, 4, (k, 260)).astype(np.float32)
    c, am = engine(semi, a, b)
    c0, am0 = oracle(semi, a, b)
    assert same_bits(c, c0)
    assert np.array_equal(am, am0)


@pytest.mark.parametrize("semi", SEMIS)
@pytest.mark.parametrize("dtype", [np.float64, np.int64])
@pytest.mark.parametrize("kind", ["normal", "ties", "increasing", "decreasing", "plateau", "special"])
def test_wide_argmax_long_k_patterns(semi, dtype, kind):
    """f64 / i64 argmax at K around multiples of 64 and up to 4100: ties,
    improvements at every k or only the first, a long plateau, and (f64)
    +-inf, NaN and signed zeros."""
    rng = np.random.default_rng(hash((semi, str(dtype), kind)) % 2**32)
    for (m, k, n) in [(130, 65, 70), (64, 128, 64), (129, 129, 65), (70, 200, 131), (33, 1000, 40), (17, 4100, 9)]:
        if kind in ("normal", "ties"):
            a = _data(rng, dtype, (m, k), kind)
            b = _data(rng, dtype, (k, n), kind)
        elif kind == "special":
            if dtype != np.float64:
                pytest.skip("special values are float")
            vals = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 2.0], np.float64)
            a = rng.choice(vals, (m, k))
            b = rng.choice(vals, (k, n))
        else:
            ramp = np.arange(k)
            if kind == "decreasing":
                ramp = -ramp
            if semi == "minplus":
                ramp = -ramp
            if kind == "plateau":
                ramp = np.zeros(k, np.int64)
                ramp[k // 3: 2 * k // 3] = 1 if semi != "minplus" else -1
            base = 3 if semi == "maxmul" else 0   # MaxMul: keep products positive and ordered
            a = np.tile(ramp - ramp.min() + base + 1 if semi == "maxmul" else ramp, (m, 1)).astype(dtype)
            b = np.ones((k, n), dtype) * (1 if semi == "maxmul" else 0)
            b = b.astype(dtype)
        if semi == "maxmul" and dtype == np.int64 and kind in ("normal",):
            a, b = a // 10, b // 10   # keep i64 products inside the exact-in-f64 range
        c, am = engine(semi, a, b)
        c0, am0 = oracle(semi, a, b)
        assert same_bits(c, c0), (m, k, n)
        assert np.array_equal(am, am0), (m, k, n)


@pytest.mark.parametrize("semi", SEMIS)
def test_wide_argmax_batched(semi):
    """f64 argmax with batches on grid.z and frequent ties."""
    rng = np.random.default_rng(31)
    a = rng.integers(-3, 4, (3, 150, 300)).astype(np.float64)
    b = rng.integers(-3, 4, (3, 300, 90)).astype(np.float64)
    c, am = engine(semi, a, b)
    c0, am0 = oracle(semi, a, b)
    assert same_bits(c, c0) and np.array_equal(am, am0)
