"""The CPU oracle pinned against the reference's golden vectors and known answers.

The oracle (oracle/tg_oracle.c) is the checker for every GPU parity test, so it
is itself checked here first: bit-exact against all in-scope JSON fixtures the
reference ships (crates/tropical-gemm-python/tests/fixtures, packed into
tests/golden/reference_fixtures.npz by tests/golden/make_golden.py), and
against the reference's hand-written known answers.
"""
import numpy as np
import pytest

from oracle import tg_oracle as O

FIX = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "reference_fixtures.npz"))
NAMES = [str(n) for n in FIX["__names__"]]


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_fixtures(name):
    a, b = FIX[name + "__a"], FIX[name + "__b"]
    c_exp, am_exp = FIX[name + "__c"], FIX[name + "__argmax"]
    semi = name.split("_")[0]
    if a.ndim == 3:
        c, am = O.gemm_batched(semi, a, b)
    else:
        c, am = O.gemm(semi, a, b)
    assert c.dtype == c_exp.dtype
    assert np.array_equal(c.view(np.uint8), c_exp.view(np.uint8)), "values not bit-exact"
    assert np.array_equal(am, am_exp)


@pytest.mark.parametrize("name", [n for n in NAMES if "f32" in n and "batched" not in n])
def test_blis_path_matches_fixtures(name):
    """The restated reference CPU argmax path (BLIS + 4x4 microkernel)."""
    a, b = FIX[name + "__a"], FIX[name + "__b"]
    c, am = O.blis_argmax_f32(name.split("_")[0], a, b, nthreads=2)
    assert np.array_equal(c, FIX[name + "__c"]) and np.array_equal(am, FIX[name + "__argmax"])


@pytest.mark.parametrize("name", [n for n in NAMES if n.startswith("maxplus_f32") and "batched" not in n])
def test_simd_value_path_matches_fixtures(name):
    """The restated reference CPU SIMD path (AVX2 8x8 microkernel, no argmax)."""
    a, b = FIX[name + "__a"], FIX[name + "__b"]
    c = O.simd_maxplus_f32(a, b, nthreads=2)
    assert np.array_equal(c.view(np.uint32), FIX[name + "__c"].view(np.uint32))


def test_simd_value_path_matches_argmax_path_across_blocks():
    """Shapes past every block size (mc = nc = 256, kc = 512) and ragged edges:
    the SIMD values equal the argmax path's (finite inputs)."""
    rng = np.random.default_rng(3)
    a = rng.standard_normal((300, 1100), dtype=np.float32)
    b = rng.standard_normal((1100, 270), dtype=np.float32)
    c_simd = O.simd_maxplus_f32(a, b, nthreads=3)
    c_ref, _ = O.blis_argmax_f32("maxplus", a, b, nthreads=3)
    assert np.array_equal(c_simd, c_ref)


@pytest.mark.parametrize("name", [n for n in NAMES if "f32" in n and "batched" not in n])
def test_simd_argmax_path_matches_fixtures(name):
    """The AVX2 argmax path (8x8 vector tiles, strict masked blend)."""
    a, b = FIX[name + "__a"], FIX[name + "__b"]
    c, am = O.simd_argmax_f32(name.split("_")[0], a, b, nthreads=2)
    assert np.array_equal(c.view(np.uint32), FIX[name + "__c"].view(np.uint32))
    assert np.array_equal(am, FIX[name + "__argmax"])


@pytest.mark.parametrize("semi", ["maxplus", "minplus", "maxmul"])
def test_simd_argmax_equals_scalar_path(semi):
    """Past every block size, ragged edges, ties (quantised values), +-inf and
    NaN entries: values and indices equal the scalar BLIS argmax path."""
    rng = np.random.default_rng(11)
    a = np.round(rng.standard_normal((270, 1100)) * 4).astype(np.float32) / 4
    b = np.round(rng.standard_normal((1100, 263)) * 4).astype(np.float32) / 4
    a[rng.random(a.shape) < 0.01] = np.inf
    b[rng.random(b.shape) < 0.01] = -np.inf
    a[rng.random(a.shape) < 0.005] = np.nan
    if semi == "maxmul":
        a, b = np.abs(a), np.abs(b)
    c_s, am_s = O.simd_argmax_f32(semi, a, b, nthreads=3)
    c_r, am_r = O.blis_argmax_f32(semi, a, b, nthreads=3)
    assert np.array_equal(c_s.view(np.uint32), c_r.view(np.uint32))
    assert np.array_equal(am_s, am_r)


def test_known_answer_2x3_3x2():
    """crates/tropical-gemm-cuda/src/lib.rs:1091-1191 (column-major data there, row-major here)."""
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    c, am = O.gemm("maxplus", a, b)
    assert c.tolist() == [[8, 9], [11, 12]] and am.tolist() == [[2, 2], [2, 2]]
    c, am = O.gemm("minplus", a, b)
    assert c.tolist() == [[2, 3], [5, 6]] and am.tolist() == [[0, 0], [0, 0]]
    c, am = O.gemm("maxmul", a, b)
    assert c.tolist() == [[15, 18], [30, 36]] and am.tolist() == [[2, 2], [2, 2]]


def test_tie_lowest_k_wins():
    """All products equal: the first k wins (cu/src/lib.rs:1194-1230, core/gemm.rs:366-418)."""
    a = np.ones((3, 5), np.float32)
    b = np.ones((5, 4), np.float32)
    for semi in ("maxplus", "minplus", "maxmul"):
        _, am = O.gemm(semi, a, b)
        assert (am == 0).all()
    a = np.array([[0, 5, 5, 1]], np.float32)
    b = np.zeros((4, 1), np.float32)
    _, am = O.gemm("maxplus", a, b)
    assert am[0, 0] == 1


def test_blis_tie_across_kc_blocks():
    """Ties across kc=256 blocks keep the earlier block (core/kernel.rs:321-359)."""
    a = np.zeros((5, 600), np.float32)
    b = np.zeros((600, 6), np.float32)
    a[:, 10] = 1.0
    a[:, 300] = 1.0
    c, am = O.blis_argmax_f32("maxplus", a, b)
    assert (am == 10).all() and (c == 1.0).all()


def test_special_values():
    """+inf MinPlus and MaxMul zeros (py/tests/test_tropical_gemm.py:529-554), NaN never wins."""
    inf = np.float32(np.inf)
    a = np.array([[inf, 1.0], [2.0, inf]], np.float32)
    b = np.array([[1.0, inf], [inf, 3.0]], np.float32)
    c, am = O.gemm("minplus", a, b)
    assert c.tolist() == [[inf, 4.0], [3.0, inf]]
    assert am.tolist() == [[0, 1], [0, 0]]
    a = np.array([[0.0, -1.0]], np.float32)
    b = np.array([[5.0], [3.0]], np.float32)
    c, am = O.gemm("maxmul", a, b)
    assert c[0, 0] == 0.0 and not np.signbit(c[0, 0]) and am[0, 0] == 0
    a = np.array([[np.nan, 1.0]], np.float32)
    b = np.array([[1.0], [1.0]], np.float32)
    c, am = O.gemm("maxplus", a, b)
    assert c[0, 0] == 2.0 and am[0, 0] == 1
    # -inf + +inf = NaN never replaces the accumulator
    a = np.array([[-inf, 0.0]], np.float32)
    b = np.array([[inf], [-3.0]], np.float32)
    c, am = O.gemm("maxplus", a, b)
    assert c[0, 0] == -3.0 and am[0, 0] == 1


def test_signed_zero_semantics():
    """argmax kernels keep the first zero's sign; value-only ones follow fmaxf/fminf."""
    a = np.array([[-0.0, 0.0]], np.float32)
    b = np.array([[-0.0], [0.0]], np.float32)
    c, am = O.gemm("maxplus", a, b)   # products: -0, +0 ; first one wins
    assert np.signbit(c[0, 0]) and am[0, 0] == 0
    c, _ = O.gemm("maxplus", a, b, with_argmax=False)
    assert not np.signbit(c[0, 0])
    c, _ = O.gemm("minplus", a[:, ::-1], b[::-1], with_argmax=False)
    assert np.signbit(c[0, 0])


def test_integer_sentinels():
    """GPU integer contract: +-46340 sentinels with saturating add (tropical_gemm.cu:15-50)."""
    INF = 46340
    a = np.array([[INF, 1], [2, INF]], np.int32)
    b = np.array([[1, INF], [INF, 3]], np.int32)
    c, am = O.gemm("minplus", a, b)
    assert c.tolist() == [[INF, 4], [3, INF]] and am.tolist() == [[0, 1], [0, 0]]
    c, am = O.gemm("maxplus", -a, -b)
    assert c.tolist() == [[-INF, -4], [-3, -INF]]
    # a finite sum equal to the sentinel never beats the initial sentinel (strict compare)
    c, am = O.gemm("minplus", np.array([[46000]], np.int32), np.array([[340]], np.int32))
    assert c[0, 0] == INF and am[0, 0] == 0
    INF64 = 3037000499
    c, am = O.gemm("minplus", np.array([[INF64, 5]], np.int64), np.array([[0], [7]], np.int64))
    assert c[0, 0] == 12 and am[0, 0] == 1


def test_backward_oracle():
    g = np.arange(6, dtype=np.float32).reshape(2, 3)
    am = np.array([[0, 1, 1], [2, 2, 9]], np.int32)  # 9 is out of range and skipped
    ga = O.backward("maxplus", True, g, am, 3)
    assert ga.tolist() == [[0, 3, 0], [0, 0, 7]]
    gb = O.backward("maxplus", False, g, am, 3)
    assert gb.tolist() == [[0, 0, 0], [0, 1, 2], [3, 4, 0]]
