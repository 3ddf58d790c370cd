"""ctypes front end of oracle/tg_oracle.c -- TEST INFRASTRUCTURE ONLY.

Row-major numpy in, numpy out.  See tg_oracle.c for the reference citations
each routine restates.  Used by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline legs; never by the product path.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libtg_oracle.so")
_lib = None

SEMIRINGS = {"maxplus": 0, "minplus": 1, "maxmul": 2}
DTYPES = {np.dtype(np.float32): 0, np.dtype(np.float64): 1, np.dtype(np.int32): 2, np.dtype(np.int64): 3}


def build() -> str:
    """Compile the oracle library (needs gcc); returns its path."""
    subprocess.check_call(["make", "-s", "-C", _HERE, "all"])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        i64, vp, i32p = ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p
        L.tg_oracle_gemm.argtypes = [ctypes.c_int, ctypes.c_int, i64, i64, i64, vp, vp, vp, i32p, ctypes.c_int]
        L.tg_oracle_blis_argmax_f32.argtypes = [ctypes.c_int, i64, i64, i64, vp, vp, vp, i32p, ctypes.c_int]
        L.tg_oracle_simd_argmax_f32.argtypes = [ctypes.c_int, i64, i64, i64, vp, vp, vp, i32p, ctypes.c_int]
        L.tg_oracle_simd_maxplus_f32.argtypes = [i64, i64, i64, vp, vp, vp, ctypes.c_int]
        L.tg_oracle_backward.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, i64, i64, i64, vp, i32p, vp, vp]
        _lib = L
    return _lib


def _ptr(x):
    return x.ctypes.data_as(ctypes.c_void_p) if x is not None else None


def gemm(semiring: str, a: np.ndarray, b: np.ndarray, with_argmax: bool = True, nthreads: int = 0):
    """C = A (x) B (row-major). Returns (C, argmax or None)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b, dtype=a.dtype)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), dtype=a.dtype)
    am = np.empty((m, n), dtype=np.int32) if with_argmax else None
    nthreads = nthreads or os.cpu_count() or 1
    rc = lib().tg_oracle_gemm(SEMIRINGS[semiring], DTYPES[a.dtype], m, n, k, _ptr(a), _ptr(b), _ptr(c), _ptr(am), nthreads)
    assert rc == 0
    return c, am


def gemm_batched(semiring: str, a: np.ndarray, b: np.ndarray, with_argmax: bool = True, nthreads: int = 0):
    cs, ams = [], []
    for i in range(a.shape[0]):
        c, am = gemm(semiring, a[i], b[i], with_argmax, nthreads)
        cs.append(c)
        ams.append(am)
    return np.stack(cs), (np.stack(ams) if with_argmax else None)


def blis_argmax_f32(semiring: str, a: np.ndarray, b: np.ndarray, nthreads: int = 1):
    """The reference's CPU argmax path (BLIS-blocked scalar 4x4 microkernel)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float32)
    am = np.empty((m, n), dtype=np.int32)
    rc = lib().tg_oracle_blis_argmax_f32(SEMIRINGS[semiring], m, n, k, _ptr(a), _ptr(b), _ptr(c), _ptr(am), nthreads)
    assert rc == 0
    return c, am


def simd_maxplus_f32(a: np.ndarray, b: np.ndarray, nthreads: int = 1):
    """The reference's AVX2 value-only MaxPlus f32 path (restated); C only."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    _, n = b.shape
    c = np.empty((m, n), dtype=np.float32)
    rc = lib().tg_oracle_simd_maxplus_f32(m, n, k, _ptr(a), _ptr(b), _ptr(c), nthreads)
    if rc != 0:
        raise RuntimeError("oracle built without AVX2")
    return c


def simd_argmax_f32(semiring: str, a: np.ndarray, b: np.ndarray, nthreads: int = 1):
    """AVX2 argmax path (8x8 vector tiles, strict masked blend); equals blis_argmax_f32 bit for bit."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float32)
    am = np.empty((m, n), dtype=np.int32)
    rc = lib().tg_oracle_simd_argmax_f32(SEMIRINGS[semiring], m, n, k, _ptr(a), _ptr(b), _ptr(c), _ptr(am), nthreads)
    if rc != 0:
        raise RuntimeError("oracle built without AVX2")
    return c, am


def backward(semiring: str, want_a: bool, grad_c: np.ndarray, argmax: np.ndarray, k: int, partner=None):
    """Ordered-sum backward: grad_A (m x k) if want_a else grad_B (k x n)."""
    grad_c = np.ascontiguousarray(grad_c)
    argmax = np.ascontiguousarray(argmax, dtype=np.int32)
    m, n = grad_c.shape
    out = np.empty((m, k) if want_a else (k, n), dtype=grad_c.dtype)
    if partner is not None:
        partner = np.ascontiguousarray(partner, dtype=grad_c.dtype)
    rc = lib().tg_oracle_backward(SEMIRINGS[semiring], DTYPES[grad_c.dtype], int(want_a), m, n, k, _ptr(grad_c),
                                  _ptr(argmax), _ptr(partner), _ptr(out))
    assert rc == 0
    return out
