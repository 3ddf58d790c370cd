"""The C-ABI library loads and exports every entry point include/*.h declares;
argument validation answers with error codes (no GPU work is done here)."""
import ctypes
import glob
import os
import re

import pytest

from tropical_gemm import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(tg_[a-z0-9_]+)\s*\(", src):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("tg_gemm", "tg_gemm_strided_batched", "tg_backward_a", "tg_backward_b", "tg_last_error"):
        assert s in syms


@pytest.mark.parametrize("sym", declared_symbols())
def test_library_exports(sym):
    L = N.lib()
    assert hasattr(L, sym), f"{sym} declared in include/ but not exported"


def test_version_and_device_count():
    assert N.version().startswith("0.2.0")
    assert N.device_count() >= 0


@pytest.mark.parametrize("args, code", [
    # bad semiring / dtype / layout / negative size: rejected before any CUDA call
    ((7, 0, 0, 4, 4, 4, 1, 4, 1, 4, 1, 4, None, None), N.TG_ERR_INVALID_ARGUMENT),
    ((0, 9, 0, 4, 4, 4, 1, 4, 1, 4, 1, 4, None, None), N.TG_ERR_INVALID_ARGUMENT),
    ((0, 0, 5, 4, 4, 4, 1, 4, 1, 4, 1, 4, None, None), N.TG_ERR_INVALID_ARGUMENT),
    ((0, 0, 0, -1, 4, 4, 1, 4, 1, 4, 1, 4, None, None), N.TG_ERR_INVALID_ARGUMENT),
    ((0, 0, 0, 4, 4, 4, None, 4, 1, 4, 1, 4, None, None), N.TG_ERR_INVALID_ARGUMENT),
    ((0, 0, 0, 4, 4, 4, 1, 3, 1, 4, 1, 4, None, None), N.TG_ERR_DIMENSION_MISMATCH),   # lda < K
    ((0, 0, 1, 4, 4, 4, 1, 4, 1, 4, 1, 3, None, None), N.TG_ERR_DIMENSION_MISMATCH),   # col-major ldc < M
])
def test_validation_error_codes(args, code):
    L = N.lib()
    rc = L.tg_gemm(*args)
    assert rc == code
    assert len(L.tg_last_error()) > 0


def test_empty_problem_is_ok_without_touching_memory():
    L = N.lib()
    assert L.tg_gemm(0, 0, 0, 0, 5, 5, None, 5, None, 5, None, 5, None, None) == N.TG_OK
    assert L.tg_gemm_strided_batched(0, 0, 0, 0, 5, 5, 5, None, 5, 25, None, 5, 25, None, 5, 25, None, None) == N.TG_OK


def test_backward_rejects_integer_types():
    L = N.lib()
    rc = L.tg_backward_a(0, 2, 0, 1, 4, 4, 4, 1, 4, 16, 1, None, 4, 16, 1, 4, 16, 0, None)
    assert rc == N.TG_ERR_UNSUPPORTED


def test_python_errors_map_to_reference_types():
    with pytest.raises(ValueError):
        N.check(N.TG_ERR_DIMENSION_MISMATCH)
    with pytest.raises(N.TropicalGemmError):
        N.check(N.TG_ERR_CUDA)


BCAST = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p,
                         ctypes.c_void_p)


def _sharded_lib():
    L = N.lib()
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    L.tg_sharded_gemm.argtypes = [ctypes.c_int, ctypes.c_int, i64, i64, i64, vp, i64, vp, i64, vp, i64, vp,
                                  ctypes.c_int, BCAST, vp, vp]
    L.tg_sharded_gemm.restype = ctypes.c_int
    return L


def test_sharded_gemm_broadcasts_before_computing():
    """A rank with no rows still takes part in the broadcast of B (strided
    extent (k-1)*ldb + n elements); a failing broadcast is reported and
    nothing is computed."""
    L = _sharded_lib()
    calls = []

    def cb(buf, nbytes, root, stream, ctx):
        calls.append((buf, nbytes, root))
        return 0

    f = BCAST(cb)
    rc = L.tg_sharded_gemm(0, 1, 0, 30, 20, None, 20, 0x1000, 32, None, 30, None, 3, f, None, None)
    assert rc == N.TG_OK and calls == [(0x1000, (19 * 32 + 30) * 8, 3)]
    fail = BCAST(lambda *a: 7)
    rc = L.tg_sharded_gemm(0, 0, 4, 4, 4, 0x10, 4, 0x20, 4, 0x30, 4, None, 0, fail, None, None)
    assert rc == N.TG_ERR_CUDA and b"code 7" in L.tg_last_error()
    rc = L.tg_sharded_gemm(0, 0, 4, 4, 4, 0x10, 4, 0x20, 4, 0x30, 4, None, 0, BCAST(0), None, None)
    assert rc == N.TG_ERR_INVALID_ARGUMENT
