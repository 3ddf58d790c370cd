"""ctypes binding of libtropical_gemm_b200.so (the C ABI in include/tropical_gemm_b200.h).

Torch is used only for device memory, streams and tensor plumbing: every
GEMM / backward runs in the library's own sm_100a kernels, launched on
torch's current CUDA stream for the tensors' device.  There is no CPU or
library fallback: if the shared library is missing, or no CUDA device is
present, calls raise.
"""
import ctypes
import os

import torch
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtropical_gemm_b200.so")

SEMIRINGS = {"maxplus": 0, "minplus": 1, "maxmul": 2}
DTYPES = {torch.float32: 0, torch.float64: 1, torch.int32: 2, torch.int64: 3}
ROW_MAJOR, COL_MAJOR = 0, 1

TG_OK = 0
TG_ERR_INVALID_ARGUMENT = 1
TG_ERR_DIMENSION_MISMATCH = 2
TG_ERR_UNSUPPORTED = 3
TG_ERR_CUDA = 4
TG_ERR_NO_DEVICE = 5


class TropicalGemmError(RuntimeError):
    """A CUDA-side failure reported by the engine."""


_lib = None


def lib() -> ctypes.CDLL:
    """Load the engine library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} not found: build it with `python __graft_entry__.py build` "
                "(or `make -C tropical-gemm_b200`)"
            )
        L = ctypes.CDLL(LIB_PATH)
        i64, vp, i32, i32p = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p
        L.tg_version.restype = ctypes.c_char_p
        L.tg_last_error.restype = ctypes.c_char_p
        L.tg_device_count.restype = ctypes.c_int
        L.tg_gemm.argtypes = [i32, i32, i32, i64, i64, i64, vp, i64, vp, i64, vp, i64, i32p, vp]
        L.tg_gemm.restype = i32
        L.tg_gemm_strided_batched.argtypes = [i32, i32, i32, i64, i64, i64, i64, vp, i64, i64, vp, i64, i64,
                                              vp, i64, i64, i32p, vp]
        L.tg_gemm_strided_batched.restype = i32
        L.tg_gemm_accumulate.argtypes = [i32, i32, i64, i64, i64, vp, i64, vp, i64, vp, i64, i32p, i32, vp]
        L.tg_gemm_accumulate.restype = i32
        for fn in (L.tg_backward_a, L.tg_backward_b):
            fn.argtypes = [i32, i32, i32, i64, i64, i64, i64, vp, i64, i64, i32p, vp, i64, i64, vp, i64, i64,
                           i32, vp]
            fn.restype = i32
        _lib = L
    return _lib


def version() -> str:
    return lib().tg_version().decode()


def device_count() -> int:
    try:
        return int(lib().tg_device_count())
    except ImportError:
        return 0


def check(status: int) -> None:
    if status == TG_OK:
        return
    msg = lib().tg_last_error().decode()
    if status in (TG_ERR_INVALID_ARGUMENT, TG_ERR_DIMENSION_MISMATCH):
        raise ValueError(msg)
    raise TropicalGemmError(f"tropical-gemm error {status}: {msg}")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*ts) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("the tropical-gemm engine needs CUDA tensors")


def gemm_out(semiring: str, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, argmax, layout: int = ROW_MAJOR,
             lda=None, ldb=None, ldc=None) -> None:
    """Raw 2-D call: writes c (and argmax when given) for C = A (x) B."""
    _require_cuda(a, b, c)
    if layout == ROW_MAJOR:
        m, k = a.shape[-2], a.shape[-1]
        n = b.shape[-1]
    else:  # the tensors hold column-major data: shapes are given as (rows, cols) of the math matrices
        m, k = a.shape[-2], a.shape[-1]
        n = b.shape[-1]
    lda = lda if lda is not None else (k if layout == ROW_MAJOR else m)
    ldb = ldb if ldb is not None else (n if layout == ROW_MAJOR else k)
    ldc = ldc if ldc is not None else (n if layout == ROW_MAJOR else m)
    with torch.cuda.device(a.device):
        check(lib().tg_gemm(SEMIRINGS[semiring], DTYPES[a.dtype], layout, m, n, k, a.data_ptr(), lda, b.data_ptr(),
                            ldb, c.data_ptr(), ldc, argmax.data_ptr() if argmax is not None else None, _stream(a)))


def _validate_pair(a: torch.Tensor, b: torch.Tensor, batched: bool) -> None:
    if a.device != b.device:
        raise ValueError(f"Tensors must be on the same device: A is on {a.device}, B is on {b.device}")
    if a.dtype != b.dtype:
        raise ValueError(f"Tensors must have the same dtype: A is {a.dtype}, B is {b.dtype}")
    if a.dtype not in DTYPES:
        raise ValueError(f"unsupported dtype {a.dtype}")
    nd = 3 if batched else 2
    if a.dim() != nd or b.dim() != nd:
        raise ValueError(f"Expected {nd}D tensors, got A with {a.dim()} dims, B with {b.dim()} dims")
    if batched and a.shape[0] != b.shape[0]:
        raise ValueError(f"Batch size mismatch: A has batch {a.shape[0]}, B has batch {b.shape[0]}")
    if a.shape[-1] != b.shape[-2]:
        raise ValueError(f"Dimension mismatch: A is {a.shape[-2]}x{a.shape[-1]}, B is {b.shape[-2]}x{b.shape[-1]}")


def gemm(semiring: str, a: torch.Tensor, b: torch.Tensor, with_argmax: bool = True):
    """Row-major C = A (x) B for 2-D CUDA tensors; returns (C, argmax int32 or None)."""
    _validate_pair(a, b, batched=False)
    _require_cuda(a, b)
    a = _rows(a)
    b = b.contiguous()
    m, k = a.shape
    n = b.shape[1]
    c = torch.empty((m, n), dtype=a.dtype, device=a.device)
    am = torch.empty((m, n), dtype=torch.int32, device=a.device) if with_argmax else None
    with torch.cuda.device(a.device):
        check(lib().tg_gemm(SEMIRINGS[semiring], DTYPES[a.dtype], ROW_MAJOR, m, n, k, a.data_ptr(), _ld(a),
                            b.data_ptr(), n, c.data_ptr(), n, am.data_ptr() if am is not None else None, _stream(a)))
    return c, am


def _rows(a: torch.Tensor) -> torch.Tensor:
    """`a` itself when its rows are contiguous (a column slice of a row-major
    matrix, for instance); a contiguous copy otherwise."""
    return a if a.dim() == 2 and a.stride(1) == 1 and a.stride(0) >= max(1, a.shape[1]) else a.contiguous()


def _ld(a: torch.Tensor) -> int:
    return max(1, a.stride(0)) if a.shape[0] > 1 else max(1, a.shape[1])


def gemm_accumulate(semiring: str, a: torch.Tensor, b: torch.Tensor, c: torch.Tensor,
                    argmax: Optional[torch.Tensor], k_offset: int) -> None:
    """In place over one K slice (f32, row-major): every output of `c`
    (and `argmax`) is replaced where a product of A[:, slice] (x) B[slice, :]
    strictly beats it; winning indices are k_offset + k.  Starting from
    gemm() over the first slice, the slices in ascending order give exactly
    gemm() over the whole K."""
    _validate_pair(a, b, batched=False)
    _require_cuda(a, b)
    if a.dtype != torch.float32:
        raise ValueError("gemm_accumulate is defined for f32")
    m, k = a.shape
    n = b.shape[1]
    if tuple(c.shape) != (m, n) or not c.is_contiguous() or c.dtype != torch.float32:
        raise ValueError("C must be a contiguous f32 (m, n) tensor")
    if argmax is not None and (tuple(argmax.shape) != (m, n) or not argmax.is_contiguous()
                               or argmax.dtype != torch.int32):
        raise ValueError("argmax must be a contiguous int32 (m, n) tensor")
    a = _rows(a)
    b = b.contiguous()
    with torch.cuda.device(a.device):
        check(lib().tg_gemm_accumulate(SEMIRINGS[semiring], ROW_MAJOR, m, n, k, a.data_ptr(), _ld(a), b.data_ptr(), n,
                                       c.data_ptr(), n, argmax.data_ptr() if argmax is not None else None,
                                       int(k_offset), _stream(a)))


def gemm_batched(semiring: str, a: torch.Tensor, b: torch.Tensor, with_argmax: bool = True):
    """Row-major strided-batched C[p] = A[p] (x) B[p] for 3-D CUDA tensors (one launch)."""
    _validate_pair(a, b, batched=True)
    _require_cuda(a, b)
    a = a.contiguous()
    b = b.contiguous()
    bs, m, k = a.shape
    n = b.shape[2]
    c = torch.empty((bs, m, n), dtype=a.dtype, device=a.device)
    am = torch.empty((bs, m, n), dtype=torch.int32, device=a.device) if with_argmax else None
    with torch.cuda.device(a.device):
        check(lib().tg_gemm_strided_batched(SEMIRINGS[semiring], DTYPES[a.dtype], ROW_MAJOR, bs, m, n, k,
                                            a.data_ptr(), k, m * k, b.data_ptr(), n, k * n, c.data_ptr(), n, m * n,
                                            am.data_ptr() if am is not None else None, _stream(a)))
    return c, am


def backward(semiring: str, want_a: bool, grad_c: torch.Tensor, argmax: torch.Tensor, k: int, partner=None):
    """Argmax-scatter gradient (row-major, 2-D or 3-D batched).

    want_a: returns grad_A (.., M, K); else grad_B (.., K, N).  partner is B
    (for grad_A) or A (for grad_B) and is required for MaxMul only.
    """
    _require_cuda(grad_c, argmax)
    grad_c = grad_c.contiguous()
    argmax = argmax.contiguous()
    if argmax.dtype != torch.int32:
        argmax = argmax.to(torch.int32)
    if grad_c.dtype not in (torch.float32, torch.float64):
        raise ValueError(f"backward needs float32/float64 gradients, got {grad_c.dtype}")
    batched = grad_c.dim() == 3
    bs = grad_c.shape[0] if batched else 1
    m, n = grad_c.shape[-2], grad_c.shape[-1]
    out_shape = (m, k) if want_a else (k, n)
    out = torch.empty(((bs,) if batched else ()) + out_shape, dtype=grad_c.dtype, device=grad_c.device)
    if partner is not None:
        partner = partner.detach().contiguous().to(grad_c.dtype)
    ldw = (n if want_a else k)
    sw = (k * n if want_a else m * k)
    fn = lib().tg_backward_a if want_a else lib().tg_backward_b
    with torch.cuda.device(grad_c.device):
        check(fn(SEMIRINGS[semiring], DTYPES[grad_c.dtype], ROW_MAJOR, bs, m, n, k, grad_c.data_ptr(), n, m * n,
                 argmax.data_ptr(), partner.data_ptr() if partner is not None else None, ldw, sw,
                 out.data_ptr(), out_shape[1], out_shape[0] * out_shape[1], 0, _stream(grad_c)))
    return out
