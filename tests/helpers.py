"""Shared helpers for the GPU parity tests (engine via the C ABI, oracle on CPU)."""
import ctypes
import os

import numpy as np
import torch

from tropical_gemm import _native as N
from oracle import tg_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SEMIS = ("maxplus", "minplus", "maxmul")
NP2T = {np.float32: torch.float32, np.float64: torch.float64, np.int32: torch.int32, np.int64: torch.int64}


def dev():
    return torch.device("cuda", 0)


def same_bits(x: np.ndarray, y: np.ndarray) -> bool:
    return x.shape == y.shape and x.dtype == y.dtype and np.array_equal(
        np.ascontiguousarray(x).view(np.uint8), np.ascontiguousarray(y).view(np.uint8))


def engine(semi, a: np.ndarray, b: np.ndarray, with_argmax=True):
    ta = torch.from_numpy(np.ascontiguousarray(a)).to(dev())
    tb = torch.from_numpy(np.ascontiguousarray(b)).to(dev())
    if a.ndim == 3:
        c, am = N.gemm_batched(semi, ta, tb, with_argmax)
    else:
        c, am = N.gemm(semi, ta, tb, with_argmax)
    torch.cuda.synchronize()
    return c.cpu().numpy(), (am.cpu().numpy() if am is not None else None)


def engine_colmajor(semi, a: np.ndarray, b: np.ndarray, with_argmax=True):
    """Same math through the column-major entry (the Rust API's convention)."""
    m, k = a.shape
    n = b.shape[1]
    ta = torch.from_numpy(np.asfortranarray(a).ravel(order="K").copy()).to(dev())
    tb = torch.from_numpy(np.asfortranarray(b).ravel(order="K").copy()).to(dev())
    c = torch.empty(m * n, dtype=ta.dtype, device=dev())
    am = torch.empty(m * n, dtype=torch.int32, device=dev()) if with_argmax else None
    N.check(N.lib().tg_gemm(N.SEMIRINGS[semi], N.DTYPES[ta.dtype], N.COL_MAJOR, m, n, k, ta.data_ptr(), m,
                            tb.data_ptr(), k, c.data_ptr(), m, am.data_ptr() if am is not None else None,
                            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    cc = c.cpu().numpy().reshape(n, m).T
    aa = am.cpu().numpy().reshape(n, m).T if am is not None else None
    return np.ascontiguousarray(cc), (np.ascontiguousarray(aa) if aa is not None else None)


def oracle(semi, a, b, with_argmax=True):
    if a.ndim == 3:
        return O.gemm_batched(semi, a, b, with_argmax)
    return O.gemm(semi, a, b, with_argmax)


from oracle.ref_gpu import ref_lib, ref_rowmajor  # noqa: E402,F401
