"""ctypes front end of oracle/_ref/libref_gpu.so -- TEST INFRASTRUCTURE ONLY.

The library is the reference's own CUDA kernel file compiled from its sources
(see oracle/Makefile and ref_gpu_launch.cu).  Used by the GPU parity tests and
by bench.py's reference arm; never by the product.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(_HERE, "_ref", "libref_gpu.so")
SEMIRINGS = {"maxplus": 0, "minplus": 1, "maxmul": 2}
DTYPES = {torch.float32: 0, torch.float64: 1, torch.int32: 2, torch.int64: 3}
_ref = None


def ref_lib():
    """Loaded library, or None when it has not been built."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB):
            return None
        L = ctypes.CDLL(REF_LIB)
        i, vp = ctypes.c_int, ctypes.c_void_p
        L.ref_gemm.argtypes = [i, i, i, i, i, i, vp, vp, vp, vp, vp]
        L.ref_gemm_batched_argmax_f32.argtypes = [i, i, i, i, i, vp, vp, vp, vp, i, i, i, vp]
        L.ref_backward.argtypes = [i, i, vp, vp, vp, i, i, i, vp]
        _ref = L
    return _ref


def ref_rowmajor(semi, ta: torch.Tensor, tb: torch.Tensor, with_argmax=True):
    """Reference kernel on row-major device tensors via its swap convention
    (crates/tropical-gemm-cuda/src/kernels.rs:416-430): C^T = B^T (x) A^T."""
    L = ref_lib()
    m, k = ta.shape
    n = tb.shape[1]
    c = torch.empty((m, n), dtype=ta.dtype, device=ta.device)
    am = torch.empty((m, n), dtype=torch.int32, device=ta.device) if with_argmax else None
    rc = L.ref_gemm(SEMIRINGS[semi], DTYPES[ta.dtype], int(with_argmax), n, m, k, tb.data_ptr(), ta.data_ptr(),
                    c.data_ptr(), am.data_ptr() if am is not None else None,
                    torch.cuda.current_stream(ta.device).cuda_stream)
    if rc != 0:
        raise RuntimeError(f"reference kernel launch failed: {rc}")
    return c, am
