"""tropical_gemm -- B200-native tropical matrix multiplication.

Drop-in for the GPU path of TensorBFS/tropical-gemm: the same module
(`tropical_gemm`, `tropical_gemm.pytorch`) and function names, computing in
hand-written sm_100a kernels (libtropical_gemm_b200.so).  C = A (x) B over
MaxPlus / MinPlus / MaxMul for f32, f64, i32 and i64, optional argmax, a
strided-batched variant and the argmax-scatter backward.

    >>> import numpy as np, tropical_gemm
    >>> a = np.random.randn(100, 50).astype(np.float32)
    >>> b = np.random.randn(50, 80).astype(np.float32)
    >>> c = tropical_gemm.maxplus_matmul(a, b)
    >>> c, argmax = tropical_gemm.maxplus_matmul_with_argmax(a, b)
"""
from tropical_gemm._core import *  # noqa: F401,F403
from tropical_gemm._core import __all__ as _core_all
from tropical_gemm._core import cuda_available  # noqa: F401

__version__ = "0.2.0"

__all__ = list(_core_all)
