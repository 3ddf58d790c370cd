"""The Python surface a reference user imports is all present (names from
crates/tropical-gemm-python/python/tropical_gemm/__init__.py:26-155,
src/lib.rs:2565-2668 and python/tropical_gemm/pytorch.py:1003-1031)."""
import numpy as np
import pytest

import tropical_gemm
import tropical_gemm.pytorch as tp

CORE = [
    "maxplus_matmul", "minplus_matmul", "maxmul_matmul",
    "maxplus_matmul_with_argmax", "minplus_matmul_with_argmax", "maxmul_matmul_with_argmax",
    "backward_a", "backward_b",
    "maxplus_matmul_f64", "minplus_matmul_f64", "maxmul_matmul_f64",
    "maxplus_matmul_with_argmax_f64", "minplus_matmul_with_argmax_f64", "maxmul_matmul_with_argmax_f64",
    "backward_a_f64", "backward_b_f64",
    "maxmul_backward_a", "maxmul_backward_b", "maxmul_backward_a_f64", "maxmul_backward_b_f64",
    "maxplus_matmul_i32", "minplus_matmul_i32", "maxmul_matmul_i32",
    "maxplus_matmul_i64", "minplus_matmul_i64", "maxmul_matmul_i64",
    "maxplus_matmul_2d", "minplus_matmul_2d", "maxmul_matmul_2d",
    "maxplus_matmul_2d_f64", "minplus_matmul_2d_f64", "maxmul_matmul_2d_f64",
    "maxplus_matmul_2d_i32", "minplus_matmul_2d_i32", "maxmul_matmul_2d_i32",
    "maxplus_matmul_2d_i64", "minplus_matmul_2d_i64", "maxmul_matmul_2d_i64",
    "maxplus_matmul_batched_with_argmax", "minplus_matmul_batched_with_argmax", "maxmul_matmul_batched_with_argmax",
    "maxplus_matmul_gpu", "minplus_matmul_gpu", "maxmul_matmul_gpu",
    "maxplus_matmul_gpu_with_argmax", "minplus_matmul_gpu_with_argmax", "maxmul_matmul_gpu_with_argmax",
    "maxplus_matmul_dlpack", "minplus_matmul_dlpack", "maxmul_matmul_dlpack",
    "maxplus_matmul_batched_dlpack", "minplus_matmul_batched_dlpack", "maxmul_matmul_batched_dlpack",
    "cuda_available",
]

TORCH = [
    "TropicalMaxPlusMatmul", "TropicalMinPlusMatmul", "TropicalMaxMulMatmul",
    "TropicalMaxPlusMatmulGPU", "TropicalMinPlusMatmulGPU", "TropicalMaxMulMatmulGPU",
    "TropicalMaxPlusMatmulBatched", "TropicalMinPlusMatmulBatched", "TropicalMaxMulMatmulBatched",
    "tropical_maxplus_matmul", "tropical_minplus_matmul", "tropical_maxmul_matmul",
    "tropical_maxplus_matmul_gpu", "tropical_minplus_matmul_gpu", "tropical_maxmul_matmul_gpu",
    "tropical_maxplus_matmul_batched", "tropical_minplus_matmul_batched", "tropical_maxmul_matmul_batched",
    "GPU_AVAILABLE", "_DLPACK_AVAILABLE",
]


@pytest.mark.parametrize("name", CORE)
def test_core_name(name):
    assert callable(getattr(tropical_gemm, name))


@pytest.mark.parametrize("name", TORCH)
def test_torch_name(name):
    assert hasattr(tp, name)


def test_dimension_mismatch_is_value_error():
    a = np.zeros((2, 3), np.float32)
    b = np.zeros((4, 2), np.float32)
    with pytest.raises(ValueError, match="Dimension mismatch"):
        tropical_gemm.maxplus_matmul(a, b)


def test_wrong_dtype_is_type_error():
    with pytest.raises(TypeError):
        tropical_gemm.maxplus_matmul(np.zeros((2, 2), np.float64), np.zeros((2, 2), np.float64))


def test_cuda_available_is_bool():
    assert isinstance(tropical_gemm.cuda_available(), bool)
