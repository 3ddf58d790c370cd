"""PyTorch autograd integration, same names as tropical_gemm.pytorch of the reference.

Reference: crates/tropical-gemm-python/python/tropical_gemm/pytorch.py (classes
:72-860, wrappers :868-1000).  What differs, by design:

* Every class computes with the B200 engine on torch's current CUDA stream.
  The reference's "CPU" classes (TropicalMaxPlusMatmul, ...) ran a Rust CPU
  kernel through numpy; here CPU tensors are moved to the current CUDA device,
  computed there, and the result is returned on the input's device (there is
  no CPU compute path).
* argmax stays int32 on the device (the reference converted it to int64 for
  scatter_add_, pytorch.py:377), and the backward is the engine's histogram
  kernel instead of zeros + two scatter_add_ + transposes (pytorch.py:386-403).
* Forward values and argmax are bit-identical to the reference's; gradients
  agree to float rounding (summation order inside a bin is unordered, as
  with the reference's scatter_add_/atomicAdd).
"""
import torch

import tropical_gemm
from . import _native as N

GPU_AVAILABLE = tropical_gemm.cuda_available()
_DLPACK_AVAILABLE = GPU_AVAILABLE
_BATCHED_DLPACK_AVAILABLE = GPU_AVAILABLE


def _compute_device(*ts) -> torch.device:
    for t in ts:
        if t.is_cuda:
            return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("tropical_gemm.pytorch needs a CUDA device (the engine has no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


def _compute_dtype(t: torch.Tensor) -> torch.dtype:
    return torch.float64 if t.dtype == torch.float64 else torch.float32


class _TropicalMatmulBase(torch.autograd.Function):
    SEMIRING = "maxplus"
    BATCHED = False
    REQUIRE_CUDA = False

    @classmethod
    def forward(cls, ctx, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
        if cls.REQUIRE_CUDA and not a.is_cuda:
            name = cls.__name__
            raise RuntimeError(f"{name} requires CUDA tensors. Use {name[:-3]} for CPU tensors.")
        if cls.BATCHED and (a.is_cuda or b.is_cuda) and a.device != b.device:
            raise RuntimeError(f"Tensors must be on the same device: a is on {a.device}, b is on {b.device}")
        dev = _compute_device(a, b)
        dt = _compute_dtype(a)
        ad = a.detach().to(device=dev, dtype=dt)
        bd = b.detach().to(device=dev, dtype=dt)
        if cls.BATCHED:
            c, am = N.gemm_batched(cls.SEMIRING, ad, bd, True)
        else:
            c, am = N.gemm(cls.SEMIRING, ad, bd, True)
        if cls.SEMIRING == "maxmul":
            ctx.save_for_backward(am, ad, bd)
        else:
            ctx.save_for_backward(am)
        ctx.k = a.shape[-1]
        ctx.out_device = a.device
        ctx.in_dtypes = (a.dtype, b.dtype)
        return c.to(a.device)

    @classmethod
    def backward(cls, ctx, grad_c: torch.Tensor):
        saved = ctx.saved_tensors
        am = saved[0]
        # contiguous once for both gradients (sum().backward() hands in a stride-0 expansion)
        g = grad_c.to(device=am.device, dtype=saved[1].dtype if len(saved) > 1 else _compute_dtype(grad_c))
        g = g.contiguous()
        if cls.SEMIRING == "maxmul":
            _, ad, bd = saved
            ga = N.backward("maxmul", True, g, am, ctx.k, bd) if ctx.needs_input_grad[0] else None
            gb = N.backward("maxmul", False, g, am, ctx.k, ad) if ctx.needs_input_grad[1] else None
        else:
            ga = N.backward(cls.SEMIRING, True, g, am, ctx.k) if ctx.needs_input_grad[0] else None
            gb = N.backward(cls.SEMIRING, False, g, am, ctx.k) if ctx.needs_input_grad[1] else None
        if ga is not None:
            ga = ga.to(device=ctx.out_device, dtype=ctx.in_dtypes[0])
        if gb is not None:
            gb = gb.to(device=ctx.out_device, dtype=ctx.in_dtypes[1])
        return ga, gb


class TropicalMaxPlusMatmul(_TropicalMatmulBase):
    """C[i,j] = max_k(A[i,k] + B[k,j]); gradient flows to A[i,argmax] and B[argmax,j]."""
    SEMIRING = "maxplus"


class TropicalMinPlusMatmul(_TropicalMatmulBase):
    """C[i,j] = min_k(A[i,k] + B[k,j])."""
    SEMIRING = "minplus"


class TropicalMaxMulMatmul(_TropicalMatmulBase):
    """C[i,j] = max_k(A[i,k] * B[k,j]); gradients use the multiplicative rule."""
    SEMIRING = "maxmul"


class TropicalMaxPlusMatmulGPU(_TropicalMatmulBase):
    """MaxPlus on CUDA tensors (raises for CPU tensors, as the reference does)."""
    SEMIRING = "maxplus"
    REQUIRE_CUDA = True


class TropicalMinPlusMatmulGPU(_TropicalMatmulBase):
    SEMIRING = "minplus"
    REQUIRE_CUDA = True


class TropicalMaxMulMatmulGPU(_TropicalMatmulBase):
    SEMIRING = "maxmul"
    REQUIRE_CUDA = True


class TropicalMaxPlusMatmulBatched(_TropicalMatmulBase):
    """C[b,i,j] = max_k(A[b,i,k] + B[b,k,j]) in one strided-batched launch."""
    SEMIRING = "maxplus"
    BATCHED = True


class TropicalMinPlusMatmulBatched(_TropicalMatmulBase):
    SEMIRING = "minplus"
    BATCHED = True


class TropicalMaxMulMatmulBatched(_TropicalMatmulBase):
    SEMIRING = "maxmul"
    BATCHED = True


def tropical_maxplus_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """MaxPlus tropical matmul (M,K) x (K,N) -> (M,N) with autograd."""
    return TropicalMaxPlusMatmul.apply(a, b)


def tropical_minplus_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """MinPlus tropical matmul (M,K) x (K,N) -> (M,N) with autograd."""
    return TropicalMinPlusMatmul.apply(a, b)


def tropical_maxmul_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """MaxMul tropical matmul (M,K) x (K,N) -> (M,N) with autograd."""
    return TropicalMaxMulMatmul.apply(a, b)


def tropical_maxplus_matmul_gpu(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """MaxPlus on CUDA tensors; raises RuntimeError for CPU tensors."""
    return TropicalMaxPlusMatmulGPU.apply(a, b)


def tropical_minplus_matmul_gpu(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return TropicalMinPlusMatmulGPU.apply(a, b)


def tropical_maxmul_matmul_gpu(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return TropicalMaxMulMatmulGPU.apply(a, b)


def tropical_maxplus_matmul_batched(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Batched MaxPlus (batch,M,K) x (batch,K,N) -> (batch,M,N) with autograd."""
    return TropicalMaxPlusMatmulBatched.apply(a, b)


def tropical_minplus_matmul_batched(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return TropicalMinPlusMatmulBatched.apply(a, b)


def tropical_maxmul_matmul_batched(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return TropicalMaxMulMatmulBatched.apply(a, b)


__all__ = [
    "TropicalMaxPlusMatmul", "TropicalMinPlusMatmul", "TropicalMaxMulMatmul",
    "TropicalMaxPlusMatmulGPU", "TropicalMinPlusMatmulGPU", "TropicalMaxMulMatmulGPU",
    "TropicalMaxPlusMatmulBatched", "TropicalMinPlusMatmulBatched", "TropicalMaxMulMatmulBatched",
    "tropical_maxplus_matmul", "tropical_minplus_matmul", "tropical_maxmul_matmul",
    "tropical_maxplus_matmul_gpu", "tropical_minplus_matmul_gpu", "tropical_maxmul_matmul_gpu",
    "tropical_maxplus_matmul_batched", "tropical_minplus_matmul_batched", "tropical_maxmul_matmul_batched",
    "GPU_AVAILABLE", "_DLPACK_AVAILABLE",
]
