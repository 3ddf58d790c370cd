"""The reference extension module's function surface, served by the B200 engine.

Every name of TensorBFS/tropical-gemm's PyO3 module `tropical_gemm._core`
(crates/tropical-gemm-python/src/lib.rs, registered at :2565-2668) exists here
with the same arguments, return shapes and error types.  All of them compute on
the GPU through libtropical_gemm_b200.so:

* numpy functions (`maxplus_matmul`, `..._with_argmax`, `..._2d`, f64/i32/i64,
  `backward_*`, batched) copy their inputs to the current CUDA device, run the
  engine and copy the result back.  Results follow the reference GPU
  semantics (the integer sentinels +-46340 / +-3037000499 with saturating
  add); for floats they equal the reference CPU results bit for bit.
* `*_matmul_gpu[_with_argmax]` keep the reference's literal buffer
  convention: the row-major numpy buffers are handed to the column-major GPU
  API unchanged and the column-major result comes back flattened
  (lib.rs:1904-1907 -> crates/tropical-gemm-cuda/src/lib.rs:198-221).
* `*_matmul_dlpack` / `*_matmul_batched_dlpack` take CUDA tensors (anything
  torch.from_dlpack accepts), run on the current stream without a host
  synchronisation, and return tensors (usable wherever the reference's
  DLPack capsules were: torch.from_dlpack accepts them).  f32 only and
  contiguous only, as in the reference (lib.rs:2193-2245, :2462-2527).
"""
import numpy as np
import torch

from . import _native as N

__all__ = []


def _export(fn):
    __all__.append(fn.__name__)
    return fn


def cuda_available() -> bool:
    """True when a CUDA device is visible and the engine library is loadable."""
    try:
        N.lib()
    except ImportError:
        return False
    return torch.cuda.is_available() and N.device_count() > 0


__all__.append("cuda_available")


def _device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA error: no CUDA device available for the tropical-gemm engine")
    return torch.device("cuda", torch.cuda.current_device())


def _as2d(x, dtype, name):
    x = np.asarray(x)
    if x.dtype != dtype:
        raise TypeError(f"argument '{name}': expected a numpy array of dtype {np.dtype(dtype)}, got {x.dtype}")
    if x.ndim != 2:
        raise TypeError(f"argument '{name}': expected a 2-D array, got {x.ndim}-D")
    return np.ascontiguousarray(x)


def _check_dims(a, b):
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"Dimension mismatch: A is {a.shape[0]}x{a.shape[1]}, B is {b.shape[0]}x{b.shape[1]}")


def _run(semiring, a, b, with_argmax):
    dev = _device()
    ta = torch.from_numpy(a).to(dev)
    tb = torch.from_numpy(b).to(dev)
    c, am = N.gemm(semiring, ta, tb, with_argmax)
    return c.cpu().numpy(), (am.cpu().numpy() if am is not None else None)


_TYPES = {"": np.float32, "_f64": np.float64, "_i32": np.int32, "_i64": np.int64}


def _make_matmul(semi, sfx, dtype, two_d):
    def fn(a, b):
        a = _as2d(a, dtype, "a")
        b = _as2d(b, dtype, "b")
        _check_dims(a, b)
        c, _ = _run(semi, a, b, False)
        return c if two_d else c.reshape(-1)
    fn.__name__ = f"{semi}_matmul{'_2d' if two_d else ''}{sfx}"
    fn.__doc__ = (f"Tropical {semi} matmul of ({np.dtype(dtype)}) A[M,K] and B[K,N]; returns C "
                  f"{'as an (M, N) array' if two_d else 'flattened (row-major)'}.")
    return fn


def _make_argmax(semi, sfx, dtype):
    def fn(a, b):
        a = _as2d(a, dtype, "a")
        b = _as2d(b, dtype, "b")
        _check_dims(a, b)
        c, am = _run(semi, a, b, True)
        return c.reshape(-1), am.reshape(-1)
    fn.__name__ = f"{semi}_matmul_with_argmax{sfx}"
    fn.__doc__ = "Returns (C, argmax) flattened row-major; argmax[i*N+j] is the winning k (int32)."
    return fn


for _semi in ("maxplus", "minplus", "maxmul"):
    for _sfx, _dt in _TYPES.items():
        for _two in (False, True):
            _f = _make_matmul(_semi, _sfx, _dt, _two)
            globals()[_f.__name__] = _export(_f)
        if _sfx in ("", "_f64"):
            _f = _make_argmax(_semi, _sfx, _dt)
            globals()[_f.__name__] = _export(_f)


def _make_backward(which, sfx, dtype, maxmul):
    want_a = which == "a"

    if maxmul:
        def fn(grad_c, argmax, partner):
            g = _as2d(grad_c, dtype, "grad_c")
            am = _as2d(argmax, np.int32, "argmax")
            p = _as2d(partner, dtype, "b" if want_a else "a")
            k = p.shape[0] if want_a else p.shape[1]
            dev = _device()
            out = N.backward("maxmul", want_a, torch.from_numpy(g).to(dev), torch.from_numpy(am).to(dev), k,
                             torch.from_numpy(p).to(dev))
            return out.cpu().numpy().reshape(-1)
        fn.__name__ = f"maxmul_backward_{which}{sfx}"
    else:
        def fn(grad_c, argmax, k):
            g = _as2d(grad_c, dtype, "grad_c")
            am = _as2d(argmax, np.int32, "argmax")
            dev = _device()
            out = N.backward("maxplus", want_a, torch.from_numpy(g).to(dev), torch.from_numpy(am).to(dev), int(k))
            return out.cpu().numpy().reshape(-1)
        fn.__name__ = f"backward_{which}{sfx}"
    fn.__doc__ = (f"Gradient w.r.t. {'A' if want_a else 'B'} through argmax (flattened row-major); "
                  "indices outside [0, K) are skipped.")
    return fn


for _which in ("a", "b"):
    for _sfx, _dt in (("", np.float32), ("_f64", np.float64)):
        for _mm in (False, True):
            _f = _make_backward(_which, _sfx, _dt, _mm)
            globals()[_f.__name__] = _export(_f)


def _make_batched(semi):
    def fn(a, b):
        a = np.asarray(a)
        b = np.asarray(b)
        if a.dtype != np.float32 or b.dtype != np.float32 or a.ndim != 3 or b.ndim != 3:
            raise TypeError("expected 3-D float32 arrays")
        if a.shape[0] != b.shape[0]:
            raise ValueError(f"Batch size mismatch: A has batch {a.shape[0]}, B has batch {b.shape[0]}")
        if a.shape[2] != b.shape[1]:
            raise ValueError(f"Dimension mismatch: A is (batch, {a.shape[1]}, {a.shape[2]}), "
                             f"B is (batch, {b.shape[1]}, {b.shape[2]})")
        dev = _device()
        c, am = N.gemm_batched(semi, torch.from_numpy(np.ascontiguousarray(a)).to(dev),
                               torch.from_numpy(np.ascontiguousarray(b)).to(dev), True)
        return c.cpu().numpy().reshape(-1), am.cpu().numpy().reshape(-1)
    fn.__name__ = f"{semi}_matmul_batched_with_argmax"
    fn.__doc__ = "Batched (batch, M, K) x (batch, K, N) with argmax; returns flattened (C, argmax)."
    return fn


for _semi in ("maxplus", "minplus", "maxmul"):
    _f = _make_batched(_semi)
    globals()[_f.__name__] = _export(_f)


# ------------------------------------------------ numpy GPU functions (literal convention)
def _make_gpu(semi, with_argmax):
    def fn(a, b):
        a = _as2d(a, np.float32, "a")
        b = _as2d(b, np.float32, "b")
        _check_dims(a, b)
        m, k = a.shape
        n = b.shape[1]
        dev = _device()
        ta = torch.from_numpy(a).to(dev)  # buffer read as column-major m x k (ld m), like the reference
        tb = torch.from_numpy(b).to(dev)
        c = torch.empty(m * n, dtype=torch.float32, device=dev)
        am = torch.empty(m * n, dtype=torch.int32, device=dev) if with_argmax else None
        with torch.cuda.device(dev):
            N.check(N.lib().tg_gemm(N.SEMIRINGS[semi], 0, N.COL_MAJOR, m, n, k, ta.data_ptr(), m, tb.data_ptr(),
                                    k, c.data_ptr(), m, am.data_ptr() if am is not None else None,
                                    torch.cuda.current_stream(dev).cuda_stream))
        if with_argmax:
            return c.cpu().numpy(), am.cpu().numpy()
        return c.cpu().numpy()
    fn.__name__ = f"{semi}_matmul_gpu{'_with_argmax' if with_argmax else ''}"
    fn.__doc__ = ("GPU matmul with the reference's buffer convention: inputs and the flattened output are "
                  "interpreted column-major.")
    return fn


for _semi in ("maxplus", "minplus", "maxmul"):
    for _wa in (False, True):
        _f = _make_gpu(_semi, _wa)
        globals()[_f.__name__] = _export(_f)


# ------------------------------------------------ DLPack-style tensor functions
def _to_tensor(x):
    return x if isinstance(x, torch.Tensor) else torch.from_dlpack(x)


def _check_tensor_pair(a, b, nd):
    if a.device.type != b.device.type:
        raise ValueError(f"Tensors must be on the same device type: A is on {a.device.type}, B is on {b.device.type}")
    if a.device != b.device:
        raise ValueError(f"Tensors must be on the same device: A is on device {a.device.index}, "
                         f"B is on device {b.device.index}")
    if a.dtype != b.dtype:
        raise ValueError(f"Tensors must have the same dtype: A is {a.dtype}, B is {b.dtype}")
    if a.dtype != torch.float32:
        raise ValueError("Only f32 tensors are supported for DLPack interface")
    if a.dim() != nd or b.dim() != nd:
        raise ValueError(f"Expected {nd}D tensors, got A with {a.dim()} dims, B with {b.dim()} dims")
    if not a.is_contiguous() or not b.is_contiguous():
        raise ValueError("Tensors must be contiguous (call .contiguous() on PyTorch tensors)")


def _make_dlpack(semi):
    def fn(a, b):
        a = _to_tensor(a)
        b = _to_tensor(b)
        _check_tensor_pair(a, b, 2)
        m, k = a.shape
        k2, n = b.shape
        if k != k2:
            raise ValueError(f"Dimension mismatch: A is {m}x{k}, B is {k2}x{n}")
        if m == 0 or k == 0 or n == 0:
            raise ValueError(f"Zero-sized dimensions not supported: m={m}, k={k}, n={n}")
        if not a.is_cuda:  # the reference's CPU-tensor branch (lib.rs:2290-2332) has no place in a GPU engine
            raise ValueError("the B200 engine takes CUDA tensors; move the tensors to a CUDA device")
        c, am = N.gemm(semi, a, b, True)
        return c.reshape(-1), am.reshape(-1)
    fn.__name__ = f"{semi}_matmul_dlpack"
    fn.__doc__ = "Row-major f32 CUDA tensors in, flattened (C, argmax int32) CUDA tensors out."
    return fn


def _make_batched_dlpack(semi):
    def fn(a, b):
        a = _to_tensor(a)
        b = _to_tensor(b)
        _check_tensor_pair(a, b, 3)
        if a.shape[0] != b.shape[0]:
            raise ValueError(f"Batch size mismatch: A has batch {a.shape[0]}, B has batch {b.shape[0]}")
        if a.shape[2] != b.shape[1]:
            raise ValueError(f"Dimension mismatch: A is (batch, {a.shape[1]}, {a.shape[2]}), "
                             f"B is (batch, {b.shape[1]}, {b.shape[2]})")
        if 0 in a.shape or b.shape[2] == 0:
            raise ValueError("Zero-sized dimensions not supported")
        if not a.is_cuda:
            raise ValueError("the B200 engine takes CUDA tensors; move the tensors to a CUDA device")
        return N.gemm_batched(semi, a, b, True)
    fn.__name__ = f"{semi}_matmul_batched_dlpack"
    fn.__doc__ = "(batch, M, K) x (batch, K, N) f32 CUDA tensors -> (C, argmax int32), one launch."
    return fn


for _semi in ("maxplus", "minplus", "maxmul"):
    for _mk in (_make_dlpack, _make_batched_dlpack):
        _f = _mk(_semi)
        globals()[_f.__name__] = _export(_f)
