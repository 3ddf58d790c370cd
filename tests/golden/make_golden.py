"""Regenerate tests/golden/reference_fixtures.npz from the reference's golden vectors.

The reference (TensorBFS/tropical-gemm v0.2.0) ships JSON fixtures produced by
TropicalNumbers.jl (crates/tropical-gemm-python/tests/fixtures/, generator
julia_generator.jl, seed 42; format in fixtures/README.md:59-95): row-major
A, B, expected C and 0-based argmax for MaxPlus/MinPlus/MaxMul x f32/f64,
including batched and special-value cases.  This script packs the in-scope ones
(the three tropical semirings; the and-or and counting semirings have no GPU
path) into one compressed .npz so tests can run where the reference tree is
absent.  Values are stored in their native dtype; argmax as int32.

Usage: python tests/golden/make_golden.py [REFERENCE_ROOT]
"""
import json
import os
import sys

import numpy as np

SEMIRINGS = ("maxplus", "minplus", "maxmul")
SCALARS = {"f32": np.float32, "f64": np.float64}


def main() -> None:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REF_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (or set REF_ROOT)")
    fdir = os.path.join(root, "crates/tropical-gemm-python/tests/fixtures")
    out = {}
    names = []
    for semi in SEMIRINGS:
        for scal, dt in SCALARS.items():
            d = os.path.join(fdir, f"{semi}_{scal}")
            for fn in sorted(os.listdir(d)):
                if not fn.endswith(".json"):
                    continue
                with open(os.path.join(d, fn)) as f:
                    fx = json.load(f)
                key = f"{semi}_{scal}__{fn[:-5]}"
                names.append(key)
                out[key + "__a"] = np.asarray(fx["a"], dtype=dt)
                out[key + "__b"] = np.asarray(fx["b"], dtype=dt)
                out[key + "__c"] = np.asarray(fx["c_expected"], dtype=dt)
                out[key + "__argmax"] = np.asarray(fx["argmax_expected"], dtype=np.int32)
    out["__names__"] = np.asarray(names)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_fixtures.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {len(names)} fixtures to {dst}")


if __name__ == "__main__":
    main()
