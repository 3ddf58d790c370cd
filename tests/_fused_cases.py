"""Parity cases for the persistent fused-resolution argmax kernel, run in a
child process started with TROPICAL_GEMM_ARGMAX_FUSED=1 so that the kernel
is used at sizes the CPU oracle checks in seconds (by default it is chosen
only for large problems).  Prints one line per case and exits non-zero on
the first mismatch."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (os.path.join(ROOT, "tropical-gemm_b200"), ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

from helpers import engine, oracle, same_bits  # noqa: E402


def data(rng, shape, kind, semi):
    if kind == "ties":
        x = rng.integers(-3, 4, shape).astype(np.float32)
    else:
        x = rng.standard_normal(shape).astype(np.float32)
    if semi == "maxmul":
        x = np.abs(x)
    return x


def pattern(semi, m, k, n, which):
    kk = np.arange(k, dtype=np.float32) * 0.01
    if semi == "minplus":
        kk = -kk
    if which == "increasing":
        a = np.tile(kk, (m, 1)) + 1.0
    elif which == "decreasing":
        a = np.tile(-kk, (m, 1)) + 1.0
    else:   # a plateau of equal products over k in [500, 1800)
        a = np.ones((m, k), np.float32)
        a[:, 500:1800] = 2.0 if semi != "minplus" else 0.5
    return a.astype(np.float32), np.ones((k, n), np.float32)


def check(tag, semi, a, b, rows=None):
    c, am = engine(semi, a, b)
    if rows is None:
        c0, am0 = oracle(semi, a, b)
        ok = same_bits(c, c0) and np.array_equal(am, am0)
    else:   # full rows (all k) of a sample
        c0, am0 = oracle(semi, np.ascontiguousarray(a[rows]), b)
        ok = same_bits(c[rows], c0) and np.array_equal(am[rows], am0)
    print(tag, "ok" if ok else "MISMATCH", flush=True)
    return ok


def main():
    rng = np.random.default_rng(2024)
    ok = True
    # odd and even k-tile counts, k tails, single- and multi-tile CTAs
    for semi in ("maxplus", "minplus", "maxmul"):
        for (m, k, n, kind) in [(300, 1100, 260, "normal"), (129, 2049, 131, "ties"), (64, 1056, 200, "ties"),
                                (200, 4096, 130, "normal"), (70, 33000, 130, "ties")]:
            a, b = data(rng, (m, k), kind, semi), data(rng, (k, n), kind, semi)
            ok &= check(f"{semi} {m}x{k}x{n} {kind}", semi, a, b)
        for which in ("increasing", "decreasing", "plateau"):
            a, b = pattern(semi, 256, 2100, 256, which)
            ok &= check(f"{semi} pattern {which}", semi, a, b)
    # more tiles than SMs: CTAs walk several tiles and cross row panels (drain passes)
    a = data(rng, (1536, 1100), "ties", "maxplus")
    b = data(rng, (1100, 1664), "ties", "maxplus")
    ok &= check("maxplus 1536x1100x1664 ties (persistent)", "maxplus", a, b, rows=rng.choice(1536, 96, replace=False))
    a = data(rng, (2048, 1500), "normal", "minplus")
    b = data(rng, (1500, 2304), "normal", "minplus")
    ok &= check("minplus 2048x1500x2304 (persistent)", "minplus", a, b, rows=rng.choice(2048, 96, replace=False))
    # special values: +-inf and signed zeros
    for semi in ("maxplus", "minplus"):
        a = data(rng, (150, 1300), "normal", semi)
        b = data(rng, (1300, 133), "normal", semi)
        for arr in (a, b):
            mask = rng.random(arr.shape)
            arr[mask < 0.05] = np.inf
            arr[(mask >= 0.05) & (mask < 0.10)] = -np.inf
            arr[(mask >= 0.10) & (mask < 0.15)] = -0.0
            arr[(mask >= 0.15) & (mask < 0.20)] = 0.0
        ok &= check(f"{semi} special values", semi, a, b)
    z = np.full((100, 1200), -0.0, np.float32)
    ok &= check("maxplus all signed zeros", "maxplus", z, np.full((1200, 90), -0.0, np.float32))
    # batched
    a = rng.integers(-5, 6, (3, 200, 2100)).astype(np.float32)
    b = rng.integers(-5, 6, (3, 2100, 300)).astype(np.float32)
    ok &= check("maxplus batched", "maxplus", a, b)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
