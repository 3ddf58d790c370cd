"""Benchmark: tropical ops/s (M*N*K/s) of f32 MaxPlus + argmax at 8192^3 on B200.

Contract (one JSON line on rank 0):
  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl engine|reference]

* N = 1: BASELINE config 2a -- MaxPlus<f32> with argmax, M = N = K = 8192,
  A and B i.i.d. standard normal from numpy seed 1 (drawn A then B).
  A step is one C = A (x) B with argmax over the whole matrix, inputs already
  in HBM.  A + B = 512 MiB > the 126 MB L2, so no explicit flush is needed.
* N > 1 (torchrun, one process per GPU, NCCL): weak scaling by row blocks of
  A -- every rank owns an 8192-row shard of A (M = 8192 * N in total), B
  (8192 x 8192) is broadcast from rank 0 over NVLink inside every timed step,
  C and argmax stay sharded (no reduction).  value = all ranks' ops / max time.
* e2e: the same step through the public API with host buffers -- pinned
  A and B copied in, tropical_gemm.maxplus_matmul_dlpack run, C and argmax
  copied back -- timed with CUDA events around everything.
* roofline: the fast kernel against the FP32 SIMT-pipe roofline
  (148 SMs x 128 tropical ops / clk, one FADD-lane slot per op).
* cpu_baseline: the reference's CPU argmax path (its BLIS + scalar 4x4
  microkernel, restated in oracle/tg_oracle.c) on a bounded row sample.
* --impl reference: times the reference's CPU implementation (the same
  restatement, all host threads) on the same config and, as an extra key,
  the reference's own CUDA kernel built from its sources (oracle/_ref).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tropical-gemm_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

M = N_ = K = 8192  # --size overrides (small cases for ncu captures)
SEED = 1
METRIC = "Tropical ops/s (M*N*K/s) f32 MaxPlus+argmax 8192^3 per B200 (weak-scaled row shards for N>1)"
UNIT = "tropical_ops/s"


class ClockSampler:
    """nvidia-smi sampling (every 100 ms) of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.mark = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a moment to start: wait for its first sample
            # (taken under the warm-up's load), then count from here on
            t_end = time.time() + 5.0
            while not self.lines and time.time() < t_end and self.proc.poll() is None:
                time.sleep(0.02)
            self.mark = len(self.lines)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # samples from the timed region; a region shorter than the sampling
        # interval falls back to the last sample before it (under warm-up load)
        lines = self.lines[self.mark:] or self.lines[max(0, self.mark - 1):self.mark]
        window = "timed region" if self.lines[self.mark:] else "last warm-up sample"
        for ln in lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for nm, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [x for x in sm if x > 0.5 * (mx or max(sm))] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "window": window}


def make_inputs(rows: int, seed: int = SEED):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((rows, K), dtype=np.float32)
    b = rng.standard_normal((K, N_), dtype=np.float32)
    return a, b


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def profile_traffic():
    """DRAM bytes per launch of the fused argmax kernel (the bench workload's dominant kernel) from the committed ncu summary (or None)."""
    path = os.path.join(ROOT, "profiles", "argmax_fused_maxplus_8192.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def launches_per_call(m: int, n: int, k: int, sms: int) -> int:
    """Kernels one f32 argmax tg_gemm call enqueues: the persistent fused
    kernel (taken for K >= 8192 with at least 16 128x128 tiles per SM, K <=
    65536, aligned rows) runs after one kernel writes both copies of B it reads (2 launches);
    the chunk kernel alone is 1."""
    env = os.environ.get("TROPICAL_GEMM_ARGMAX_FUSED", "")
    tiles = ((m + 127) // 128) * ((n + 127) // 128)
    auto = 8192 <= k and tiles >= 16 * sms
    fused = k <= 65536 and k > 1024 and n % 4 == 0 and k % 4 == 0 and (env == "1" or (env != "0" and auto))
    return 2 if fused else 1


def cpu_baseline(rows: int, threads: int):
    """Reference CPU argmax path (restated) on `rows` rows of the workload."""
    from oracle import tg_oracle
    a, b = make_inputs(rows, seed=SEED)
    t0 = time.perf_counter()
    tg_oracle.blis_argmax_f32("maxplus", a, b, nthreads=threads)
    dt = time.perf_counter() - t0
    return rows * N_ * K / dt, dt


def cpu_config1(threads: int):
    """MaxPlus f32 + argmax, 1024^3, A and B uniform in
    [-1, 1) from seed 0, on the reference's CPU argmax path (restated), one
    thread and all host threads."""
    from oracle import tg_oracle
    rng = np.random.default_rng(0)
    a = (2 * rng.random((1024, 1024), dtype=np.float32) - 1).astype(np.float32)
    b = (2 * rng.random((1024, 1024), dtype=np.float32) - 1).astype(np.float32)
    res = {}
    for nt in (1, threads):
        t0 = time.perf_counter()
        tg_oracle.blis_argmax_f32("maxplus", a, b, nthreads=nt)
        dt = time.perf_counter() - t0
        res[f"threads_{nt}"] = {"ops_per_s": 1024.0 ** 3 / dt, "s": dt}
        # the reference's AVX2 path (values only; it has no SIMD argmax path)
        t0 = time.perf_counter()
        tg_oracle.simd_maxplus_f32(a, b, nthreads=nt)
        dt = time.perf_counter() - t0
        res[f"simd_values_only_threads_{nt}"] = {"ops_per_s": 1024.0 ** 3 / dt, "s": dt}
        t0 = time.perf_counter()
        tg_oracle.simd_argmax_f32("maxplus", a, b, nthreads=nt)
        dt = time.perf_counter() - t0
        res[f"simd_argmax_threads_{nt}"] = {"ops_per_s": 1024.0 ** 3 / dt, "s": dt}
    return res


def cpu_simd_argmax(rows: int, threads: int):
    """AVX2 argmax path (8x8 vector tiles with an index vector per row; the
    reference's argmax path is scalar) on `rows` rows of the workload."""
    from oracle import tg_oracle
    a, b = make_inputs(rows, seed=SEED)
    t0 = time.perf_counter()
    tg_oracle.simd_argmax_f32("maxplus", a, b, nthreads=threads)
    dt = time.perf_counter() - t0
    return rows * N_ * K / dt, dt


def cpu_simd_values(rows: int, threads: int):
    """Reference CPU SIMD value-only path (AVX2 8x8, restated) on `rows` rows."""
    from oracle import tg_oracle
    a, b = make_inputs(rows, seed=SEED)
    t0 = time.perf_counter()
    tg_oracle.simd_maxplus_f32(a, b, nthreads=threads)
    dt = time.perf_counter() - t0
    return rows * N_ * K / dt, dt


def _time_ms(fn, reps=3, warm=1):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def extras(dev):
    """The other BASELINE configs on one GPU (informational keys, same metric)."""
    from tropical_gemm import _native as Nat
    from tropical_gemm.pytorch import tropical_maxplus_matmul_batched
    res = {}
    rng = np.random.default_rng(1)
    # 2a without argmax
    a = torch.from_numpy(rng.standard_normal((8192, 8192), dtype=np.float32)).to(dev)
    b = torch.from_numpy(rng.standard_normal((8192, 8192), dtype=np.float32)).to(dev)
    ms = _time_ms(lambda: Nat.gemm("maxplus", a, b, False))
    res["maxplus_f32_value_only_8192"] = {"ops_per_s": 8192.0 ** 3 / (ms * 1e-3), "ms": ms}
    # 2b: MinPlus f32 + argmax, values U[0,100) with 90% +inf
    mats = []
    for _ in range(2):
        v = (100 * rng.random((8192, 8192))).astype(np.float32)
        v[rng.random((8192, 8192)) < 0.9] = np.inf
        mats.append(torch.from_numpy(v).to(dev))
    ms = _time_ms(lambda: Nat.gemm("minplus", mats[0], mats[1], True))
    res["minplus_f32_argmax_90pct_inf_8192"] = {"ops_per_s": 8192.0 ** 3 / (ms * 1e-3), "ms": ms}
    del a, b, mats
    # 3: batched autograd forward + backward, 64 x [512x256] . [256x512]
    g = torch.Generator().manual_seed(0)
    ab = torch.randn((64, 512, 256), generator=g).to(dev).requires_grad_(True)
    bb = torch.randn((64, 256, 512), generator=g).to(dev).requires_grad_(True)

    def step():
        ab.grad = None
        bb.grad = None
        tropical_maxplus_matmul_batched(ab, bb).sum().backward()

    ms = _time_ms(step, reps=10, warm=3)
    ms_f = _time_ms(lambda: Nat.gemm_batched("maxplus", ab.detach(), bb.detach(), True), reps=10, warm=3)
    _, amb = Nat.gemm_batched("maxplus", ab.detach(), bb.detach(), True)
    gcb = torch.ones((64, 512, 512), device=dev)
    ms_b = _time_ms(lambda: (Nat.backward("maxplus", True, gcb, amb, 256),
                             Nat.backward("maxplus", False, gcb, amb, 256)), reps=10, warm=3)
    res["batched_autograd_fwd_bwd_64x512x256x512"] = {"ms": ms, "fwd_ops_per_s": 64 * 512 * 256 * 512 / (ms * 1e-3),
                                                       "fwd_kernel_ms": ms_f, "bwd_kernels_ms": ms_b}
    # 4: one APSP squaring, MinPlus i32, n = 16384, 5% density, weights 1..1000, missing = 46340
    n = 16384
    mask = rng.random((n, n)) < 0.05
    d = np.where(mask, rng.integers(1, 1001, (n, n)), 46340).astype(np.int32)
    np.fill_diagonal(d, 0)
    td = torch.from_numpy(d).to(dev)
    ms = _time_ms(lambda: Nat.gemm("minplus", td, td, True), reps=2)
    res["apsp_minplus_i32_argmax_16384_one_squaring"] = {"ops_per_s": float(n) ** 3 / (ms * 1e-3), "ms": ms,
                                                         "14_squarings_s": 14 * ms / 1e3}
    del td
    # 5: one rank's row block of the sharded config (4096 of 32768 rows)
    gg = torch.Generator(device=dev).manual_seed(2)
    a5 = torch.randn((4096, 8192), generator=gg, device=dev)
    b5 = torch.randn((8192, 32768), generator=gg, device=dev)
    ms = _time_ms(lambda: Nat.gemm("maxplus", a5, b5, True), reps=2)
    res["5_row_block_4096x32768x8192_maxplus_f32_argmax"] = {"ms": ms, "ops_per_s": 4096.0 * 32768 * 8192 / (ms * 1e-3)}
    del a5, b5
    a5 = torch.rand((4096, 8192), generator=gg, device=dev, dtype=torch.float64)
    b5 = torch.rand((8192, 32768), generator=gg, device=dev, dtype=torch.float64)
    ms = _time_ms(lambda: Nat.gemm("maxmul", a5, b5, False), reps=2)
    res["5_row_block_4096x32768x8192_maxmul_f64_values"] = {"ms": ms,
                                                            "ops_per_s": 4096.0 * 32768 * 8192 / (ms * 1e-3)}
    return res


CASES = ("backward", "batched_fwd", "f64", "f64_values", "apsp_step", "minplus_inf", "pipe_rates")

PIPE_VARIANTS = ("pair_fadd2_fmnmx3", "fadd2_alone", "fmnmx3_alone", "fadd_alone", "fmnmx_alone",
                 "fadd_x2_fmnmx3", "fadd2_fmnmx_x2", "fadd_fmnmx", "engine_ktile_body",
                 "engine_ktile_body_with_barrier", "ktile_body_bpair_outer", "ktile_body_two_kpairs",
                 "ktile_body_two_kpairs_tree", "ktile_body_kquad_swapped", "ktile_body_kquad_aligned",
                 "pair_b_lds128", "pair_b_lds64", "pair_b_lds128_prefetched",
                 "f64_dadd_alone", "f64_fmax_alone", "f64_dadd_fmax", "f64_dadd_strict_select",
                 "f64_dadd_select_with_index")


def pipe_rates(blocks_per_sm=(1, 2), iters=20000, variants=PIPE_VARIANTS):
    # the k-tile body variants run one CTA per SM (their register use)
    """Register-only instruction-mix rates (products per clock per SM) from
    the probe library (tropical-gemm_b200/csrc/probe/tg_pipe_rates.cu)."""
    import ctypes
    path = os.path.join(ROOT, "tropical-gemm_b200", "tropical_gemm", "libtg_pipe_rates.so")
    lib = ctypes.CDLL(path)
    lib.tg_probe_pipe_rate.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
    res = {}
    for name in variants:
        v = PIPE_VARIANTS.index(name)
        row = {}
        body = 8 <= v < 15
        for occ in ((1,) if body else blocks_per_sm):
            it = max(1, iters // 32) if body else iters
            r, ms = ctypes.c_double(), ctypes.c_double()
            rc = lib.tg_probe_pipe_rate(v, occ, 256, it, ctypes.byref(r), ctypes.byref(ms))
            if rc != 0:
                raise RuntimeError(f"pipe-rate probe {name} failed with CUDA error {rc}")
            row[f"warps_per_sm_{8 * occ}"] = round(r.value, 2)
        res[name] = row
    return res


def run_case(args):
    """One secondary workload, timed alone (CUDA events, `--steps` launches after
    `--warmup`), for per-kernel numbers and ncu captures; prints one JSON line.
    Not the driver's bench line (that is the default mode)."""
    from tropical_gemm import _native as Nat
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(1)
    out = {"case": args.case, "steps": args.steps, "warmup": args.warmup}
    if args.case == "backward":
        # BASELINE config 3 shapes: grad_A and grad_B of a batch of 64 [512x256].[256x512]
        bs, m, k, n = 64, 512, 256, 512
        a = torch.from_numpy(rng.standard_normal((bs, m, k), dtype=np.float32)).to(dev)
        b = torch.from_numpy(rng.standard_normal((bs, k, n), dtype=np.float32)).to(dev)
        _, am = Nat.gemm_batched("maxplus", a, b, True)
        gc = torch.ones((bs, m, n), dtype=torch.float32, device=dev)

        def step():
            Nat.backward("maxplus", True, gc, am, k)
            Nat.backward("maxplus", False, gc, am, k)

        ms = _time_ms(step, reps=args.steps, warm=args.warmup)
        # per gradient: read grad_C (4 B) + argmax (4 B) per output, write the gradient once
        alg = 2 * bs * m * n * 8 + bs * (m * k + k * n) * 4
        out.update({"ms": ms, "algorithmic_bytes": alg, "gbs": alg / (ms * 1e-3) / 1e9,
                    "config": {"batch": bs, "m": m, "k": k, "n": n, "dtype": "f32"}})
    elif args.case == "batched_fwd":
        # BASELINE config 3 forward: MaxPlus f32 + argmax, batch 64 of [512x256].[256x512]
        bs, m, k, n = 64, 512, 256, 512
        a = torch.from_numpy(rng.standard_normal((bs, m, k), dtype=np.float32)).to(dev)
        b = torch.from_numpy(rng.standard_normal((bs, k, n), dtype=np.float32)).to(dev)
        ms = _time_ms(lambda: Nat.gemm_batched("maxplus", a, b, True), reps=args.steps, warm=args.warmup)
        out.update({"ms": ms, "ops_per_s": float(bs) * m * n * k / (ms * 1e-3),
                    "config": {"batch": bs, "m": m, "k": k, "n": n, "dtype": "f32", "argmax": True}})
    elif args.case in ("f64", "f64_values"):
        sz = args.size if args.size != 8192 else 4096
        a = torch.rand((sz, sz), dtype=torch.float64, device=dev)
        b = torch.rand((sz, sz), dtype=torch.float64, device=dev)
        wa = args.case == "f64"
        ms = _time_ms(lambda: Nat.gemm("maxplus", a, b, wa), reps=args.steps, warm=args.warmup)
        out.update({"ms": ms, "ops_per_s": float(sz) ** 3 / (ms * 1e-3),
                    "config": {"m": sz, "n": sz, "k": sz, "dtype": "f64", "argmax": wa}})
    elif args.case == "apsp_step":
        n = args.size
        mask = rng.random((n, n)) < 0.05
        d = np.where(mask, rng.integers(1, 1001, (n, n)), 46340).astype(np.int32)
        np.fill_diagonal(d, 0)
        td = torch.from_numpy(d).to(dev)
        ms = _time_ms(lambda: Nat.gemm("minplus", td, td, True), reps=args.steps, warm=args.warmup)
        out.update({"ms": ms, "ops_per_s": float(n) ** 3 / (ms * 1e-3),
                    "config": {"n": n, "dtype": "i32", "density": 0.05, "argmax": True}})
    elif args.case == "pipe_rates":
        out.update({"unit": "products per clock per SM", "rates": pipe_rates()})
    elif args.case == "minplus_inf":
        n = args.size
        mats = []
        for _ in range(2):
            v = (100 * rng.random((n, n))).astype(np.float32)
            v[rng.random((n, n)) < 0.9] = np.inf
            mats.append(torch.from_numpy(v).to(dev))
        ms = _time_ms(lambda: Nat.gemm("minplus", mats[0], mats[1], True), reps=args.steps, warm=args.warmup)
        out.update({"ms": ms, "ops_per_s": float(n) ** 3 / (ms * 1e-3),
                    "config": {"n": n, "dtype": "f32", "inf_fraction": 0.9, "argmax": True}})
    print(json.dumps(out), flush=True)


def sharded_extras(dist, rank, world, dev):
    """BASELINE config 5 at this world size: M = N = 32768, K = 8192, rows of A
    sharded across the ranks (strong scaling), B broadcast from rank 0 with
    NCCL inside every timed step, C (+ argmax) sharded.  MaxPlus f32 with
    argmax (A, B ~ N(0,1)) and MaxMul f64 value-only (A, B ~ U[0,1)), seed 2.
    Every rank must call this (it runs collectives); rank 0 uses the result."""
    from tropical_gemm import _native as Nat
    m, n, k = 32768, 32768, 8192
    if m % world:
        return {"skipped": f"{m} rows do not split over {world} ranks"}
    rows = m // world
    lib = Nat.lib()
    stream = torch.cuda.current_stream(dev)
    res = {"m": m, "n": n, "k": k, "rows_per_rank": rows, "n_gpus": world,
           "data": "torch generator seed 2 (+ rank for A) on the device"}
    for name, dtype, semi, with_am in (("maxplus_f32_argmax", torch.float32, 0, True),
                                       ("maxmul_f64", torch.float64, 2, False)):
        g = torch.Generator(device=dev).manual_seed(2 + rank)
        gb = torch.Generator(device=dev).manual_seed(2)
        if dtype == torch.float32:
            a = torch.randn((rows, k), generator=g, device=dev, dtype=dtype)
            b = torch.randn((k, n), generator=gb, device=dev, dtype=dtype)
        else:
            a = torch.rand((rows, k), generator=g, device=dev, dtype=dtype)
            b = torch.rand((k, n), generator=gb, device=dev, dtype=dtype)
        c = torch.empty((rows, n), device=dev, dtype=dtype)
        am = torch.empty((rows, n), device=dev, dtype=torch.int32) if with_am else None
        pipelined = dist is not None and dtype == torch.float32
        from tropical_gemm import distributed as D

        def gemm_only():
            Nat.check(lib.tg_gemm(semi, Nat.DTYPES[dtype], 0, rows, n, k, a.data_ptr(), k, b.data_ptr(), n,
                                  c.data_ptr(), n, am.data_ptr() if am is not None else None, stream.cuda_stream))

        def step():
            if dist is not None:
                dist.broadcast(b, src=0)
            gemm_only()
            return c, am

        def step_pipelined():   # B's K slices broadcast while the previous slice computes
            return D.pipelined_sharded_matmul("maxplus", a, b, src=0, with_argmax=True, chunks=4)

        def timed(fn, steps=2):
            fn()
            if dist is not None:
                dist.barrier()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            t = e0.elapsed_time(e1) / steps
            if dist is not None:
                tt = torch.tensor([t], device=dev)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                t = float(tt.item())
            return t

        ms = timed(step)
        res[name] = {"ms_per_step": ms, "ops_per_s": float(m) * n * k / (ms * 1e-3), "steps": 2,
                     "timing": "CUDA events per rank, max over ranks, B broadcast inside each step"}
        res[name]["gemm_alone_ms"] = timed(gemm_only)
        if dist is not None:
            res[name]["broadcast_alone_ms"] = timed(lambda: dist.broadcast(b, src=0))
            if pipelined:
                # the K-pipelined form: its time, and its result against one pass, bit for bit
                res[name]["pipelined_4_slices_ms"] = timed(step_pipelined)
                cp, amp = step_pipelined()
                gemm_only()
                ok = torch.tensor([int(torch.equal(cp.view(torch.int32), c.view(torch.int32)) and
                                       torch.equal(amp, am))], device=dev)
                dist.all_reduce(ok, op=dist.ReduceOp.MIN)
                res[name]["pipelined_equals_one_pass_on_every_rank"] = bool(ok.item())
        del a, b, c, am
        torch.cuda.empty_cache()
    return res


def dist_setup(n_gpus: int):
    if n_gpus > 1 or "RANK" in os.environ:
        import torch.distributed as dist
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        from tropical_gemm import distributed as D
        D.init("nccl", timeout_s=300, device_id=torch.device("cuda", local))
        return dist, rank, world, local
    torch.cuda.set_device(0)
    return None, 0, 1, 0


def run_engine(args):
    from tropical_gemm import _native as Nat
    import tropical_gemm

    dist, rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    a_np, b_np = make_inputs(M, seed=SEED + rank)  # rank r owns rows [8192 r, 8192 (r+1)) of A
    if rank != 0:
        b_np = make_inputs(1, seed=SEED)[1]
    a = torch.from_numpy(a_np).to(dev)
    b = torch.from_numpy(b_np).to(dev)
    c = torch.empty((M, N_), device=dev)
    am = torch.empty((M, N_), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    lib = Nat.lib()

    def gemm():
        Nat.check(lib.tg_gemm(0, 0, 0, M, N_, K, a.data_ptr(), K, b.data_ptr(), N_, c.data_ptr(), N_,
                              am.data_ptr(), stream.cuda_stream))

    from tropical_gemm import distributed as D

    def step():
        # one broadcast of B, then the GEMM: the broadcast is ~0.5 % of a step
        # on NVLink, and a K-pipelined step measured slower (each K slice pays
        # the argmax resolution again), so the one-shot form is the timed one
        if dist is not None:
            dist.broadcast(b, src=0)
        gemm()

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
            torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    with ClockSampler(local) as clk:
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            ev[2 * i].record(stream)
            step()
            ev[2 * i + 1].record(stream)
        t1.record(stream)
        barrier()
    total_ms = t0.elapsed_time(t1)
    kern_ms = [ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)]
    if dist is not None:   # the kernel alone, for the roofline (the steps above include the broadcast)
        for i in range(args.steps):
            ev[2 * i].record(stream)
            gemm()
            ev[2 * i + 1].record(stream)
        torch.cuda.synchronize()
        kern_ms = [ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)]
    if dist is not None:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ops_step = float(M) * N_ * K * world
    value = ops_step * args.steps / (total_ms * 1e-3)

    e2e_value = None
    if not args.no_e2e:
        # e2e through the public API with host buffers (pinned), rank-local
        a_h = torch.from_numpy(a_np).pin_memory()
        b_h = torch.from_numpy(b_np).pin_memory() if rank == 0 else None
        c_h = torch.empty((M * N_,), dtype=torch.float32).pin_memory()
        am_h = torch.empty((M * N_,), dtype=torch.int32).pin_memory()
        e2e_steps = max(3, args.steps)

        # Pipelined over three streams so that step i+1's host->device copies and
        # step i-1's device->host copies overlap step i's kernel; every step still
        # moves its own inputs in and its own C + argmax out inside the timed region.
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        slots = [dict(da=torch.empty((M, K), device=dev), db=torch.empty((K, N_), device=dev),
                      ev_in=torch.cuda.Event(), ev_comp=torch.cuda.Event(), ev_out=torch.cuda.Event())
                 for _ in range(2)]
        for sl in slots:
            sl["ev_comp"].record(stream)
            sl["ev_out"].record(stream)

        def e2e_step(i):
            sl = slots[i % 2]
            with torch.cuda.stream(s_in):
                s_in.wait_event(sl["ev_comp"])            # compute of step i-2 is done with these buffers
                sl["da"].copy_(a_h.view(M, K), non_blocking=True)
                if rank == 0:   # other ranks receive B over NVLink (the broadcast below)
                    sl["db"].copy_(b_h.view(K, N_), non_blocking=True)
                sl["ev_in"].record(s_in)
            stream.wait_event(sl["ev_in"])
            if dist is not None:
                dist.broadcast(sl["db"], src=0)
            cc, aa = tropical_gemm.maxplus_matmul_dlpack(sl["da"], sl["db"])
            sl["ev_comp"].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(sl["ev_comp"])
                cc.record_stream(s_out)
                aa.record_stream(s_out)
                c_h.copy_(cc, non_blocking=True)
                am_h.copy_(aa, non_blocking=True)
                sl["ev_out"].record(s_out)

        e2e_step(0)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s_in)
        for i in range(e2e_steps):
            e2e_step(i)
        e1.record(s_out)
        barrier()
        e2e_ms = e0.elapsed_time(e1)
        if dist is not None:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e_value = ops_step * e2e_steps / (e2e_ms * 1e-3)

    config5 = None
    if not args.no_extras and args.size == 8192:
        config5 = sharded_extras(dist, rank, world, dev)

    if rank == 0:
        peaks = measured_peaks()
        clocks = clk.summary()
        props = torch.cuda.get_device_properties(dev)
        sm_max = peaks.get("sm_max_mhz") or clocks.get("sm_max_mhz") or 1965.0
        peak = props.multi_processor_count * 128 * sm_max * 1e6
        avg_kern_s = statistics.mean(kern_ms) * 1e-3
        achieved = float(M) * N_ * K / avg_kern_s
        # second denominator: the measured rate of the kernel's own instruction
        # mix (FADD2 + 3-input FMNMX, register-only probe, 8 warps per SM)
        try:
            pr = pipe_rates(blocks_per_sm=(1,), iters=4000, variants=("pair_fadd2_fmnmx3", "pair_b_lds128"))
            mix = pr["pair_fadd2_fmnmx3"]["warps_per_sm_8"]
            mix_smem = pr["pair_b_lds128"]["warps_per_sm_8"]
        except Exception:  # the probe library is optional for the contract line
            mix = mix_smem = None
        mix_peak = props.multi_processor_count * mix * sm_max * 1e6 if mix else None
        out = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic: numpy default_rng(seed 1 + rank) standard normal, A then B (BASELINE config 2a)",
            "config": {"workload": "maxplus_f32_argmax", "m_per_gpu": M, "n": N_, "k": K,
                       "m_total": M * world, "layout": "row-major",
                       "b_broadcast": "nccl broadcast from rank 0 inside each step" if world > 1 else "none",
                       "l2": "inputs (A+B = 512 MiB) exceed the 126 MB L2; no flush"},
            "roofline": {"bound": "simt", "achieved": achieved / 1e12, "peak": peak / 1e12, "unit": "Tops/s",
                         "frac": achieved / peak, "traffic": profile_traffic(),
                         "peak_basis": f"{props.multi_processor_count} SMs x 128 ops/clk x {sm_max:.0f} MHz "
                                       "(FP32 SIMT pipes; tropical GEMM cannot use tensor cores)",
                         "frac_at_sampled_clock": (achieved / (props.multi_processor_count * 128 * clocks["sm_mhz"] * 1e6))
                         if clocks.get("sm_mhz") else None,
                         "mix_peak": mix_peak / 1e12 if mix_peak else None,
                         "frac_mix": achieved / mix_peak if mix_peak else None,
                         "mix_basis": (f"measured FADD2 + FMNMX3 issue rate {mix:.1f} products/clk/SM "
                                       f"(bench.py --case pipe_rates) x {props.multi_processor_count} SMs x "
                                       f"{sm_max:.0f} MHz") if mix else None,
                         "smem_fed_peak": (props.multi_processor_count * mix_smem * sm_max * 1e6 / 1e12)
                         if mix_smem else None,
                         "frac_smem_fed": (achieved / (props.multi_processor_count * mix_smem * sm_max * 1e6))
                         if mix_smem else None,
                         "smem_fed_basis": (f"the same pair with its B operands reloaded from shared memory every "
                                            f"iteration: {mix_smem:.1f} products/clk/SM") if mix_smem else None},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    # whole job: every rank's A shard and rank 0's B in, every rank's C + argmax out
                    "h2d_bytes_per_step": 4 * (M * K * world + K * N_),
                    "d2h_bytes_per_step": 8 * M * N_ * world, "api": "tropical_gemm.maxplus_matmul_dlpack"},
            "gpu_launches": args.steps * launches_per_call(M, N_, K, props.multi_processor_count),
            "clocks": clocks,
            "kernel_ms": {"mean": statistics.mean(kern_ms), "min": min(kern_ms), "max": max(kern_ms)},
        }
        if world == 1 and not args.no_extras and args.size == 8192:
            out["extras"] = extras(dev)
        if config5 is not None:
            out["config5_sharded_32768x32768x8192"] = config5
        if world == 1 and not args.no_cpu:
            rows = args.cpu_baseline_rows
            threads = os.cpu_count() or 1
            v, dt = cpu_baseline(rows, threads)
            out["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                                   "sample": f"{rows} x {N_} x {K} rows of the same workload, {dt:.1f} s, "
                                             "reference BLIS argmax path (mc=nc=64,kc=256, 4x4 scalar) restated "
                                             "in C, OpenMP over column blocks"}
            # the reference runs one GEMM on one thread: the faithful figure
            v1, dt1 = cpu_baseline(64, 1)
            out["cpu_baseline"]["single_thread"] = {"value": v1, "cores": 1,
                                                    "sample": f"64 x {N_} x {K} rows, {dt1:.1f} s"}
            try:
                vs, dts = cpu_simd_values(rows, threads)
                out["cpu_baseline"]["simd_values_only"] = {
                    "value": vs, "cores": threads,
                    "sample": f"{rows} x {N_} x {K} rows, {dts:.1f} s: the reference's AVX2 value-only MaxPlus "
                              "path (8x8 f32x8 microkernel, mc=nc=256, kc=512) restated in C; no argmax"}
            except RuntimeError as e:
                out["cpu_baseline"]["simd_values_only"] = {"unavailable": str(e)}
            try:
                va, dta = cpu_simd_argmax(rows, threads)
                out["cpu_baseline"]["simd_argmax"] = {
                    "value": va, "cores": threads,
                    "sample": f"{rows} x {N_} x {K} rows, {dta:.1f} s: AVX2 argmax path (8x8 f32x8 tiles with "
                              "an index vector per row, mc=nc=256, kc=512), bit-exact with the scalar path"}
            except RuntimeError as e:
                out["cpu_baseline"]["simd_argmax"] = {"unavailable": str(e)}
            out["config1_cpu_1024"] = cpu_config1(threads)
        print(json.dumps(out), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def _ev_ms(fn, reps=3, warm=1):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def reference_gpu_configs(dev):
    """The reference's CUDA kernels (oracle/_ref, compiled from its .cu with
    nvcc -O3 for sm_100a) on each BASELINE configuration, same inputs as the
    engine's extras: ms per launch and tropical ops/s."""
    from oracle.ref_gpu import ref_lib, ref_rowmajor
    L = ref_lib()
    if L is None:
        return {"unavailable": "reference kernels not built (oracle/_ref)"}
    res = {"kernels": "crates/tropical-gemm-cuda/kernels/tropical_gemm.cu, reference launch geometry"}
    rng = np.random.default_rng(1)
    # 2a: MaxPlus f32 + argmax 8192^3 (and values only)
    a_np, b_np = make_inputs(8192)
    a = torch.from_numpy(a_np).to(dev)
    b = torch.from_numpy(b_np).to(dev)
    ms = _ev_ms(lambda: ref_rowmajor("maxplus", a, b, True))
    res["2a_maxplus_f32_argmax_8192"] = {"ms": ms, "ops_per_s": 8192.0 ** 3 / (ms * 1e-3)}
    ms = _ev_ms(lambda: ref_rowmajor("maxplus", a, b, False))
    res["2a_maxplus_f32_values_8192"] = {"ms": ms, "ops_per_s": 8192.0 ** 3 / (ms * 1e-3)}
    del a, b
    # 2b: MinPlus f32 + argmax, U[0,100) with 90 % +inf
    mats = []
    for _ in range(2):
        v = (100 * rng.random((8192, 8192))).astype(np.float32)
        v[rng.random((8192, 8192)) < 0.9] = np.inf
        mats.append(torch.from_numpy(v).to(dev))
    ms = _ev_ms(lambda: ref_rowmajor("minplus", mats[0], mats[1], True))
    res["2b_minplus_f32_argmax_90pct_inf_8192"] = {"ms": ms, "ops_per_s": 8192.0 ** 3 / (ms * 1e-3)}
    del mats
    # 3: batched forward (reference batched argmax kernel) + backward as the
    # reference's torch path does it (pytorch.py:386-403: two scatter_add_)
    g = torch.Generator().manual_seed(0)
    ab = torch.randn((64, 512, 256), generator=g).to(dev)
    bb = torch.randn((64, 256, 512), generator=g).to(dev)
    cb = torch.empty((64, 512, 512), device=dev)
    amb = torch.empty((64, 512, 512), dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream

    def fwd():
        rc = L.ref_gemm_batched_argmax_f32(0, 64, 512, 512, 256, bb.data_ptr(), ab.data_ptr(), cb.data_ptr(),
                                           amb.data_ptr(), 256 * 512, 512 * 256, 512 * 512, st)
        assert rc == 0

    ms_f = _ev_ms(fwd, reps=10, warm=3)
    gc = torch.ones((64, 512, 512), device=dev)
    am64 = amb.long()

    def bwd():
        ga = torch.zeros((64, 512, 256), device=dev)
        ga.scatter_add_(2, am64, gc)
        gbt = torch.zeros((64, 512, 256), device=dev)
        gbt.scatter_add_(2, am64.transpose(1, 2), gc.transpose(1, 2))
        return ga, gbt.transpose(1, 2)

    ms_b = _ev_ms(bwd, reps=10, warm=3)
    res["3_batched_64x512x256x512"] = {"fwd_ms": ms_f, "fwd_ops_per_s": 64 * 512 * 256 * 512 / (ms_f * 1e-3),
                                       "bwd_ms_torch_scatter": ms_b, "fwd_bwd_ms": ms_f + ms_b}
    del ab, bb, cb, amb, gc, am64
    # 4: one APSP squaring, MinPlus i32 + argmax, n = 16384
    n = 16384
    mask = rng.random((n, n)) < 0.05
    d = np.where(mask, rng.integers(1, 1001, (n, n)), 46340).astype(np.int32)
    np.fill_diagonal(d, 0)
    td = torch.from_numpy(d).to(dev)
    ms = _ev_ms(lambda: ref_rowmajor("minplus", td, td, True), reps=1)
    res["4_apsp_minplus_i32_argmax_16384_one_squaring"] = {"ms": ms, "ops_per_s": float(n) ** 3 / (ms * 1e-3),
                                                           "14_squarings_s": 14 * ms / 1e3}
    del td
    # 5: one rank's row block of the sharded config (4096 of 32768 rows)
    gg = torch.Generator(device=dev).manual_seed(2)
    a5 = torch.randn((4096, 8192), generator=gg, device=dev)
    b5 = torch.randn((8192, 32768), generator=gg, device=dev)
    ms = _ev_ms(lambda: ref_rowmajor("maxplus", a5, b5, True), reps=1)
    res["5_row_block_4096x32768x8192_maxplus_f32_argmax"] = {"ms": ms, "ops_per_s": 4096.0 * 32768 * 8192 / (ms * 1e-3)}
    del a5, b5
    a5 = torch.rand((4096, 8192), generator=gg, device=dev, dtype=torch.float64)
    b5 = torch.rand((8192, 32768), generator=gg, device=dev, dtype=torch.float64)
    ms = _ev_ms(lambda: ref_rowmajor("maxmul", a5, b5, False), reps=1)
    res["5_row_block_4096x32768x8192_maxmul_f64_values"] = {"ms": ms,
                                                            "ops_per_s": 4096.0 * 32768 * 8192 / (ms * 1e-3)}
    return res


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    rows = args.cpu_rows
    for _ in range(args.warmup):
        cpu_baseline(max(8, rows // 8), threads)
    vals, secs = [], 0.0
    for _ in range(args.steps):
        v, dt = cpu_baseline(rows, threads)
        vals.append(v)
        secs += dt
    value = float(np.mean(vals))
    out = {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: numpy default_rng(seed 1) standard normal (BASELINE config 2a), row sample",
        "config": {"workload": "maxplus_f32_argmax", "m_per_gpu": M, "n": N_, "k": K},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{rows} rows x {N_} x {K} per step: the reference CPU argmax path "
                                   "(BLIS + 4x4 scalar microkernel) restated in C (the Rust reference cannot be "
                                   "built here), all host threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    # The reference's own CUDA kernels on this GPU (built from its sources),
    # on every BASELINE configuration.
    try:
        if torch.cuda.is_available():
            out["reference_gpu"] = reference_gpu_configs(torch.device("cuda", 0))
    except Exception as e:  # the CPU figure above is the arm's value; this key is informational
        out["reference_gpu"] = {"error": str(e)[:200]}
    print(json.dumps(out), flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="engine", choices=["engine", "reference"])
    p.add_argument("--cpu-rows", type=int, default=1024, help="rows of A per step of the reference arm")
    p.add_argument("--cpu-baseline-rows", type=int, default=8192,
                   help="rows of A timed in the engine line's cpu_baseline (8192 = the whole workload)")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-extras", action="store_true", help="skip the other BASELINE configs (extra keys)")
    p.add_argument("--size", type=int, default=8192, help="square size (8192 = BASELINE config 2a)")
    p.add_argument("--case", choices=CASES, help="time one secondary workload alone (for profiling)")
    args = p.parse_args()
    if args.case:
        run_case(args)
        return
    global M, N_, K
    M = N_ = K = args.size
    if args.impl == "reference":
        run_reference(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
