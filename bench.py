#!/usr/bin/env python
"""Benchmark: kernel-matvec TFLOP/s at n=1M, d=16, t=16 (RBF-ARD) on 1..8 B200.

One step = one matrix-free K(X,X)·V + sigma^2 V with t=16 right-hand sides over
the seeded config-3 inputs (X ~ N(0, I)^{1e6 x 16}, l ~ U[0.5, 3]^16), inputs
resident in HBM. With N GPUs the training rows are sharded (each rank owns
n/N rows of the output; X and V are replicated) and every step ends with the
NCCL all-gather of the output row blocks, as one CG iteration needs.

Prints one JSON line (rank 0). `--impl reference` times the reference's CPU
route on the host cores instead: its own NumPy kernel evaluator
(KernelNode.evaluate, installed unmodified under baseline/_ref) + BLAS, or the
restatement in oracle/cpu_baseline.py where that install is absent.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "kernel-matvec TFLOP/s & fit s/iter at n=1M,d=16,t=16"
UNIT = "TFLOP/s"
F_PER_PAIR_RBF = lambda d, t: 3 * d + 3 + 2 * t  # algorithmic flops per kernel entry
# Tensor-core flops the Gram-form kernel issues per kernel entry (d padded to
# DP = 16): MMA1 3xTF32 on x·y (3 * 2 * DP) + the norm k-step (2 * 8), MMA2
# three tf32 products into t = 16 columns (3 * 2 * t).
TC_PER_PAIR_GRAM = lambda dp, t: 3 * 2 * dp + 2 * 8 + 3 * 2 * t
# fp16 Gram kernel (kind::f16, K = 16 per MMA): MMA1 is 4 k-steps of 16 at
# DP = 16 (xh.bh, xl.bh, xh.bl, norms) or 2 at DP = 8, MMA2 one N = 32 and one
# N = 16 product per column.
TC_PER_PAIR_GRAMH = lambda dp, t: (4 if dp > 8 else 2) * 2 * 16 + 2 * 2 * t + 2 * t
MUFU_PER_SM_CLK = 16  # MUFU (ex2) results per SM per clock on B200: 4 per sub-partition
# DRAM bytes (read + write) of one fp16 Gram tile-kernel launch at n = 1e6, d = 16, t = 16 on one
# GPU, from the one-pass ncu capture in profiles/kv_tile_gramh_rbf_ard_d16_t16.md.
GRAMH_TRAFFIC_C3 = 784.76e6 + 196.19e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--rows", dest="n", type=int, default=1_000_000)
    ap.add_argument("--dims", dest="d", type=int, default=16)
    ap.add_argument("--rhs", dest="t", type=int, default=16)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--workload", default="c3", choices=["c1", "c2", "c3", "c3fit", "c4", "c5", "materialized"],
                    help="c3: the headline K·V / fit line (default); c3fit: the config-3 fit alone "
                         "(--cfg-iters iterations, rows sharded); materialized: matrix-free K·V "
                         "against the reference's materialized route (dense K + SGEMM) at "
                         "n = 4e4; c1, c2, c4: the other "
                         "fit configurations (1 GPU); c5: LOVE prediction at scale")
    ap.add_argument("--cfg-iters", type=int, default=50,
                    help="c1 / c2 / c4: outer fit iterations")
    ap.add_argument("--test-rows", type=int, default=0,
                    help="c5: test points (default = --rows)")
    ap.add_argument("--love-rank", type=int, default=256)
    ap.add_argument("--fit-iters", type=int, default=2,
                    help="outer fit iterations for the fit block of the c3 line (0 = skip); "
                         "--workload c3fit runs the full fit")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None
        self.gpu = gpu_index

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().strip().splitlines() if r]
        os.unlink(self.file.name)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for nm, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def run_fit(X, y, iters: int, local: int, comm) -> dict:
    """SingleOutputGP(RBF(ard=True)).fit(X, y, method="matrix_free",
    num_probes=15) for `iters` outer iterations; s/iter is the median host wall
    time per iteration over iterations 5..K (jit_training.mojo:855-860) when
    K > 5, else over all K (labelled)."""
    from mojogp_b200.gp import SingleOutputGP
    from mojogp_b200.kernel import RBF
    gp = SingleOutputGP(RBF(ard=True), device=local)
    t0 = time.perf_counter()
    res = gp.fit(X, y, max_iterations=iters, method="matrix_free", num_probes=15, comm=comm)
    total = time.perf_counter() - t0
    it = np.asarray(res.iter_times_ms, np.float64) / 1e3
    window = "iterations 5..K" if it.size > 5 else f"all {it.size} iterations"
    s_iter = float(np.median(it[4:] if it.size > 5 else it))
    if comm:
        s_iter = comm.allreduce_max(s_iter)
        total = comm.allreduce_max(total)
    info = gp._train_info
    kinds = info.get("tile_kernels", [])
    return {"s_per_iter": s_iter, "window": window, "iterations": int(res.iterations),
            "fit_total_s": total,
            "cg_iters_per_iter": [int(c) for c in res.cg_iterations_history],
            "tile_kernel_per_iter": {k: kinds.count(k) for k in sorted(set(kinds))},
            "settings": {"api": "SingleOutputGP(RBF(ard=True)).fit(method='matrix_free', "
                                "num_probes=15)", "max_cg_iter": info["max_cg_iterations"],
                         "cg_tol": info["cg_tolerance"],
                         "max_tridiag_iter": info["max_tridiag_iter"],
                         "precond_rank": info["precond_rank"], "initial_noise": 0.1},
            "final_nll": float(res.nll),
            "history": {"iter_s": it.tolist(), "nll": [float(v) for v in res.nll_history],
                        "tile_kernels": kinds}}


def reference_matvec_sample(X, V, ell, target_s: float, max_rows: int, threads: int):
    """Time the reference's own CPU route where it is installed (baseline/_ref):
    its NumPy kernel evaluator KernelNode.evaluate (mojogp/kernel.py:722-923)
    on row blocks x all columns, then a BLAS product with V, row blocks spread
    over host threads. Returns (result dict, kind), kind "reference"; falls
    back to the restatement in oracle/cpu_baseline.py (kind "port") when the
    reference package does not import."""
    import concurrent.futures as cf
    ref_dir = ROOT / "baseline" / "_ref"
    try:
        if str(ref_dir) not in sys.path:
            sys.path.insert(0, str(ref_dir))
        from mojogp.kernel import RBF as RefRBF, make_ard_kernel as ref_ard
    except Exception:  # the reference is not installed here: use the restatement
        from oracle import cpu_baseline
        return cpu_baseline.time_matvec_sample(X, V, ell, 1.0, target_s=target_s, threads=threads,
                                               max_rows=max_rows), "port"
    d = X.shape[1]
    kern = ref_ard(RefRBF(ard=True), d)
    params = np.concatenate([np.asarray(ell, np.float64), [1.0]])
    V64 = V.astype(np.float64)
    n = X.shape[0]

    def rows_block(r0, r1):
        K = kern.evaluate(X[r0:r1], X, params=params)
        return np.asarray(K, np.float64) @ V64

    def run(nrows, blk=16):  # 16 rows x n columns of float64 temporaries per thread
        t0 = time.perf_counter()
        with cf.ThreadPoolExecutor(threads) as ex:
            list(ex.map(lambda r: rows_block(r, min(r + blk, nrows)), range(0, nrows, blk)))
        return time.perf_counter() - t0

    dt = run(min(64, n))
    nrows = int(min(max_rows, n, max(64, 64 * target_s / max(dt, 1e-3))))
    nrows = max(64, nrows // 64 * 64)
    dt = run(nrows)
    return {"seconds": dt, "rows": nrows, "pairs": nrows * n, "pairs_per_s": nrows * n / dt,
            "threads": threads}, "reference"


def run_reference(args, rank: int, world: int) -> None:
    """CPU arm: the reference's NumPy route on the host cores (rank 0 only)."""
    if rank != 0:
        return
    from mojogp_b200 import synthetic
    X, _, ell = synthetic.config3(n=args.n, d=args.d)
    V = synthetic.probes_v(args.n, args.t, seed=1)
    threads = os.cpu_count() or 1
    per_step = []
    kind = "port"
    for it in range(args.warmup + args.steps):
        r, kind = reference_matvec_sample(
            X, V, ell, target_s=max(2.0, 30.0 / max(args.steps + args.warmup, 1)),
            max_rows=2048, threads=threads)
        if it >= args.warmup:
            per_step.append(r)
    F = F_PER_PAIR_RBF(args.d, args.t)
    tflops = [r["pairs_per_s"] * F / 1e12 for r in per_step]
    value = statistics.median(tflops)
    rows = per_step[-1]["rows"]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * statistics.median(r["seconds"] for r in per_step),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (config 3 recipe, seed 3)",
        "config": {"workload": "config3 K(X,X)V RBF-ARD", "n": args.n, "d": args.d, "t": args.t,
                   "sample": f"{rows} rows x {args.n} columns per step"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{rows} output rows x all {args.n} columns: "
                                   + ("the reference's KernelNode.evaluate (baseline/_ref) + BLAS"
                                      if kind == "reference" else
                                      "float64 NumPy evaluator restated (kernel.py:804-923) + BLAS")},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_love(args, rank: int, world: int, local: int) -> None:
    """Config 5: LOVE prediction at scale through the public API with host
    arrays (alpha CG, rank-r Lanczos root, predictive mean and variance for
    every test point). Training rows are sharded for the alpha solve and the
    root; test rows are sharded for the cross products. One timed pass after a
    small warm-up run that loads every kernel; the phases are wall-clocked on
    the host with a device synchronisation at each boundary, max over ranks."""
    from mojogp_b200 import synthetic
    from mojogp_b200.kernel import RBF, make_ard_kernel
    from mojogp_b200.prediction import PredictionCache, compute_alpha
    from mojogp_b200.provider import Provider

    comm = None
    if world > 1:
        from mojogp_b200.distributed import Communicator
        comm = Communicator.from_env(device=local)
    n, m, r = args.n, args.test_rows or args.n, args.love_rank
    d = 8
    kern = make_ard_kernel(RBF(ard=True), d)

    def one_pass(nn, mm, rr):
        X, y, Xs, params, noise = synthetic.config5(n=nn, n_test=mm, d=d)
        prov = Provider(X, kern, params, noise, device=local)
        yc = y - y.mean()
        if comm:
            comm.barrier()
        t0 = time.perf_counter()
        alpha, iters = compute_alpha(prov, yc, 300, 1e-3, comm=comm)
        t1 = time.perf_counter()
        cache = PredictionCache(prov, alpha, float(y.mean()), rr, comm=comm)
        t2 = time.perf_counter()
        if comm:
            mean, var = cache.predict_sharded(Xs, comm)
        else:
            mean, var = cache.predict(Xs)
        std = np.sqrt(var)
        t3 = time.perf_counter()
        cache.destroy()
        ph = [t1 - t0, t2 - t1, t3 - t2]
        if comm:
            ph = [comm.allreduce_max(v) for v in ph]
        return ph, iters, float(np.mean(std)), prov.matvec_layout(1), prov.matvec_layout(16)

    one_pass(min(n, 20000), min(m, 20000), min(r, 64))  # warm-up: kernel loads, attributes
    sampler = ClockSampler(local)
    sampler.start()
    (a_s, r_s, p_s), iters, mean_std, lay1, lay16 = one_pass(n, m, r)
    clocks = sampler.stop()
    total = a_s + r_s + p_s
    chunks = -(-(r + 1) // 16)
    entries = {"alpha": float(iters + 1) * n * n, "root": float(r) * n * n,
               "predict": float(chunks) * m * n}
    line = {
        "metric": "LOVE predict s (alpha CG + rank-r Lanczos root + mean/std at every test point)",
        "value": total, "unit": "s", "n_gpus": world, "steps": 1, "warmup": 1,
        "ms_per_step": total * 1e3, "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (config 5 recipe: X, X* ~ U[0,1]^8, l ~ U[0.2,1], os 1, noise 0.01, seed 5)",
        "config": {"workload": "config5 LOVE prediction", "n": n, "n_test": m, "d": d,
                   "love_rank": r, "parallelism": f"train rows x{world} (alpha, root), "
                                                  f"test rows x{world} (mean/std)",
                   "tile_kernels": {"1 column": lay1, "16 columns": lay16}},
        "phases_s": {"alpha_cg": a_s, "love_root": r_s, "mean_std": p_s},
        "alpha_cg_iters": iters,
        "kernel_entries_per_s": {k: entries[k] / v for k, v in
                                 zip(("alpha", "root", "predict"), (a_s, r_s, p_s)) if v > 0},
        "mean_std": mean_std,
        "e2e": {"value": total, "unit": "s", "h2d_bytes_per_step": int(4 * (n * d + n + m * d)),
                "d2h_bytes_per_step": int(4 * (n + 2 * m))},
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if comm:
        comm.close()


def run_c3fit(args, rank: int, world: int, local: int) -> None:
    """Config 3 fit alone: the public API at the reference's defaults for
    --cfg-iters outer iterations, rows sharded over the ranks (north_star's
    50-iteration fit at n = 1e6, d = 16)."""
    from mojogp_b200 import synthetic
    comm = None
    if world > 1:
        from mojogp_b200.distributed import Communicator
        comm = Communicator.from_env(device=local)
    X, y, _ = synthetic.config3(n=args.n, d=args.d)
    sampler = ClockSampler(local)
    sampler.start()
    fit = run_fit(X, y, args.cfg_iters, local, comm)
    clocks = sampler.stop()
    line = {
        "metric": "fit s/iter", "value": fit["s_per_iter"], "unit": "s", "n_gpus": world,
        "steps": fit["iterations"], "warmup": 0, "ms_per_step": fit["s_per_iter"] * 1e3,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (config 3 recipe: X~N(0,I), y = RFF prior draw + noise, seed 3)",
        "config": {"workload": "config3 fit RBF-ARD matrix-free, t=16", "n": args.n,
                   "d": args.d, "parallelism": f"row-shard x{world}"},
        "fit": fit, "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if comm:
        comm.close()


def run_materialized(args, rank: int, world: int, local: int) -> None:
    """The reference's materialized route (fn_ptr_module.py:363-421: K filled
    densely once per parameter update, then every product is an fp32 SGEMM
    with use_tf32=False) against this library's matrix-free K·V at the size
    that route serves (n = 4e4, RBF-ARD, t = 16). The dense side runs in torch
    (fp32 cuBLAS, TF32 off) as the measurement of a plain library GEMM; both
    sides are CUDA-event timed with inputs resident."""
    if rank != 0:
        return
    import torch  # before the library: its NCCL must be the one loaded
    import ctypes as C
    from mojogp_b200 import _lib, synthetic
    from mojogp_b200.kernel import RBF, make_ard_kernel
    from mojogp_b200.provider import DeviceBuffer, Provider
    torch.backends.cuda.matmul.allow_tf32 = False
    n, d, t = (args.n if args.n != 1_000_000 else 40_000), 8, 16
    X, _ = synthetic.config2(n=n, d=d)
    ell = np.random.default_rng(4).uniform(0.5, 3.0, size=d).astype(np.float32)
    params = np.concatenate([ell, [1.0]]).astype(np.float32)
    prov = Provider(X, make_ard_kernel(RBF(ard=True), d), params, 0.01, device=local)
    V = synthetic.probes_v(n, t, seed=1)
    vd = DeviceBuffer.from_host(np.ascontiguousarray(V.T), local)
    od = DeviceBuffer((t, n), local)
    steps = max(args.steps, 5)
    step_ms = np.zeros(steps)
    kern_ms = np.zeros(steps)
    launches = np.zeros(steps, dtype=np.int64)
    _lib.call("gpb_benchmark_forward", prov.h, vd.cptr, od.cptr, t, args.warmup, steps, 0,
              C.c_void_p(step_ms.ctypes.data), C.c_void_p(kern_ms.ctypes.data),
              C.c_void_p(launches.ctypes.data))
    mf_ms = float(np.median(step_ms))
    dev = torch.device("cuda", local)
    Xt = torch.from_numpy(X).to(dev) / torch.from_numpy(ell).to(dev)
    Vt = torch.from_numpy(V).to(dev)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def fill():
        sq = (Xt * Xt).sum(1)
        K = sq[:, None] + sq[None, :] - 2.0 * (Xt @ Xt.T)
        return torch.exp(-0.5 * K.clamp_min_(0.0))

    K = fill()
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(3):
        K = fill()
    ev[1].record()
    torch.cuda.synchronize()
    fill_ms = ev[0].elapsed_time(ev[1]) / 3
    out = K @ Vt + 0.01 * Vt
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        ev[2].record()
        out = K @ Vt
        out.add_(Vt, alpha=0.01)
        ev[3].record()
        torch.cuda.synchronize()
        times.append(ev[2].elapsed_time(ev[3]))
    gemm_ms = float(np.median(times))
    ref = od.download().T
    err = float(np.linalg.norm(out.cpu().numpy() - ref) / np.linalg.norm(ref))
    line = {
        "metric": "K·V ms per product (matrix-free vs materialized)", "value": mf_ms, "unit": "ms",
        "n_gpus": 1, "steps": steps, "warmup": args.warmup, "ms_per_step": mf_ms,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (config 2 recipe inputs, RBF-ARD)",
        "config": {"workload": "materialized-route comparison", "n": n, "d": d, "t": t,
                   "tile_kernel": prov.matvec_layout(t)},
        "materialized": {"fill_ms": fill_ms, "sgemm_ms": gemm_ms, "K_bytes": 4 * n * n,
                         "sgemm_gbs": 4.0 * n * n / (gemm_ms * 1e-3) / 1e9,
                         "products_to_amortise_fill": (fill_ms / (mf_ms - gemm_ms)
                                                       if mf_ms > gemm_ms else None)},
        "matrix_free_vs_sgemm_rel_diff": err,
    }
    print(json.dumps(line), flush=True)


def run_config(args, rank: int, world: int, local: int) -> None:
    """Configs 1, 2 and 4 through the public model API on one GPU: a full fit
    (fit s/iter = median per-iteration time; the LMC fit, which records no
    per-iteration times, is total / iterations) and, for config 1, the LOVE
    prediction of 128 test points. Config 1 also times the reference's NumPy
    exact-Cholesky fit iteration on the host cores as its CPU baseline."""
    if rank != 0:
        return
    from mojogp_b200 import synthetic
    from mojogp_b200.gp import SingleOutputGP
    from mojogp_b200.kernel import RBF, Matern32, Matern52
    from mojogp_b200.multi_output_gp import MultiOutputLMCGP
    wl, iters = args.workload, args.cfg_iters
    sampler = ClockSampler(local)
    extra = {}
    if wl in ("c1", "c2"):
        if wl == "c1":
            X, y, Xs = synthetic.config1()
            make = lambda: SingleOutputGP(RBF(), device=local)
            kw = dict(method="matrix_free")
            cfg = {"workload": "config1 RBF 1-D fit + LOVE predict", "n": 2000, "d": 1,
                   "t": 11, "n_test": 128}
        else:
            X, y = synthetic.config2()
            Xs = None
            make = lambda: SingleOutputGP(Matern52(ard=True), device=local)
            kw = dict(method="matrix_free", num_probes=15, preconditioner="greedy",
                      preconditioner_rank=100)
            cfg = {"workload": "config2 Matern-5/2 ARD fit, pivoted-Cholesky rank 100",
                   "n": X.shape[0], "d": X.shape[1], "t": 16}
        make().fit(X, y, max_iterations=2, **kw)  # warm-up: kernel loads
        gp = make()
        sampler.start()
        t0 = time.perf_counter()
        res = gp.fit(X, y, max_iterations=iters, **kw)
        fit_s = time.perf_counter() - t0
        if Xs is not None:
            t1 = time.perf_counter()
            mean, std = gp.predict(Xs, return_std=True, variance_method="love")
            extra["predict_s"] = time.perf_counter() - t1
            extra["mean_std"] = float(np.mean(std))
        clocks = sampler.stop()
        it = np.asarray(res.iter_times_ms, np.float64)
        s_iter = float(np.median(it[4:] if it.size > 5 else it)) / 1e3
        extra.update({"final_nll": float(res.nll), "iterations": int(res.iterations),
                      "cg_iters_median": float(np.median(res.cg_iterations_history))})
    else:
        X, Y = synthetic.config4()
        make = lambda: MultiOutputLMCGP(kernels=[RBF(), Matern32(), RBF(ard=True)],
                                        num_probes=15, device=local)
        make().fit(X, Y, max_iterations=2, method="matrix_free")
        gp = make()
        sampler.start()
        t0 = time.perf_counter()
        gp.fit(X, Y, max_iterations=iters, method="matrix_free")
        fit_s = time.perf_counter() - t0
        clocks = sampler.stop()
        done = len(gp.nll_history)
        s_iter = fit_s / max(done, 1)
        extra.update({"final_nll": float(gp.final_nll), "iterations": done,
                      "cg_iters_median": float(np.median(gp.cg_iterations_history)),
                      "cg_iters_max": int(np.max(gp.cg_iterations_history)),
                      "precond_rebuilds": int(gp.precond_rebuild_count),
                      "tile_kernels": [p.matvec_layout(16) for p in gp._lmc.providers]})
        cfg = {"workload": "config4 LMC T=4, R=3 (RBF, Matern-3/2, RBF-ARD) fit",
               "n": X.shape[0], "d": X.shape[1], "T": 4, "R": 3, "t": 16}
    line = {
        "metric": "fit s/iter", "value": s_iter, "unit": "s", "n_gpus": 1, "steps": iters,
        "warmup": 2, "ms_per_step": s_iter * 1e3, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic ({wl} recipe)", "config": cfg, "fit_total_s": fit_s,
        **extra, "clocks": clocks,
    }
    if wl == "c1" and not args.no_cpu_baseline:
        from oracle import cpu_baseline
        gpp = gp.get_params()
        sec = cpu_baseline.time_exact_fit_iteration(
            X, y - gpp["mean"], np.array([gpp["rbf_lengthscale"]]), gpp["rbf_outputscale"],
            gpp["noise"], reps=3)
        line["cpu_baseline"] = {"value": sec, "unit": "s", "cores": os.cpu_count() or 1,
                                "kind": "port",
                                "sample": "one exact-Cholesky fit iteration at n = 2000 (LML + "
                                          "gradient, float64 NumPy + BLAS)"}
    print(json.dumps(line, default=float), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "c5":
        run_love(args, rank, world, local)
        return
    if args.workload in ("c1", "c2", "c4"):
        run_config(args, rank, world, local)
        return
    if args.workload == "c3fit":
        run_c3fit(args, rank, world, local)
        return
    if args.workload == "materialized":
        run_materialized(args, rank, world, local)
        return

    from mojogp_b200 import _lib, synthetic
    from mojogp_b200.kernel import RBF, make_ard_kernel
    from mojogp_b200.provider import DeviceBuffer, Provider, pinned
    import ctypes as C

    comm = None
    if world > 1:
        from mojogp_b200.distributed import Communicator
        comm = Communicator.from_env(device=local)

    n, d, t = args.n, args.d, args.t
    X, y_fit, ell = synthetic.config3(n=n, d=d)
    params = np.concatenate([ell, [1.0]]).astype(np.float32)
    kern = make_ard_kernel(RBF(ard=True), d)
    prov = Provider(X, kern, params, noise=0.0025, device=local)
    V = synthetic.probes_v(n, t, seed=1)
    Vc = np.ascontiguousarray(V.T)
    vd = DeviceBuffer.from_host(Vc, local)
    r0, r1 = (rank * n) // world, ((rank + 1) * n) // world
    od = DeviceBuffer((t, n), local)

    F = F_PER_PAIR_RBF(d, t)
    flops_total = float(n) * n * F  # whole job per step
    flops_local = float(r1 - r0) * n * F

    # Measured FP32 roofline denominator.
    peak_tf, peak_ms = C.c_double(), C.c_double()
    _lib.call("gpb_measure_fp32_peak", local, C.byref(peak_tf), C.byref(peak_ms))

    sampler = ClockSampler(local)
    if comm:
        comm.barrier()
    sampler.start()
    steps, warm = args.steps, args.warmup
    step_ms = np.zeros(steps)
    kern_ms = np.zeros(steps)
    launches = np.zeros(steps, dtype=np.int64)
    if comm is None:
        _lib.call("gpb_benchmark_forward", prov.h, vd.cptr, od.cptr, t, warm, steps, 1,
                  C.c_void_p(step_ms.ctypes.data), C.c_void_p(kern_ms.ctypes.data),
                  C.c_void_p(launches.ctypes.data))
    else:
        res = comm.benchmark_sharded_forward(prov, vd, od, t, warm, steps, r0, r1)
        step_ms[:], kern_ms[:], launches[:] = res
    clocks = sampler.stop()

    total_ms = float(step_ms.sum())
    if comm:
        total_ms = comm.allreduce_max(total_ms)
        kmean = comm.allreduce_max(float(kern_ms.mean()))
    else:
        kmean = float(kern_ms.mean())
    value = flops_total * steps / (total_ms * 1e-3) / 1e12

    # End to end through the C ABI with host buffers (H2D V, matvec, D2H out).
    e2e_tf = None
    if comm is None:
        out_h = np.empty_like(Vc)
        # Host buffers are page-locked once, outside the timed region, as a
        # caller staging inputs in pinned memory would have them.
        with pinned(Vc, out_h):
            t0 = time.perf_counter()
            for _ in range(max(1, min(steps, 3))):
                _lib.call("gpb_forward_matvec_host", prov.h, C.c_void_p(out_h.ctypes.data),
                          C.c_void_p(Vc.ctypes.data), t)
            e2e_s = (time.perf_counter() - t0) / max(1, min(steps, 3))
        e2e_tf = flops_total / e2e_s / 1e12
    else:
        e2e_tf = comm.e2e_sharded(prov, Vc, t, r0, r1, flops_total)

    # Fit s/iter through the public model API at the reference's resolved
    # defaults for this route (gp.py:800-807, 1437-1456: max CG 100, tol 1e-2,
    # max_tridiag 30, no preconditioner for matrix-free RBF-ARD; initial noise
    # 0.1 and default kernel parameters), 15 probes (t = 16), rows sharded like
    # the matvec.
    fit = None
    if args.fit_iters > 0:
        fit = run_fit(X, y_fit, args.fit_iters, local, comm)
        fit.pop("history", None)

    achieved = flops_local / (kmean * 1e-3) / 1e12
    layout = prov.matvec_layout(t)
    pairs_per_s = float(r1 - r0) * n / (kmean * 1e-3)
    sm_mhz = (clocks or {}).get("sm_mhz") or 1965.0
    fp32_peak = {"achieved": achieved, "peak": peak_tf.value, "unit": "TFLOP/s",
                 "frac": achieved / peak_tf.value, "flops_per_pair": F,
                 "peak_source": "measured FFMA probe (gpb_measure_fp32_peak) on this GPU"}
    if layout in ("gram-tensor-core", "gram-tensor-core-tf32"):
        f16 = layout == "gram-tensor-core"
        peaks_path = Path(__file__).resolve().parent / "MEASURED_PEAKS.json"
        try:
            bf16 = float(json.loads(peaks_path.read_text())["bf16_tflops"])
            src = "of measured: MEASURED_PEAKS.json bf16_tflops (burst)"
        except (OSError, KeyError, ValueError):
            bf16, src = 1590.0, "of fallback: 1.59 PFLOP/s bf16"
        peak = bf16 if f16 else bf16 / 2
        src += " = dense f16" if f16 else " / 2 = dense tf32"
        dp = 16 if d > 8 else 8
        tc = TC_PER_PAIR_GRAMH(dp, 16) if f16 else TC_PER_PAIR_GRAM(dp, 16)
        tc_achieved = pairs_per_s * tc / 1e12
        traffic = (GRAMH_TRAFFIC_C3 if f16 and world == 1 and (n, d, t) == (1_000_000, 16, 16)
                   else None)
        roofline = {"bound": "tensor", "achieved": tc_achieved, "peak": peak,
                    "unit": "TFLOP/s", "frac": tc_achieved / peak, "traffic": traffic,
                    "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                       "launch at this size (profiles/kv_tile_gramh_rbf_ard_d16_t16.md)"
                                       if traffic else "not captured for this configuration"),
                    "peak_source": src, "tensor_flops_per_pair": tc,
                    "mufu": {"achieved_per_sm_clk": pairs_per_s / 148 / (sm_mhz * 1e6),
                             "peak_per_sm_clk": MUFU_PER_SM_CLK,
                             "frac": pairs_per_s / 148 / (sm_mhz * 1e6) / MUFU_PER_SM_CLK},
                    "fp32_equivalent": fp32_peak}
    else:
        roofline = dict(bound="fp32", traffic=None,
                        nominal_peak=148 * 128 * 2 * 1.965e9 / 1e12, **fp32_peak)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": total_ms / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (config 3 recipe: X~N(0,I), l~U[0.5,3], seed 3)",
        "config": {"workload": "config3 K(X,X)V RBF-ARD matrix-free, t=16", "n": n, "d": d,
                   "t": t, "parallelism": f"row-shard x{world}", "tile_kernel": layout,
                   "l2": "256 MB flush before every step; packed column tiles 128 MB"},
        "gpu_launches": int(launches.sum()),
        "step_split_ms": {"tile_kernel": kmean, "pack_and_exchange": total_ms / steps - kmean,
                          "note": "mean over the timed steps, max over ranks; pack_and_exchange "
                                  "= packing, the colmax all-reduce and the NCCL all-gather of "
                                  "the packed column tiles (0 exchange on 1 GPU)"},
        "e2e": {"value": e2e_tf, "unit": UNIT, "h2d_bytes_per_step": int(Vc.nbytes),
                "d2h_bytes_per_step": int(Vc.nbytes)},
        "roofline": roofline,
        "clocks": clocks,
        "fit": fit,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r, kind = reference_matvec_sample(X, V, ell, target_s=args.cpu_seconds, max_rows=1024,
                                          threads=os.cpu_count() or 1)
        line["cpu_baseline"] = {
            "value": r["pairs_per_s"] * F / 1e12, "unit": UNIT, "cores": r["threads"],
            "kind": kind,
            "sample": f"{r['rows']} output rows x all {n} columns: "
                      + ("the reference's KernelNode.evaluate (baseline/_ref) + BLAS"
                         if kind == "reference" else
                         "float64 NumPy evaluator restated (kernel.py:804-923) + BLAS")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if comm:
        comm.close()


if __name__ == "__main__":
    main()
