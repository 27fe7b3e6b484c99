#!/usr/bin/env python3
"""PSGD-Kron optimizer step benchmark on B200: steps/sec with a preconditioner update every step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload llama-1.1b|gpt2-medium|vit-tiny|config1]
                    [--impl b200|reference] [--no-extra]
N > 1 is launched by torch.distributed.run (one rank per GPU over NCCL): parameters are partitioned across ranks
by FLOP-balanced assignment and the updated parameters are all-gathered every step (psgd_pro_b200.dist).

One step = one full KronWhiten.step_math over the whole parameter set (damping-noise draws, preconditioner update
of every factor, preconditioned gradient, clip, parameter update, and for N > 1 the all-gather). Gradients are
synthetic N(0, std^2) tensors of the workload's shapes, pre-generated on the device (two sets, alternating; each
larger than L2). The timed region is bracketed by barrier + synchronize, timed with CUDA events, max over ranks.
Launch-level CUDA events inside the timed region give each kernel launch's duration for the roofline line.

At N = 1 the line also carries sub-records measured after the headline (outside its timed region): the other
parameter sets of the benchmark plan (GPT-2-medium, the north-star target; ViT-Tiny; the 256 x 512 config 1) and
the triangle-stored SYRK / SYMM / TRMM microbenchmark with cuBLAS timed beside it (--no-extra skips them).

--impl reference times the reference algorithm's CPU implementation (the numpy restatement in oracle/, fp32, every
host thread) on rank 0: one timed step per unique parameter shape, extrapolated by the shape multiplicities.
"""
import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_NOTE = "inputs larger than L2 (two alternating gradient sets of GBs)"


def load_peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="llama-1.1b")
    ap.add_argument("--precision", default=None, choices=[None, "fp32", "bf16"])
    ap.add_argument("--max-skew", default="inf")
    ap.add_argument("--max-size", type=float, default=8192)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the sub-records (other workloads, SYRK table)")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--buckets", type=int, default=None, help="N > 1: all-gather buckets per rank (default 4)")
    return ap.parse_args()


def config_of(args, shapes, desc, world):
    """The config dict both arms print (same keys and values for the same workload and N)."""
    return {"workload": args.workload, "parameter_set": desc, "tensors": len(shapes),
            "params": sum(math.prod(s) for s in shapes), "max_precond_size": args.max_size,
            "max_skew": args.max_skew, "parallelism": f"precond-shard{world}+allgather" if world > 1 else "single",
            "l2": L2_NOTE}


# ---- CPU reference (oracle) timing ------------------------------------------------------------------------------
def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [d.get("num_threads", 0) for d in threadpool_info() if d.get("user_api") == "blas"]
        if n:
            return max(n)
    except Exception:
        pass
    return os.cpu_count() or 1


def use_all_host_threads():
    """Every host thread for the BLAS the oracle calls (torchrun sets OMP_NUM_THREADS=1 in its workers)."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n, user_api="blas")
    except Exception:
        pass
    return n


class CpuReference:
    """The reference algorithm on the host (oracle/psgd_oracle.py, fp32 numpy): one optimizer per unique parameter
    shape, each timed over one full step; the full-step time is the multiplicity-weighted sum."""

    def __init__(self, shapes, max_size, max_skew, grad_std, seed=0):
        import numpy as np
        from oracle import psgd_oracle as O
        self.np, self.O = np, O
        uniq = {}
        for s in shapes:
            sq = tuple(x for x in s if x != 1)
            uniq[sq] = uniq.get(sq, 0) + 1
        self.shapes = sorted(uniq, key=lambda s: -math.prod(s) if s else 0)
        self.mult = uniq
        rng = np.random.default_rng(seed)
        self.units = []
        for s in self.shapes:
            p = rng.standard_normal(s if s else (), dtype=np.float32) * np.float32(0.02)
            opt = O.KronWhitenOracle([np.asarray(p)], preconditioner_max_size=max_size,
                                     preconditioner_max_skew=max_skew, dtype=np.float32)
            g = np.asarray(rng.standard_normal(s if s else (), dtype=np.float32) * np.float32(grad_std))
            draws = opt.make_draws(rng, [g], coins=[1.0])
            draws["update"] = 0.0
            self.units.append((opt, g, draws))
        self.t = {}

    def time_shape(self, k):
        opt, g, draws = self.units[k]
        t0 = time.perf_counter()
        opt.step([g], draws)
        dt = time.perf_counter() - t0
        self.t[self.shapes[k]] = dt
        return dt

    def full_step_seconds(self):
        return sum(self.t[s] * self.mult[s] for s in self.shapes)

    def per_shape(self):
        return [{"shape": list(s), "count": self.mult[s], "seconds": round(self.t[s], 4)} for s in self.shapes]

    def describe(self):
        return (f"one fp32 step of each of the {len(self.shapes)} unique parameter shapes (numpy oracle), "
                f"scaled by multiplicity to the {sum(self.mult.values())}-tensor set (extrapolated)")


# ---- clocks during the timed region --------------------------------------------------------------------------------
class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index, path):
        self.path, self.idx = path, gpu_index
        self.proc = None
        try:
            self.f = open(path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(gpu_index)], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                c = [x.strip() for x in line.split(",")]
                if len(c) < 9:
                    continue
                try:
                    sm.append(float(c[1]))
                    smax.append(float(c[2]))
                except ValueError:
                    continue
                for nm, v in zip(names, c[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(nm)
        if not sm:  # a timed region shorter than one sampling interval: take one reading now
            try:
                out = subprocess.run(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-i",
                                      str(self.idx)], capture_output=True, text=True, timeout=10).stdout
                c = [x.strip() for x in out.strip().split(",")]
                sm, smax = [float(c[1])], [float(c[2])]
                reasons = {nm for nm, v in zip(names, c[5:9]) if v.lower().startswith("active")}
            except Exception:
                return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---- the reference arm --------------------------------------------------------------------------------------------
def run_reference(args, rank, world):
    from psgd_pro_b200.workloads import WORKLOADS
    shapes_fn, pdt, gdt, std, desc = WORKLOADS[args.workload]
    if rank != 0:
        return
    cores = use_all_host_threads()
    shapes = shapes_fn()
    ref = CpuReference(shapes, args.max_size, float(args.max_skew), std)
    n = len(ref.shapes)
    for k in range(n):  # one untimed rotation fills the table (initialisation and first-call costs)
        ref.time_shape(k)
    for w in range(args.warmup):
        ref.time_shape(w % n)
    vals = []
    for i in range(args.steps):
        ref.time_shape(i % n)
        vals.append(1.0 / ref.full_step_seconds())
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": "psgd_kron_steps_per_sec", "value": v, "unit": "steps/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / v,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_of(args, shapes, desc, world),
            "cpu_baseline": {"value": v, "unit": "steps/s", "cores": cores, "kind": "port",
                             "sample": ref.describe() + "; each timed step re-times one shape in rotation",
                             "extrapolated": True, "per_shape": ref.per_shape()},
            "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- device-timed steps of one optimizer ---------------------------------------------------------------------------
def timed_steps(opt, inners, grads, steps, warmup, barrier, nvtx=False, before_timed=None):
    """warmup untimed steps, then `steps` timed ones with launch-level events (each optimizer's trace hook) for the
    phase table. Returns (ms per step on this rank, {phase: ms per step, summed over the optimizers})."""
    import torch
    for w in range(warmup):
        opt.step_math(grads[w % 2])
    torch.cuda.synchronize()
    for inner in inners:
        inner.check_errors()
    events = []

    def trace(name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        events.append((name, ev))
    for inner in inners:
        inner.trace = trace
    if before_timed is not None:
        before_timed()
    barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if nvtx:
        torch.cuda.nvtx.range_push("timed")  # profilers filter on this range (ncu --nvtx --nvtx-include timed/)
    t0.record()
    for i in range(steps):
        opt.step_math(grads[i % 2])
    t1.record()
    if nvtx:
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    ms = t0.elapsed_time(t1) / steps
    for inner in inners:
        inner.trace = None
        inner.check_errors()
    phase_ms = {}
    for (a, ea), (b, eb) in zip(events[:-1], events[1:]):
        if b == "start":
            continue
        phase_ms[b] = phase_ms.get(b, 0.0) + ea.elapsed_time(eb)
    return ms, {k: v / max(1, steps) for k, v in phase_ms.items()}


def roofline_of(inners, phase_ms, peaks, peak_src):
    """The dominant tensor-core phase: algorithmic FLOPs of its launches (summed over the optimizers) / their event
    duration, against the measured sustained bf16 peak (a kernel timed inside a long step)."""
    if not inners or not phase_ms:
        return None
    groups = {}
    for inner in inners:
        for n, g in inner._plan.phase_groups():
            groups.setdefault(n, []).append(g)
    cand = [(phase_ms.get(n, 0.0), n) for n in groups]
    tm, dominant = max(cand)
    flops = sum(g.flops for g in groups[dominant])
    achieved = flops / (tm * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    kind = groups[dominant][0].kind
    kernel = (f"gemm_pair_kernel<256,3,{kind & 7}>" if kind & 8 else
              (f"gemm_group_kernel<1,256,4,{kind}>" if inners[0]._split == 1 else
               f"gemm_group_kernel<3,128,3,{kind}>"))
    # DRAM traffic of the Procrustes pair-kernel launch, from one ncu capture (dram__bytes_read.sum +
    # dram__bytes_write.sum) of the one-layer Llama case (the same factor sizes), scaled to this launch by FLOPs
    traffic = None
    if dominant in ("procrustes", "qupdate") and kind == 9:
        traffic = flops * (2.663e9 / 1.2609e12)
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "traffic": traffic, "traffic_unit": "bytes per launch", "kernel": kernel, "phase": dominant,
            "flops_per_launch": flops, "ms_per_launch": tm,
            "peak_source": f"{peak_src} sustained bf16 (MEASURED_PEAKS.json)" if peak_src == "measured"
            else "fallback"}


def workload_tensors(name, dev, max_size, max_skew, world=1, owner=None, buckets=1):
    import torch
    from psgd_pro_b200.dist import assignment_for, make_flat_params
    from psgd_pro_b200.workloads import WORKLOADS
    shapes_fn, pdt, gdt, std, desc = WORKLOADS[name]
    shapes = shapes_fn()
    dt = {"bf16": torch.bfloat16, "fp32": torch.float32}
    if owner is None:
        owner = assignment_for([tuple(x for x in s if x != 1) for s in shapes], world, max_size, max_skew)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    params, flat, seg = make_flat_params(shapes, owner, world, dt[pdt], dev,
                                         init=lambda s: torch.randn(s, device=dev, generator=gen) * 0.02,
                                         buckets=buckets, max_size=max_size, max_skew=max_skew)
    grads = [[(torch.randn(s, device=dev, generator=gen) * std).to(dt[gdt]) for s in shapes] for _ in range(2)]
    return shapes, desc, std, owner, params, flat, seg, grads


# ---- sub-records at N = 1 ---------------------------------------------------------------------------------------------
def sub_workload(name, dev, args, peaks, peak_src, steps, warmup):
    """steps/s of another parameter set of the benchmark plan on this GPU, with its phase table and roofline."""
    import torch
    from psgd_pro_b200 import KronWhiten
    from psgd_pro_b200.dist import falg
    max_skew = float(args.max_skew)
    shapes, desc, std, owner, params, flat, seg, grads = workload_tensors(name, dev, args.max_size, max_skew)
    opt = KronWhiten(params, preconditioner_max_size=args.max_size, preconditioner_max_skew=max_skew,
                     precision=args.precision, cuda_graphs=False)
    torch.manual_seed(0)
    torch.cuda.manual_seed(0)
    ms, phase_ms = timed_steps(opt, [opt], grads, steps, warmup, lambda: None)
    F = sum(falg(tuple(x for x in s if x != 1), args.max_size, max_skew) for s in shapes)
    rec = {"workload": name, "parameter_set": desc, "tensors": len(shapes),
           "params": sum(math.prod(s) for s in shapes), "steps": steps, "warmup": warmup, "ms_per_step": ms,
           "value": 1000.0 / ms, "unit": "steps/s", "f_alg_tflop_per_step": F / 1e12,
           "whole_step_tflops": F / (ms * 1e-3) / 1e12,
           "whole_step_frac_of_burst": F / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"],
           "whole_step_frac_of_sustained": F / (ms * 1e-3) / 1e12 / peaks.get("bf16_tflops_sustained",
                                                                              peaks["bf16_tflops"]),
           "roofline": roofline_of([opt], phase_ms, peaks, peak_src), "gpu_launches_per_step":
               opt._plan.launches_per_step(True),
           "phases_ms": {k: round(v, 4) for k, v in sorted(phase_ms.items(), key=lambda x: -x[1])}}
    if name == "gpt2-medium":  # north star: >= 60% of the bf16 dense peak on one GPU
        rec["north_star"] = {"target_frac_of_burst": 0.6, "met": rec["whole_step_frac_of_burst"] >= 0.6,
                             "target_ms_per_step": F / (0.6 * peaks["bf16_tflops"] * 1e12) * 1e3}
    del opt, params, grads, flat
    torch.cuda.empty_cache()
    return rec


class CublasRef:
    """cuBLAS fp32 SYRK / SYMM / TRMM (the library calls of the reference's kernels/blas.cpp:20-65 and a TRMM) through
    its C API, on the current stream; the comparators of the SYRK table. Column-major conventions: a row-major
    n x n matrix is the column-major transpose."""

    def __init__(self, torch):
        import glob
        import nvidia
        cand = glob.glob(os.path.join(os.path.dirname(nvidia.__path__[0]), "nvidia", "cublas", "lib",
                                      "libcublas.so*"))
        self.lib = ctypes.CDLL(sorted(cand)[-1] if cand else "libcublas.so.12")
        self.h = ctypes.c_void_p()
        if self.lib.cublasCreate_v2(ctypes.byref(self.h)) != 0:
            raise RuntimeError("cublasCreate failed")
        self.lib.cublasSetStream_v2(self.h, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        self.one, self.zero = ctypes.c_float(1.0), ctypes.c_float(0.0)

    def ssyrk(self, A, C, n, k):  # C (upper, column-major) = A^T A with A column-major k x n (= row-major n x k)
        return self.lib.cublasSsyrk_v2(self.h, 0, 1, n, k, ctypes.byref(self.one), ctypes.c_void_p(A.data_ptr()), k,
                                       ctypes.byref(self.zero), ctypes.c_void_p(C.data_ptr()), n)

    def ssymm(self, S, X, C, n, p):  # C = S X, S symmetric (upper), column-major n x n, X n x p
        return self.lib.cublasSsymm_v2(self.h, 0, 0, n, p, ctypes.byref(self.one), ctypes.c_void_p(S.data_ptr()), n,
                                       ctypes.c_void_p(X.data_ptr()), n, ctypes.byref(self.zero),
                                       ctypes.c_void_p(C.data_ptr()), n)

    def strmm(self, T, X, C, n, p):  # C = triu(T) X (column-major, out of place)
        return self.lib.cublasStrmm_v2(self.h, 0, 0, 0, 0, n, p, ctypes.byref(self.one),
                                       ctypes.c_void_p(T.data_ptr()), n, ctypes.c_void_p(X.data_ptr()), n,
                                       ctypes.c_void_p(C.data_ptr()), n)

    def close(self):
        self.lib.cublasDestroy_v2(self.h)


def event_time(torch, fn, reps, flush):
    """Median device time of fn over reps runs, L2 flushed (a buffer larger than L2 written) before each run."""
    ts = []
    for _ in range(reps):
        flush.add_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def syrk_table(dev, reps=5):
    """Config 3: C = A A^T stored as the packed upper triangle, n = k in {1024, 2048, 4096, 8192}, A ~ N(0, 1/n),
    bf16 (one bf16 MMA, fp32 accumulation) and fp32 (bf16 hi/lo pairs, three MMAs) inputs; SYMM-from-triangle S X and
    TRMM triu(T) X at the same n in fp32. TFLOP/s on the algorithmic counts n(n+1)k (SYRK), 2n^3 (SYMM), n^2(n+1)
    (TRMM). "kernel": the tensor-core product with its operands resident; "op": the call a plug-in user makes, fp32
    storage in, fp32 out (operand staging from the stored triangle included). Beside it cuBLAS: Ssyrk / Ssymm /
    Strmm (fp32, FMA units, what kernels/blas.cpp calls) and the bf16 GEMM A A^T (full square)."""
    import torch
    from psgd_pro_b200 import kernels as K, ops
    torch.backends.cuda.matmul.allow_tf32 = False
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > L2
    cb = CublasRef(torch)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = []
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    try:
        for n in (1024, 2048, 4096, 8192):
            A32 = torch.randn(n, n, device=dev, generator=g) / math.sqrt(n)
            A16 = A32.to(torch.bfloat16)
            P = torch.empty(n * (n + 1) // 2, device=dev)
            f_syrk = n * (n + 1) * n
            rec = {"n": n, "k": n}
            # bf16 SYRK, packed output: the operand is the bf16 matrix itself (row pitch n, 16-byte aligned)
            spec = K.make_spec((A16, None), (A16, None), n, n, n, bn=256, mode=K.PSGD_GEMM_SYRK, out_packed=P)
            grp = K.GemmGroup([spec], 1, dev)
            t = event_time(torch, lambda: grp.launch(err), reps, flush)
            rec["syrk_bf16"] = {"ms": t, "tflops": f_syrk / t / 1e9, "kernel": "pair" if grp.kind & 8 else "one-cta"}
            # fp32 SYRK: hi/lo operand staged once (kernel), or per call (op)
            (hi, lo), keep = K.to_operand(A32, split=True)
            spec3 = K.make_spec((hi, lo), (hi, lo), n, n, n, bn=128, mode=K.PSGD_GEMM_SYRK, out_packed=P)
            grp3 = K.GemmGroup([spec3], 3, dev)
            t = event_time(torch, lambda: grp3.launch(err), reps, flush)
            rec["syrk_fp32_kernel"] = {"ms": t, "tflops": f_syrk / t / 1e9}
            t = event_time(torch, lambda: ops.syrk_packed_impl(A32, False), reps, flush)
            rec["syrk_fp32_op"] = {"ms": t, "tflops": f_syrk / t / 1e9}
            C = torch.empty(n, n, device=dev)
            t = event_time(torch, lambda: cb.ssyrk(A32, C, n, n), reps, flush)
            rec["cublas_ssyrk_fp32"] = {"ms": t, "tflops": f_syrk / t / 1e9}
            t = event_time(torch, lambda: torch.matmul(A16, A16.T), reps, flush)
            rec["cublas_gemm_bf16_full"] = {"ms": t, "tflops_useful": f_syrk / t / 1e9,
                                            "tflops_raw": 2 * n ** 3 / t / 1e9}
            # SYMM from the triangle and TRMM, fp32
            S = (A32 + A32.T).triu()
            X = torch.randn(n, n, device=dev, generator=g) / math.sqrt(n)
            t = event_time(torch, lambda: ops.symm_impl(S, X), reps, flush)
            rec["symm_fp32_op"] = {"ms": t, "tflops": 2 * n ** 3 / t / 1e9}
            t = event_time(torch, lambda: cb.ssymm(S, X, C, n, n), reps, flush)
            rec["cublas_ssymm_fp32"] = {"ms": t, "tflops": 2 * n ** 3 / t / 1e9}
            T = A32 + torch.eye(n, device=dev)
            t = event_time(torch, lambda: ops.trmm_impl(T, X), reps, flush)
            rec["trmm_fp32_op"] = {"ms": t, "tflops": n * n * (n + 1) / t / 1e9}
            t = event_time(torch, lambda: cb.strmm(T, X, C, n, n), reps, flush)
            rec["cublas_strmm_fp32"] = {"ms": t, "tflops": n * n * (n + 1) / t / 1e9}
            out.append(rec)
            del A32, A16, P, C, S, X, T, hi, lo, keep, grp, grp3
        ops.check_errors()
        if int(err.item()) != 0:
            raise RuntimeError(f"device error flags {int(err.item()):#x}")
    finally:
        cb.close()
        torch.cuda.empty_cache()
    return out


def e2e_reduce_scatter(params, owner, flat, seg, kw, grads, steps, dev, world, barrier):
    """steps/s of the sharded step with the gradient reduce-scatter fused in, each step's full local gradient set
    copied from pinned host memory (the next step's copy starts once this step's reduce-scatters have read the
    buffer) and the clip scales read back."""
    import torch
    import torch.distributed as dist
    from psgd_pro_b200.dist import ShardedKronWhiten
    opt = ShardedKronWhiten(params, assignment=owner, flat=(flat, seg), reduce_scatter=True, **kw)
    views = opt.local_grads()
    host = [g.cpu().pin_memory() for g in grads[0]]
    met = torch.empty(max(1, len(opt.owned)), dtype=torch.float32).pin_memory()
    cs, main = torch.cuda.Stream(), torch.cuda.current_stream()
    for _ in range(2):  # warm-up: plans, first-call costs
        for h, v in zip(host, views):
            v.copy_(h, non_blocking=True)
        opt.step_math(views)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    copied = torch.cuda.Event()
    e0.record()
    for i in range(steps):
        with torch.cuda.stream(cs):
            if opt.rs_consumed is not None:
                cs.wait_event(opt.rs_consumed)
            for h, v in zip(host, views):
                v.copy_(h, non_blocking=True)
            copied.record(cs)
        main.wait_event(copied)
        opt.step_math(views)
        opt.clip_scales_into(met)
        torch.cuda.current_stream().synchronize()
        _ = float(met[0])
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    h2d = sum(h.numel() * h.element_size() for h in host) * world
    for o in opt.inners:
        o.check_errors()
    del opt
    torch.cuda.empty_cache()
    return {"value": 1000.0 / ms, "unit": "steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": met.numel() * 4,
            "inputs": "every rank copies in its whole local gradient set (as N = 1 does); the step reduce-scatters "
                      "it (NCCL, average over ranks) bucket by bucket before each bucket's update"}


def gemm_vs_cublas(dev):
    """This package's tcgen05 GEMM beside cuBLAS's bf16 GEMM (torch.matmul) on the step's largest shapes, random
    data, each looped for about 1.5 s so both run under the same 1000 W cap: TFLOP/s, joules per launch (NVML energy
    counter) and the median SM clock. Epilogues: plain (bf16 out, as cuBLAS), aux (fp32 read and written plus the
    transposed bf16 copy: the q-update / Procrustes form) and SYRK (the upper tiles only, n^3 useful FLOPs)."""
    import torch
    from psgd_pro_b200 import kernels as K
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        energy = lambda: pynvml.nvmlDeviceGetTotalEnergyConsumption(h) / 1000.0
    except Exception:
        energy = None
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def loop(fn, flops, seconds=1.5):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        reps = max(5, int(seconds / max(a.elapsed_time(b) * 1e-3, 1e-6)))
        phys = os.environ["CUDA_VISIBLE_DEVICES"].split(",")[dev.index] if "CUDA_VISIBLE_DEVICES" in os.environ \
            else dev.index
        import tempfile
        clk = ClockSampler(phys, os.path.join(tempfile.gettempdir(), "psgd_gemm_vs_cublas_clocks.csv"))
        e0 = energy() if energy else None
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        e1 = energy() if energy else None
        c = clk.stop()
        ms = a.elapsed_time(b) / reps
        rec = {"ms": ms, "tflops": flops / ms / 1e9, "sm_mhz": c["sm_mhz"] if c else None}
        if e0 is not None:
            rec["J_per_launch"] = (e1 - e0) / reps
            rec["tflop_per_J"] = flops / rec["J_per_launch"] / 1e12 if rec["J_per_launch"] > 0 else None
        return rec

    out = []
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    for n in (5632, 8192):
        A = torch.randn(n, n, device=dev, generator=g).to(torch.bfloat16)
        B = torch.randn(n, n, device=dev, generator=g).to(torch.bfloat16)
        C = torch.empty(n, n, device=dev, dtype=torch.bfloat16)
        Q = torch.randn(n, n, device=dev, generator=g)
        rec = {"n": n, "cublas_bf16_gemm": loop(lambda: torch.matmul(A, B.T, out=C), 2 * n ** 3)}
        gp = K.GemmGroup([K.make_spec((A, None), (B, None), n, n, n, bn=256, out_hi=C)], 1, dev)
        rec["ours_plain"] = loop(lambda: gp.launch(err), 2 * n ** 3)
        ga = K.GemmGroup([K.make_spec((A, None), (B, None), n, n, n, bn=256, alpha=-1e-3, beta=1.0, aux=Q, out_f32=Q,
                                      out_hi_t=C)], 1, dev)
        rec["ours_aux"] = loop(lambda: ga.launch(err), 2 * n ** 3)
        gs = K.GemmGroup([K.make_spec((A, None), (A, None), n, n, n, bn=256, mode=K.PSGD_GEMM_SYRK, out_hi=C)], 1, dev)
        rec["ours_syrk_useful"] = loop(lambda: gs.launch(err), n ** 3)
        rec["kernels"] = {"plain": gp.kind, "aux": ga.kind, "syrk": gs.kind}
        out.append(rec)
        del A, B, C, Q, gp, ga, gs
    torch.cuda.synchronize()
    if int(err.item()) != 0:
        raise RuntimeError(f"device error flags {int(err.item()):#x}")
    torch.cuda.empty_cache()
    return out


# ---- the B200 arm ---------------------------------------------------------------------------------------------------
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    from psgd_pro_b200.dist import ShardedKronWhiten, falg

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    max_skew = float(args.max_skew)
    nb = (args.buckets or 4) if world > 1 else 1
    shapes, desc, std, owner, params, flat, seg, grads = workload_tensors(args.workload, dev, args.max_size,
                                                                          max_skew, world, buckets=nb)
    kw = dict(preconditioner_max_size=args.max_size, preconditioner_max_skew=max_skew, precision=args.precision,
              cuda_graphs=False)
    opt = ShardedKronWhiten(params, assignment=owner, flat=(flat, seg) if world > 1 else None, **kw)
    inners = opt.inners
    torch.manual_seed(0)
    torch.cuda.manual_seed(0)

    def barrier():
        if world > 1:
            dist.barrier()

    import tempfile
    phys = os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local] if "CUDA_VISIBLE_DEVICES" in os.environ else local
    clocks = {}

    def start_clocks():  # sampled during the timed region only
        clocks["c"] = ClockSampler(phys, os.path.join(tempfile.gettempdir(), f"psgd_bench_clocks_rank{rank}.csv"))
    if world > 1:
        opt.timing = []
    ms, phase_ms = timed_steps(opt, inners, grads, args.steps, args.warmup, barrier, nvtx=True,
                               before_timed=start_clocks)
    clk = clocks["c"].stop()
    clk = clk if rank == 0 else None
    comm = None
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        # per-rank compute (step start to the last bucket's compute end) and the exposed all-gather tail
        tm = opt.timing_ms()[-args.steps:]
        comp = statistics.median(x["compute_ms"] for x in tm)
        tail = statistics.median(x["exposed_gather_ms"] for x in tm)
        gat = statistics.median(x["gather_ms"] for x in tm)
        v = torch.tensor([comp, -comp, tail, gat], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        comm = {"collective": "all_gather_into_tensor (NCCL) of the updated parameters, bf16, "
                              f"{opt.nbuckets} buckets per rank, each started on a side stream when its bucket's "
                              "step has finished",
                "bytes_per_rank_per_step": opt.gather_bytes(), "compute_ms_max_rank": float(v[0]),
                "compute_ms_min_rank": float(-v[1]), "exposed_gather_ms_max_rank": float(v[2]),
                "gather_ms_max_rank": float(v[3]),
                "note": "compute = this rank's buckets, start to end; exposed gather = time from the end of the "
                        "last bucket's compute to the end of the last all-gather"}
        opt.timing = None
    peaks, peak_src = load_peaks()
    roofline = roofline_of(inners, phase_ms, peaks, peak_src)

    # end to end through the public API: every step's gradients are copied in from pinned host memory and the
    # step's metric (per-parameter clip scales) is read back to the host. Pipelined as a training loop would run
    # it: step i + 1's gradients travel on a copy stream into the second of two device buffers while step i
    # computes, and step i's metric is read once the step has finished; all of it inside the timed region.
    ek = args.e2e_steps or max(2, min(args.steps, 5))
    # each rank copies in the gradients of the parameters it owns: the sharded step reads only those (at N = 1, all)
    own = list(opt.owned)
    host = [[grads[j][i].cpu().pin_memory() for i in own] for j in range(2)]
    bufs = [[grads[j][i] for i in own] for j in range(2)]
    mets = [torch.empty(max(1, len(own)), dtype=torch.float32).pin_memory() for _ in range(2)]
    main, copy_stream = torch.cuda.current_stream(), torch.cuda.Stream()
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    met_ready = [torch.cuda.Event(), torch.cuda.Event()]
    seen = []
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()

    def h2d(i):  # step i's inputs into buffer i % 2, after the step that last used that buffer finished
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(done[b])
            for hg, dgt in zip(host[b], bufs[b]):
                dgt.copy_(hg, non_blocking=True)
            copied[b].record(copy_stream)

    h2d(0)
    for i in range(ek):
        b = i % 2
        if i + 1 < ek:
            h2d(i + 1)
        main.wait_event(copied[b])
        opt.step_math(grads[b])  # bufs[b] holds grads[b]'s owned tensors, just refilled
        opt.clip_scales_into(mets[b])
        met_ready[b].record(main)
        done[b].record(main)
        if i >= 1:  # the previous step's metric on the host
            met_ready[(i - 1) % 2].synchronize()
            seen.append(float(mets[(i - 1) % 2][0]))
    met_ready[(ek - 1) % 2].synchronize()
    seen.append(float(mets[(ek - 1) % 2][0]))
    e1.record()
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1) / ek
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    h2d_bytes = sum(g.numel() * g.element_size() for g in host[0])
    if world > 1:  # whole job: every rank's copies
        t = torch.tensor([float(h2d_bytes)], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        h2d_bytes = int(t.item())
    e2e = {"value": 1000.0 / e_ms, "unit": "steps/s", "h2d_bytes_per_step": h2d_bytes,
           "d2h_bytes_per_step": mets[0].numel() * 4, "overlap": "next step's H2D copy during this step"}
    if world > 1:
        e2e["inputs"] = ("each rank copies in the gradients of the parameters it owns (the sharded step reads no "
                         "others, as a reduce-scatter would deliver them); N = 1 copies all of them")

    # at N > 1 also the data-parallel loop as it runs in training: every rank copies in its whole set of local
    # gradients (as at N = 1) and the step reduce-scatters them (average over ranks) before the sharded update
    e2e_rs = None
    if world > 1:
        e2e_rs = e2e_reduce_scatter(params, owner, flat, seg, kw, grads, ek, dev, world, barrier)
        e2e["reduce_scatter"] = e2e_rs

    F = sum(falg(tuple(x for x in s if x != 1), args.max_size, max_skew) for s in shapes)
    launches = sum(o._plan.launches_per_step(True) for o in inners) * args.steps
    if world > 1:
        t = torch.tensor([float(launches)], device=dev)
        dist.all_reduce(t)
        launches = int(t.item())

    # CPU baseline and the sub-records (rank 0, one GPU only), after the headline's timed regions
    cpu, extra = None, None
    if rank == 0 and world == 1:
        prec = inners[0].precision
        del opt, inners, params, grads, flat, bufs
        torch.cuda.empty_cache()
        if not args.no_cpu_baseline:
            cores = use_all_host_threads()
            ref = CpuReference(shapes, args.max_size, max_skew, std)
            for k in range(len(ref.shapes)):
                ref.time_shape(k)
            v = 1.0 / ref.full_step_seconds()
            cpu = {"value": v, "unit": "steps/s", "cores": cores, "kind": "port", "sample": ref.describe(),
                   "extrapolated": True, "per_shape": ref.per_shape()}
        if not args.no_extra:
            extra = {}
            for name, st in (("gpt2-medium", max(5, args.steps // 2)), ("vit-tiny", max(5, args.steps)),
                             ("config1", max(5, args.steps))):
                if name != args.workload:
                    extra[name] = sub_workload(name, dev, args, peaks, peak_src, st, max(3, args.warmup))
            extra["syrk_config3"] = syrk_table(dev)
            extra["gemm_vs_cublas"] = gemm_vs_cublas(dev)
    else:
        prec = inners[0].precision if inners else args.precision
    if rank == 0:
        line = {"metric": "psgd_kron_steps_per_sec", "value": 1000.0 / ms, "unit": "steps/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if prec == "bf16" else "bf16x3",
                "data": "synthetic", "config": config_of(args, shapes, desc, world),
                "f_alg_tflop_per_step": F / 1e12,
                "whole_step_tflops": F / (ms * 1e-3) / 1e12,
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clk, "collective": comm,
                "phases_ms": {k: round(v, 4) for k, v in sorted(phase_ms.items(), key=lambda x: -x[1])}}
        if extra is not None:
            line["extra"] = extra
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
