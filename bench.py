#!/usr/bin/env python3
"""PSGD-Kron optimizer step benchmark on B200: steps/sec with a preconditioner update every step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload llama-1.1b|gpt2-medium|vit-tiny|config1]
                    [--impl b200|reference]
N > 1 is launched by torch.distributed.run (one rank per GPU over NCCL): parameters are partitioned across ranks
by FLOP-balanced assignment and the updated parameters are all-gathered every step (psgd_pro_b200.dist).

One step = one full KronWhiten.step_math over the whole parameter set (damping-noise draws, preconditioner update
of every factor, preconditioned gradient, clip, parameter update, and for N > 1 the all-gather). Gradients are
synthetic N(0, std^2) tensors of the workload's shapes, pre-generated on the device (two sets, alternating; each
larger than L2). The timed region is bracketed by barrier + synchronize, timed with CUDA events, max over ranks.
Launch-level CUDA events inside the timed region give each kernel launch's duration for the roofline line.

--impl reference times the reference algorithm's CPU implementation (the numpy restatement in oracle/, fp32, all
host threads) on rank 0: one timed step per unique parameter shape, extrapolated by the shape multiplicities.
"""
import argparse
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
    ap.add_argument("--e2e-steps", type=int, default=None)
    return ap.parse_args()


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

    def describe(self):
        return (f"one fp32 step of each of the {len(self.shapes)} unique parameter shapes (numpy oracle), "
                f"scaled by multiplicity to the {sum(self.mult.values())}-tensor set")


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
def run_reference(args, rank):
    from psgd_pro_b200.workloads import WORKLOADS
    shapes_fn, pdt, gdt, std, desc = WORKLOADS[args.workload]
    if rank != 0:
        return
    ref = CpuReference(shapes_fn(), args.max_size, float(args.max_skew), std)
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
            "data": "synthetic", "config": {"workload": args.workload, "parameter_set": desc,
                                            "max_precond_size": args.max_size, "max_skew": args.max_skew},
            "cpu_baseline": {"value": v, "unit": "steps/s", "cores": cpu_threads(), "kind": "port",
                             "sample": ref.describe() + "; each timed step re-times one shape in rotation"},
            "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- the B200 arm ---------------------------------------------------------------------------------------------------
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch
    import torch.distributed as dist
    from psgd_pro_b200 import KronWhiten
    from psgd_pro_b200.dist import ShardedKronWhiten, assignment_for, make_flat_params, falg
    from psgd_pro_b200.workloads import WORKLOADS

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    shapes_fn, pdt, gdt, std, desc = WORKLOADS[args.workload]
    shapes = shapes_fn()
    max_skew = float(args.max_skew)
    dt = {"bf16": torch.bfloat16, "fp32": torch.float32}
    owner = assignment_for([tuple(x for x in s if x != 1) for s in shapes], world, args.max_size, max_skew)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    params, flat, seg = make_flat_params(shapes, owner, world, dt[pdt], dev,
                                         init=lambda s: torch.randn(s, device=dev, generator=gen) * 0.02)
    grads = [[(torch.randn(s, device=dev, generator=gen) * std).to(dt[gdt]) for s in shapes] for _ in range(2)]
    kw = dict(preconditioner_max_size=args.max_size, preconditioner_max_skew=max_skew, precision=args.precision,
              cuda_graphs=False)
    opt = ShardedKronWhiten(params, assignment=owner, flat=(flat, seg) if world > 1 else None, **kw)
    inner = opt.inner
    torch.manual_seed(0)
    torch.cuda.manual_seed(0)

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up (builds the plan, first-call costs)
    for w in range(args.warmup):
        opt.step_math(grads[w % 2])
    torch.cuda.synchronize()
    if inner is not None:
        inner.check_errors()

    # timed region: launch-level events for the roofline
    events = []
    if inner is not None:
        def trace(name):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            events.append((name, ev))
        inner.trace = trace
    import tempfile
    phys = os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local] if "CUDA_VISIBLE_DEVICES" in os.environ else local
    clocks = ClockSampler(phys, os.path.join(tempfile.gettempdir(), f"psgd_bench_clocks_rank{rank}.csv"))
    barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")  # profilers filter on this range (ncu --nvtx --nvtx-include timed/)
    t0.record()
    for i in range(args.steps):
        opt.step_math(grads[i % 2])
    t1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop() if rank == 0 else None
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    if inner is not None:
        inner.trace = None
        inner.check_errors()

    # per-launch durations inside the timed region
    phase_ms = {}
    for (a, ea), (b, eb) in zip(events[:-1], events[1:]):
        if b == "start":
            continue
        phase_ms[b] = phase_ms.get(b, 0.0) + ea.elapsed_time(eb)
    nsteps = max(1, args.steps)
    phase_ms = {k: v / nsteps for k, v in phase_ms.items()}
    roofline, dominant = None, None
    peaks, peak_src = load_peaks()
    if inner is not None and phase_ms:
        groups = dict(inner._plan.phase_groups())
        cand = [(phase_ms.get(n, 0.0), n) for n in groups]
        tm, dominant = max(cand)
        flops = groups[dominant].flops
        achieved = flops / (tm * 1e-3) / 1e12
        peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        kind = groups[dominant].kind
        kernel = (f"gemm_pair_kernel<256,6,{kind & 7}>" if kind & 8 else
                  (f"gemm_group_kernel<1,256,4,{kind}>" if inner._split == 1 else f"gemm_group_kernel<3,128,3,{kind}>"))
        # DRAM traffic of the q-update / Procrustes pair kernel, from one ncu capture (dram__bytes_read.sum +
        # dram__bytes_write.sum) of the Procrustes launch of the one-layer Llama case (the same factor sizes),
        # scaled to this launch by FLOPs: 3.357 GB for 1.2609 TFLOP
        traffic = None
        if dominant in ("procrustes", "qupdate") and kind == 9:
            traffic = flops * (3.357e9 / 1.2609e12)
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "traffic": traffic, "traffic_unit": "bytes per launch",
                    "kernel": kernel, "phase": dominant, "flops_per_launch": flops, "ms_per_launch": tm,
                    "peak_source": f"{peak_src} sustained bf16 (MEASURED_PEAKS.json)" if peak_src == "measured"
                    else "fallback"}

    # end to end through the public API: every step's gradients are copied in from pinned host memory and the
    # step's metric (per-parameter clip scales) is read back to the host. Pipelined as a training loop would run
    # it: step i + 1's gradients travel on a copy stream into the second of two device buffers while step i
    # computes, and step i's metric is read once the step has finished; all of it inside the timed region.
    e2e = None
    ek = args.e2e_steps or max(2, min(args.steps, 5))
    # each rank copies in the gradients of the parameters it owns: the sharded step reads only those (at N = 1, all)
    own = list(opt.owned)
    host = [[grads[j][i].cpu().pin_memory() for i in own] for j in range(2)]
    bufs = [[grads[j][i] for i in own] for j in range(2)]
    nown = len(inner._plan.params) if inner is not None else 0
    mets = [torch.empty(max(1, nown), dtype=torch.float32).pin_memory() for _ in range(2)]
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
        if inner is not None:
            mets[b].copy_(inner._plan.clip[:max(1, nown)], non_blocking=True)
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
    h2d = sum(g.numel() * g.element_size() for g in host[0])
    if world > 1:  # whole job: every rank's copies
        t = torch.tensor([float(h2d)], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        h2d = int(t.item())
    e2e = {"value": 1000.0 / e_ms, "unit": "steps/s", "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": mets[0].numel() * 4, "overlap": "next step's H2D copy during this step"}

    # CPU baseline (rank 0, one GPU only): the reference algorithm on the host cores
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = CpuReference(shapes, args.max_size, max_skew, std)
        for k in range(len(ref.shapes)):
            ref.time_shape(k)
        v = 1.0 / ref.full_step_seconds()
        cpu = {"value": v, "unit": "steps/s", "cores": cpu_threads(), "kind": "port", "sample": ref.describe()}

    F = sum(falg(tuple(x for x in s if x != 1), args.max_size, max_skew) for s in shapes)
    launches = inner._plan.launches_per_step(True) * args.steps if inner is not None else 0
    if world > 1:
        t = torch.tensor([float(launches)], device=dev)
        dist.all_reduce(t)
        launches = int(t.item())
    if rank == 0:
        prec = inner.precision if inner is not None else args.precision
        line = {"metric": "psgd_kron_steps_per_sec", "value": 1000.0 / ms, "unit": "steps/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if prec == "bf16" else "bf16x3",
                "data": "synthetic",
                "config": {"workload": args.workload, "parameter_set": desc, "tensors": len(shapes),
                           "params": sum(math.prod(s) for s in shapes), "precision": prec,
                           "max_precond_size": args.max_size, "max_skew": args.max_skew,
                           "parallelism": f"precond-shard{world}+allgather" if world > 1 else "single",
                           "l2": "inputs larger than L2 (two alternating gradient sets of GBs)"},
                "f_alg_tflop_per_step": F / 1e12,
                "whole_step_tflops": F / (ms * 1e-3) / 1e12,
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "clocks": clk,
                "phases_ms": {k: round(v, 4) for k, v in sorted(phase_ms.items(), key=lambda x: -x[1])}}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
