#!/usr/bin/env python
"""bench.py -- effective FP64 TFLOP/s of the emulated grouped DGEMM on B200.

Metric: effective FP64 TFLOP/s = sum_g 2 m_g n_g k_g / t for one
ggemm_grouped_dgemm call over the whole group (EMU_GROUPED path, adaptive moduli), next to
cuBLAS native DGEMM on the same data, plus the certified fraction of outputs.

Default workload (configs[1] of BASELINE.json, "C2"): G = 64 problems, m, n, k drawn uniformly
from {128, 192, ..., 2048}; entries (U - 0.5) exp(2 N(0,1)); alpha ~ U(0.5, 2), beta = 0.5,
C ~ U[-1, 1); num_moduli = 0 with target 1e-15.  Synthetic seeded data of those shapes and
distributions (no dataset is involved).  Inputs (about 1.8 GB) exceed the 126 MB L2.

One JSON line on rank 0.  `value` times K calls with inputs resident in HBM; `e2e` times K
calls through the same public API with each step's A, B, C copied in from pinned host memory
and C copied back, steps pipelined over two device buffer sets (step i + 1's copy in overlaps
step i's compute and copy out).  Multi-GPU (torchrun): the global group has 64 problems per rank, partitioned
by ggemm_shard_group (cost-balanced, no collective on the data path); timing is the max over
ranks.  `--impl reference` times the reference's host FP64 path (the naive triple loop of its
tests, restated in oracle/) on all host threads, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tests"))

PHI = 2.0
SIZES = list(range(128, 2049, 64))
PROBS_PER_GPU = 64
SEED = 20261201


# ----------------------------------------------------------------------------- workload
def c2_shapes(num: int, seed: int = SEED):
    rng = np.random.default_rng(seed)
    m = rng.choice(SIZES, num)
    n = rng.choice(SIZES, num)
    k = rng.choice(SIZES, num)
    alpha = rng.uniform(0.5, 2.0, num)
    return [(int(m[i]), int(n[i]), int(k[i]), float(alpha[i]), 0.5) for i in range(num)]


def c3_shapes(num: int):
    """Config C3 of the survey: num problems of 8192^3, alpha = 1, beta = 0 (INT8-bound)."""
    return [(8192, 8192, 8192, 1.0, 0.0)] * num


def fill_phi(t, phi: float, seed: int):
    """(U - 0.5) * exp(phi * N(0,1)) in place (device generator, deterministic per seed)."""
    import torch

    g = torch.Generator(device=t.device)
    g.manual_seed(seed)
    u = torch.rand(t.shape, generator=g, device=t.device, dtype=torch.float64)
    if phi == 0.0:
        t.copy_(u - 0.5)
    else:
        z = torch.randn(t.shape, generator=g, device=t.device, dtype=torch.float64)
        t.copy_((u - 0.5) * torch.exp(phi * z))


class Group:
    """Device buffers of one rank's problems (tight leading dimensions)."""

    def __init__(self, g2, shapes, seeds, device, phi=PHI):
        import torch

        self.shapes = shapes
        na = sum(m * k for m, n, k, _, _ in shapes)
        nb = sum(k * n for m, n, k, _, _ in shapes)
        nc = sum(m * n for m, n, k, _, _ in shapes)
        self.na, self.nb, self.nc = na, nb, nc
        self.A = torch.empty(max(na, 1), dtype=torch.float64, device=device)
        self.B = torch.empty(max(nb, 1), dtype=torch.float64, device=device)
        self.C = torch.empty(max(nc, 1), dtype=torch.float64, device=device)
        self.C0 = torch.empty(max(nc, 1), dtype=torch.float64, device=device)
        oa = ob = oc = 0
        entries = []
        for (m, n, k, alpha, beta), sd in zip(shapes, seeds):
            fill_phi(self.A[oa:oa + m * k], phi, sd * 4 + 1)
            fill_phi(self.B[ob:ob + k * n], phi, sd * 4 + 2)
            fill_phi(self.C0[oc:oc + m * n], 0.0, sd * 4 + 3)
            self.C0[oc:oc + m * n].mul_(2.0)  # U[-1, 1)
            entries.append(dict(m=m, n=n, k=k, A=self.A.data_ptr() + 8 * oa, lda=m,
                                B=self.B.data_ptr() + 8 * ob, ldb=k,
                                C=self.C.data_ptr() + 8 * oc, ldc=m, alpha=alpha, beta=beta))
            oa += m * k
            ob += k * n
            oc += m * n
        self.C.copy_(self.C0)
        self.problems = g2.make_problems(entries)
        self.num = len(shapes)
        self.flops = sum(2.0 * m * n * k for m, n, k, _, _ in shapes)
        self.g2 = g2

    def problems_on(self, A, B, C):
        """The same problems with their operands in other device buffers of the same sizes."""
        oa = ob = oc = 0
        entries = []
        for m, n, k, alpha, beta in self.shapes:
            entries.append(dict(m=m, n=n, k=k, A=A.data_ptr() + 8 * oa, lda=m,
                                B=B.data_ptr() + 8 * ob, ldb=k, C=C.data_ptr() + 8 * oc,
                                ldc=m, alpha=alpha, beta=beta))
            oa += m * k
            ob += k * n
            oc += m * n
        return self.g2.make_problems(entries)

    def algorithmic(self, N: int):
        """Algorithmic bytes / ops of the three stages for moduli count N (per call)."""
        prep = recon = ops = 0.0
        for m, n, k, alpha, beta in self.shapes:
            kp = (k + 31) // 32 * 32
            prep += 8.0 * (m * k + k * n) + (N + 1) * (m + n) * kp + 16.0 * (m + n)
            # products read by the reconstruct: N digit bytes + the int32 abs product per entry
            # (digit layout), or N + 1 int32 products (int32 layout, narrow problems)
            per_entry = (N + 4.0) if digit_layout(m, n, N) else 4.0 * (N + 1)
            recon += per_entry * m * n + (8.0 * m * n if beta != 0 else 0) + 8.0 * m * n \
                + 16.0 * (m + n)
            ops += 2.0 * m * n * kp * (N + 1)
        return prep, ops, recon


def digit_layout(m: int, n: int, N: int) -> bool:
    """The library's per-problem product layout choice (digit layout unless it is larger)."""
    plane = ((n + 31) // 32 * m * 32 + 255) // 256 * 256
    return (N + 4) * plane <= 4 * (N + 1) * ((m * n + 63) // 64 * 64)


# ------------------------------------------------------------------------------ helpers
class ClockSampler:
    """SM clock and clock-event reasons sampled every ~10 ms during the timed region (NVML in a
    background thread; read-only queries)."""

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.samples = []
        self.reasons = set()
        self.err = None

    def start(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.dev = pynvml.nvmlDeviceGetHandleByUUID(self.uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.dev, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report why
            self.err = f"nvml unavailable: {e}"
            return
        self.stop_flag = threading.Event()
        names = {"hw_slowdown": self.nv.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": self.nv.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": self.nv.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": self.nv.nvmlClocksEventReasonSwPowerCap,
                 "hw_power_brake": self.nv.nvmlClocksEventReasonHwPowerBrakeSlowdown}

        def loop():
            while not self.stop_flag.is_set():
                try:
                    self.samples.append(
                        self.nv.nvmlDeviceGetClockInfo(self.dev, self.nv.NVML_CLOCK_SM))
                    r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.dev)
                    for nm, bit in names.items():
                        if r & bit:
                            self.reasons.add(nm)
                except Exception as e:
                    self.err = str(e)
                    return
                time.sleep(0.01)

        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()

    def stop(self):
        if self.err and not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err]}
        self.stop_flag.set()
        self.thread.join(timeout=2)
        sm = self.samples
        out = {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": float(self.max_mhz),
               "samples": len(sm), "reasons": sorted(self.reasons)}
        try:
            self.nv.nvmlShutdown()
        except Exception:
            pass
        return out


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def int8_peak_tops(torch):
    """cuBLASLt INT8 GEMM (torch._int_mm, 8192^3, int32 accumulate): the library reference for
    the INT8 tensor-core roofline, measured in this run (best of 5)."""
    a = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device="cuda")
    b = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b)
    best = 1e30
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e) / 1e3)
    del a, b
    return 2.0 * 8192 ** 3 / best / 1e12


def traffic_from_profiles(kernel: str):
    """DRAM bytes per launch of `kernel` on the bench workload from profiles/dram_traffic.txt
    (lines: <kernel> <bytes_per_launch> <how>), or None."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == kernel and not line.startswith("#"):
                    return float(parts[1])
    except OSError:
        pass
    return None


def cpu_reference(oracle, shapes, target_s=12.0, threads=0):
    """Naive FP64 triple loop on host threads over a column sample of every problem.
    Returns (TFLOP/s, threads, sample description)."""
    rng = np.random.default_rng(7)
    data = []
    for m, n, k, alpha, beta in shapes:
        A = rng.random(m * k) - 0.5
        B = rng.random(k * n) - 0.5
        C = rng.random(m * n) - 0.5
        data.append((m, n, k, alpha, beta, A, B, C))
    nthreads = threads if threads > 0 else oracle.L.ozo_max_threads()

    def run(cols):
        flops = 0.0
        t0 = time.perf_counter()
        for m, n, k, alpha, beta, A, B, C in data:
            c = min(n, cols)
            oracle.dgemm_naive(m, n, k, alpha, A, m, B, k, beta, C, m, 0, c, nthreads)
            flops += 2.0 * m * c * k
        return flops, time.perf_counter() - t0

    cols = max(1, nthreads)
    flops, dt = run(cols)
    while dt < 0.5 and cols < 4096:
        cols *= 4
        flops, dt = run(cols)
    scale = max(1.0, target_s / max(dt, 1e-6))
    cols = int(min(4096, cols * scale))
    flops, dt = run(cols)
    sample = (f"first {cols} columns of each of the {len(shapes)} problems "
              f"({flops / 2e9:.1f} GFMA, {dt:.1f} s)")
    return flops / dt / 1e12, nthreads, sample


# --------------------------------------------------------------------------------- arms
def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import g2util

    oracle = g2util.Oracle()
    shapes = c2_shapes(PROBS_PER_GPU * args.gpus)
    target = max(1.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_reference(oracle, shapes, target_s=min(target, 5.0))
    vals = []
    t0 = time.perf_counter()
    last = None
    for _ in range(args.steps):
        last = cpu_reference(oracle, shapes, target_s=target)
        vals.append(last[0])
    wall = time.perf_counter() - t0
    v = float(np.median(vals))
    flops = sum(2.0 * m * n * k for m, n, k, _, _ in shapes)
    line = {
        "impl": "reference", "metric": "effective FP64 TFLOP/s (2*sum(mnk)/t)", "value": v,
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": flops / (v * 1e12) * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "C2: G=64*N ragged m,n,k in {128..2048 step 64}, phi=2, "
                               "alpha~U(0.5,2), beta=0.5", "path": "host FP64 triple loop"},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": last[1], "kind": "port",
                         "sample": last[2]},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": wall,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist

    import g2util

    g2 = g2util.load_pkg()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    # global group, then this rank's shard
    c3 = args.workload == "c3"
    gshapes = c3_shapes(args.problems * world) if c3 else c2_shapes(args.problems * world)
    if world > 1:
        logical = g2.make_problems([dict(m=m, n=n, k=k, A=0x1000 * (i + 1), lda=m,
                                         B=0x100000000 * (i + 1), ldb=k,
                                         C=0x10000000000 * (i + 1), ldc=m, alpha=a, beta=b)
                                    for i, (m, n, k, a, b) in enumerate(gshapes)])
        subs, shard, src = g2.shard_group(logical, len(gshapes), world)
        mine = [i for i in range(len(shard)) if shard[i] == rank]
        shapes = []
        seeds = []
        for i in mine:
            p = subs[i]
            shapes.append((p.m, p.n, p.k, p.alpha, p.beta))
            seeds.append(SEED + 1000 * src[i] + (p.C - logical[src[i]].C) // 8)
    else:
        shapes = gshapes
        seeds = [SEED + 1000 * i for i in range(len(shapes))]
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    grp = Group(g2, shapes, seeds, dev, phi=0.5 if c3 else PHI)
    torch.cuda.synchronize()
    sptr = stream.cuda_stream
    handle = g2.Handle(max(1, grp.num), grp.na, grp.nb, grp.nc, stream=sptr)
    cfg = g2.config(num_moduli=16 if c3 else 0, target_rel_err=1e-15, allow_fallback=1)

    def call(path=g2.PATH_EMU_GROUPED):
        rc, st = handle.grouped_dgemm(path, cfg, grp.problems, grp.num)
        if rc != 0:
            raise RuntimeError(f"ggemm_grouped_dgemm rc={rc}")
        return st

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def total_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    # ---------------------------------------------------------------- device-resident timing
    for _ in range(args.warmup):
        st = call()
    barrier()
    launches_per_call = st.kernel_launches
    nmod = st.moduli_max
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    for es in ev:
        for e in es:
            e.record(stream)
    barrier()
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    clocks = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    clocks.start()
    time.sleep(0.05)
    t_start, t_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    t_start.record(stream)
    for s in range(args.steps):
        handle.set_stage_events(ev[s])
        call()
    t_stop.record(stream)
    barrier()
    clk = clocks.stop()
    handle.set_stage_events(None)
    elapsed = t_start.elapsed_time(t_stop) / 1e3
    stage_ms = np.array([[es[0].elapsed_time(es[1]), es[1].elapsed_time(es[2]),
                          es[2].elapsed_time(es[3])] for es in ev]).mean(axis=0)
    status = handle.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}")
    t_max = max_over_ranks(elapsed)
    flops_all = total_over_ranks(grp.flops)
    value = flops_all * args.steps / t_max / 1e12

    if args.quick:
        line = {"quick": True, "workload": args.workload, "value": value, "unit": "TFLOP/s",
                "ms_per_step": t_max / args.steps * 1e3,
                "stage_ms": [float(x) for x in stage_ms], "problems_per_gpu": grp.num,
                "moduli": nmod}
        if c3:  # cuBLAS DGEMM on the same data, and the GEMM stage's INT8 rate
            for _ in range(2):
                call(g2.PATH_NATIVE_GROUPED)
            barrier()
            n0, n1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n0.record(stream)
            for _ in range(args.steps):
                call(g2.PATH_NATIVE_GROUPED)
            n1.record(stream)
            barrier()
            line["cublas_dgemm_tflops"] = flops_all * args.steps / max_over_ranks(
                n0.elapsed_time(n1) / 1e3) / 1e12
            ops = sum(2.0 * m * n * ((k + 31) // 32 * 32) * (nmod + 1)
                      for m, n, k, _, _ in grp.shapes)
            line["gemm_int8_tops"] = ops / (stage_ms[1] / 1e3) / 1e12
        if rank == 0:
            print(json.dumps(line), flush=True)
        handle.close()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    # ------------------------------------------------------------------- end-to-end timing
    # Every step copies its inputs A, B, C from pinned host memory, runs the public call and
    # copies C back.  Steps are pipelined over two device buffer sets and three streams, as a
    # serving loop would run them: step i + 1's host->device copy overlaps step i's compute
    # and device->host copy.
    hA = torch.empty(grp.A.shape, dtype=torch.float64, pin_memory=True)
    hB = torch.empty(grp.B.shape, dtype=torch.float64, pin_memory=True)
    hC0 = torch.empty(grp.C0.shape, dtype=torch.float64, pin_memory=True)
    hC = torch.empty(grp.C.shape, dtype=torch.float64, pin_memory=True)
    hA.copy_(grp.A)
    hB.copy_(grp.B)
    hC0.copy_(grp.C0)
    bufs = [(grp.A, grp.B, grp.C, grp.problems)]
    A2, B2, C2 = torch.empty_like(grp.A), torch.empty_like(grp.B), torch.empty_like(grp.C)
    bufs.append((A2, B2, C2, grp.problems_on(A2, B2, C2)))
    s_in = torch.cuda.Stream(device=dev)
    s_out = torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    for e in ev_free:
        e.record(s_out)
    torch.cuda.synchronize()

    def e2e_step(i):
        b = i & 1
        A, B, C, probs = bufs[b]
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_free[b])  # step i - 2 is done with this buffer set
            A.copy_(hA, non_blocking=True)
            B.copy_(hB, non_blocking=True)
            C.copy_(hC0, non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        rc, _ = handle.grouped_dgemm(g2.PATH_EMU_GROUPED, cfg, probs, grp.num)
        if rc != 0:
            raise RuntimeError(f"ggemm_grouped_dgemm rc={rc}")
        ev_done[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[b])
            hC.copy_(C, non_blocking=True)
            ev_free[b].record(s_out)

    for i in range(max(1, args.warmup)):
        e2e_step(i)
    barrier()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(s_in)
    for i in range(args.steps):
        e2e_step(i)
    s_in.wait_stream(s_out)
    e_stop.record(s_in)
    barrier()
    e_elapsed = max_over_ranks(e_start.elapsed_time(e_stop) / 1e3)
    e2e_value = flops_all * args.steps / e_elapsed / 1e12
    h2d = total_over_ranks((grp.na + grp.nb + grp.nc) * 8.0)
    d2h = total_over_ranks(grp.nc * 8.0)
    del hA, hB, hC0, hC, bufs, A2, B2, C2

    # ------------------------------------------------------- cuBLAS native DGEMM, same data
    for _ in range(2):
        call(g2.PATH_NATIVE_GROUPED)
    barrier()
    n_start, n_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_start.record(stream)
    for _ in range(args.steps):
        call(g2.PATH_NATIVE_GROUPED)
    n_stop.record(stream)
    barrier()
    native_value = flops_all * args.steps / max_over_ranks(
        n_start.elapsed_time(n_stop) / 1e3) / 1e12

    # ------------------------------------------------------------ certified fraction (untimed)
    os.environ["GGEMM_STATS_REPAIR"] = "1"
    h2 = g2.Handle(max(1, grp.num), grp.na, grp.nb, grp.nc, stream=sptr)
    os.environ.pop("GGEMM_STATS_REPAIR", None)
    rc, st2 = h2.grouped_dgemm(g2.PATH_EMU_GROUPED, cfg, grp.problems, grp.num)
    torch.cuda.synchronize()
    h2.close()
    entries = total_over_ranks(float(sum(m * n for m, n, k, _, _ in grp.shapes)))
    flagged = total_over_ranks(float(max(0, st2.num_uncertified) + max(0, st2.num_repaired)
                                     + max(0, st2.num_safety_fallback)))
    certified = 100.0 * (1.0 - flagged / max(entries, 1.0))

    # ------------------------------------------------------------------------ roofline
    hbm, bf16, peak_kind = measured_peaks()
    try:
        int8 = int8_peak_tops(torch) if rank == 0 else None
    except RuntimeError:
        int8 = None
    prep_b, gemm_ops, recon_b = grp.algorithmic(nmod)
    stages = {
        "prep_kernel": {"ms": float(stage_ms[0]), "bound": "hbm", "unit": "GB/s",
                        "achieved": prep_b / (stage_ms[0] / 1e3) / 1e9, "peak": hbm,
                        "algorithmic_bytes": prep_b},
        "gemm_kernel": {"ms": float(stage_ms[1]), "bound": "tensor", "unit": "TOP/s",
                        "achieved": gemm_ops / (stage_ms[1] / 1e3) / 1e12, "peak": int8,
                        "algorithmic_ops": gemm_ops},
        "recon_kernel": {"ms": float(stage_ms[2]), "bound": "hbm", "unit": "GB/s",
                         "achieved": recon_b / (stage_ms[2] / 1e3) / 1e9, "peak": hbm,
                         "algorithmic_bytes": recon_b},
    }
    for k_, v_ in stages.items():
        v_["frac"] = (v_["achieved"] / v_["peak"]) if v_["peak"] else None
    dom = max(stages, key=lambda s: stages[s]["ms"])
    d = stages[dom]
    traffic = traffic_from_profiles(dom)
    roofline = {"kernel": dom, "bound": d["bound"], "achieved": d["achieved"], "peak": d["peak"],
                "unit": d["unit"], "frac": d["frac"], "traffic": traffic,
                "peak_source": (f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if d["bound"] == "hbm"
                                else "cuBLASLt int8 8192^3 measured in this run")}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        oracle = g2util.Oracle()
        v, cores, sample = cpu_reference(oracle, grp.shapes, target_s=args.cpu_seconds)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": "effective FP64 TFLOP/s (2*sum(mnk)/t), EMU_GROUPED vs cuBLAS DGEMM",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic",
            "config": {"workload": "C2: G=64 per GPU, m,n,k uniform in {128..2048 step 64}, "
                                   "phi=2, alpha~U(0.5,2), beta=0.5, C~U[-1,1), "
                                   "num_moduli=0 target 1e-15",
                       "path": "EMU_GROUPED (repair COUNT)", "moduli": nmod,
                       "problems_per_gpu": grp.num, "l2": "inputs 1.8 GB/GPU > 126 MB L2",
                       "parallelism": f"group sharded over {world} GPU(s), no collective"},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "schedule": "2 buffer sets; copy in / call / copy out on 3 streams",
                    "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": roofline,
            "stages": stages,
            "cublas_dgemm": {"value": native_value, "unit": "TFLOP/s",
                             "path": "NATIVE_GROUPED (cublasDgemmGroupedBatched)"},
            "speedup_vs_cublas": value / native_value,
            "certified_pct": certified,
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": launches_per_call * args.steps,
            "peaks": {"hbm_gbs": hbm, "bf16_tflops": bf16, "source": peak_kind,
                      "int8_tops_cublaslt": int8},
        }
        print(json.dumps(line), flush=True)
    handle.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--problems", type=int, default=PROBS_PER_GPU,
                    help="problems per GPU (64 = the C2 workload; fewer for profiling)")
    ap.add_argument("--workload", choices=["c2", "c3"], default="c2",
                    help="c2: the bench line's workload; c3: 8192^3 problems, N = 16, "
                         "--quick only (device timing, cuBLAS DGEMM beside it)")
    ap.add_argument("--quick", action="store_true",
                    help="device-resident timing only (profiling runs): no e2e, cuBLAS, "
                         "certified or CPU legs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload == "c3":
        if args.impl == "reference":
            ap.error("--workload c3 times this library only")
        args.quick = True
        if args.problems == PROBS_PER_GPU:
            args.problems = 8
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
