#!/usr/bin/env python
"""bench.py -- effective FP64 TFLOP/s of the emulated grouped DGEMM on B200.

Metric: effective FP64 TFLOP/s = sum_g 2 m_g n_g k_g / t for one
ggemm_grouped_dgemm call over the whole group, next to cuBLAS native DGEMM on the same data, the
reference library (its own sources built for sm_100a, oracle/_ref) on the same device buffers,
the INT8-roofline-implied bound and the certified fraction of outputs.

Workloads are the five BASELINE configurations (tests/workloads.py); the default is C5, the
largest configuration that fits one B200 (512 problems, 16 shared 4096^2 A operands, operand
reuse, 36.5 GB of FP64 operands).  C3 and C5 spread one fixed group over the GPUs (strong
scaling, ggemm_shard_group: reuse components kept whole, no collective on the data path); C2
gives every GPU its own 64-problem group (weak scaling; rank 0's group is the N = 1 group).
Inputs exceed the 126 MB L2 in every timed workload but C1.

One JSON line on rank 0.  `value` times K calls with inputs resident in HBM; `e2e` times K
calls through the same public API with each step's A, B, C copied in from pinned host memory
and C copied back, steps pipelined over two device buffer sets.  `--impl reference` times the
reference's host FP64 path (the naive triple loop of its tests, restated in oracle/) on all
host threads, on a bounded sample of the same workload.
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

METRIC = "Effective FP64 TFLOP/s (2Σmnk/t) at 1/2/4/8 B200 vs cuBLAS DGEMM; certified %"
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libggemm_ref.so")


def make_workload(name: str, world: int, rank: int, problems: int = 0, path: str = ""):
    """(whole workload, this rank's workload) -- they differ only for weak scaling (C2).
    problems > 0 keeps the first `problems` problems (small cases for profiling); a non-empty
    `path` (a ggemm_path_t name) replaces the configuration's own path."""
    import dataclasses

    import workloads as W

    if name == "c2":
        mine = W.c2(64, W.C2_SEED + rank)
    else:
        mine = W.CONFIGS[name]()
    if problems > 0:
        mine = W.Workload(mine.name, mine.items[:problems], mine.phi, mine.num_moduli,
                          mine.path_name, mine.min_k, mine.nonfinite_frac, mine.seed,
                          mine.scaling, mine.describe + f" (first {problems} problems)",
                          mine.allow_fallback, mine.target_rel_err)
    if path:
        mine = dataclasses.replace(mine, path_name=path,
                                   describe=mine.describe + f" (path {path})")
    return mine, mine


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


def int8_peak_tops(torch, sustained_s: float = 2.0):
    """cuBLASLt INT8 GEMM (torch._int_mm, 8192^3, int32 accumulate): the library reference for
    the INT8 tensor-core roofline, measured in this run.  Returns (burst, sustained) TOP/s: the
    best of 5 single calls, and back-to-back calls for about `sustained_s` seconds (the rate
    under the power cap, comparable with a GEMM stage timed inside a long step)."""
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
    reps = max(3, int(sustained_s / best))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        torch._int_mm(a, b)
    e.record()
    e.synchronize()
    sustained = s.elapsed_time(e) / 1e3 / reps
    del a, b
    ops = 2.0 * 8192 ** 3
    return ops / best / 1e12, ops / sustained / 1e12


def traffic_from_profiles(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` on `workload` from profiles/dram_traffic.txt
    (lines: <kernel> <workload> <bytes_per_launch> <how>), or None."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if line.startswith("#") or len(parts) < 3:
                    continue
                if parts[0] == kernel and parts[1] == workload:
                    return float(parts[2])
    except OSError:
        pass
    return None


def moduli_of(g2, grp, cfg, path):
    """Moduli count the planner gives each problem (0 for native routes)."""
    num = grp.num
    route = (ctypes.c_int * max(1, num))()
    nmod = (ctypes.c_int * max(1, num))()
    tile = (ctypes.c_int * max(1, num))()
    rc = g2.lib.ggemm_stage_plan(grp.problems, num, ctypes.byref(cfg), path, 148, 0.0, 0.0, 0.0,
                                 -1.0, 0.0, route, nmod, tile)  # the library's own model
    if rc != 0:
        raise RuntimeError(f"ggemm_stage_plan rc={rc}")
    return [nmod[i] if route[i] == 0 else 0 for i in range(num)]


def digit_layout(m: int, n: int, N: int) -> bool:
    """The library's per-problem product layout choice (digit layout unless it is larger)."""
    plane = ((n + 31) // 32 * m * 32 + 255) // 256 * 256
    return (N + 4) * plane <= 4 * (N + 1) * ((m * n + 63) // 64 * 64)


def align(x, a=256):
    return (x + a - 1) // a * a


def img_bytes(g2, rows, k, N):
    return (N + 1) * align(g2.img_plane_bytes(rows, k))


def pool_need(g2, grp, nmods, reuse: bool):
    """Bytes of residue images and products one chunk of the whole group needs."""
    a_seen, b_seen = set(), set()
    need = 0
    for p, N in zip(grp.pieces, nmods):
        if N <= 0:
            continue
        it = grp.wl.items[p.src]
        akey = it.a if reuse else ("p", p.src, p.col0)
        bkey = it.b if reuse else ("p", p.src, p.col0)
        if akey not in a_seen:
            a_seen.add(akey)
            need += img_bytes(g2, it.m, it.k, N)
        if bkey not in b_seen:
            b_seen.add(bkey)
            need += img_bytes(g2, p.n, it.k, N)
        if digit_layout(it.m, p.n, N):
            need += align(N * g2.digit_plane_bytes(it.m, p.n) + 4 * g2.digit_plane_bytes(it.m, p.n))
        else:
            need += align(4 * (N + 1) * ((it.m * p.n + 63) // 64 * 64))
    return need + (64 << 20)


def algorithmic(grp, nmods, reuse: bool):
    """Algorithmic bytes of prep and reconstruct and INT8 ops of the GEMM, per call."""
    prep = recon = ops = 0.0
    a_seen, b_seen = set(), set()
    for p, N in zip(grp.pieces, nmods):
        if N <= 0:
            continue
        it = grp.wl.items[p.src]
        m, n, k = it.m, p.n, it.k
        kp = (k + 31) // 32 * 32
        akey = it.a if reuse else ("p", p.src, p.col0)
        bkey = it.b if reuse else ("p", p.src, p.col0)
        if akey not in a_seen:
            a_seen.add(akey)
            prep += 8.0 * m * k + (N + 1) * m * kp + 16.0 * m
        if bkey not in b_seen:
            b_seen.add(bkey)
            prep += 8.0 * k * n + (N + 1) * n * kp + 16.0 * n
        per_entry = (N + 4.0) if digit_layout(m, n, N) else 4.0 * (N + 1)
        recon += per_entry * m * n + (8.0 * m * n if it.beta != 0 else 0) + 8.0 * m * n \
            + 16.0 * (m + n)
        ops += 2.0 * m * n * kp * (N + 1)
    return prep, ops, recon


class RefLib:
    """The reference library (its own sources built for sm_100a into oracle/_ref) through its
    public API: ggemm_create_ex / ggemm_grouped_dgemm / ggemm_destroy."""

    def __init__(self):
        L = ctypes.CDLL(REF_SO)
        L.ggemm_create_ex.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                      ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t,
                                      ctypes.c_void_p, ctypes.c_int]
        L.ggemm_create_ex.restype = ctypes.c_int
        L.ggemm_grouped_dgemm.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        L.ggemm_grouped_dgemm.restype = ctypes.c_int
        L.ggemm_destroy.argtypes = [ctypes.c_void_p]
        self.L = L


def ref_calls(wl, grp):
    """Sub-groups for the reference library, each small enough for its handle: the reference
    sizes A/B residues as 21 planes x 2 x the summed element budgets and C32 as 21 x 4 bytes per
    C entry (src/ggemm.cu:228-341), so a group is cut at reuse-component boundaries (C5) or
    whenever that estimate passes 48 GB."""
    cap = 48e9
    out, cur, ca, cb, cc = [], [], 0, 0, 0
    last_a = None
    for i, p in enumerate(grp.pieces):
        it = wl.items[p.src]
        a, b, c = it.m * it.k, it.k * p.n, it.m * p.n
        est = 42.0 * (ca + a) + 42.0 * (cb + b) + 84.0 * (cc + c)
        boundary = cur and ((wl.path_name == "emu_grouped_reuse" and it.a != last_a) or est > cap)
        if boundary:
            out.append(cur)
            cur, ca, cb, cc = [], 0, 0, 0
        cur.append(i)
        ca, cb, cc = ca + a, cb + b, cc + c
        last_a = it.a
    if cur:
        out.append(cur)
    return out


def time_reference_library(g2, wl, grp, cfg, path, stream, steps, torch):
    """Effective TFLOP/s of the reference library on the same device buffers (its own handle,
    same path and configuration), CUDA events on the same stream.  Sub-groups (ref_calls) run
    one after another, each with its own handle created and warmed up outside the timed region;
    a step's time is the sum of its sub-group calls."""
    if not os.path.exists(REF_SO):
        return {"value": None, "unavailable": "oracle/_ref/libggemm_ref.so not built"}
    ref = RefLib()
    subs = ref_calls(wl, grp)
    entries = grp.entries_on(grp.A, grp.B, grp.C)
    reps = max(1, min(steps, 3))
    per_step = 0.0
    for sub in subs:
        probs = g2.make_problems([entries[i] for i in sub])
        ta = sum(entries[i]["m"] * entries[i]["k"] for i in sub) + 1
        tb = sum(entries[i]["k"] * entries[i]["n"] for i in sub) + 1
        tc = sum(entries[i]["m"] * entries[i]["n"] for i in sub) + 1
        h = ctypes.c_void_p()
        rc = ref.L.ggemm_create_ex(ctypes.byref(h), len(sub), ta, tb, tc,
                                   ctypes.c_void_p(stream), wl.min_k)
        if rc != 0:
            return {"value": None, "unavailable": f"reference ggemm_create_ex rc={rc}"}
        try:
            for r in range(reps + 1):  # one warm-up call, then reps timed calls
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                rc = ref.L.ggemm_grouped_dgemm(h, path, ctypes.addressof(cfg),
                                               ctypes.addressof(probs), len(sub), None)
                s1.record()
                s1.synchronize()
                if rc != 0:
                    return {"value": None, "unavailable": f"reference ggemm_grouped_dgemm rc={rc}"}
                if r > 0:
                    per_step += s0.elapsed_time(s1) / 1e3 / reps
        finally:
            torch.cuda.synchronize()
            ref.L.ggemm_destroy(h)
    return {"value": grp.flops / per_step / 1e12, "unit": "TFLOP/s", "calls_per_step": len(subs),
            "ms_per_step": per_step * 1e3,
            "how": "oracle/_ref/libggemm_ref.so (reference sources built for sm_100a), same device "
                   "buffers, path and config, mean of " + str(reps) + " timed steps; " + (
                       f"{len(subs)} calls per step (its handle cannot hold the whole group)"
                       if len(subs) > 1 else "one call per step")}


def cpu_reference(oracle, shapes, target_s=12.0, threads=0, a_limit=2**26):
    """Naive FP64 triple loop (the reference's host FP64 path) on host threads over a sample of
    the group: the first `cols` columns of the first `probs` problems, grown from one problem
    until a run takes at least 0.5 s, then scaled to about target_s.  shapes: (m, n, k, alpha,
    beta, a_id) per problem; problems sharing an a_id share their A matrix (at most a_limit
    elements of A are generated).  Returns (TFLOP/s, threads, sample description)."""
    rng = np.random.default_rng(7)
    nthreads = threads if threads > 0 else oracle.L.ozo_max_threads()
    a_mats, a_elems, data = {}, 0, []
    for m, n, k, alpha, beta, aid in shapes:
        if aid not in a_mats:
            if data and a_elems + m * k > a_limit:
                break
            a_mats[aid] = rng.random(m * k) - 0.5
            a_elems += m * k
        data.append((m, n, k, alpha, beta, a_mats[aid]))

    def run(probs, cols):
        flops = 0.0
        work = []
        for m, n, k, alpha, beta, A in data[:probs]:
            c = min(n, cols)
            work.append((m, c, k, alpha, beta, A, rng.random(k * c) - 0.5, rng.random(m * c) - 0.5))
        t0 = time.perf_counter()
        for m, c, k, alpha, beta, A, B, C in work:
            oracle.dgemm_naive(m, c, k, alpha, A, m, B, k, beta, C, m, 0, c, nthreads)
            flops += 2.0 * m * c * k
        return flops, time.perf_counter() - t0

    nmax = max(d[1] for d in data)
    probs, cols = 1, min(nthreads, nmax)
    flops, dt = run(probs, cols)
    while dt < 0.5 and (cols < nmax or probs < len(data)):
        if cols < nmax:
            cols = min(nmax, cols * 4)
        else:
            probs = min(len(data), probs * 4)
        flops, dt = run(probs, cols)
    if dt < 0.5 * target_s:  # scale the sample up towards target_s (a long first run is kept)
        f = target_s / max(dt, 1e-6)
        if cols < nmax:
            cols = int(min(nmax, cols * f))
        else:
            probs = int(min(len(data), probs * f))
        flops, dt = run(probs, cols)
    sample = (f"first {min(cols, nmax)} columns of the first {probs} of the {len(shapes)} problems "
              f"({flops / 2e9:.1f} GFMA, {dt:.1f} s)")
    return flops / dt / 1e12, nthreads, sample


def config_of(wl, world):
    return {"workload": wl.describe, "path": wl.path_name,
            "parallelism": (f"group sharded over {world} GPU(s) by ggemm_shard_group, no collective"
                            if wl.scaling == "strong" else
                            f"one group per GPU on {world} GPU(s), no collective")}


# --------------------------------------------------------------------------------- arms
def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    import g2util

    wl, _ = make_workload(args.workload, world, 0, args.problems, args.path)
    oracle = g2util.Oracle()
    shapes = [(it.m, it.n, it.k, it.alpha, it.beta, it.a) for it in wl.items]
    if wl.scaling == "weak":  # the whole job: every rank's group
        for r in range(1, world):
            w2, _ = make_workload(args.workload, world, r, args.problems, args.path)
            shapes += [(it.m, it.n, it.k, it.alpha, it.beta, (r, it.a)) for it in w2.items]
    target = max(1.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_reference(oracle, shapes, target_s=min(target, 3.0))
    vals = []
    t0 = time.perf_counter()
    last = None
    for _ in range(args.steps):
        last = cpu_reference(oracle, shapes, target_s=target)
        vals.append(last[0])
    wall = time.perf_counter() - t0
    v = float(np.median(vals))
    flops = sum(2.0 * s[0] * s[1] * s[2] for s in shapes)
    line = {
        "impl": "reference", "metric": METRIC, "value": v,
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": flops / (v * 1e12) * 1e3, "higher_is_better": True,
        "scaling": wl.scaling, "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": dict(config_of(wl, world), path="host FP64 triple loop (reference tests)"),
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
    import workloads as W

    g2 = g2util.load_pkg()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    args.gpus = world
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def reduce(x: float, op) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op)
        return float(t.item())

    def max_over_ranks(x):
        return reduce(x, dist.ReduceOp.MAX if world > 1 else None)

    def total_over_ranks(x):
        return reduce(x, dist.ReduceOp.SUM if world > 1 else None)

    phase_t0 = time.perf_counter()
    phases = {}

    def phase(name):
        nonlocal phase_t0
        now = time.perf_counter()
        phases[name] = round(now - phase_t0, 2)
        phase_t0 = now

    wl_all, wl = make_workload(args.workload, world, rank, args.problems, args.path)
    pieces = (W.shard_pieces(g2, wl, world, rank) if wl.scaling == "strong"
              else W.shard_pieces(g2, wl, 1, 0))
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    grp = W.DeviceGroup(g2, wl, pieces, dev)
    torch.cuda.synchronize()
    sptr = stream.cuda_stream
    path = W.path_id(g2, wl.path_name)
    cfg = g2.config(num_moduli=wl.num_moduli, target_rel_err=wl.target_rel_err,
                    allow_fallback=wl.allow_fallback)
    reuse = path == g2.PATH_EMU_GROUPED_REUSE
    nmods = moduli_of(g2, grp, cfg, path) if grp.num else []
    # a pool that holds the whole call in one chunk (stage events need a single chunk), at most
    # 55 % of the device
    total_mem = torch.cuda.get_device_properties(local).total_memory
    need = pool_need(g2, grp, nmods, reuse)
    os.environ["GGEMM_WORKSPACE_FRACTION"] = str(min(0.55, need / total_mem + 0.002))
    handle = g2.Handle(max(1, grp.num), grp.budget[0] + 1, grp.budget[1] + 1, grp.budget[2] + 1,
                       stream=sptr, min_k=wl.min_k)

    phase("setup")

    def call(p=path, probs=None):
        if grp.num == 0:
            return g2.Stats()
        rc, st = handle.grouped_dgemm(p, cfg, grp.problems if probs is None else probs, grp.num)
        if rc != 0:
            raise RuntimeError(f"ggemm_grouped_dgemm rc={rc}")
        return st

    # ---------------------------------------------------------------- device-resident timing
    for _ in range(args.warmup):
        st = call()
    barrier()
    # kernel_launches counts the pipeline's kernels (and cuBLAS calls); every call also launches
    # one kernel that uploads its descriptor blob
    launches_per_call = st.kernel_launches + 1
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
    host_s = []
    t_start.record(stream)
    for s in range(args.steps):
        handle.set_stage_events(ev[s])
        h0 = time.perf_counter()
        call()
        host_s.append(time.perf_counter() - h0)  # the call returns once its work is enqueued
    t_stop.record(stream)
    barrier()
    clk = clocks.stop()
    handle.set_stage_events(None)
    elapsed = t_start.elapsed_time(t_stop) / 1e3
    # per-stage times (recorded by the library when the call runs as one chunk)
    stage_ms = np.array([[es[0].elapsed_time(es[1]), es[1].elapsed_time(es[2]),
                          es[2].elapsed_time(es[3])] for es in ev]).mean(axis=0)
    if not all(x > 0 for x in stage_ms):
        stage_ms = np.array([float("nan")] * 3)
    status = handle.device_status()
    if status != 0:
        raise RuntimeError(f"device status {status}")
    t_max = max_over_ranks(elapsed)
    flops_all = total_over_ranks(grp.flops)
    value = flops_all * args.steps / t_max / 1e12
    prep_b, gemm_ops, recon_b = algorithmic(grp, nmods, reuse)
    phase("device_timing")
    if args.quick:
        line = {"quick": True, "workload": args.workload, "value": value, "unit": "TFLOP/s",
                "ms_per_step": t_max / args.steps * 1e3, "n_gpus": world,
                "stage_ms": [float(x) for x in stage_ms], "problems_per_gpu": grp.num,
                "moduli": nmod, "launches_per_call": launches_per_call,
                "host_us_per_call": float(np.min(host_s)) * 1e6 if host_s else None,
                "gemm_int8_tops": gemm_ops / (stage_ms[1] / 1e3) / 1e12 if stage_ms[1] > 0 else None,
                "prep_gbs": prep_b / (stage_ms[0] / 1e3) / 1e9 if stage_ms[0] > 0 else None,
                "recon_gbs": recon_b / (stage_ms[2] / 1e3) / 1e9 if stage_ms[2] > 0 else None,
                "clocks": clk}
        if rank == 0:
            print(json.dumps(line), flush=True)
        handle.close()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0

    # ------------------------------------------------------------------- end-to-end timing
    # Every step copies its inputs A, B (each unique operand once) and C from pinned host memory,
    # runs the public call and copies C back.  Steps are pipelined over two device buffer sets
    # and three streams, as a serving loop would run them: step i + 1's host->device copy
    # overlaps step i's compute and device->host copy.
    c_in = any(it.beta != 0.0 for it in wl.items)
    hA = torch.empty(grp.A.shape, dtype=torch.float64, pin_memory=True)
    hB = torch.empty(grp.B.shape, dtype=torch.float64, pin_memory=True)
    hC0 = torch.empty(grp.C.shape, dtype=torch.float64, pin_memory=True)
    hC = torch.empty(grp.C.shape, dtype=torch.float64, pin_memory=True)
    hA.copy_(grp.A)
    hB.copy_(grp.B)
    hC0.copy_(grp.C)
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
            if c_in:
                C.copy_(hC0, non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        call(probs=probs)
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
    h2d = total_over_ranks((grp.na + grp.nb + (grp.nc if c_in else 0)) * 8.0)
    d2h = total_over_ranks(grp.nc * 8.0)
    del hA, hB, hC0, hC, bufs, A2, B2, C2
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    phase("e2e")

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
    phase("cublas")

    # ------------------------------------------------------------ certified fraction (untimed)
    os.environ["GGEMM_STATS_REPAIR"] = "1"
    handle.close()
    h2 = g2.Handle(max(1, grp.num), grp.budget[0] + 1, grp.budget[1] + 1, grp.budget[2] + 1,
                   stream=sptr, min_k=wl.min_k)
    os.environ.pop("GGEMM_STATS_REPAIR", None)
    st2 = g2.Stats()
    if grp.num:
        rc, st2 = h2.grouped_dgemm(path, cfg, grp.problems, grp.num)
        if rc != 0:
            raise RuntimeError(f"stats call rc={rc}")
    torch.cuda.synchronize()
    h2.close()
    entries = total_over_ranks(float(sum(it[0] * it[1] for it in grp.shapes())))
    flagged = total_over_ranks(float(max(0, st2.num_uncertified) + max(0, st2.num_repaired)
                                     + max(0, st2.num_safety_fallback)))
    certified = 100.0 * (1.0 - flagged / max(entries, 1.0))
    torch.cuda.empty_cache()
    phase("certified")

    # ------------------------------------- the reference library built for sm_100a, same data
    refv = None
    if not args.no_ref_lib:
        try:
            refv = time_reference_library(g2, wl, grp, cfg, path, sptr, args.steps, torch)
        except Exception as e:  # reported, never fatal
            refv = {"value": None, "unavailable": f"{type(e).__name__}: {e}"}
        v = refv.get("value")
        per = max_over_ranks(grp.flops / (v * 1e12) if v else 0.0)
        refv["value"] = (flops_all / per / 1e12) if v and per > 0 else None
    torch.cuda.empty_cache()
    phase("reference_library")

    # ------------------------------------------------------------------------ roofline
    hbm, bf16, peak_kind = measured_peaks()
    try:
        int8_burst, int8 = int8_peak_tops(torch)
    except RuntimeError:
        int8_burst = int8 = None
    phase("int8_reference")
    stages = {
        "prep_kernel": {"ms": float(stage_ms[0]), "bound": "hbm", "unit": "GB/s",
                        "achieved": prep_b / (stage_ms[0] / 1e3) / 1e9, "peak": hbm,
                        "algorithmic_bytes": prep_b},
        "gemm_kernel": {"ms": float(stage_ms[1]), "bound": "tensor", "unit": "TFLOP/s",
                        "ops": "int8 (TOP/s)",
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
    roofline = {"kernel": dom, "bound": d["bound"], "achieved": d["achieved"], "peak": d["peak"],
                "unit": d["unit"], "frac": d["frac"],
                "traffic": traffic_from_profiles(dom, args.workload),
                "peak_source": (f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if d["bound"] == "hbm"
                                else "cuBLASLt INT8 8192^3 (torch._int_mm) back to back for ~2 s "
                                     "in this run (sustained, under the power cap); burst "
                                     f"{int8_burst:.0f}" if int8_burst else "unavailable")}
    # INT8-roofline-implied bound on the metric: INT8 peak x sum 2mnk / sum 2mn Kp (N+1)
    fl = sum(2.0 * s[0] * s[1] * s[2] for s, N in zip(grp.shapes(), nmods) if N > 0)
    bound = {"int8_implied_tflops": (int8 * fl / gemm_ops) * (flops_all / max(grp.flops, 1))
             if int8 and gemm_ops else None,
             "how": "in-run sustained cuBLASLt INT8 x sum 2mnk / sum 2mn Kp (N+1) (abs plane "
                    "counted)"}
    if bound["int8_implied_tflops"]:
        bound["frac"] = value / bound["int8_implied_tflops"]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        oracle = g2util.Oracle()
        shp = [(it.m, it.n, it.k, it.alpha, it.beta, it.a) for it in wl.items]
        v, cores, sample = cpu_reference(oracle, shp, target_s=args.cpu_seconds)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}
    phase("cpu_baseline")

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max / args.steps * 1e3,
            "higher_is_better": True, "scaling": wl.scaling, "vs_baseline": None,
            "dtype": "f64", "data": "synthetic",
            "config": dict(config_of(wl_all, world), moduli=nmod, problems_rank0=grp.num,
                           l2=("inputs of every step exceed the 126 MB L2"
                               if (grp.na + grp.nb) * 8 > 126e6 else "inputs fit L2")),
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "schedule": "2 buffer sets; copy in / call / copy out on 3 streams",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": roofline,
            "stages": stages,
            "cublas_dgemm": {"value": native_value, "unit": "TFLOP/s",
                             "path": "NATIVE_GROUPED (cublasDgemmGroupedBatched)"},
            "speedup_vs_cublas": value / native_value,
            "ref_ggemm_sm100a": refv,
            "speedup_vs_ref_ggemm": (value / refv["value"]) if refv and refv.get("value") else None,
            "int8_bound": bound,
            "certified_pct": certified,
            "cpu_baseline": cpu,
            "clocks": clk,
            "gpu_launches": launches_per_call * args.steps,
            "phase_s": phases,
            # least over steps: a later call also waits for the descriptor slot of the call two
            # before it to be consumed by the GPU
            "host_us_per_call": float(np.min(host_s)) * 1e6 if host_s else None,
            "peaks": {"hbm_gbs": hbm, "bf16_tflops": bf16, "source": peak_kind,
                      "int8_tops_cublaslt_sustained": int8,
                      "int8_tops_cublaslt_burst": int8_burst},
        }
        print(json.dumps(line), flush=True)
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
    ap.add_argument("--workload", choices=["c1", "c2", "c3", "c4", "c5"], default="c5",
                    help="BASELINE configuration (tests/workloads.py); c5 is the headline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-lib", action="store_true",
                    help="skip timing the reference library built for sm_100a")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--problems", type=int, default=0,
                    help="keep only the first N problems of the workload (profiling cases)")
    ap.add_argument("--path", default="",
                    choices=["", "native_loop", "native_grouped", "emu_loop", "emu_loop_batched",
                             "emu_grouped", "auto", "emu_grouped_reuse"],
                    help="run the workload on this path instead of its configured one")
    ap.add_argument("--quick", action="store_true",
                    help="device-resident timing only (profiling runs): no e2e, cuBLAS, "
                         "certified, reference or CPU legs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
