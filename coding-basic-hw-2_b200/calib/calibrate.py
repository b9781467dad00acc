#!/usr/bin/env python
"""calibrate.py -- fits this library's B200 cost model (the AUTO path's emulate-or-native choice)
from timings on the GPU it runs on, and writes it as JSON.

  python coding-basic-hw-2_b200/calib/calibrate.py [--out coding-basic-hw-2_b200/calib/b200.json]

The reference fits its planner from microbenchmarks (bench/calib/calib.cu, fit.py) and reads the
fit from params_<gpu>.json (src/planner.cpp:57-92); this is the same idea for this library's
kernels.  A sweep of uniform groups (problem sizes from 32 to 4096, square and K-heavy / K-light
shapes) runs through ggemm_grouped_dgemm on path EMU_GROUPED, with per-stage CUDA events
(ggemm_set_stage_events), and through NATIVE_GROUPED (cuBLAS).  Non-negative least squares then
fits, per stage, a time per algorithmic unit and a time per work item:

  prep   t = bytes / prep_bw    + blocks x prep_block_s / SMs      (blocks: 32 A rows / 8 B columns)
  gemm   t = ops / gemm_ops     + tiles x gemm_tile_s / SMs        (ops over 128-row padded tiles)
  recon  t = bytes / recon_bw   + blocks x recon_block_s / SMs     (blocks: 128 rows x 16 columns)
  native t = 2 m n k / fp64_flops + problem_s                      (per problem of a grouped call)

with the byte and op counts of the kernels' own data flow (residue images of N + 1 planes, the
digit product layout, C read when beta != 0).  planner.cpp evaluates the same formulas.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)


def load_pkg():
    spec = importlib.util.spec_from_file_location("ggemm_b200", os.path.join(PKG, "__init__.py"),
                                                  submodule_search_locations=[PKG])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ggemm_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def units(m, n, k, N, beta):
    """Algorithmic units of one emulated problem (the formulas planner.cpp evaluates)."""
    kp = (k + 31) // 32 * 32
    prep_bytes = 8.0 * (m * k + k * n) + (N + 1) * (m + n) * kp + 16.0 * (m + n)
    prep_blocks = (m + 31) // 32 + (n + 7) // 8
    mp = (m + 127) // 128 * 128
    ne = (n + 15) // 16 * 16
    ops = 2.0 * mp * ne * kp * (N + 1)
    tiles = (N + 1) * ((m + 127) // 128) * ((n + 255) // 256 if n > 128 else 1)
    recon_bytes = (N + 4.0) * m * n + 8.0 * m * n * (2 if beta != 0 else 1) + 16.0 * (m + n)
    recon_blocks = ((n + 15) // 16) * ((m + 127) // 128)
    return prep_bytes, prep_blocks, ops, tiles, recon_bytes, recon_blocks


def nnls(A, b):
    """Non-negative least squares on relative error (rows scaled by 1 / b)."""
    from scipy.optimize import nnls as _nnls

    w = 1.0 / np.maximum(b, 1e-9)
    x, _ = _nnls(A * w[:, None], b * w)
    return x


def shapes():
    out = []
    for s in (32, 48, 64, 96, 128, 192, 256, 384, 512, 768, 1024, 1536, 2048, 3072, 4096):
        out.append((s, s, s))
        if s <= 1024:
            out.append((s, s, 4 * s))
        if s >= 128:
            out.append((s, s, max(32, s // 8)))
        if 64 <= s <= 2048:
            out.append((2 * s, s // 2, s))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "b200.json"))
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    import torch

    g2 = load_pkg()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    props = torch.cuda.get_device_properties(0)
    sms = props.multi_processor_count
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    rows = []
    for (m, n, k) in shapes():
        per = 2.0 * m * n * k
        G = int(max(1, min(512, 4e10 / per)))
        while G > 1 and G * 8 * (m * k + k * n + 2 * m * n) > 6e9:
            G //= 2
        gen = torch.Generator(device=dev)
        gen.manual_seed(m * 7 + n * 13 + k)
        A = (torch.rand(G * m * k, generator=gen, device=dev, dtype=torch.float64) - 0.5)
        B = (torch.rand(G * k * n, generator=gen, device=dev, dtype=torch.float64) - 0.5)
        C = torch.zeros(G * m * n, device=dev, dtype=torch.float64)
        probs = g2.make_problems([dict(m=m, n=n, k=k, A=A.data_ptr() + 8 * g * m * k, lda=m,
                                       B=B.data_ptr() + 8 * g * k * n, ldb=k,
                                       C=C.data_ptr() + 8 * g * m * n, ldc=m, alpha=1.0,
                                       beta=0.0) for g in range(G)])
        cfg = g2.config(0, 1e-15, 1, 0)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        for e in ev:
            e.record(stream)
        with g2.Handle(G, G * m * k, G * k * n, G * m * n, stream=stream.cuda_stream) as h:
            h.set_stage_events(ev)
            st_ms = []
            for r in range(args.reps + 1):
                rc, st = h.grouped_dgemm(g2.PATH_EMU_GROUPED, cfg, probs, G)
                assert rc == 0
                torch.cuda.synchronize()
                if r:
                    st_ms.append([ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]),
                                  ev[2].elapsed_time(ev[3])])
            h.set_stage_events(None)
            N = st.moduli_max
            nat = []
            for r in range(args.reps + 1):
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record(stream)
                rc, _ = h.grouped_dgemm(g2.PATH_NATIVE_GROUPED, cfg, probs, G)
                s1.record(stream)
                s1.synchronize()
                assert rc == 0
                if r:
                    nat.append(s0.elapsed_time(s1))
        t = np.median(np.array(st_ms), axis=0) / 1e3
        u = units(m, n, k, N, 0.0)
        rows.append(dict(m=m, n=n, k=k, G=G, N=N, prep_s=t[0], gemm_s=t[1], recon_s=t[2],
                         native_s=float(np.median(nat)) / 1e3, units=[G * x for x in u]))
        print(json.dumps(rows[-1]), flush=True)
        del A, B, C
    # fits (per stage: a per-unit and a per-item term, plus a per-launch constant)
    U = np.array([r["units"] for r in rows])
    one = np.ones(len(rows))
    pre = nnls(np.stack([U[:, 0], U[:, 1] / sms, one], 1), np.array([r["prep_s"] for r in rows]))
    gem = nnls(np.stack([U[:, 2], U[:, 3] / sms, one], 1), np.array([r["gemm_s"] for r in rows]))
    rec = nnls(np.stack([U[:, 4], U[:, 5] / sms, one], 1), np.array([r["recon_s"] for r in rows]))
    nat_flops = np.array([r["G"] * 2.0 * r["m"] * r["n"] * r["k"] for r in rows])
    nat = nnls(np.stack([nat_flops, np.array([r["G"] for r in rows], float), one], 1),
               np.array([r["native_s"] for r in rows]))
    fit = {
        "gpu": props.name, "sms": sms,
        "when": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
        "how": "coding-basic-hw-2_b200/calib/calibrate.py: stage CUDA events over a sweep of "
               f"{len(rows)} uniform groups, non-negative least squares on relative error",
        "prep_bw": 1.0 / max(pre[0], 1e-30), "prep_block_s": pre[1],
        "gemm_ops": 1.0 / max(gem[0], 1e-30), "gemm_tile_s": gem[1],
        "recon_bw": 1.0 / max(rec[0], 1e-30), "recon_block_s": rec[1],
        "fp64_flops": 1.0 / max(nat[0], 1e-30), "native_problem_s": nat[1],
        "launch_s": {"prep": pre[2], "gemm": gem[2], "recon": rec[2], "native": nat[2]},
        "samples": rows,
    }
    with open(args.out, "w") as f:
        json.dump(fit, f, indent=1)
    print(json.dumps({k: v for k, v in fit.items() if k != "samples"}))


if __name__ == "__main__":
    main()
