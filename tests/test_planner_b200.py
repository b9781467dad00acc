"""AUTO's emulate-or-native choice on B200: the calibrated cost model of this library's kernels.

calib/b200.json holds the model fitted on a B200 by calib/calibrate.py; the library reads it
from beside itself.  These tests restate the model's formulas here, evaluate them per problem of
every BASELINE configuration, and require the planner seam (ggemm_stage_plan, AUTO, calibrated
model) to route each problem the same way; they also record the routes per configuration.
"""
import ctypes
import json
import os

import pytest

import workloads as W
from g2util import PKG_DIR

CALIB = os.path.join(PKG_DIR, "calib", "b200.json")
EMU, TINY, UNPROFITABLE, SMALL_K, ALPHA_ZERO = 0, 4, 5, 7, 8


def model(m, n, k, beta, N, d, sms=148):
    kp = (k + 31) // 32 * 32
    prep = (8.0 * (m * k + k * n) + (N + 1) * (m + n) * kp + 16.0 * (m + n)) / d["prep_bw"] + \
        ((m + 31) // 32 + (n + 7) // 8) * d["prep_block_s"] / sms
    gemm = 2.0 * ((m + 127) // 128 * 128) * ((n + 15) // 16 * 16) * kp * (N + 1) / d["gemm_ops"] + \
        (N + 1) * ((m + 127) // 128) * ((n + 255) // 256 if n > 128 else 1) * d["gemm_tile_s"] / sms
    recon = ((N + 4.0) * m * n + 8.0 * m * n * (2 if beta != 0 else 1) + 16.0 * (m + n)) / \
        d["recon_bw"] + ((n + 15) // 16) * ((m + 127) // 128) * d["recon_block_s"] / sms
    native = 2.0 * m * n * k / d["fp64_flops"] + d["native_problem_s"]
    return prep + gemm + recon, native


def plan(g2, wl):
    P = W.logical_problems(g2, wl)
    n = len(wl.items)
    r, nm, t = (ctypes.c_int * n)(), (ctypes.c_int * n)(), (ctypes.c_int * n)()
    cfg = g2.config(wl.num_moduli, wl.target_rel_err, 1, 0)
    assert g2.lib.ggemm_stage_plan(P, n, ctypes.byref(cfg), g2.PATH_AUTO, 148, 0.0, 0.0, 0.0,
                                   -1.0, 0.0, r, nm, t) == 0
    return [r[i] for i in range(n)], [nm[i] for i in range(n)]


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_auto_routes_follow_the_calibrated_model(g2, name):
    d = json.load(open(CALIB))
    wl = W.CONFIGS[name]()
    routes, nmods = plan(g2, wl)
    for it, r, N in zip(wl.items, routes, nmods):
        if it.alpha == 0.0:
            assert r == ALPHA_ZERO
        elif it.k <= 16:
            assert r == SMALL_K
        elif it.m * it.n * it.k < 32 ** 3:
            assert r == TINY
        else:
            t_emu, t_nat = model(it.m, it.n, it.k, it.beta, N, d)
            assert r == (EMU if t_emu <= t_nat else UNPROFITABLE), (it, t_emu, t_nat)


def test_auto_routes_per_config(g2):
    """The routes AUTO takes on each configuration on a B200 (recorded; the large dense configs
    emulate everything, the small-problem ones go to cuBLAS)."""
    counts = {}
    for name in ["c1", "c2", "c3", "c4", "c5"]:
        routes, _ = plan(g2, W.CONFIGS[name]())
        counts[name] = {r: routes.count(r) for r in set(routes)}
    assert counts["c3"] == {EMU: 8}
    assert counts["c5"] == {EMU: 512}
    assert counts["c1"] == {UNPROFITABLE: 4}  # 256^3: cuBLAS is faster on a B200
    assert counts["c4"].get(ALPHA_ZERO) == 51 and counts["c4"].get(EMU, 0) < 50
    assert 0 < counts["c2"].get(EMU, 0) < 64  # the larger problems emulate, the smaller do not
