"""AUTO through the public call on B200, against the planner seam and against the pure paths.

The handle plans with the calibrated model (calib/b200.json beside the library); the number of
problems it sends to cuBLAS as fallbacks (stats.num_fallback) must equal what the planner seam
predicts with the same model.  On the ragged C2 group, where the model splits the problems
between emulation and cuBLAS, AUTO must be no slower than the better of EMU_GROUPED and
NATIVE_GROUPED (within 15 %: timing on a shared machine).
"""
import ctypes
import os

import numpy as np
import pytest

import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FALLBACK_ROUTES = (3, 4, 5, 6, 7)  # K_TOO_LARGE, TINY, UNPROFITABLE, PRECISION, SMALL_K


def seam_fallbacks(g2, wl):
    P = W.logical_problems(g2, wl)
    n = len(wl.items)
    r, nm, t = (ctypes.c_int * n)(), (ctypes.c_int * n)(), (ctypes.c_int * n)()
    cfg = g2.config(wl.num_moduli, wl.target_rel_err, 1, 0)
    assert g2.lib.ggemm_stage_plan(P, n, ctypes.byref(cfg), g2.PATH_AUTO, 148, 0.0, 0.0, 0.0,
                                   -1.0, 0.0, r, nm, t) == 0
    return sum(1 for i in range(n) if r[i] in FALLBACK_ROUTES)


def timed(h, g2, grp, path, cfg, reps=5):
    s = torch.cuda.current_stream()
    out = []
    for i in range(reps + 1):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        rc, st = h.grouped_dgemm(path, cfg, grp.problems, grp.num)
        e1.record(s)
        e1.synchronize()
        assert rc == 0
        if i:
            out.append(e0.elapsed_time(e1))
    return float(np.median(out)), st


@pytest.mark.parametrize("name", ["c2", "c4"])
def test_auto_fallbacks_equal_the_seam(g2, cuda, name):
    wl = W.CONFIGS[name]()
    grp = W.DeviceGroup(g2, wl, W.shard_pieces(g2, wl, 1, 0), torch.device("cuda", 0))
    cfg = g2.config(wl.num_moduli, wl.target_rel_err, 1, 0)
    with g2.Handle(grp.num, grp.budget[0] + 1, grp.budget[1] + 1, grp.budget[2] + 1,
                   stream=torch.cuda.current_stream().cuda_stream, min_k=wl.min_k) as h:
        rc, st = h.grouped_dgemm(g2.PATH_AUTO, cfg, grp.problems, grp.num)
        torch.cuda.synchronize()
        assert rc == 0 and h.device_status() == 0
    assert st.num_fallback == seam_fallbacks(g2, wl)


def test_auto_on_c2_no_slower_than_the_better_pure_path(g2, cuda):
    wl = W.c2()
    grp = W.DeviceGroup(g2, wl, W.shard_pieces(g2, wl, 1, 0), torch.device("cuda", 0))
    cfg = g2.config(0, 1e-15, 1, g2.REPAIR_COUNT)  # one repair mode for all three paths
    with g2.Handle(grp.num, grp.budget[0] + 1, grp.budget[1] + 1, grp.budget[2] + 1,
                   stream=torch.cuda.current_stream().cuda_stream) as h:
        t_emu, _ = timed(h, g2, grp, g2.PATH_EMU_GROUPED, cfg)
        t_nat, _ = timed(h, g2, grp, g2.PATH_NATIVE_GROUPED, cfg)
        t_auto, st = timed(h, g2, grp, g2.PATH_AUTO, cfg)
    print(f"C2: AUTO {t_auto:.3f} ms ({st.num_fallback} of 64 native), EMU_GROUPED {t_emu:.3f} ms, "
          f"NATIVE_GROUPED {t_nat:.3f} ms")
    assert t_auto <= 1.15 * min(t_emu, t_nat)
