"""Host-side cost of a call at a large group size (C4: 1024 problems, AUTO).

The reference's host planning took longer than its GPU work at G = 1024 (618.9 us of host plan
against a 603.5 us GPU span, docs/report.md:622).  Here the direct call (plan, reuse, chunking,
descriptor blob, H2D copy and launches, then return) and the graph path (ggemm_execute_plan of a
plan made once) are timed on the host, and the direct call is compared with its own GPU span.
The figures are printed; the bounds are loose (a shared machine).
"""
import ctypes
import time

import numpy as np
import pytest

import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_host_cost_at_g1024(g2, cuda):
    wl = W.c4()
    grp = W.DeviceGroup(g2, wl, W.shard_pieces(g2, wl, 1, 0), torch.device("cuda", 0))
    cfg = g2.config(0, 1e-15, 1, 0)
    s = torch.cuda.current_stream()
    with g2.Handle(grp.num, grp.budget[0] + 1, grp.budget[1] + 1, grp.budget[2] + 1,
                   stream=s.cuda_stream, min_k=wl.min_k) as h:
        host, gpu = [], []
        for i in range(8):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            t0 = time.perf_counter()
            rc, _ = h.grouped_dgemm(g2.PATH_AUTO, cfg, grp.problems, grp.num)
            t1 = time.perf_counter()
            e1.record(s)
            e1.synchronize()
            assert rc == 0
            if i >= 3:
                host.append((t1 - t0) * 1e6)
                gpu.append(e0.elapsed_time(e1) * 1e3)
        err = ctypes.c_int(0)
        plan = g2.lib.ggemm_make_plan_ex(h.ptr, g2.PATH_AUTO, ctypes.byref(cfg), grp.problems,
                                         grp.num, ctypes.byref(err))
        assert plan and err.value == 0
        try:
            ex = []
            for i in range(8):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                assert g2.lib.ggemm_execute_plan(plan, ctypes.c_void_p(s.cuda_stream)) == 0
                t1 = time.perf_counter()
                torch.cuda.synchronize()
                if i >= 3:
                    ex.append((t1 - t0) * 1e6)
        finally:
            g2.lib.ggemm_destroy_plan(plan)
    h_direct, g_direct, h_plan = (float(np.median(x)) for x in (host, gpu, ex))
    print(f"C4 (G=1024, AUTO): direct call host {h_direct:.1f} us, GPU span {g_direct:.1f} us; "
          f"ggemm_execute_plan host {h_plan:.1f} us")
    assert h_direct < 5000.0
    assert h_plan < h_direct
