"""bench.py's host-side helpers (no GPU): workload selection with --problems / --path, and the
per-workload DRAM traffic table it reads from profiles/ for roofline.traffic."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_make_workload_keeps_the_configured_path_by_default():
    whole, mine = bench.make_workload("c5", 1, 0)
    assert whole is mine
    assert mine.path_name == "emu_grouped_reuse" and len(mine.items) == 512


def test_make_workload_path_override_and_problem_cut():
    _, mine = bench.make_workload("c4", 1, 0, problems=10, path="emu_grouped")
    assert mine.path_name == "emu_grouped"
    assert len(mine.items) == 10
    assert "(path emu_grouped)" in mine.describe and "(first 10 problems)" in mine.describe
    # the override changes nothing else of the configuration
    _, ref = bench.make_workload("c4", 1, 0, problems=10)
    assert [(i.m, i.n, i.k, i.alpha) for i in mine.items] == \
        [(i.m, i.n, i.k, i.alpha) for i in ref.items]
    assert mine.min_k == ref.min_k and mine.nonfinite_frac == ref.nonfinite_frac


def test_c2_is_weak_scaling_with_a_group_per_rank():
    _, r0 = bench.make_workload("c2", 2, 0)
    _, r1 = bench.make_workload("c2", 2, 1)
    assert r0.scaling == "weak" and len(r0.items) == len(r1.items) == 64
    assert [(i.m, i.n, i.k) for i in r0.items] != [(i.m, i.n, i.k) for i in r1.items]


def test_traffic_table_lookup():
    for kernel in ("prep_kernel", "gemm_kernel", "recon_kernel"):
        for wl in ("c5", "c2"):
            v = bench.traffic_from_profiles(kernel, wl)
            assert v is not None and v > 1e9, (kernel, wl)
    assert bench.traffic_from_profiles("gemm_kernel", "c9") is None
