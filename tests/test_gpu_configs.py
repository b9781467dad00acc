"""Parity on the five BASELINE configurations at their stated sizes, through the public call.

Each test builds a configuration exactly as BASELINE.json states it (tests/workloads.py: shapes,
distributions, alpha / beta, moduli settings, min_k), runs ggemm_grouped_dgemm of this library and
the reference's own ggemm_grouped_dgemm (its sources built for sm_100a into oracle/_ref,
src/ggemm.cu:698-741) on the same device buffers, and compares the FP64 outputs word for word and
the stats counters (GGEMM_STATS_REPAIR=1 in both).

  C1  verbatim (4 x 256^3, N = 14), also gated entrywise against the FP64 triple loop with the
      reference's own test gate: entries with |C - C_exact| > gamma_{k+2} (|alpha||A||B| +
      |beta||C|) must not outnumber the certificate's uncertified count
      (tests/test_grouped.cu:44-57, tests/reference.h:8)
  C2  full size (64 ragged problems, adaptive N)
  C3  one 8192^3 problem at N = 16 (the 16-plane images, residues near |x| ~ T_16)
  C4  full size (1024 problems, NaN / +Inf, alpha = 0, min_k 16) on EMU_GROUPED with REPAIR_ON
      (bitwise); AUTO is gated against cuBLAS FP64 (its routes follow this library's own B200
      cost model, so they need not equal the reference planner's)
  C5  one full reuse component (1 A of 4096^2 x 32 problems) on EMU_GROUPED_REUSE, and two
      components with a workspace pool that forces this library to run the call in chunks
"""
import ctypes
import os
from ctypes import c_void_p

import numpy as np
import pytest

import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _ref_api(ref):
    L = ref.L
    L.ggemm_create_ex.argtypes = [ctypes.POINTER(c_void_p), ctypes.c_int, ctypes.c_size_t,
                                  ctypes.c_size_t, ctypes.c_size_t, c_void_p, ctypes.c_int]
    L.ggemm_grouped_dgemm.argtypes = [c_void_p, ctypes.c_int, c_void_p, c_void_p, ctypes.c_int,
                                      c_void_p]
    L.ggemm_destroy.argtypes = [c_void_p]
    return L


def _budget(grp):
    return grp.budget[0] + 1, grp.budget[1] + 1, grp.budget[2] + 1


def run_ours(g2, grp, path, cfg, min_k, pool_fraction=None):
    """One call of this library on grp (C reset first); returns (rc, stats, C copy)."""
    os.environ["GGEMM_STATS_REPAIR"] = "1"
    if pool_fraction is not None:
        os.environ["GGEMM_WORKSPACE_FRACTION"] = str(pool_fraction)
    try:
        grp.reset()
        torch.cuda.synchronize()
        with g2.Handle(grp.num, *_budget(grp), stream=torch.cuda.current_stream().cuda_stream,
                       min_k=min_k) as h:
            rc, st = h.grouped_dgemm(path, cfg, grp.problems, grp.num)
            torch.cuda.synchronize()
            status = h.device_status()
    finally:
        os.environ.pop("GGEMM_STATS_REPAIR", None)
        os.environ.pop("GGEMM_WORKSPACE_FRACTION", None)
    assert status == 0
    return rc, st, grp.C.clone()


def run_reference(g2, ref, grp, path, cfg, min_k, subsets=None):
    """The reference library on the same buffers (C reset first), one call per subset of
    problems (its handle sizes workspace from summed budgets); returns (rc, stats, C copy)."""
    L = _ref_api(ref)
    entries = grp.entries_on(grp.A, grp.B, grp.C)
    subsets = subsets or [list(range(grp.num))]
    total = g2.Stats()
    os.environ["GGEMM_STATS_REPAIR"] = "1"
    try:
        grp.reset()
        torch.cuda.synchronize()
        for sub in subsets:
            probs = g2.make_problems([entries[i] for i in sub])
            h = c_void_p()
            ta = sum(entries[i]["m"] * entries[i]["k"] for i in sub) + 1
            tb = sum(entries[i]["k"] * entries[i]["n"] for i in sub) + 1
            tc = sum(entries[i]["m"] * entries[i]["n"] for i in sub) + 1
            assert L.ggemm_create_ex(ctypes.byref(h), len(sub), ta, tb, tc,
                                     torch.cuda.current_stream().cuda_stream, min_k) == 0
            st = g2.Stats()
            rc = L.ggemm_grouped_dgemm(h, path, ctypes.addressof(cfg), ctypes.addressof(probs),
                                       len(sub), ctypes.addressof(st))
            torch.cuda.synchronize()
            L.ggemm_destroy(h)
            if rc != 0:
                return rc, st, None
            for f in ("num_repaired", "num_uncertified", "num_safety_fallback", "num_fallback"):
                setattr(total, f, getattr(total, f) + getattr(st, f))
            total.moduli_max = max(total.moduli_max, st.moduli_max)
            total.moduli_min = st.moduli_min if total.moduli_min == 0 else min(total.moduli_min,
                                                                               st.moduli_min)
    finally:
        os.environ.pop("GGEMM_STATS_REPAIR", None)
    return 0, total, grp.C.clone()


def differing_words(a, b):
    return int((a.view(torch.int64) != b.view(torch.int64)).sum().item())


def assert_same(ours, theirs, what):
    rc, st, C = ours
    rc2, st2, C2 = theirs
    assert rc == 0 and rc2 == 0, (rc, rc2)
    diff = differing_words(C, C2)
    assert diff == 0, f"{what}: {diff} FP64 output words differ from the reference library"
    for f in ("num_repaired", "num_uncertified", "num_safety_fallback", "num_fallback",
              "moduli_min", "moduli_max"):
        assert getattr(st, f) == getattr(st2, f), (what, f, getattr(st, f), getattr(st2, f))


def group(g2, wl, pieces=None):
    pieces = pieces if pieces is not None else W.shard_pieces(g2, wl, 1, 0)
    return W.DeviceGroup(g2, wl, pieces, torch.device("cuda", 0), keep_c0=True)


def cfg_of(g2, wl, repair=0):
    return g2.config(wl.num_moduli, wl.target_rel_err, wl.allow_fallback, repair)


def gamma(n):
    u = 2.0 ** -53
    return n * u / (1.0 - n * u)


# ------------------------------------------------------------------------------------- C1
def test_c1_verbatim_vs_reference_and_host_triple_loop(g2, ref, oracle, cuda):
    wl = W.c1()
    grp = group(g2, wl)
    cfg = cfg_of(g2, wl)
    path = W.path_id(g2, wl.path_name)
    ours = run_ours(g2, grp, path, cfg, wl.min_k)
    assert_same(ours, run_reference(g2, ref, grp, path, cfg, wl.min_k), "C1")
    # entrywise against the host FP64 triple loop (the reference's host path) and an extended
    # precision product: the certificate must count every entry beyond gamma_{k+2} den
    rc, st, C = ours
    A, B, C0, Cg = (x.cpu().numpy() for x in (grp.A, grp.B, grp.c0, C))
    over = 0
    for i, it in enumerate(wl.items):
        m, n, k = it.m, it.n, it.k
        a = A[grp.a_off[it.a]:grp.a_off[it.a] + m * k].reshape(k, m).T
        b = B[grp.b_off[it.b]:grp.b_off[it.b] + k * n].reshape(n, k).T
        c0 = C0[grp.c_off[i]:grp.c_off[i] + m * n].reshape(n, m).T
        got = Cg[grp.c_off[i]:grp.c_off[i] + m * n].reshape(n, m).T
        naive = np.ascontiguousarray(c0.T).reshape(-1).copy()
        oracle.dgemm_naive(m, n, k, it.alpha, np.ascontiguousarray(a.T).reshape(-1), m,
                           np.ascontiguousarray(b.T).reshape(-1), k, it.beta,
                           naive, m)
        naive = naive.reshape(n, m).T
        exact = it.alpha * (a.astype(np.longdouble) @ b.astype(np.longdouble)) + \
            it.beta * c0.astype(np.longdouble)
        den = abs(it.alpha) * (np.abs(a) @ np.abs(b)) + abs(it.beta) * np.abs(c0)
        g = gamma(k + 2)
        err = np.abs((got.astype(np.longdouble) - exact)).astype(np.float64)
        over += int(np.count_nonzero(~(err <= g * den)))
        # the naive FP64 loop meets the same bound, so the two agree within 2 gamma den
        assert np.all(np.abs(got - naive) <= 2 * g * den), f"C1 problem {i}"
    assert st.num_uncertified >= over, (st.num_uncertified, over)


# ------------------------------------------------------------------------------------- C2
def test_c2_full_size_vs_reference(g2, ref, cuda):
    wl = W.c2()
    grp = group(g2, wl)
    cfg = cfg_of(g2, wl)
    path = W.path_id(g2, wl.path_name)
    ours = run_ours(g2, grp, path, cfg, wl.min_k)
    assert ours[1].moduli_max == 15 and ours[1].kernel_launches == 3
    assert_same(ours, run_reference(g2, ref, grp, path, cfg, wl.min_k), "C2")


# ------------------------------------------------------------------------------------- C3
def test_c3_one_8192_cubed_problem_n16_vs_reference(g2, ref, cuda):
    wl = W.c3()
    grp = group(g2, wl, [W.Piece(0, 0, 8192)])
    cfg = cfg_of(g2, wl)
    path = W.path_id(g2, wl.path_name)
    ours = run_ours(g2, grp, path, cfg, wl.min_k)
    assert ours[1].moduli_max == 16
    assert_same(ours, run_reference(g2, ref, grp, path, cfg, wl.min_k), "C3")


# ------------------------------------------------------------------------------------- C4
def test_c4_full_size_emu_grouped_repair_on_vs_reference(g2, ref, cuda):
    wl = W.c4()
    grp = group(g2, wl)
    cfg = cfg_of(g2, wl, repair=g2.REPAIR_ON)
    path = g2.PATH_EMU_GROUPED
    ours = run_ours(g2, grp, path, cfg, wl.min_k)
    assert ours[1].num_safety_fallback > 0  # NaN / Inf rows went through the FP64 dot
    assert_same(ours, run_reference(g2, ref, grp, path, cfg, wl.min_k), "C4 EMU_GROUPED/ON")


def test_c4_full_size_auto_against_cublas_fp64(g2, cuda):
    """AUTO (repair ON) on the full C4 group: every finite entry within 2 gamma_{k+2} den of
    cuBLAS FP64 (both lie within gamma_{k+2} den of the exact value), non-finite entries of the
    same class (NaN / +Inf / -Inf) as cuBLAS, alpha = 0 problems (routed to cuBLAS) identical
    to the native call."""
    wl = W.c4()
    grp = group(g2, wl)
    rc, st, C = run_ours(g2, grp, g2.PATH_AUTO, cfg_of(g2, wl), wl.min_k)
    assert rc == 0
    native = run_ours(g2, grp, g2.PATH_NATIVE_GROUPED, cfg_of(g2, wl), wl.min_k)[2]
    for i, it in enumerate(wl.items):
        m, n, k = it.m, it.n, it.k
        got = C[grp.c_off[i]:grp.c_off[i] + m * n]
        want = native[grp.c_off[i]:grp.c_off[i] + m * n]
        if it.alpha == 0.0:
            # alpha = 0 goes to cuBLAS, as in the reference (src/planner.cpp:307-308); its
            # grouped DGEMM still forms A B, so NaN / Inf in A reach C: same bytes as the
            # native path
            assert torch.equal(got.view(torch.int64), want.view(torch.int64)), f"alpha=0, {i}"
            continue
        a = grp.A[grp.a_off[it.a]:grp.a_off[it.a] + m * k].view(k, m).t()
        b = grp.B[grp.b_off[it.b]:grp.b_off[it.b] + k * n].view(n, k).t()
        c0 = grp.c0[grp.c_off[i]:grp.c_off[i] + m * n].view(n, m).t()
        den = (abs(it.alpha) * (a.abs().nan_to_num(0.0, 0.0) @ b.abs())
               + abs(it.beta) * c0.abs()).t().reshape(-1)
        fin = torch.isfinite(want)
        assert torch.equal(torch.isnan(got), torch.isnan(want)), f"NaN pattern, problem {i}"
        assert torch.equal(got[torch.isinf(want)], want[torch.isinf(want)]), f"Inf, problem {i}"
        err = (got[fin] - want[fin]).abs()
        assert bool((err <= 2 * gamma(k + 2) * den[fin]).all()), f"problem {i} ({m},{n},{k})"


# ------------------------------------------------------------------------------------- C5
def test_c5_one_reuse_component_vs_reference(g2, ref, cuda):
    wl = W.c5()
    grp = group(g2, wl, [W.Piece(p, 0, 1024) for p in range(32)])
    cfg = cfg_of(g2, wl)
    path = W.path_id(g2, wl.path_name)
    ours = run_ours(g2, grp, path, cfg, wl.min_k)
    assert ours[1].num_unique_A == 1 and ours[1].num_unique_B == 32
    assert_same(ours, run_reference(g2, ref, grp, path, cfg, wl.min_k), "C5 component")


def test_c5_two_components_chunked_vs_reference(g2, ref, cuda):
    """Two reuse components (64 problems) with a pool of about 6 GB (one component needs about
    4.9 GB): this library splits the call into chunks, preparing the second component's A again
    in the chunk that continues it; the reference runs one call per component.  Identical
    bytes."""
    wl = W.c5()
    grp = group(g2, wl, [W.Piece(p, 0, 1024) for p in range(64)])
    cfg = cfg_of(g2, wl)
    path = W.path_id(g2, wl.path_name)
    total = torch.cuda.get_device_properties(0).total_memory
    ours = run_ours(g2, grp, path, cfg, wl.min_k, pool_fraction=6e9 / total)
    assert ours[1].kernel_launches > 3  # chunked
    theirs = run_reference(g2, ref, grp, path, cfg, wl.min_k,
                           subsets=[list(range(32)), list(range(32, 64))])
    assert_same(ours, theirs, "C5 chunked")
