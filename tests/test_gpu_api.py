"""The public call (ggemm_grouped_dgemm / plans) on B200, modelled on the reference's
tests/test_grouped.cu, test_graph.cu and test_reuse_e2e.cu.

Gate (never relaxed, tests/test_grouped.cu:5-12): |C - Cref| <= gamma_n (|alpha||A||B| +
|beta||C0|) componentwise, n = k + [alpha != 1] + [beta != 0], with Cref from an 80-bit
long-double product.  Strict for native paths and repair ON; for repair COUNT the number of
violating entries must not exceed the certificate's uncertified count.
"""
import ctypes
import os

import numpy as np
import pytest

from g2util import col_major, gen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

U = 2.0 ** -53


class Group:
    def __init__(self, shapes, phi, alpha, beta, seed, pad=0, nan_c=False, poison=None):
        rng = np.random.default_rng(seed)
        self.items = []
        for i, (m, n, k) in enumerate(shapes):
            a = alpha(i) if callable(alpha) else alpha
            A, B, C0 = gen(rng, (m, k), phi), gen(rng, (k, n), phi), gen(rng, (m, n), 0.0)
            if poison:
                poison(i, A, B)
            if nan_c:
                C0[:] = np.nan
            lda, ldb, ldc = max(1, m + pad), max(1, k + pad), max(1, m + pad)
            self.items.append(dict(m=m, n=n, k=k, alpha=a, beta=beta, A=A, B=B, C0=C0, lda=lda,
                                   ldb=ldb, ldc=ldc))
        self.reset()

    def reset(self):
        self.dev = []
        for it in self.items:
            dA = torch.from_numpy(col_major(it["A"], it["lda"])).cuda()
            dB = torch.from_numpy(col_major(it["B"], it["ldb"])).cuda()
            dC = torch.from_numpy(col_major(it["C0"], it["ldc"])).cuda()
            self.dev.append((dA, dB, dC))

    def problems(self, g2):
        return g2.make_problems([dict(m=it["m"], n=it["n"], k=it["k"], A=dA.data_ptr(), lda=it["lda"],
                                      B=dB.data_ptr(), ldb=it["ldb"], C=dC.data_ptr(), ldc=it["ldc"],
                                      alpha=it["alpha"], beta=it["beta"])
                                 for it, (dA, dB, dC) in zip(self.items, self.dev)])

    def budgets(self):
        return (sum(it["m"] * it["k"] for it in self.items) + 1,
                sum(it["k"] * it["n"] for it in self.items) + 1,
                sum(it["m"] * it["n"] for it in self.items) + 1)

    def outputs(self):
        res = []
        for it, (_, _, dC) in zip(self.items, self.dev):
            c = dC.cpu().numpy()
            if it["m"] and it["n"]:
                res.append(c[: it["ldc"] * it["n"]].reshape(it["n"], it["ldc"])[:, : it["m"]].T.copy())
            else:
                res.append(np.zeros((it["m"], it["n"])))
        return res

    def gate(self, outs):
        """(entries over gamma_n incl. non-finite, max err / (gamma_n den))."""
        over, worst = 0, 0.0
        for it, C in zip(self.items, outs):
            m, n, k = it["m"], it["n"], it["k"]
            if not (m and n):
                continue
            A = it["A"].astype(np.longdouble)
            B = it["B"].astype(np.longdouble)
            C0 = it["C0"].astype(np.longdouble)
            ab = A @ B if k else np.zeros((m, n), dtype=np.longdouble)
            absab = np.abs(A) @ np.abs(B) if k else np.zeros((m, n), dtype=np.longdouble)
            al, be = np.longdouble(it["alpha"]), np.longdouble(it["beta"])
            ref = al * ab + (be * C0 if it["beta"] != 0 else 0)
            den = abs(al) * absab + (abs(be) * np.abs(C0) if it["beta"] != 0 else 0)
            nt = k + (it["alpha"] != 1.0) + (it["beta"] != 0.0)
            g = max(nt, 1) * U / (1 - max(nt, 1) * U)
            finite_ref = np.isfinite(ref)
            err = np.abs(C.astype(np.longdouble) - ref)
            bad = finite_ref & ~(err <= g * den)
            bad |= finite_ref & ~np.isfinite(C)
            over += int(bad.sum())
            with np.errstate(divide="ignore", invalid="ignore"):
                r = np.where(finite_ref & (den > 0), err / (g * den), 0)
            worst = max(worst, float(np.nanmax(r)) if r.size else 0.0)
        return over, worst


def run(g2, grp, path, cfg, stats_env=True, min_k=32, stream=None):
    if stats_env:
        os.environ["GGEMM_STATS_REPAIR"] = "1"
    try:
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream
        h = g2.Handle(max(1, len(grp.items)), *grp.budgets(), stream=s, min_k=min_k)
    finally:
        os.environ.pop("GGEMM_STATS_REPAIR", None)
    rc, st = h.grouped_dgemm(path, cfg, grp.problems(g2), len(grp.items))
    torch.cuda.synchronize()
    h.close()
    return rc, st


WORKLOADS = {
    "uniform64": [(64, 64, 64)] * 8,
    "ragged": [(7, 13, 33), (100, 70, 50), (33, 65, 200), (128, 96, 300), (1, 300, 64),
               (300, 1, 129), (40, 24, 72), (65, 3, 31)],
    "longk": [(16, 16, 2048), (32, 8, 4096)],
    # an odd number of problems: NATIVE_GROUPED's pointer table (3 x 8 bytes per problem) is then
    # not a multiple of 16 bytes, so the descriptor upload kernel copies a tail
    "odd3": [(48, 40, 96), (17, 33, 5), (64, 80, 128)],
}
PATHS = [0, 1, 2, 3, 4, 5, 6]


@pytest.mark.parametrize("wl", list(WORKLOADS))
@pytest.mark.parametrize("phi,alpha,beta", [(0.5, 1.0, 0.0), (2.0, 1.5, -0.75)])
@pytest.mark.parametrize("path", PATHS)
def test_gate_every_path(g2, cuda, wl, phi, alpha, beta, path):
    grp = Group(WORKLOADS[wl], phi, alpha, beta, seed=100 * len(wl) + int(10 * phi), pad=3 if wl == "ragged" else 0)
    cfg = g2.config(0, 1e-15, 1 if path == 4 else 0, 0)
    rc, st = run(g2, grp, path, cfg)
    assert rc == 0
    over, worst = grp.gate(grp.outputs())
    if path in (2, 3, 5, 6):  # repair COUNT: the certificate may over-report, never miss
        assert st.num_uncertified >= 0 and over <= st.num_uncertified, (over, st.num_uncertified)
    else:
        assert over == 0, (over, worst)
    assert st.num_problems == len(grp.items)
    computable = sum(1 for it in grp.items if it["m"] and it["n"] and it["k"])
    if path >= 2 and computable - st.num_fallback >= 1:
        assert 2 <= st.moduli_min <= st.moduli_max <= 20


def test_emulated_paths_bitwise_identical(g2, cuda):
    """EMU_LOOP, EMU_LOOP_BATCHED, EMU_GROUPED and EMU_GROUPED_REUSE run the same kernels on
    the same residues: identical bytes (reference tests/test_reuse_e2e.cu:1-14)."""
    shapes = WORKLOADS["ragged"] + WORKLOADS["uniform64"][:3]
    outs = {}
    for path in (2, 3, 5, 6):
        grp = Group(shapes, 1.0, 1.25, 0.5, seed=99)
        rc, st = run(g2, grp, path, g2.config(15, 1e-15, 0, g2.REPAIR_COUNT), stats_env=False)
        assert rc == 0
        outs[path] = grp.outputs()
    for path in (2, 5, 6):
        for a, b in zip(outs[3], outs[path]):
            assert np.array_equal(a.view(np.uint64), b.view(np.uint64)), path


def test_launch_count_independent_of_group_size(g2, cuda):
    launches = []
    for G in (16, 1024):
        grp = Group([(32, 32, 32)] * G, 0.5, 1.0, 0.0, seed=G)
        rc, st = run(g2, grp, 3, g2.config(0, 1e-15, 0, 0), stats_env=False)
        assert rc == 0
        launches.append(st.kernel_launches)
    assert launches[0] == launches[1] == 3


@pytest.mark.parametrize("path", [3, 4, 5])
def test_bitwise_reproducible(g2, cuda, path):
    grp = Group(WORKLOADS["ragged"], 2.0, 1.0, 0.0, seed=5)
    s = torch.cuda.current_stream().cuda_stream
    h = g2.Handle(len(grp.items), *grp.budgets(), stream=s)
    cfg = g2.config(0, 1e-15, 1, 0)
    rc1, _ = h.grouped_dgemm(path, cfg, grp.problems(g2), len(grp.items))
    torch.cuda.synchronize()
    r1 = [c.copy() for c in grp.outputs()]
    for _, _, dC in grp.dev:
        dC.zero_()
    rc2, _ = h.grouped_dgemm(path, cfg, grp.problems(g2), len(grp.items))
    torch.cuda.synchronize()
    r2 = grp.outputs()
    h.close()
    assert rc1 == rc2 == 0
    for a, b in zip(r1, r2):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))


EDGE_CASES = {
    "one_100x70x50": ([(100, 70, 50)], 1.0, 0.0, False),
    "one_1x1x1": ([(1, 1, 1)], 1.0, 0.0, False),
    "zero_dims_mix": ([(0, 32, 32), (32, 0, 32), (32, 32, 0), (48, 40, 36), (0, 0, 0)], 1.5, -0.5, False),
    "all_empty": ([(0, 16, 16), (16, 0, 16)], 1.0, 0.0, False),
    "beta0_nanC": ([(40, 24, 72), (17, 33, 5)], 1.0, 0.0, True),
    "k_not_mult32": ([(33, 31, 1), (65, 3, 31), (5, 129, 97)], -2.0, 1.0, False),
}


@pytest.mark.parametrize("case", list(EDGE_CASES))
@pytest.mark.parametrize("path", PATHS)
def test_edge_cases(g2, cuda, case, path):
    shapes, alpha, beta, nan_c = EDGE_CASES[case]
    grp = Group(shapes, 1.0, alpha, beta, seed=len(case), nan_c=nan_c)
    rc, st = run(g2, grp, path, g2.config(0, 1e-15, 1 if path == 4 else 0, 0), min_k=1)
    assert rc == 0
    over, worst = grp.gate(grp.outputs())
    if path in (2, 3, 5, 6):
        assert over <= max(0, st.num_uncertified)
    else:
        assert over == 0


def test_zero_problems_null_pointer(g2, cuda):
    s = torch.cuda.current_stream().cuda_stream
    with g2.Handle(4, 64, 64, 64, stream=s) as h:
        for path in PATHS:
            st = g2.Stats()
            rc = g2.lib.ggemm_grouped_dgemm(h.ptr, path, None, None, 0, ctypes.byref(st))
            assert rc == 0 and st.num_problems == 0 and st.num_fallback == 0
    torch.cuda.synchronize()


def test_big_k_fallback(g2, cuda):
    grp = Group([(4, 4, 140000), (64, 64, 64), (8, 8, 8)], 0.5, 1.0, 0.0, seed=3)
    rc, st = run(g2, grp, 4, g2.config(0, 1e-15, 1, 0))
    assert rc == 0 and st.num_fallback >= 1
    assert grp.gate(grp.outputs())[0] == 0
    for path in (3, 4):
        grp.reset()
        rc, st = run(g2, grp, path, g2.config(0, 1e-15, 0, 0))
        assert rc == g2.ERR_UNSAFE


def test_capacity_and_argument_violations(g2, cuda):
    grp = Group([(16, 16, 16)] * 3, 0.0, 1.0, 0.0, seed=1)
    s = torch.cuda.current_stream().cuda_stream
    for path in PATHS:
        with g2.Handle(2, 4096, 4096, 4096, stream=s) as h:
            rc, _ = h.grouped_dgemm(path, g2.config(), grp.problems(g2), 3)
            assert rc == g2.ERR_INVALID
        with g2.Handle(8, 100, 100, 100, stream=s) as h:
            rc, _ = h.grouped_dgemm(path, g2.config(), grp.problems(g2), 3)
            assert rc == g2.ERR_WORKSPACE
    with g2.Handle(8, 4096, 4096, 4096, stream=s) as h:
        for bad in (1, 21, -1):
            rc, _ = h.grouped_dgemm(3, g2.config(bad), grp.problems(g2), 3)
            assert rc == g2.ERR_INVALID
        rc, _ = h.grouped_dgemm(3, g2.config(0, 1e-15, 1, 7), grp.problems(g2), 3)
        assert rc == g2.ERR_INVALID
    torch.cuda.synchronize()


def test_operand_reuse_counts_and_bits(g2, cuda):
    """Shared A (LoRA-like) and shared B (tensor-parallel-like): unique-operand counts, and the
    same bytes as EMU_GROUPED (reference tests/test_reuse_e2e.cu:1-14)."""
    rng = np.random.default_rng(17)
    k = 96
    A_shared = col_major(gen(rng, (64, k), 1.0), 64)
    B_shared = col_major(gen(rng, (k, 48), 1.0), k)
    B_own = [col_major(gen(rng, (k, 40), 1.0), k) for _ in range(3)]
    A_own = [col_major(gen(rng, (32, k), 1.0), 32) for _ in range(3)]
    outs = {}
    for path in (3, 5):
        dA = torch.from_numpy(A_shared).cuda()
        dB = torch.from_numpy(B_shared).cuda()
        keep, entries, Cs = [], [], []
        for g in range(3):
            Bg = torch.from_numpy(B_own[g]).cuda()
            C = torch.zeros(64 * 40, dtype=torch.float64, device="cuda")
            keep.append(Bg)
            Cs.append(C)
            entries.append(dict(m=64, n=40, k=k, A=dA.data_ptr(), lda=64, B=Bg.data_ptr(), ldb=k,
                                C=C.data_ptr(), ldc=64, alpha=1.0, beta=0.0))
        for g in range(3):
            Ag = torch.from_numpy(A_own[g]).cuda()
            C = torch.zeros(32 * 48, dtype=torch.float64, device="cuda")
            keep.append(Ag)
            Cs.append(C)
            entries.append(dict(m=32, n=48, k=k, A=Ag.data_ptr(), lda=32, B=dB.data_ptr(), ldb=k,
                                C=C.data_ptr(), ldc=32, alpha=1.0, beta=0.0))
        P = g2.make_problems(entries)
        with g2.Handle(6, 64 * k * 6, k * 48 * 6, 64 * 48 * 6,
                       stream=torch.cuda.current_stream().cuda_stream) as h:
            rc, st = h.grouped_dgemm(path, g2.config(15, 1e-15, 0, 0), P, 6)
            torch.cuda.synchronize()
        assert rc == 0
        if path == 5:
            assert st.reuse_enabled == 1 and st.num_unique_A == 4 and st.num_unique_B == 4
        else:
            assert st.num_unique_A == 6 and st.num_unique_B == 6
        outs[path] = [C.cpu().numpy() for C in Cs]
    for a, b in zip(outs[3], outs[5]):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))


def test_nonfinite_alpha_zero_small_k_auto(g2, cuda):
    """Config-4-like: NaN/Inf rows, alpha = 0 problems, k < 32 on a min_k = 16 handle."""
    def poison(i, A, B):
        if i % 3 == 0 and A.size:
            A[0, 0] = np.nan
        if i % 3 == 1 and A.size:
            A[-1, -1] = np.inf
    shapes = [(40, 30, 16), (33, 20, 100), (64, 64, 17), (16, 200, 512), (128, 16, 40), (20, 20, 300)]
    grp = Group(shapes, 4.0, lambda i: 0.0 if i == 4 else 1.0, 0.5, seed=44, poison=poison)
    rc, st = run(g2, grp, 4, g2.config(0, 1e-15, 1, 0), min_k=16)
    assert rc == 0
    assert grp.gate(grp.outputs())[0] == 0
    grp.reset()
    rc, st = run(g2, grp, 3, g2.config(0, 1e-15, 1, g2.REPAIR_ON), min_k=16)
    assert rc == 0 and st.num_safety_fallback > 0
    assert grp.gate(grp.outputs())[0] == 0


def test_group_beyond_cached_tile_schedule(g2, cuda):
    """More GEMM jobs than the per-CTA tile schedule caches (4096): the GEMM decodes each tile
    itself.  Same bytes as the group run in two calls below that size."""
    shapes = [(16 + (i % 5) * 8, 24 + (i % 3) * 8, 40 + (i % 7) * 16) for i in range(4200)]
    grp = Group(shapes, 1.0, 1.0, 0.5, seed=42)
    cfg = g2.config(15, 1e-15, 0, 0)
    rc, _ = run(g2, grp, 3, cfg, stats_env=False)
    assert rc == 0
    whole = [c.copy() for c in grp.outputs()]
    parts = []
    for lo, hi in ((0, 2100), (2100, 4200)):
        sub = Group(shapes[lo:hi], 1.0, 1.0, 0.5, seed=0)
        sub.items = grp.items[lo:hi]
        sub.reset()
        rc, _ = run(g2, sub, 3, cfg, stats_env=False)
        assert rc == 0
        parts += sub.outputs()
    for a, b in zip(whole, parts):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))


def test_chunked_group_matches_single_pass(g2, cuda):
    """A handle whose workspace holds only a few problems runs the group in chunks, with the
    same bytes as one pass."""
    shapes = [(128, 128, 128)] * 12
    grp = Group(shapes, 1.0, 1.0, 0.0, seed=12)
    rc, st = run(g2, grp, 3, g2.config(15, 1e-15, 0, 0), stats_env=False)
    assert rc == 0 and st.kernel_launches == 3
    one = [c.copy() for c in grp.outputs()]
    total = torch.cuda.get_device_properties(0).total_memory
    os.environ["GGEMM_WORKSPACE_FRACTION"] = str(3.5e6 / total)
    try:
        grp.reset()
        rc, st = run(g2, grp, 3, g2.config(15, 1e-15, 0, 0), stats_env=False)
    finally:
        os.environ.pop("GGEMM_WORKSPACE_FRACTION", None)
    assert rc == 0 and st.kernel_launches > 3
    for a, b in zip(one, grp.outputs()):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))


def test_graph_plan_matches_direct_call(g2, cuda):
    """ggemm_make_plan + ggemm_execute_plan equal a direct call bit for bit, on the handle's
    stream and on another stream; update_pointers retargets the plan (tests/test_graph.cu)."""
    shapes = WORKLOADS["ragged"][:5] + [(3, 3, 3000000 // 1000)]
    grp = Group(shapes, 1.0, 1.0, 0.5, seed=8)
    s = torch.cuda.current_stream().cuda_stream
    h = g2.Handle(len(shapes), *grp.budgets(), stream=s)
    cfg = g2.config(0, 1e-15, 1, 0)
    rc, st = h.grouped_dgemm(4, cfg, grp.problems(g2), len(shapes))
    torch.cuda.synchronize()
    direct = [c.copy() for c in grp.outputs()]
    grp.reset()
    err = ctypes.c_int(-1)
    plan = g2.lib.ggemm_make_plan_ex(h.ptr, 4, ctypes.byref(cfg), grp.problems(g2), len(shapes),
                                     ctypes.byref(err))
    assert plan and err.value == 0
    assert g2.lib.ggemm_execute_plan(plan, ctypes.c_void_p(s)) == 0
    torch.cuda.synchronize()
    for a, b in zip(direct, grp.outputs()):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))
    # another stream
    grp2 = Group(shapes, 1.0, 1.0, 0.5, seed=8)
    other = torch.cuda.Stream()
    A = (ctypes.c_void_p * len(shapes))(*[d[0].data_ptr() for d in grp2.dev])
    B = (ctypes.c_void_p * len(shapes))(*[d[1].data_ptr() for d in grp2.dev])
    C = (ctypes.c_void_p * len(shapes))(*[d[2].data_ptr() for d in grp2.dev])
    assert g2.lib.ggemm_plan_update_pointers(plan, A, B, C) == 0
    assert g2.lib.ggemm_execute_plan(plan, ctypes.c_void_p(other.cuda_stream)) == 0
    torch.cuda.synchronize()
    for a, b in zip(direct, grp2.outputs()):
        assert np.array_equal(a.view(np.uint64), b.view(np.uint64))
    st2 = g2.Stats()
    assert g2.lib.ggemm_plan_get_stats(plan, ctypes.byref(st2)) == 0
    assert st2.kernel_launches == st.kernel_launches
    g2.lib.ggemm_destroy_plan(plan)
    h.close()
