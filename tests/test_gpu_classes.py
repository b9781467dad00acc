"""Calls that mix moduli counts of different kernel instances.

prep and the reconstruct are compiled per class of moduli counts (N = 14, 15, 16 each, the
others together); the host sorts the descriptors of a call by class and launches one kernel per
class present.  These tests mix the classes in one call and check every output bit for bit
against the CPU oracle, the launch count, and the stage seam's prep with mixed N.
"""
import ctypes

import numpy as np
import pytest

from g2util import col_major, gen

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

# k = 16 -> N = 14, 33..4096 -> 15, 8192 -> 16 at a 1e-15 target; 12..13 at 1e-12
MIXED = [(40, 50, 16), (70, 33, 100), (64, 48, 8192), (31, 90, 12), (50, 20, 3000),
         (20, 36, 9000), (129, 65, 257)]


def _run(g2, oracle, target, seed):
    rng = np.random.default_rng(seed)
    probs, keep, wants, Ns = [], [], [], []
    for i, (m, n, k) in enumerate(MIXED):
        A, B, C0 = gen(rng, (m, k), 1.0), gen(rng, (k, n), 1.0), gen(rng, (m, n), 0.0)
        lda, ldb, ldc = m + 1, k + 2, m + 3
        alpha, beta = (1.0, 0.0) if i % 2 else (0.75, -0.5)
        Af, Bf, Cf = col_major(A, lda), col_major(B, ldb), col_major(C0, ldc)
        N = max(2, oracle.choose(k, target))
        want = Cf.copy()
        oracle.emulated(m, n, k, N, alpha, beta, Af, lda, Bf, ldb, want, ldc, 1)
        dA, dB, dC = (torch.from_numpy(x).cuda() for x in (Af, Bf, Cf.copy()))
        keep.append((dA, dB, dC))
        wants.append(want)
        Ns.append(N)
        probs.append(dict(m=m, n=n, k=k, A=dA.data_ptr(), lda=lda, B=dB.data_ptr(), ldb=ldb,
                          C=dC.data_ptr(), ldc=ldc, alpha=alpha, beta=beta))
    P = g2.make_problems(probs)
    ta = sum(m * k for m, n, k in MIXED)
    tb = sum(k * n for m, n, k in MIXED)
    tc = sum(m * n for m, n, k in MIXED)
    with g2.Handle(len(MIXED), ta, tb, tc, stream=torch.cuda.current_stream().cuda_stream) as h:
        rc, st = h.grouped_dgemm(g2.PATH_EMU_GROUPED, g2.config(0, target, 0, 0), P, len(MIXED))
        torch.cuda.synchronize()
    assert rc == 0, rc
    for (_, _, dC), want, (m, n, k) in zip(keep, wants, MIXED):
        got = dC.cpu().numpy()
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), (m, n, k)
    return st, Ns


def test_mixed_dedicated_classes(g2, oracle, cuda):
    """N = 14, 15 and 16 in one call: three prep and three reconstruct instances."""
    st, Ns = _run(g2, oracle, 1e-15, 3)
    assert sorted(set(Ns)) == [14, 15, 16]
    assert (st.moduli_min, st.moduli_max) == (14, 16)
    assert st.kernel_launches == 3 + 1 + 3


def test_generic_classes(g2, oracle, cuda):
    """Counts below 14 share the dispatching instances: one prep and one reconstruct launch."""
    st, Ns = _run(g2, oracle, 1e-12, 4)
    assert max(Ns) < 14
    assert st.kernel_launches == 3


def test_stage_prep_mixed_counts(g2, oracle, cuda):
    """One ggemm_stage_prep call over descriptors of five classes (N = 8, 14, 15, 16, 20),
    given in an order the library re-sorts: every image and workspace as the oracle's."""
    rng = np.random.default_rng(11)
    cases = [(37, 300, 20, 0), (29, 200, 15, 1), (40, 150, 8, 0), (33, 90, 16, 1),
             (21, 400, 14, 0), (45, 64, 15, 0)]
    descs = (g2.PrepDesc * len(cases))()
    keep, outs = [], []
    for i, (rows, k, N, kind) in enumerate(cases):
        mat = gen(rng, (rows, k), 2.0)
        if kind == 0:
            ld = rows + 2
            X = col_major(mat, ld)
        else:
            ld = k + 3
            X = col_major(mat.T, ld)
        pb = (g2.img_plane_bytes(rows, k) + 255) // 256 * 256
        Xd = torch.from_numpy(np.ascontiguousarray(X)).cuda()
        img = torch.full(((N + 1) * pb,), 0x5A, dtype=torch.int8, device="cuda")
        ws = torch.zeros(4 * rows, dtype=torch.int32, device="cuda")
        keep += [Xd, img, ws]
        outs.append((X, rows, k, ld, N, kind, img, pb, ws))
        descs[i] = g2.PrepDesc(Xd.data_ptr(), ld, rows, k, N, kind, img.data_ptr(), pb,
                               ws.data_ptr())
    scr = torch.empty(g2.lib.ggemm_stage_scratch_bytes(len(cases)), dtype=torch.uint8,
                      device="cuda")
    cnt = torch.zeros(64, dtype=torch.uint8, device="cuda")
    rc = g2.lib.ggemm_stage_prep(descs, len(cases), scr.data_ptr(), scr.numel(), cnt.data_ptr(),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(cnt.cpu().numpy()[32:36].view(np.uint32)[0]) == 0
    for X, rows, k, ld, N, kind, img, pb, ws in outs:
        ref_planes, ref_ws, _ = oracle.prep(X, rows, k, ld, N, kind)
        h = img.cpu().numpy()
        for l in range(N + 1):
            got = g2.unpack_plane(h[l * pb:(l + 1) * pb], rows, k)
            assert np.array_equal(got, ref_planes[l]), (rows, k, N, kind, l)
        np.testing.assert_array_equal(ws.cpu().numpy(), ref_ws)
