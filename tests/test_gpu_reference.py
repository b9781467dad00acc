"""Bit-exact parity with the REFERENCE's own kernels (moneychen168/Coding-Basic-HW-2 built for
sm_100a from its sources into oracle/_ref, run on the same B200 on the same inputs).

  residues + row/column workspace  vs oz2_prep_grouped        (src/ozaki2_numerics.cu:609-623)
  int32 residue products           vs i8_grouped_gemm         (src/int8_grouped_gemm.cu:741-780)
  FP64 outputs, all repair modes   vs oz2_reconstruct_grouped (src/ozaki2_numerics.cu:625-637)
  the public call                  vs ggemm_grouped_dgemm     (src/ggemm.cu:698-741)
"""
import ctypes
from ctypes import c_double, c_int, c_size_t, c_void_p

import numpy as np
import pytest

from g2util import col_major, gen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


class Oz2Problem(ctypes.Structure):
    """oz2_problem (src/ozaki2_numerics.h:23-30)."""

    _fields_ = [("m", c_int), ("n", c_int), ("k", c_int), ("kp", c_int), ("num_moduli", c_int),
                ("lda", c_int), ("ldb", c_int), ("ldc", c_int), ("A", c_void_p), ("B", c_void_p),
                ("C", c_void_p), ("alpha", c_double), ("beta", c_double), ("A8", c_void_p),
                ("B8", c_void_p), ("a8_mod_stride", c_size_t), ("b8_mod_stride", c_size_t),
                ("C32", c_void_p), ("c32_mod_stride", c_size_t), ("row_shift", c_void_p),
                ("col_shift", c_void_p)]


class I8Problem(ctypes.Structure):
    """i8_problem (src/int8_grouped_gemm.h:16-23)."""

    _fields_ = [("m", c_int), ("n", c_int), ("kp", c_int), ("A", c_void_p), ("B", c_void_p),
                ("C", c_void_p), ("tile_cfg", c_int)]


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_struct_sizes(ref):
    assert ref.L.ozr_sizeof_oz2_problem() == ctypes.sizeof(Oz2Problem)
    assert ref.L.ozr_sizeof_i8_problem() == ctypes.sizeof(I8Problem)


SHAPES = [(200, 150, 777, 20, 1.0, 1.0, 0.0), (1, 300, 64, 16, 0.5, -2.5, 1.0),
          (300, 1, 129, 12, 2.0, 0.75, -0.5), (77, 55, 1, 8, 1.0, 1.0, 2.0),
          (64, 48, 512, 18, 1.0, 1.0, 0.0), (33, 65, 2048, 10, 4.0, 1.0, 0.25),
          (16, 16, 16, 15, 2.0, 1.0, 0.0), (128, 96, 1000, 15, 2.0, 1.0, 0.5),
          (256, 256, 256, 14, 0.0, 1.0, 0.0)]


def _make(seed, special=None):
    rng = np.random.default_rng(seed)
    probs = []
    for (m, n, k, N, phi, alpha, beta) in SHAPES:
        A = gen(rng, (m, k), phi)
        B = gen(rng, (k, n), phi)
        C0 = gen(rng, (m, n), 0.0)
        if special == "mixed" and m > 40 and k > 20:
            A[3, :] = 0.0
            A[5, 17] = np.nan
            B[11 % k, 0] = np.inf
        lda, ldb, ldc = m + 7, k + 3, m + 1
        probs.append(dict(m=m, n=n, k=k, N=N, alpha=alpha, beta=beta, lda=lda, ldb=ldb, ldc=ldc,
                          A=col_major(A, lda), B=col_major(B, ldb), C0=col_major(C0, ldc)))
    return probs


def _ref_pipeline(ref, probs, mode):
    """Runs the reference's prep, INT8 GEMM and reconstruct; returns per problem
    (planes A [N+1,m,kp], planes B, ws A, ws B, C32 [N+1, m*n], C)."""
    keep, ozs, i8s, meta = [], [], [], []
    for p in probs:
        m, n, k, N = p["m"], p["n"], p["k"], p["N"]
        kp = (k + 31) // 32 * 32
        P = N + 1
        dA, dB = torch.from_numpy(p["A"]).cuda(), torch.from_numpy(p["B"]).cuda()
        dC = torch.from_numpy(p["C0"].copy()).cuda()
        A8 = torch.full((P * m * kp + 16,), 0x5A, dtype=torch.int8, device="cuda")
        B8 = torch.full((P * n * kp + 16,), 0x5A, dtype=torch.int8, device="cuda")
        C32 = torch.zeros(P * m * n + 16, dtype=torch.int32, device="cuda")
        rs = torch.zeros(4 * m + 4, dtype=torch.int32, device="cuda")
        cs = torch.zeros(4 * n + 4, dtype=torch.int32, device="cuda")
        keep += [dA, dB, dC, A8, B8, C32, rs, cs]
        ozs.append(Oz2Problem(m, n, k, kp, N, p["lda"], p["ldb"], p["ldc"], dA.data_ptr(),
                              dB.data_ptr(), dC.data_ptr(), p["alpha"], p["beta"], A8.data_ptr(),
                              B8.data_ptr(), m * kp, n * kp, C32.data_ptr(), m * n, rs.data_ptr(),
                              cs.data_ptr()))
        for l in range(P):
            i8s.append(I8Problem(m, n, kp, A8.data_ptr() + l * m * kp, B8.data_ptr() + l * n * kp,
                                 C32.data_ptr() + 4 * l * m * n, 0))
        meta.append((A8, B8, C32, rs, cs, dC))
    num = len(ozs)
    h_oz = (Oz2Problem * num)(*ozs)
    d_oz = torch.frombuffer(bytearray(bytes(h_oz)), dtype=torch.uint8).cuda()
    h_i8 = (I8Problem * len(i8s))(*i8s)
    d_i8 = torch.frombuffer(bytearray(bytes(h_i8)), dtype=torch.uint8).cuda()
    ws_bytes = ref.L.ozr_i8_sched_ws_bytes(len(i8s))
    d_ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    mm = max(p["m"] for p in probs)
    nn = max(p["n"] for p in probs)
    s = _stream()
    ref.L.ozr_read_counters(None, 1, s)
    assert ref.L.ozr_prep_grouped(d_oz.data_ptr(), num, mm, nn, s) == 0
    assert ref.L.ozr_i8_grouped_gemm(d_i8.data_ptr(), len(i8s), ctypes.addressof(h_i8),
                                     d_ws.data_ptr(), ws_bytes, s) == 0
    assert ref.L.ozr_reconstruct_grouped(d_oz.data_ptr(), num, mm, nn, s, mode) == 0
    cnt = (ctypes.c_ulonglong * 4)()
    assert ref.L.ozr_read_counters(ctypes.addressof(cnt), 1, s) == 0
    torch.cuda.synchronize()
    out = []
    for p, (A8, B8, C32, rs, cs, dC) in zip(probs, meta):
        m, n, k, N = p["m"], p["n"], p["k"], p["N"]
        kp = (k + 31) // 32 * 32
        P = N + 1
        out.append((A8.cpu().numpy()[:P * m * kp].reshape(P, m, kp),
                    B8.cpu().numpy()[:P * n * kp].reshape(P, n, kp),
                    rs.cpu().numpy()[:4 * m], cs.cpu().numpy()[:4 * n],
                    C32.cpu().numpy()[:P * m * n].reshape(P, m * n), dC.cpu().numpy()))
    return out, list(cnt)


def _our_pipeline(g2, probs, mode):
    """Our three stages on the same inputs; same outputs as _ref_pipeline."""
    keep, preps, gemms, recons, meta = [], [], [], [], []
    for p in probs:
        m, n, k, N = p["m"], p["n"], p["k"], p["N"]
        P = N + 1
        pa = (g2.img_plane_bytes(m, k) + 255) // 256 * 256
        pb = (g2.img_plane_bytes(n, k) + 255) // 256 * 256
        cp = (m * n + 63) // 64 * 64
        dA, dB = torch.from_numpy(p["A"]).cuda(), torch.from_numpy(p["B"]).cuda()
        dC = torch.from_numpy(p["C0"].copy()).cuda()
        ia = torch.zeros(P * pa + 256, dtype=torch.int8, device="cuda")
        ib = torch.zeros(P * pb + 256, dtype=torch.int8, device="cuda")
        c32 = torch.zeros(P * cp + 64, dtype=torch.int32, device="cuda")
        rs = torch.zeros(4 * m + 4, dtype=torch.int32, device="cuda")
        cs = torch.zeros(4 * n + 4, dtype=torch.int32, device="cuda")
        keep += [dA, dB, dC, ia, ib, c32, rs, cs]
        preps.append(g2.PrepDesc(dA.data_ptr(), p["lda"], m, k, N, 0, ia.data_ptr(), pa, rs.data_ptr()))
        preps.append(g2.PrepDesc(dB.data_ptr(), p["ldb"], n, k, N, 1, ib.data_ptr(), pb, cs.data_ptr()))
        gemms.append(g2.GemmDesc(ia.data_ptr(), ib.data_ptr(), c32.data_ptr(), pa, pb, cp, m, n, k, P))
        recons.append(g2.ReconDesc(m, n, k, N, dA.data_ptr(), p["lda"], dB.data_ptr(), p["ldb"],
                                   dC.data_ptr(), p["ldc"], p["alpha"], p["beta"], c32.data_ptr(),
                                   cp, rs.data_ptr(), cs.data_ptr()))
        meta.append((ia, ib, c32, rs, cs, dC, pa, pb, cp))
    num = len(probs)
    scr = torch.empty(g2.lib.ggemm_stage_scratch_bytes(2 * num), dtype=torch.uint8, device="cuda")
    cnt = torch.zeros(64, dtype=torch.uint8, device="cuda")
    s = _stream()
    assert g2.lib.ggemm_stage_prep((g2.PrepDesc * (2 * num))(*preps), 2 * num, scr.data_ptr(),
                                   scr.numel(), cnt.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert g2.lib.ggemm_stage_gemm((g2.GemmDesc * num)(*gemms), num, scr.data_ptr(), scr.numel(),
                                   cnt.data_ptr(), s) == 0
    torch.cuda.synchronize()
    assert g2.lib.ggemm_stage_recon((g2.ReconDesc * num)(*recons), num, mode, scr.data_ptr(),
                                    scr.numel(), cnt.data_ptr(), s) == 0
    torch.cuda.synchronize()
    out = []
    for p, (ia, ib, c32, rs, cs, dC, pa, pb, cp) in zip(probs, meta):
        m, n, k, N = p["m"], p["n"], p["k"], p["N"]
        P = N + 1
        ha, hb = ia.cpu().numpy(), ib.cpu().numpy()
        A8 = np.stack([g2.unpack_plane(ha[l * pa:(l + 1) * pa], m, k) for l in range(P)])
        B8 = np.stack([g2.unpack_plane(hb[l * pb:(l + 1) * pb], n, k) for l in range(P)])
        hc = c32.cpu().numpy()
        out.append((A8, B8, rs.cpu().numpy()[:4 * m], cs.cpu().numpy()[:4 * n],
                    np.stack([hc[l * cp:l * cp + m * n] for l in range(P)]), dC.cpu().numpy()))
    c = cnt.cpu().numpy().view(np.uint64)
    return out, [int(x) for x in c[:4]]


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("special", [None, "mixed"])
def test_stages_bit_exact_vs_reference_kernels(g2, ref, cuda, mode, special):
    probs = _make(77 + mode, special)
    theirs, cnt_ref = _ref_pipeline(ref, probs, mode)
    ours, cnt = _our_pipeline(g2, probs, mode)
    for p, t, o in zip(probs, theirs, ours):
        tag = (p["m"], p["n"], p["k"], p["N"])
        assert np.array_equal(o[0], t[0]), f"A residues differ {tag}"
        assert np.array_equal(o[1], t[1]), f"B residues differ {tag}"
        assert np.array_equal(o[2], t[2]), f"row workspace differs {tag}"
        assert np.array_equal(o[3], t[3]), f"col workspace differs {tag}"
        assert np.array_equal(o[4], t[4]), f"int32 products differ {tag}"
        diff = np.count_nonzero(o[5].view(np.uint64) != t[5].view(np.uint64))
        assert diff == 0, f"{diff} FP64 outputs differ {tag}"
    assert cnt == cnt_ref


def test_public_call_bit_exact_vs_reference_library(g2, ref, cuda):
    """Same inputs through the reference's ggemm_grouped_dgemm and ours (EMU_GROUPED, fixed N
    and adaptive N, repair COUNT): identical bytes."""
    L = ref.L
    L.ggemm_create.argtypes = [ctypes.POINTER(c_void_p), c_int, c_size_t, c_size_t, c_size_t,
                               c_void_p]
    L.ggemm_grouped_dgemm.argtypes = [c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p]
    L.ggemm_destroy.argtypes = [c_void_p]
    probs = _make(4242)
    for num_moduli in (15, 0):
        outs = []
        for which in ("ref", "ours"):
            keep, entries = [], []
            for p in probs:
                dA, dB = torch.from_numpy(p["A"]).cuda(), torch.from_numpy(p["B"]).cuda()
                dC = torch.from_numpy(p["C0"].copy()).cuda()
                keep.append((dA, dB, dC))
                entries.append(dict(m=p["m"], n=p["n"], k=p["k"], A=dA.data_ptr(), lda=p["lda"],
                                    B=dB.data_ptr(), ldb=p["ldb"], C=dC.data_ptr(), ldc=p["ldc"],
                                    alpha=p["alpha"], beta=p["beta"]))
            P = g2.make_problems(entries)
            ta = sum(p["m"] * p["k"] for p in probs) + 1
            tb = sum(p["k"] * p["n"] for p in probs) + 1
            tc = sum(p["m"] * p["n"] for p in probs) + 1
            cfg = g2.config(num_moduli, 1e-15, 0, 0)
            if which == "ref":
                h = c_void_p()
                assert L.ggemm_create(ctypes.byref(h), len(probs), ta, tb, tc,
                                      torch.cuda.current_stream().cuda_stream) == 0
                rc = L.ggemm_grouped_dgemm(h, g2.PATH_EMU_GROUPED, ctypes.addressof(cfg),
                                           ctypes.addressof(P), len(probs), None)
                torch.cuda.synchronize()
                L.ggemm_destroy(h)
            else:
                with g2.Handle(len(probs), ta, tb, tc,
                               stream=torch.cuda.current_stream().cuda_stream) as hh:
                    rc, _ = hh.grouped_dgemm(g2.PATH_EMU_GROUPED, cfg, P, len(probs))
                    torch.cuda.synchronize()
            assert rc == 0
            outs.append([dC.cpu().numpy() for _, _, dC in keep])
        for a, b, p in zip(outs[0], outs[1], probs):
            assert np.array_equal(a.view(np.uint64), b.view(np.uint64)), (p["m"], p["n"], p["k"])
