"""Stage-by-stage parity of the CUDA path against the CPU oracle (bit-exact).

prep: residues of every plane, row/column workspace {shift, abs shift, ||dX||, ||X'||} and the
non-finite counter (reference src/ozaki2_numerics.cu:242-442).  GEMM: exact int32 products of
every plane (src/int8_grouped_gemm.h:4-10).  Reconstruct: FP64 outputs and counters for every
repair mode (src/ozaki2_numerics.cu:454-586).  Inputs are seeded; the checker runs on the CPU.
"""
import ctypes

import numpy as np
import pytest

from g2util import col_major, decode_tables, gen

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _scratch(g2, num):
    return torch.empty(g2.lib.ggemm_stage_scratch_bytes(num), dtype=torch.uint8, device="cuda")


def _counters():
    return torch.zeros(64, dtype=torch.uint8, device="cuda")


def _counter_values(c):
    v = c.cpu().numpy().view(np.uint64)
    return [int(x) for x in v[:4]], int(c.cpu().numpy()[32:36].view(np.uint32)[0])


def run_prep(g2, X: np.ndarray, rows, k, ld, N, kind, poison=0x5A):
    pb = (g2.img_plane_bytes(rows, k) + 255) // 256 * 256
    Xd = torch.from_numpy(np.ascontiguousarray(X)).cuda()
    img = torch.full(((N + 1) * pb + 256,), poison, dtype=torch.int8, device="cuda")
    ws = torch.zeros(4 * max(rows, 1), dtype=torch.int32, device="cuda")
    d = (g2.PrepDesc * 1)()
    d[0] = g2.PrepDesc(Xd.data_ptr(), ld, rows, k, N, kind, img.data_ptr(), pb, ws.data_ptr())
    scr, cnt = _scratch(g2, 1), _counters()
    rc = g2.lib.ggemm_stage_prep(d, 1, scr.data_ptr(), scr.numel(), cnt.data_ptr(),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    img_h = img.cpu().numpy()
    planes = np.stack([g2.unpack_plane(img_h[l * pb:(l + 1) * pb], rows, k) for l in range(N + 1)])
    return planes, ws.cpu().numpy()[: 4 * rows], _counter_values(cnt), img_h, pb


PREP_CASES = [
    # rows, k, N, kind, phi, special
    (37, 100, 1, 0, 2.0, None),
    (37, 100, 8, 0, 2.0, None),
    (37, 100, 13, 0, 2.0, None),
    (37, 100, 20, 0, 2.0, None),
    (29, 100, 15, 1, 2.0, None),
    (29, 100, 20, 1, 4.0, None),
    (64, 777, 15, 0, 1.0, None),
    (48, 777, 16, 1, 0.5, None),
    (5, 3000, 15, 0, 2.0, None),
    (33, 33, 14, 1, 0.0, None),
    (40, 300, 14, 0, 1.0, "zero_row"),
    (40, 300, 14, 1, 1.0, "zero_row"),
    (20, 512, 18, 0, 1.0, "tiny"),
    (20, 512, 18, 1, 1.0, "huge"),
    (50, 200, 16, 0, 1.0, "nan"),
    (40, 200, 16, 1, 1.0, "inf"),
    (1, 1, 15, 0, 1.0, None),
    (1, 1, 15, 1, 1.0, None),
    (300, 64, 16, 0, 4.0, None),
]


@pytest.mark.parametrize("rows,k,N,kind,phi,special", PREP_CASES)
def test_prep_matches_oracle(g2, oracle, cuda, rows, k, N, kind, phi, special):
    rng = np.random.default_rng(1000 + rows * 7 + k + N * 13 + kind)
    mat = gen(rng, (rows, k), phi)  # row r, depth q
    if special == "zero_row":
        mat[3, :] = 0.0
    elif special == "tiny":
        mat *= 2.0 ** -700
    elif special == "huge":
        mat *= 2.0 ** 650
    elif special == "nan":
        mat[2, 17] = np.nan
    elif special == "inf":
        mat[4, 33] = np.inf
    if kind == 0:
        ld = rows + 3
        X = col_major(mat, ld)  # A: element (r, q) at r + q*ld
    else:
        ld = k + 5
        X = col_major(mat.T, ld)  # B (k x n): element (q, r) at q + r*ld
    planes, ws, (cnt, status), img_h, pb = run_prep(g2, X, rows, k, ld, N, kind)
    ref_planes, ref_ws, ref_nf = oracle.prep(X, rows, k, ld, N, kind)
    assert status == 0
    np.testing.assert_array_equal(ws, ref_ws)
    for l in range(N + 1):
        bad = np.argwhere(planes[l] != ref_planes[l])
        assert bad.size == 0, f"plane {l}: {len(bad)} mismatches, first {bad[:4].tolist()}"
    assert cnt[0] == ref_nf
    # padding rows of the last row group are zero in every plane
    kp = (k + 31) // 32 * 32
    rg = (rows + 7) // 8
    if rows % 8:
        for l in range(N + 1):
            r = np.arange(rows, rg * 8)[:, None]
            q = np.arange(kp)[None, :]
            rr, qq = r & 7, q & 31
            off = ((q >> 5) * rg + (r >> 3)) * 256 + rr * 32 + (((qq >> 4) ^ (rr >> 2)) << 4) + (qq & 15)
            assert np.all(img_h[l * pb + off] == 0)


def qscale_planes(planes: np.ndarray, N: int, t) -> np.ndarray:
    """Residue planes of x -> residue planes of q_l x (GGEMM_PREP_QSCALED): the symmetric
    representative for odd p_l, the two's complement low byte for p_0 = 256; abs plane kept."""
    out = planes.copy()
    for l in range(N):
        p, q = int(t["p"][l]), int(t["qinv"][N][l])
        s = (planes[l].astype(np.int64) % p) * q % p
        s = np.where(2 * s > p, s - p, s)
        out[l] = (s & 255).astype(np.uint8).view(np.int8)
    return out


@pytest.mark.parametrize("rows,k,N,kind,phi,special",
                         [c for c in PREP_CASES if c[3] == 0 and c[5] in (None, "nan", "tiny")])
def test_prep_qscaled_matches_oracle(g2, oracle, cuda, rows, k, N, kind, phi, special):
    """kind | GGEMM_PREP_QSCALED: plane l < N holds the residues of q_l x, the workspace and the
    abs plane are those of the unscaled prep."""
    rng = np.random.default_rng(2000 + rows * 7 + k + N * 13)
    mat = gen(rng, (rows, k), phi)
    if special == "tiny":
        mat *= 2.0 ** -700
    elif special == "nan":
        mat[2, 17] = np.nan
    ld = rows + 3
    X = col_major(mat, ld)
    planes, ws, (cnt, status), _, _ = run_prep(g2, X, rows, k, ld, N, kind | g2.PREP_QSCALED)
    ref_planes, ref_ws, ref_nf = oracle.prep(X, rows, k, ld, N, kind)
    assert status == 0
    np.testing.assert_array_equal(ws, ref_ws)
    want = qscale_planes(ref_planes, N, decode_tables(oracle.tables_bytes()))
    for l in range(N + 1):
        bad = np.argwhere(planes[l] != want[l])
        assert bad.size == 0, f"plane {l}: {len(bad)} mismatches, first {bad[:4].tolist()}"
    assert cnt[0] == ref_nf


def run_gemm(g2, A8s, B8s, ks):
    """A8s[i]: planes x m x kp int8, B8s[i]: planes x n x kp.  Returns list of planes x m*n."""
    descs = (g2.GemmDesc * len(A8s))()
    keep = []
    outs = []
    for i, (A8, B8, k) in enumerate(zip(A8s, B8s, ks)):
        P, m, _ = A8.shape
        n = B8.shape[1]
        pa = (g2.img_plane_bytes(m, k) + 255) // 256 * 256
        pbb = (g2.img_plane_bytes(n, k) + 255) // 256 * 256
        ha = np.zeros(P * pa, dtype=np.int8)
        hb = np.zeros(P * pbb, dtype=np.int8)
        for l in range(P):
            ha[l * pa:l * pa + g2.img_plane_bytes(m, k)] = g2.pack_plane(A8[l], k)
            hb[l * pbb:l * pbb + g2.img_plane_bytes(n, k)] = g2.pack_plane(B8[l], k)
        da = torch.from_numpy(ha).cuda()
        db = torch.from_numpy(hb).cuda()
        cp = (m * n + 63) // 64 * 64
        dc = torch.full((P * cp + 64,), 0x7F7F7F7F, dtype=torch.int32, device="cuda")
        keep += [da, db]
        outs.append((dc, P, m, n, cp))
        descs[i] = g2.GemmDesc(da.data_ptr(), db.data_ptr(), dc.data_ptr(), pa, pbb, cp, m, n, k, P)
    scr, cnt = _scratch(g2, len(A8s)), _counters()
    rc = g2.lib.ggemm_stage_gemm(descs, len(A8s), scr.data_ptr(), scr.numel(), cnt.data_ptr(),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    _, status = _counter_values(cnt)
    assert status == 0
    res = []
    for dc, P, m, n, cp in outs:
        h = dc.cpu().numpy()
        res.append(np.stack([h[l * cp:l * cp + m * n] for l in range(P)]))
    return res


def _i8(rng, shape, k):
    a = rng.integers(-128, 128, size=shape, dtype=np.int16).astype(np.int8)
    kp = (k + 31) // 32 * 32
    out = np.zeros(shape[:-1] + (kp,), dtype=np.int8)
    out[..., :k] = a[..., :k]
    return out


def _ref_gemm(A8, B8):
    return np.stack([(A8[l].astype(np.int64) @ B8[l].astype(np.int64).T).T.reshape(-1)
                     for l in range(A8.shape[0])])


GEMM_SHAPES = [(1, 1, 1), (7, 13, 33), (128, 128, 128), (130, 257, 1000), (33, 65, 2048),
               (300, 200, 4096), (256, 384, 96), (129, 127, 31)]


def test_gemm_bit_exact_grouped(g2, cuda):
    rng = np.random.default_rng(1234)
    A8s, B8s, ks = [], [], []
    for i, (m, n, k) in enumerate(GEMM_SHAPES):
        P = 1 + (i % 3)
        A8s.append(_i8(rng, (P, m, k), k))
        B8s.append(_i8(rng, (P, n, k), k))
        ks.append(k)
    outs = run_gemm(g2, A8s, B8s, ks)
    for (m, n, k), A8, B8, C in zip(GEMM_SHAPES, A8s, B8s, outs):
        ref = _ref_gemm(A8, B8)
        assert np.array_equal(C.astype(np.int64), ref), f"mismatch for {(m, n, k)}"


def test_gemm_int32_edge_all_minus128(g2, cuda):
    """kp = 131040 with every residue -128: |sum| = 128^2 * 131040 < 2^31 (the exactness limit
    of the reference, src/int8_grouped_gemm.h:10)."""
    k = 131040
    A8 = np.full((1, 8, k), -128, dtype=np.int8)
    B8 = np.full((1, 16, k), -128, dtype=np.int8)
    C = run_gemm(g2, [A8], [B8], [k])[0]
    assert np.all(C == 128 * 128 * k)


def _oracle_pipeline_inputs(oracle, m, n, k, N, phi, seed, pad=3):
    rng = np.random.default_rng(seed)
    A = gen(rng, (m, k), phi)
    B = gen(rng, (k, n), phi)
    C0 = gen(rng, (m, n), 0.0)
    lda, ldb, ldc = m + pad, k + pad, m + pad
    Af, Bf, Cf = col_major(A, lda), col_major(B, ldb), col_major(C0, ldc)
    kp = (k + 31) // 32 * 32
    A8, rs, _ = oracle.prep(Af, m, k, lda, N, 0)
    B8, cs, _ = oracle.prep(Bf, n, k, ldb, N, 1)
    C32 = np.concatenate([oracle.i8_gemm(A8[l], B8[l]) for l in range(N + 1)])
    return Af, Bf, Cf, lda, ldb, ldc, C32, rs, cs, kp


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("m,n,k,N,phi,alpha,beta", [
    (40, 30, 100, 15, 1.0, 1.0, 0.0),
    (64, 48, 512, 15, 2.0, -1.5, 0.75),
    (16, 16, 16, 15, 2.0, 1.0, 0.0),
    (33, 65, 2048, 10, 4.0, 1.0, 0.25),
    (7, 13, 33, 20, 0.5, 2.0, 1.0),
])
def test_recon_matches_oracle(g2, oracle, cuda, mode, m, n, k, N, phi, alpha, beta):
    Af, Bf, Cf, lda, ldb, ldc, C32, rs, cs, kp = _oracle_pipeline_inputs(
        oracle, m, n, k, N, phi, seed=m * 31 + n * 7 + k + N)
    want = Cf.copy()
    cnt_ref = oracle.reconstruct(m, n, k, N, alpha, beta, Af, lda, Bf, ldb, want, ldc, C32, rs,
                                 cs, mode)
    dA, dB = torch.from_numpy(Af).cuda(), torch.from_numpy(Bf).cuda()
    dC = torch.from_numpy(Cf.copy()).cuda()
    dC32 = torch.from_numpy(C32).cuda()
    drs, dcs = torch.from_numpy(rs).cuda(), torch.from_numpy(cs).cuda()
    d = (g2.ReconDesc * 1)()
    d[0] = g2.ReconDesc(m, n, k, N, dA.data_ptr(), lda, dB.data_ptr(), ldb, dC.data_ptr(), ldc,
                        alpha, beta, dC32.data_ptr(), m * n, drs.data_ptr(), dcs.data_ptr())
    scr, cnt = _scratch(g2, 1), _counters()
    rc = g2.lib.ggemm_stage_recon(d, 1, mode, scr.data_ptr(), scr.numel(), cnt.data_ptr(),
                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), \
        f"{np.count_nonzero(got.view(np.uint64) != want.view(np.uint64))} entries differ"
    c, _ = _counter_values(cnt)
    assert c[1:] == [int(x) for x in cnt_ref[1:]]


def test_full_api_emu_grouped_matches_oracle(g2, oracle, cuda):
    rng = np.random.default_rng(7)
    shapes = [(200, 150, 777), (1, 300, 64), (300, 1, 129), (77, 55, 1), (64, 48, 512),
              (40, 33, 300), (33, 65, 2048), (16, 16, 16)]
    N = 15
    mode = 1  # COUNT (EMU_GROUPED default)
    probs, keep, wants = [], [], []
    for i, (m, n, k) in enumerate(shapes):
        A = gen(rng, (m, k), 1.0)
        B = gen(rng, (k, n), 1.0)
        C0 = gen(rng, (m, n), 0.0)
        lda, ldb, ldc = m + 2, k + 1, m + 3
        alpha, beta = (1.0, 0.0) if i % 2 == 0 else (-1.25, 0.5)
        Af, Bf, Cf = col_major(A, lda), col_major(B, ldb), col_major(C0, ldc)
        want = Cf.copy()
        oracle.emulated(m, n, k, N, alpha, beta, Af, lda, Bf, ldb, want, ldc, mode)
        dA, dB, dC = (torch.from_numpy(x).cuda() for x in (Af, Bf, Cf.copy()))
        keep.append((dA, dB, dC))
        wants.append(want)
        probs.append(dict(m=m, n=n, k=k, A=dA.data_ptr(), lda=lda, B=dB.data_ptr(), ldb=ldb,
                          C=dC.data_ptr(), ldc=ldc, alpha=alpha, beta=beta))
    P = g2.make_problems(probs)
    tot_a = sum(m * k for m, n, k in shapes)
    tot_b = sum(k * n for m, n, k in shapes)
    tot_c = sum(m * n for m, n, k in shapes)
    stream = torch.cuda.current_stream().cuda_stream
    with g2.Handle(len(shapes), tot_a, tot_b, tot_c, stream=stream) as h:
        cfg = g2.config(num_moduli=N, allow_fallback=0)
        rc, st = h.grouped_dgemm(g2.PATH_EMU_GROUPED, cfg, P, len(shapes))
        torch.cuda.synchronize()
        assert rc == 0, rc
        assert st.kernel_launches == 3
        for (dA, dB, dC), want in zip(keep, wants):
            got = dC.cpu().numpy()
            assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
