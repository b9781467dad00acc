"""Parity of the digit product layout (GGEMM_PRODUCTS_DIGITS) against the CPU oracle.

The reference hands int32 products C_l from its GEMM to its reconstruct, which first reduces
each to the CRT digit y_l = (C_l mod p_l) q_l mod p_l (src/ozaki2_numerics.cu:509-517).  This
library's GEMM epilogue writes y_l directly (one byte per entry and plane, the abs plane as
int32, in 32-column records).  These tests check (1) the digits and abs products the GEMM writes
against digits computed from exact int64 products, including the int32 extremes, and (2) the
reconstruct from digits against the oracle's reconstruct from the int32 products, bit for bit.
"""
import ctypes

import numpy as np
import pytest

from g2util import col_major, decode_tables, gen

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _scratch(g2, num):
    return torch.empty(g2.lib.ggemm_stage_scratch_bytes(num), dtype=torch.uint8, device="cuda")


def _counters():
    return torch.zeros(64, dtype=torch.uint8, device="cuda")


@pytest.fixture(scope="module")
def tables(oracle):
    return decode_tables(oracle.tables_bytes())


def digits_of(C: np.ndarray, N: int, t) -> np.ndarray:
    """(N+1, m, n) int64 products -> (N, m, n) CRT digits."""
    p = t["p"][:N].astype(np.int64)[:, None, None]
    q = t["qinv"][N][:N].astype(np.int64)[:, None, None]
    return (C[:N] % p) * q % p


def records_of(M: np.ndarray, m: int, n: int, w: int) -> np.ndarray:
    """(m, n) matrix -> its records of w columns of one row, the records of a column block row
    after row (the digit layout: w = 16 digit bytes or w = 4 int32 abs products), padded with
    zeros to whole 32-column chunks."""
    nrec = (n + 31) // 32 * (32 // w)
    pad = np.zeros((m, nrec * w), dtype=M.dtype)
    pad[:, :n] = M
    return pad.reshape(m, nrec, w).transpose(1, 0, 2).reshape(-1)


def to_records(Y: np.ndarray, m: int, n: int, yp: int, N: int) -> np.ndarray:
    """(N, m, n) digits -> the digit planes of the layout (padding zero)."""
    out = np.zeros((N, yp), dtype=np.uint8)
    for l in range(N):
        r = records_of(Y[l], m, n, 16)
        out[l, :r.size] = r
    return out


def from_records(buf: np.ndarray, m: int, n: int, w: int = 16) -> np.ndarray:
    """One plane of w-column records -> its (m, n) matrix (padding columns dropped)."""
    nrec = (n + 31) // 32 * (32 // w)
    return buf[:nrec * m * w].reshape(nrec, m, w).transpose(1, 0, 2).reshape(m, nrec * w)[:, :n]


def _rand_planes(rng, P, rows, k, lo=-128, hi=128):
    kp = (k + 31) // 32 * 32
    a = np.zeros((P, rows, kp), dtype=np.int8)
    a[..., :k] = rng.integers(lo, hi, size=(P, rows, k), dtype=np.int16).astype(np.int8)
    return a


def run_gemm_digits(g2, A8s, B8s, ks, Ns, layout=None):
    layout = g2.PRODUCTS_DIGITS if layout is None else layout
    descs = (g2.GemmDesc * len(A8s))()
    keep, outs = [], []
    for i, (A8, B8, k, N) in enumerate(zip(A8s, B8s, ks, Ns)):
        P, m, _ = A8.shape
        n = B8.shape[1]
        assert P == N + 1
        pa = (g2.img_plane_bytes(m, k) + 255) // 256 * 256
        pb = (g2.img_plane_bytes(n, k) + 255) // 256 * 256
        ha = np.zeros(P * pa, dtype=np.int8)
        hb = np.zeros(P * pb, dtype=np.int8)
        for l in range(P):
            ha[l * pa:l * pa + g2.img_plane_bytes(m, k)] = g2.pack_plane(A8[l], k)
            hb[l * pb:l * pb + g2.img_plane_bytes(n, k)] = g2.pack_plane(B8[l], k)
        da, db = torch.from_numpy(ha).cuda(), torch.from_numpy(hb).cuda()
        yp = g2.digit_plane_bytes(m, n)
        dy = torch.full((N * yp + 4 * yp,), 0x5A, dtype=torch.uint8, device="cuda")
        keep += [da, db]
        outs.append((dy, m, n, N, yp))
        descs[i] = g2.GemmDesc(da.data_ptr(), db.data_ptr(), dy.data_ptr(), pa, pb, yp, m, n, k,
                               P, N, layout)
    scr, cnt = _scratch(g2, len(A8s)), _counters()
    assert g2.lib.ggemm_stage_gemm(descs, len(A8s), scr.data_ptr(), scr.numel(), cnt.data_ptr(),
                                   _stream()) == 0
    torch.cuda.synchronize()
    assert int(cnt.cpu().numpy()[32:36].view(np.uint32)[0]) == 0
    res = []
    for dy, m, n, N, yp in outs:
        h = dy.cpu().numpy()
        Y = np.stack([from_records(h[l * yp:(l + 1) * yp], m, n) for l in range(N)])
        L = from_records(h[N * yp:].view(np.int32), m, n, 4)
        res.append((Y, L))
    return res


def _exact(A8, B8):
    return np.stack([A8[l].astype(np.int64) @ B8[l].astype(np.int64).T for l in range(A8.shape[0])])


DIGIT_SHAPES = [(1, 1, 1, 2), (7, 13, 33, 20), (128, 128, 128, 15), (130, 257, 1000, 15),
                (33, 65, 2048, 10), (300, 200, 512, 15), (129, 127, 31, 8), (64, 300, 96, 3)]


def test_gemm_digits_grouped(g2, cuda, tables):
    rng = np.random.default_rng(99)
    A8s, B8s, ks, Ns = [], [], [], []
    for m, n, k, N in DIGIT_SHAPES:
        A8s.append(_rand_planes(rng, N + 1, m, k))
        B8s.append(_rand_planes(rng, N + 1, n, k))
        ks.append(k)
        Ns.append(N)
    outs = run_gemm_digits(g2, A8s, B8s, ks, Ns)
    for (m, n, k, N), A8, B8, (Y, L) in zip(DIGIT_SHAPES, A8s, B8s, outs):
        C = _exact(A8, B8)
        assert np.array_equal(Y.astype(np.int64), digits_of(C, N, tables)), (m, n, k, N)
        assert np.array_equal(L.astype(np.int64), C[N]), (m, n, k, N)


def qscale(A8: np.ndarray, N: int, t) -> np.ndarray:
    """A residue planes -> q_l-scaled planes (GGEMM_PREP_QSCALED); the abs plane is kept."""
    out = A8.copy()
    for l in range(N):
        p, q = int(t["p"][l]), int(t["qinv"][N][l])
        s = (A8[l].astype(np.int64) % p) * q % p
        out[l] = (np.where(2 * s > p, s - p, s) & 255).astype(np.uint8).view(np.int8)
    return out


def test_gemm_digits_qscaled(g2, cuda, tables):
    """GGEMM_PRODUCTS_DIGITS_QSCALED: from q-scaled A images the epilogue reduces C'_l mod p_l
    only; the digits equal those of the unscaled products."""
    rng = np.random.default_rng(199)
    A8s, As, B8s, ks, Ns = [], [], [], [], []
    for m, n, k, N in DIGIT_SHAPES:
        A8 = _rand_planes(rng, N + 1, m, k)
        A8s.append(A8)
        As.append(qscale(A8, N, tables))
        B8s.append(_rand_planes(rng, N + 1, n, k))
        ks.append(k)
        Ns.append(N)
    outs = run_gemm_digits(g2, As, B8s, ks, Ns, g2.PRODUCTS_DIGITS_QSCALED)
    for (m, n, k, N), A8, B8, (Y, L) in zip(DIGIT_SHAPES, A8s, B8s, outs):
        C = _exact(A8, B8)
        assert np.array_equal(Y.astype(np.int64), digits_of(C, N, tables)), (m, n, k, N)
        assert np.array_equal(L.astype(np.int64), C[N]), (m, n, k, N)


@pytest.mark.parametrize("sa,sb", [(-128, -128), (-128, 127), (127, -128), (127, 127)])
def test_gemm_digits_qscaled_int32_extremes(g2, cuda, tables, sa, sb):
    """The q-scaled digit at the int32 limit: k = 131040 with constant scaled residues, so that
    C'_l sits at +-128^2 k or +-127^2 k."""
    k, N = 131040, 20
    A8 = np.full((N + 1, 8, k), sa, dtype=np.int8)
    B8 = np.full((N + 1, 40, k), sb, dtype=np.int8)
    Y, L = run_gemm_digits(g2, [A8], [B8], [k], [N], g2.PRODUCTS_DIGITS_QSCALED)[0]
    # A8 here already stands for the scaled residues: the digit is C' mod p_l
    p = tables["p"][:N].astype(np.int64)[:, None, None]
    assert np.array_equal(Y.astype(np.int64), np.full((N, 8, 40), sa * sb * k, np.int64) % p)
    assert np.array_equal(L.astype(np.int64), np.full((8, 40), sa * sb * k, np.int64))


@pytest.mark.parametrize("sa,sb", [(-128, -128), (-128, 127), (127, -128)])
def test_gemm_digits_int32_extremes(g2, cuda, tables, sa, sb):
    """k = 131040 with constant residues: products at +-128^2 k (the int32 exactness limit of
    the reference, src/int8_grouped_gemm.h:10) still give exact digits."""
    k, N = 131040, 20
    A8 = np.full((N + 1, 8, k), sa, dtype=np.int8)
    B8 = np.full((N + 1, 40, k), sb, dtype=np.int8)
    Y, L = run_gemm_digits(g2, [A8], [B8], [k], [N])[0]
    C = np.full((N + 1, 8, 40), sa * sb * k, dtype=np.int64)
    assert np.array_equal(Y.astype(np.int64), digits_of(C, N, tables))
    assert np.array_equal(L.astype(np.int64), C[N])


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("m,n,k,N,phi,alpha,beta", [
    (40, 30, 100, 15, 1.0, 1.0, 0.0),
    (64, 48, 512, 15, 2.0, -1.5, 0.75),
    (70, 100, 16, 15, 2.0, 1.0, 0.0),
    (33, 65, 2048, 10, 4.0, 1.0, 0.25),
    (7, 13, 33, 20, 0.5, 2.0, 1.0),
    (129, 33, 300, 2, 1.0, 0.5, -2.0),
])
def test_recon_digits_matches_oracle(g2, oracle, cuda, tables, mode, m, n, k, N, phi, alpha,
                                     beta):
    rng = np.random.default_rng(m * 131 + n * 17 + k + N)
    A, B, C0 = gen(rng, (m, k), phi), gen(rng, (k, n), phi), gen(rng, (m, n), 0.0)
    lda, ldb, ldc = m + 3, k + 1, m + 2
    Af, Bf, Cf = col_major(A, lda), col_major(B, ldb), col_major(C0, ldc)
    A8, rs, _ = oracle.prep(Af, m, k, lda, N, 0)
    B8, cs, _ = oracle.prep(Bf, n, k, ldb, N, 1)
    C32 = np.concatenate([oracle.i8_gemm(A8[l], B8[l]) for l in range(N + 1)])
    want = Cf.copy()
    cnt_ref = oracle.reconstruct(m, n, k, N, alpha, beta, Af, lda, Bf, ldb, want, ldc, C32, rs,
                                 cs, mode)
    # int32 products (column-major planes) -> digit layout
    C = C32.astype(np.int64).reshape(N + 1, n, m).transpose(0, 2, 1)
    yp = g2.digit_plane_bytes(m, n)
    buf = np.zeros(N * yp + 4 * yp, dtype=np.uint8)
    buf[:N * yp] = to_records(digits_of(C, N, tables).astype(np.uint8), m, n, yp, N).reshape(-1)
    Lrec = np.zeros(yp, dtype=np.int32)
    r = records_of(C[N].astype(np.int32), m, n, 4)
    Lrec[:r.size] = r
    buf[N * yp:] = Lrec.view(np.uint8)
    dA, dB = torch.from_numpy(Af).cuda(), torch.from_numpy(Bf).cuda()
    dC = torch.from_numpy(Cf.copy()).cuda()
    dY = torch.from_numpy(buf).cuda()
    drs, dcs = torch.from_numpy(rs).cuda(), torch.from_numpy(cs).cuda()
    d = (g2.ReconDesc * 1)()
    d[0] = g2.ReconDesc(m, n, k, N, dA.data_ptr(), lda, dB.data_ptr(), ldb, dC.data_ptr(), ldc,
                        alpha, beta, dY.data_ptr(), yp, drs.data_ptr(), dcs.data_ptr(),
                        g2.PRODUCTS_DIGITS)
    scr, cnt = _scratch(g2, 1), _counters()
    assert g2.lib.ggemm_stage_recon(d, 1, mode, scr.data_ptr(), scr.numel(), cnt.data_ptr(),
                                    _stream()) == 0
    torch.cuda.synchronize()
    got = dC.cpu().numpy()
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), \
        f"{np.count_nonzero(got.view(np.uint64) != want.view(np.uint64))} entries differ"
    c = [int(x) for x in cnt.cpu().numpy().view(np.uint64)[:4]]
    assert c[1:] == [int(x) for x in cnt_ref[1:]]


def test_stage_rejects_bad_digit_descs(g2, cuda):
    """Digit descriptors with a misaligned plane stride or N out of range are refused."""
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    d = (g2.GemmDesc * 1)()
    p = buf.data_ptr()
    for N, yp, planes in [(0, 256, 1), (21, 256, 22), (4, 250, 5), (4, 256, 6), (4, 0, 5)]:
        d[0] = g2.GemmDesc(p, p, p, 256, 256, yp, 8, 8, 32, planes, N, g2.PRODUCTS_DIGITS)
        scr, cnt = _scratch(g2, 1), _counters()
        assert g2.lib.ggemm_stage_gemm(d, 1, scr.data_ptr(), scr.numel(), cnt.data_ptr(),
                                       _stream()) == g2.ERR_INVALID, (N, yp, planes)
