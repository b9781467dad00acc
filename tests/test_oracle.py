"""The CPU oracle pinned before it is trusted.

1. Its CRT tables are byte-identical to the reference's own (src/moduli.h:124-181, built from
   the reference sources in oracle/_ref) and to the product library's host tables.
2. Published values: the choose(k, 1e-15) table printed by the reference
   (results/numerics_perf_511101.log:1-15) and the per-N constants re-derived from the
   reference's host code (log2 P, log2 u1, T, bounds).
3. Exact residue check in the style of the reference's test_numerics_standalone.cu:210-258:
   trunc(2^s a) computed with exact rational arithmetic, residues with Python integers.
"""
import ctypes
import math
from fractions import Fraction

import numpy as np
import pytest

from g2util import col_major, decode_tables, gen

MODULI = [256, 255, 253, 251, 247, 239, 233, 229, 227, 223, 217, 211, 199, 197, 193, 191, 181,
          179, 173, 167]


_tables = decode_tables


def test_tables_identical_to_reference(oracle, ref):
    assert oracle.tables_bytes() == ref.tables_bytes()


def test_product_tables_identical_to_oracle(g2, oracle):
    n = g2.lib.ggemm_stage_crt_tables(None, 0)
    buf = (ctypes.c_ubyte * n)()
    assert g2.lib.ggemm_stage_crt_tables(buf, n) == n
    assert bytes(buf) == oracle.tables_bytes()


def test_tables_exact_integers(oracle):
    """Integer constants re-derived with Python big integers."""
    t = _tables(oracle.tables_bytes())
    assert list(t["p"]) == MODULI
    for N in (1, 8, 14, 15, 16, 20):
        P = math.prod(MODULI[:N])
        M = [P // p for p in MODULI[:N]]
        sh = max(x.bit_length() for x in M) - 49
        assert t["log2_u1"][N] == sh
        for l in range(N):
            assert (M[l] % MODULI[l]) * int(t["qinv"][N][l]) % MODULI[l] == 1 % MODULI[l]
            assert int(t["s1"][N][l]) == (M[l] >> sh if sh >= 0 else M[l] << -sh)
        assert int(t["P1"][N]) == (P >> sh if sh >= 0 else P << -sh)


def test_published_constants(oracle):
    """Values of the reference host code (src/moduli.h:124-181, src/ozaki2_numerics.cu:639-673,
    re-derived from its sources): log2 P, log2 u1, T, bounds."""
    t = _tables(oracle.tables_bytes())
    rows = {
        8: (63.50, 7, 2.5551e9, 2.505e-8, 1.002e-7, 1.417e-7),
        13: (102.25, 46, 1.7353e15, 3.699e-14, 1.476e-13, 2.087e-13),
        14: (109.87, 54, 2.4356e16, 2.740e-15, 1.062e-14, 1.498e-14),
        15: (117.46, 61, 3.3837e17, 3.008e-16, 8.683e-16, 1.182e-15),
        16: (125.04, 69, 4.6763e18, 1.257e-16, 1.667e-16, 1.894e-16),
        20: (154.84, 99, 1.4307e23, 1.123e-16, 1.123e-16, 1.124e-16),
    }
    for N, (lp, lu1, T, b256, b4096, b8192) in rows.items():
        assert round(float(t["log2P"][N]), 2) == lp
        assert t["log2_u1"][N] == lu1
        assert float(t["T"][N]) == pytest.approx(T, rel=1e-4)
        assert oracle.error_bound(256, N) == pytest.approx(b256, rel=1e-3)
        assert oracle.error_bound(4096, N) == pytest.approx(b4096, rel=1e-3)
        assert oracle.error_bound(8192, N) == pytest.approx(b8192, rel=1e-3)


def test_choose_tables(oracle):
    """The published choose table, results/numerics_perf_511101.log:1-15."""
    got = {k: oracle.choose(k, 1e-15) for k in (256, 1024, 4096, 16384, 65536, 131072)}
    assert got == {256: 15, 1024: 15, 4096: 15, 16384: 16, 65536: 16, 131072: -1}
    assert oracle.choose(16, 1e-15) == 14
    for k in (32, 64, 1000, 2048, 4096):
        assert oracle.choose(k, 1e-15) == 15
    for k in (8192, 50000, 131040):
        assert oracle.choose(k, 1e-15) == 16
    for k in (17, 100, 2048):
        assert oracle.choose_cw(k, 16.0) == 15
    for k in (4096, 20000, 131040):
        assert oracle.choose_cw(k, 16.0) == 14


def test_bounds_and_choice_match_reference(oracle, ref, g2):
    for k in list(range(0, 300, 7)) + [1000, 4096, 8192, 65536, 131040, 131041]:
        for N in range(1, 21):
            b = oracle.error_bound(k, N)
            assert b == ref.L.ozr_error_bound(k, N)
            assert b == g2.lib.ggemm_stage_error_bound(k, N)
        for target in (1e-15, 1e-12, 1e-8, 3e-16):
            assert oracle.choose(k, target) == ref.L.ozr_choose(k, target)
        for rho in (1.0, 16.0, 100.0):
            assert oracle.choose_cw(k, rho) == ref.L.ozr_choose_cw(k, rho)


def _exact_residues(X, rows, k, ld, kind, ws, N, T):
    """Returns the exact expected planes [N, rows, kp] from the oracle's shifts."""
    kp = (k + 31) // 32 * 32
    out = np.zeros((N, rows, kp), dtype=np.int64)
    for r in range(rows):
        s = int(ws[r])
        if s == -(2**31):
            continue
        n2 = 0
        for q in range(k):
            a = X[r + q * ld] if kind == 0 else X[q + r * ld]
            x = Fraction(float(a)) * (Fraction(2) ** s)
            xi = math.trunc(x)
            n2 += xi * xi
            for l in range(N):
                p = MODULI[l]
                v = xi % p
                if v > (p - 1) // 2:
                    v -= p
                out[l, r, q] = v
        assert math.isqrt(n2) <= T
    return out


@pytest.mark.parametrize("N,kind", [(1, 0), (8, 0), (13, 1), (20, 0), (15, 1)])
def test_oracle_residues_exact(oracle, N, kind):
    rows, k = 11, 45
    rng = np.random.default_rng(N * 10 + kind)
    mat = gen(rng, (rows, k), 2.0)
    mat[3, :] = 0.0
    if kind == 0:
        ld = rows + 2
        X = col_major(mat, ld)
    else:
        ld = k + 3
        X = col_major(mat.T, ld)
    planes, ws, _ = oracle.prep(X, rows, k, ld, N, kind)
    t = _tables(oracle.tables_bytes())
    want = _exact_residues(X, rows, k, ld, kind, ws, N, float(t["T"][N]))
    assert np.array_equal(planes[:N].astype(np.int64), want)
    # abs plane in [0, 127], zero row -> zero abs shift marker
    assert planes[N].min() >= 0 and planes[N].max() <= 127
    assert ws[rows + 3] == -(2**31) + 1


def test_oracle_gemm_and_crt_roundtrip(oracle):
    """The CRT of exact products reproduces A'B' exactly (up to the u1 rounding of xr)."""
    rng = np.random.default_rng(5)
    m, n, k, N = 6, 5, 70, 15
    A = gen(rng, (m, k), 1.0)
    B = gen(rng, (k, n), 1.0)
    Af, Bf = col_major(A, m), col_major(B, k)
    A8, rs, _ = oracle.prep(Af, m, k, m, N, 0)
    B8, cs, _ = oracle.prep(Bf, n, k, k, N, 1)
    t = _tables(oracle.tables_bytes())
    for i in range(m):
        for j in range(n):
            ap = [math.trunc(Fraction(float(A[i, q])) * Fraction(2) ** int(rs[i])) for q in range(k)]
            bp = [math.trunc(Fraction(float(B[q, j])) * Fraction(2) ** int(cs[j])) for q in range(k)]
            X = sum(a * b for a, b in zip(ap, bp))
            planes = np.array([oracle.i8_gemm(A8[l, i:i + 1], B8[l, j:j + 1])[0]
                               for l in range(N + 1)], dtype=np.int32)
            S1 = ctypes.c_uint64()
            S2 = ctypes.c_uint32()
            Q = ctypes.c_double()
            xr = ctypes.c_double()
            oracle.L.ozo_crt_entry(N, planes.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), 1,
                                   ctypes.byref(S1), ctypes.byref(S2), ctypes.byref(Q),
                                   ctypes.byref(xr))
            u1 = Fraction(2) ** int(t["log2_u1"][N])
            err = abs(Fraction(xr.value) - Fraction(X) / u1)
            assert err <= Fraction(N * 255, 2 ** 19) + Fraction(1, 2 ** 10) + abs(Fraction(X) / u1) / 2 ** 51
