"""Shared test helpers: package loader, ctypes bindings of the checkers, seeded inputs.

The checkers are test infrastructure: the plain-C restatement in oracle/ (liboz2_oracle.so)
and the reference implementation built from its own sources (oracle/_ref/libggemm_ref.so).
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import sys
from ctypes import POINTER, c_double, c_int, c_size_t, c_uint64, c_void_p

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "coding-basic-hw-2_b200")
ORACLE_SO = os.path.join(ROOT, "oracle", "liboz2_oracle.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libggemm_ref.so")


def load_pkg():
    """Imports the product package (its directory name is not a Python identifier)."""
    if "ggemm_b200" in sys.modules:
        return sys.modules["ggemm_b200"]
    spec = importlib.util.spec_from_file_location(
        "ggemm_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ggemm_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def gen(rng: np.random.Generator, shape, phi: float) -> np.ndarray:
    """(U(0,1) - 0.5) * exp(phi * N(0,1)): the reference's test-matrix convention
    (bench/workloads.h:26-27)."""
    u = rng.random(shape)
    if phi == 0.0:
        return u - 0.5
    return (u - 0.5) * np.exp(phi * rng.standard_normal(shape))


def col_major(a: np.ndarray, ld: int) -> np.ndarray:
    """rows x cols matrix -> flat column-major buffer with leading dimension ld (padding 0)."""
    rows, cols = a.shape
    buf = np.zeros(ld * max(cols, 1), dtype=np.float64)
    if rows and cols:
        buf.reshape(max(cols, 1), ld)[:cols, :rows] = a.T
    return buf


_i8p = POINTER(ctypes.c_int8)
_i32p = POINTER(ctypes.c_int32)
_f64p = POINTER(c_double)
_u64p = POINTER(c_uint64)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class Oracle:
    """ctypes view of oracle/liboz2_oracle.so."""

    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} missing: make -C oracle")
        L = ctypes.CDLL(ORACLE_SO)
        L.ozo_tables_size.restype = c_size_t
        L.ozo_error_bound.restype = c_double
        L.ozo_error_bound.argtypes = [c_int, c_int]
        L.ozo_choose_num_moduli.argtypes = [c_int, c_double]
        L.ozo_choose_num_moduli_cw.argtypes = [c_int, c_double]
        L.ozo_prep_rows.argtypes = [_f64p, c_int, c_int, c_int, c_int, c_int, _i8p, _i32p, _u64p]
        L.ozo_prep_cols.argtypes = [_f64p, c_int, c_int, c_int, c_int, c_int, _i8p, _i32p, _u64p]
        L.ozo_i8_gemm.argtypes = [_i8p, _i8p, c_int, c_int, c_int, _i32p]
        L.ozo_reconstruct.argtypes = [c_int, c_int, c_int, c_int, c_double, c_double, _f64p, c_int,
                                      _f64p, c_int, _f64p, c_int, _i32p, _i32p, _i32p, c_int, _u64p]
        L.ozo_crt_entry.argtypes = [c_int, _i32p, c_size_t, _u64p, POINTER(ctypes.c_uint32),
                                    _f64p, _f64p]
        L.ozo_emulated_dgemm.argtypes = [c_int, c_int, c_int, c_int, c_double, c_double, _f64p,
                                         c_int, _f64p, c_int, _f64p, c_int, c_int, _u64p]
        L.ozo_dgemm_naive.argtypes = [c_int, c_int, c_int, c_double, _f64p, c_int, _f64p, c_int,
                                      c_double, _f64p, c_int, c_int, c_int, c_int]
        self.L = L

    def tables_bytes(self) -> bytes:
        n = self.L.ozo_tables_size()
        b = (ctypes.c_ubyte * n)()
        assert self.L.ozo_build_tables(b) == 0
        return bytes(b)

    def error_bound(self, k, N):
        return self.L.ozo_error_bound(k, N)

    def choose(self, k, target):
        return self.L.ozo_choose_num_moduli(k, target)

    def choose_cw(self, k, rho):
        return self.L.ozo_choose_num_moduli_cw(k, rho)

    def prep(self, X: np.ndarray, rows: int, k: int, ld: int, N: int, kind: int):
        """X flat column-major buffer.  Returns (planes [(N+1), rows, kp] int8, ws [4 rows] int32,
        nonfinite count)."""
        kp = (k + 31) // 32 * 32
        out = np.zeros((N + 1) * max(rows, 1) * max(kp, 1), dtype=np.int8)
        ws = np.zeros(4 * max(rows, 1), dtype=np.int32)
        nf = np.zeros(1, dtype=np.uint64)
        X = np.ascontiguousarray(X, dtype=np.float64)
        fn = self.L.ozo_prep_rows if kind == 0 else self.L.ozo_prep_cols
        fn(_ptr(X, _f64p), rows, k, ld, N, kp, _ptr(out, _i8p), _ptr(ws, _i32p), _ptr(nf, _u64p))
        return (out[: (N + 1) * rows * kp].reshape(N + 1, rows, kp), ws[: 4 * rows], int(nf[0]))

    def i8_gemm(self, A8: np.ndarray, B8: np.ndarray) -> np.ndarray:
        """A8 m x kp, B8 n x kp (int8) -> C32 m x n, returned as the column-major flat buffer."""
        m, kp = A8.shape
        n = B8.shape[0]
        A8 = np.ascontiguousarray(A8, dtype=np.int8)
        B8 = np.ascontiguousarray(B8, dtype=np.int8)
        C = np.zeros(max(m * n, 1), dtype=np.int32)
        assert self.L.ozo_i8_gemm(_ptr(A8, _i8p), _ptr(B8, _i8p), m, n, kp, _ptr(C, _i32p)) == 0
        return C[: m * n]

    def reconstruct(self, m, n, k, N, alpha, beta, A, lda, B, ldb, C, ldc, C32, rs, cs, mode):
        """C (flat column-major, ldc) updated in place; returns counters [4]."""
        cnt = np.zeros(4, dtype=np.uint64)
        A = np.ascontiguousarray(A, dtype=np.float64)
        B = np.ascontiguousarray(B, dtype=np.float64)
        C32 = np.ascontiguousarray(C32, dtype=np.int32)
        rs = np.ascontiguousarray(rs, dtype=np.int32)
        cs = np.ascontiguousarray(cs, dtype=np.int32)
        self.L.ozo_reconstruct(m, n, k, N, alpha, beta, _ptr(A, _f64p), lda, _ptr(B, _f64p), ldb,
                               _ptr(C, _f64p), ldc, _ptr(C32, _i32p), _ptr(rs, _i32p),
                               _ptr(cs, _i32p), mode, _ptr(cnt, _u64p))
        return cnt

    def emulated(self, m, n, k, N, alpha, beta, A, lda, B, ldb, C, ldc, mode):
        cnt = np.zeros(4, dtype=np.uint64)
        A = np.ascontiguousarray(A, dtype=np.float64)
        B = np.ascontiguousarray(B, dtype=np.float64)
        rc = self.L.ozo_emulated_dgemm(m, n, k, N, alpha, beta, _ptr(A, _f64p), lda,
                                       _ptr(B, _f64p), ldb, _ptr(C, _f64p), ldc, mode,
                                       _ptr(cnt, _u64p))
        assert rc == 0
        return cnt

    def dgemm_naive(self, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, j0=0, j1=None,
                    threads=0):
        j1 = n if j1 is None else j1
        self.L.ozo_dgemm_naive(m, n, k, alpha, _ptr(A, _f64p), lda, _ptr(B, _f64p), ldb, beta,
                               _ptr(C, _f64p), ldc, j0, j1, threads)


class Reference:
    """ctypes view of oracle/_ref/libggemm_ref.so (the reference's own code)."""

    def __init__(self, path=REF_SO):
        L = ctypes.CDLL(path)
        L.ozr_tables_size.restype = c_size_t
        L.ozr_build_tables.argtypes = [c_void_p, c_size_t]
        L.ozr_error_bound.restype = c_double
        L.ozr_error_bound.argtypes = [c_int, c_int]
        L.ozr_choose.argtypes = [c_int, c_double]
        L.ozr_choose_cw.argtypes = [c_int, c_double]
        for f in ("ozr_sizeof_problem", "ozr_sizeof_plan_entry", "ozr_sizeof_oz2_problem",
                  "ozr_sizeof_i8_problem", "ozr_i8_sched_ws_bytes"):
            getattr(L, f).restype = c_size_t
        L.ozr_i8_sched_ws_bytes.argtypes = [c_int]
        L.ozr_plan.argtypes = [c_void_p, c_int, c_void_p, c_int, c_int, c_double, c_double,
                               c_double, c_double, c_void_p]
        L.ozr_reuse.argtypes = [c_void_p, c_int, c_void_p, c_int, c_void_p]
        L.ozr_prep_grouped.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p]
        L.ozr_reconstruct_grouped.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p, c_int]
        L.ozr_i8_grouped_gemm.argtypes = [c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_void_p]
        L.ozr_read_counters.argtypes = [c_void_p, c_int, c_void_p]
        L.ozr_force_prep_split.argtypes = [c_int]
        self.L = L

    @classmethod
    def load(cls):
        if not os.path.exists(REF_SO):
            return None
        return cls()

    def tables_bytes(self) -> bytes:
        n = self.L.ozr_tables_size()
        b = (ctypes.c_ubyte * n)()
        assert self.L.ozr_build_tables(b, n) == 0
        return bytes(b)


def problem_dict(m, n, k, A, lda, B, ldb, C, ldc, alpha, beta):
    return dict(m=m, n=n, k=k, A=A, lda=lda, B=B, ldb=ldb, C=C, ldc=ldc, alpha=alpha, beta=beta)


def decode_tables(buf: bytes):
    """Decodes the oz2_crt_tables layout."""
    off = 0

    def take(dtype, count):
        nonlocal off
        a = np.frombuffer(buf, dtype=dtype, count=count, offset=off)
        off += a.nbytes
        return a

    t = {}
    t["p"] = take(np.int32, 20)
    t["magic"] = take(np.uint32, 20)
    t["pow2"] = take(np.uint8, 20 * 128).reshape(20, 128)
    t["s1"] = take(np.uint64, 21 * 20).reshape(21, 20)
    t["s2"] = take(np.uint32, 21 * 20).reshape(21, 20)
    t["qinv"] = take(np.int32, 21 * 20).reshape(21, 20)
    off = (off + 7) // 8 * 8
    t["P1"] = take(np.int64, 21)
    t["P2"] = take(np.float64, 21)
    t["inv_Pu"] = take(np.float64, 21)
    t["log2_u1"] = take(np.int32, 21)
    off = (off + 7) // 8 * 8
    t["T"] = take(np.float64, 21)
    t["log2P"] = take(np.float64, 21)
    return t
