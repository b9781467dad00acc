"""ggemm_b200 -- Python view of the B200 grouped FP64-via-INT8 GEMM library.

The product is the C-ABI shared library ``libggemm_b200.so`` built from ``csrc/`` (declared in
``include/ggemm.h``, ``include/ggemm_graph.h`` and ``include/ggemm_stages.h``).  This module
binds it with ctypes, mirroring the reference's C API (moneychen168/Coding-Basic-HW-2,
``include/ggemm.h``): the same structs, path enum, repair modes and GGEMM_ERR_* codes, so tests
and benchmarks drive exactly the entry points a C caller would.  There is no fallback: when the
shared library is missing, importing this module raises.

Device memory, streams and multi-process plumbing come from PyTorch; pointers are passed as
integers (``tensor.data_ptr()``, ``torch.cuda.current_stream().cuda_stream``).
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_int, c_longlong, c_size_t, c_void_p

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libggemm_b200.so")

# ----------------------------------------------------------------------------- public enums
PATH_NATIVE_LOOP = 0
PATH_NATIVE_GROUPED = 1
PATH_EMU_LOOP = 2
PATH_EMU_GROUPED = 3
PATH_AUTO = 4
PATH_EMU_GROUPED_REUSE = 5
PATH_EMU_LOOP_BATCHED = 6
PATH_NAMES = {
    PATH_NATIVE_LOOP: "native_loop",
    PATH_NATIVE_GROUPED: "native_grouped",
    PATH_EMU_LOOP: "emu_loop",
    PATH_EMU_GROUPED: "emu_grouped",
    PATH_AUTO: "auto",
    PATH_EMU_GROUPED_REUSE: "emu_grouped_reuse",
    PATH_EMU_LOOP_BATCHED: "emu_loop_batched",
}

MAX_MODULI = 20
REPAIR_DEFAULT, REPAIR_OFF, REPAIR_COUNT, REPAIR_ON = 0, 1, 2, 3
STAGE_REPAIR_OFF, STAGE_REPAIR_COUNT, STAGE_REPAIR_ON = 0, 1, 2

OK = 0
ERR_INVALID = 1
ERR_WORKSPACE = 2
ERR_UNSAFE = 3
ERR_CUDA = 4
ERR_CUBLAS = 5
ERR_NUMERICS = 6
ERR_I8GEMM = 7
ERR_ALLOC = 8

SHIFT_NONFINITE = -(2**31)
SHIFT_ZERO = -(2**31) + 1

ROUTE_EMU, ROUTE_EMPTY, ROUTE_K_ZERO, ROUTE_K_TOO_LARGE = 0, 1, 2, 3
ROUTE_TINY, ROUTE_UNPROFITABLE, ROUTE_PRECISION, ROUTE_SMALL_K, ROUTE_ALPHA_ZERO = 4, 5, 6, 7, 8
MAX_K_EXACT = 131040


# ---------------------------------------------------------------------------- C structures
class Problem(ctypes.Structure):
    """ggemm_problem_t (include/ggemm.h)."""

    _fields_ = [
        ("m", c_int), ("n", c_int), ("k", c_int),
        ("A", c_void_p), ("lda", c_int),
        ("B", c_void_p), ("ldb", c_int),
        ("C", c_void_p), ("ldc", c_int),
        ("alpha", c_double), ("beta", c_double),
    ]


class Config(ctypes.Structure):
    """ggemm_config_t."""

    _fields_ = [("num_moduli", c_int), ("target_rel_err", c_double),
                ("allow_fallback", c_int), ("repair_mode", c_int)]


class Stats(ctypes.Structure):
    """ggemm_stats_t."""

    _fields_ = [
        ("num_problems", c_int), ("num_fallback", c_int), ("kernel_launches", c_int),
        ("moduli_min", c_int), ("moduli_max", c_int),
        ("reuse_enabled", c_int), ("num_unique_A", c_int), ("num_unique_B", c_int),
        ("num_promoted", c_int),
        ("num_repaired", c_longlong), ("num_uncertified", c_longlong),
        ("num_safety_fallback", c_longlong),
    ]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class PrepDesc(ctypes.Structure):
    """ggemm_prep_desc_t (include/ggemm_stages.h)."""

    _fields_ = [("X", c_void_p), ("ld", c_longlong), ("rows", c_int), ("k", c_int),
                ("N", c_int), ("kind", c_int), ("img", c_void_p), ("plane_bytes", c_longlong),
                ("ws", c_void_p)]


class GemmDesc(ctypes.Structure):
    """ggemm_gemm_desc_t."""

    _fields_ = [("A", c_void_p), ("B", c_void_p), ("C", c_void_p), ("a_plane", c_longlong),
                ("b_plane", c_longlong), ("c_plane", c_longlong), ("m", c_int), ("n", c_int),
                ("k", c_int), ("planes", c_int), ("N", c_int), ("layout", c_int)]


class ReconDesc(ctypes.Structure):
    """ggemm_recon_desc_t."""

    _fields_ = [("m", c_int), ("n", c_int), ("k", c_int), ("N", c_int),
                ("A", c_void_p), ("lda", c_longlong), ("B", c_void_p), ("ldb", c_longlong),
                ("C", c_void_p), ("ldc", c_longlong), ("alpha", c_double), ("beta", c_double),
                ("C32", c_void_p), ("c_plane", c_longlong), ("rs", c_void_p), ("cs", c_void_p),
                ("layout", c_int), ("reserved", c_int)]


# Product layouts between the residue GEMM and the reconstruct (ggemm_stages.h).
PRODUCTS_INT32 = 0
PRODUCTS_DIGITS = 1
PRODUCTS_DIGITS_QSCALED = 2  # GEMM stage only: A images prepared with PREP_QSCALED
PREP_QSCALED = 2  # flag in PrepDesc.kind: plane l holds residues of q_l x


def digit_plane_bytes(m, n):
    """ggemm_digit_plane_bytes: bytes of one digit plane of an m x n problem."""
    return ((n + 31) // 32 * m * 32 + 255) // 256 * 256



COUNTER_BYTES = 64


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C coding-basic-hw-2_b200` "
            "(or __graft_entry__.build()); there is no fallback implementation")
    lib = ctypes.CDLL(LIB_PATH)
    sig = {
        "ggemm_create": (c_int, [POINTER(c_void_p), c_int, c_size_t, c_size_t, c_size_t, c_void_p]),
        "ggemm_create_ex": (c_int, [POINTER(c_void_p), c_int, c_size_t, c_size_t, c_size_t,
                                    c_void_p, c_int]),
        "ggemm_destroy": (None, [c_void_p]),
        "ggemm_grouped_dgemm": (c_int, [c_void_p, c_int, POINTER(Config), POINTER(Problem), c_int,
                                        POINTER(Stats)]),
        "ggemm_make_plan": (c_void_p, [c_void_p, c_int, POINTER(Config), POINTER(Problem), c_int]),
        "ggemm_make_plan_ex": (c_void_p, [c_void_p, c_int, POINTER(Config), POINTER(Problem),
                                          c_int, POINTER(c_int)]),
        "ggemm_execute_plan": (c_int, [c_void_p, c_void_p]),
        "ggemm_plan_update_pointers": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
        "ggemm_plan_get_stats": (c_int, [c_void_p, POINTER(Stats)]),
        "ggemm_destroy_plan": (None, [c_void_p]),
        "ggemm_stage_scratch_bytes": (c_size_t, [c_int]),
        "ggemm_stage_prep": (c_int, [POINTER(PrepDesc), c_int, c_void_p, c_size_t, c_void_p,
                                     c_void_p]),
        "ggemm_stage_gemm": (c_int, [POINTER(GemmDesc), c_int, c_void_p, c_size_t, c_void_p,
                                     c_void_p]),
        "ggemm_stage_recon": (c_int, [POINTER(ReconDesc), c_int, c_int, c_void_p, c_size_t,
                                      c_void_p, c_void_p]),
        "ggemm_stage_plan": (c_int, [POINTER(Problem), c_int, POINTER(Config), c_int, c_int,
                                     c_double, c_double, c_double, c_double, c_double,
                                     POINTER(c_int), POINTER(c_int), POINTER(c_int)]),
        "ggemm_stage_reuse": (c_int, [POINTER(Problem), c_int, POINTER(c_int), c_int,
                                      POINTER(c_int)]),
        "ggemm_set_stage_events": (c_int, [c_void_p, c_void_p]),
        "ggemm_device_status": (c_int, [c_void_p]),
        "ggemm_shard_group": (c_int, [POINTER(Problem), c_int, c_int, POINTER(Problem),
                                      POINTER(c_int), POINTER(c_int), c_int, POINTER(c_int)]),
        "ggemm_stage_crt_tables": (c_size_t, [c_void_p, c_size_t]),
        "ggemm_stage_error_bound": (c_double, [c_int, c_int]),
        "ggemm_dgemm_noalloc": (c_int, [POINTER(Problem), c_int, c_int, c_void_p]),
        "ggemm_dgemm_noalloc_status": (c_int, [c_void_p]),
        "ggemm_stage_wait_probe": (c_int, [c_void_p, c_longlong, c_void_p]),
        "ggemm_device_count": (c_int, []),
        "ggemm_version": (c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


# --------------------------------------------------------------------------- layout helpers
def img_plane_bytes(rows: int, k: int) -> int:
    """Bytes of one residue plane (include/ggemm_stages.h: ggemm_img_plane_bytes)."""
    return ((rows + 7) // 8) * ((k + 31) // 32) * 256


def _img_index(rows: int, k: int) -> np.ndarray:
    kp = (k + 31) // 32 * 32
    rg = (rows + 7) // 8
    r = np.arange(rows, dtype=np.int64)[:, None]
    q = np.arange(kp, dtype=np.int64)[None, :]
    rr, qq = r & 7, q & 31
    return ((q >> 5) * rg + (r >> 3)) * 256 + rr * 32 + (((qq >> 4) ^ (rr >> 2)) << 4) + (qq & 15)


def unpack_plane(buf: np.ndarray, rows: int, k: int) -> np.ndarray:
    """Image bytes of one plane -> int8 array rows x round_up(k, 32) (row-major, K contiguous)."""
    return np.asarray(buf, dtype=np.int8).reshape(-1)[_img_index(rows, k)]


def pack_plane(mat: np.ndarray, k: int) -> np.ndarray:
    """int8 rows x kp (kp >= round_up(k, 32); extra columns must be 0) -> image bytes."""
    rows = mat.shape[0]
    kp = (k + 31) // 32 * 32
    out = np.zeros(img_plane_bytes(rows, k), dtype=np.int8)
    full = np.zeros((rows, kp), dtype=np.int8)
    full[:, : min(kp, mat.shape[1])] = mat[:, :kp]
    out[_img_index(rows, k)] = full
    return out


# ------------------------------------------------------------------------------ API helpers
def make_problems(entries) -> ctypes.Array:
    """entries: iterable of dicts with keys m, n, k, A, lda, B, ldb, C, ldc, alpha, beta
    (pointers as ints)."""
    entries = list(entries)
    arr = (Problem * max(1, len(entries)))()
    for i, e in enumerate(entries):
        arr[i] = Problem(e["m"], e["n"], e["k"], e["A"], e["lda"], e["B"], e["ldb"], e["C"],
                         e["ldc"], float(e["alpha"]), float(e["beta"]))
    return arr


def config(num_moduli=0, target_rel_err=1e-15, allow_fallback=1, repair_mode=0) -> Config:
    return Config(num_moduli, target_rel_err, allow_fallback, repair_mode)


class Handle:
    """Owns a ggemm_handle_t (ggemm_create_ex) bound to the current device and `stream`."""

    def __init__(self, max_problems, max_a, max_b, max_c, stream=0, min_k=32):
        self.ptr = c_void_p()
        rc = lib.ggemm_create_ex(ctypes.byref(self.ptr), int(max_problems), int(max_a),
                                 int(max_b), int(max_c), c_void_p(stream or None), int(min_k))
        if rc != OK:
            raise RuntimeError(f"ggemm_create_ex failed: {rc}")

    def grouped_dgemm(self, path, cfg, problems, num):
        st = Stats()
        rc = lib.ggemm_grouped_dgemm(self.ptr, int(path), ctypes.byref(cfg) if cfg else None,
                                     problems, int(num), ctypes.byref(st))
        return rc, st

    def set_stage_events(self, events):
        """events: 4 torch.cuda.Event (already recorded once, so the CUDA events exist) or
        None to stop recording."""
        if events is None:
            return lib.ggemm_set_stage_events(self.ptr, None)
        arr = (c_void_p * 4)(*[e.cuda_event for e in events])
        return lib.ggemm_set_stage_events(self.ptr, arr)

    def device_status(self):
        return lib.ggemm_device_status(self.ptr)

    def close(self):
        if self.ptr:
            lib.ggemm_destroy(self.ptr)
            self.ptr = c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shard_group(problems, num, num_shards, out_cap=None):
    """ggemm_shard_group: returns (sub-problem array, shard list, source-problem list)."""
    cap = out_cap or max(16, 4 * num + 64 * num_shards)
    out = (Problem * cap)()
    sh = (c_int * cap)()
    src = (c_int * cap)()
    nout = c_int(0)
    rc = lib.ggemm_shard_group(problems, int(num), int(num_shards), out, sh, src, cap,
                               ctypes.byref(nout))
    if rc != OK:
        raise RuntimeError(f"ggemm_shard_group failed: {rc}")
    n = nout.value
    return out, [sh[i] for i in range(n)], [src[i] for i in range(n)]


def version() -> str:
    return lib.ggemm_version().decode()
