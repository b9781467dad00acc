"""The safety fallback (entries in a row of A or a column of B that holds NaN or Inf) against the
reference library, through the public call, bit for bit.

The reference computes every such entry as alpha * dot + beta * C with dot the sequential FP64
fma chain over k (src/ozaki2_numerics.cu:445-452, 492-497).  This library computes them in
64 x 64 tiles inside the reconstruct launch; the chains are the same operations in the same
order.  The group puts poisoned rows and columns in several row / column tiles (side R and side
C items, and entries poisoned on both sides), uses padded leading dimensions, k that is not a
multiple of the 32-position staging chunk, a problem whose every row is poisoned, beta = 0 and
beta != 0, and runs in the three repair modes.  Outputs and stats counters must equal the
reference's.
"""
import ctypes
import os
from ctypes import c_void_p

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

# (m, n, k, alpha, beta, poisoned A rows, poisoned B columns)
SHAPES = [
    (200, 150, 777, 1.0, 0.0, [0, 63, 64, 130, 199], [5, 70, 149]),
    (130, 70, 33, -2.5, 0.5, [7], [0, 64, 69]),
    (64, 64, 64, 1.0, 1.0, list(range(64)), []),
    (1, 300, 100, 0.75, -1.0, [0], [299]),
    (300, 1, 50, 2.0, 0.25, [150, 151], []),
    (96, 130, 1000, 1.0, 0.0, [], [1, 2, 128]),
    (70, 90, 2048, 0.5, 2.0, [3, 69], [44]),
]


def _build(seed, device):
    rng = np.random.default_rng(seed)
    keep, entries = [], []
    for (m, n, k, alpha, beta, rows, cols) in SHAPES:
        lda, ldb, ldc = m + 5, k + 3, m + 2
        A = (rng.random((lda, k)) - 0.5) * np.exp(rng.standard_normal((lda, k)))
        B = (rng.random((ldb, n)) - 0.5) * np.exp(rng.standard_normal((ldb, n)))
        C = rng.random((ldc, n)) - 0.5
        for r in rows:
            A[r, rng.integers(k)] = np.nan if r % 2 else np.inf
        for c in cols:
            B[rng.integers(k), c] = -np.inf if c % 2 else np.nan
        # column-major buffers: element (i, q) of A at i + q * lda
        tA = torch.from_numpy(np.asfortranarray(A).ravel(order="F")).to(device)
        tB = torch.from_numpy(np.asfortranarray(B).ravel(order="F")).to(device)
        tC = torch.from_numpy(np.asfortranarray(C).ravel(order="F")).to(device)
        keep.append((tA, tB, tC, tC.clone()))
        entries.append(dict(m=m, n=n, k=k, A=tA.data_ptr(), lda=lda, B=tB.data_ptr(), ldb=ldb,
                            C=tC.data_ptr(), ldc=ldc, alpha=alpha, beta=beta))
    return keep, entries


def _budgets():
    return (sum(m * k for m, n, k, *_ in SHAPES) + 1, sum(k * n for m, n, k, *_ in SHAPES) + 1,
            sum(m * n for m, n, k, *_ in SHAPES) + 1)


def _reset(keep):
    for (_, _, C, C0) in keep:
        C.copy_(C0)
    torch.cuda.synchronize()


@pytest.mark.parametrize("repair", [1, 2, 3])  # GGEMM_REPAIR_OFF, COUNT, ON
def test_safety_fallback_vs_reference(g2, ref, cuda, repair):
    keep, entries = _build(11 + repair, cuda)
    probs = g2.make_problems(entries)
    cfg = g2.config(0, 1e-15, 1, repair)
    s = torch.cuda.current_stream().cuda_stream
    os.environ["GGEMM_STATS_REPAIR"] = "1"
    try:
        _reset(keep)
        with g2.Handle(len(entries), *_budgets(), stream=s, min_k=16) as h:
            rc, st = h.grouped_dgemm(g2.PATH_EMU_GROUPED, cfg, probs, len(entries))
            torch.cuda.synchronize()
            assert rc == 0 and h.device_status() == 0
        ours = [C.clone() for (_, _, C, _) in keep]
        _reset(keep)
        L = ref.L
        L.ggemm_create_ex.argtypes = [ctypes.POINTER(c_void_p), ctypes.c_int, ctypes.c_size_t,
                                      ctypes.c_size_t, ctypes.c_size_t, c_void_p, ctypes.c_int]
        L.ggemm_grouped_dgemm.argtypes = [c_void_p, ctypes.c_int, c_void_p, c_void_p,
                                          ctypes.c_int, c_void_p]
        L.ggemm_destroy.argtypes = [c_void_p]
        hr = c_void_p()
        assert L.ggemm_create_ex(ctypes.byref(hr), len(entries), *_budgets(), s, 16) == 0
        st2 = g2.Stats()
        rc2 = L.ggemm_grouped_dgemm(hr, g2.PATH_EMU_GROUPED, ctypes.addressof(cfg),
                                    ctypes.addressof(probs), len(entries), ctypes.addressof(st2))
        torch.cuda.synchronize()
        L.ggemm_destroy(hr)
        assert rc2 == 0
    finally:
        os.environ.pop("GGEMM_STATS_REPAIR", None)
    for x, ((m, n, k, *_), mine, (_, _, theirs, _)) in enumerate(zip(SHAPES, ours, keep)):
        diff = int((mine.view(torch.int64) != theirs.view(torch.int64)).sum().item())
        assert diff == 0, f"problem {x} ({m}x{n}x{k}): {diff} words differ"
    for f in ("num_repaired", "num_uncertified", "num_safety_fallback", "num_fallback"):
        assert getattr(st, f) == getattr(st2, f), (f, getattr(st, f), getattr(st2, f))
    assert st.num_safety_fallback > 0
