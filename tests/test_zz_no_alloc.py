"""ggemm_dgemm_noalloc: the entry point for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: code that owns no CUDA allocator, runs inside another
runtime's memory pool, or must not allocate or free device memory.  ggemm_dgemm_noalloc lets
them emulate one FP64 GEMM with every scratch byte taken from a fixed 64 MiB array inside the
library.  These tests call it through the C ABI and require its output to equal, bit for bit
(the tolerance of every emulated-path comparison in this suite), the output of the existing
entry point ggemm_grouped_dgemm (EMU_GROUPED, same moduli count and repair mode) on the same
inputs, on calls in a row that share the array.  The cases cover both product layouts (digits,
and int32 for n below about 10), adaptive and fixed moduli counts (N = 16 uses the prep instance
with the accumulator bias), every repair mode, alpha = 0 and k = 0 (C = beta C, which the grouped
call computes with cuBLAS: equal values, zeros of either sign), beta = 0 with NaN in C (C not
read) and signed zeros.  This
file is collected last so that a failure here cannot hide any other test; it passes alone in a
fresh process as well.
"""
import ctypes

import numpy as np
import pytest

from g2util import col_major, gen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ERR_WORKSPACE = 2
PROBE_TIMEOUT = 3


def _inputs(rng, m, n, k, phi, pad, c_fill=None):
    A, B, C0 = gen(rng, (m, max(k, 1)), phi), gen(rng, (max(k, 1), n), phi), gen(rng, (m, n), 0.0)
    if c_fill is not None:
        C0[:] = c_fill
    lda, ldb, ldc = m + pad, max(k, 1) + pad, m + pad
    return (torch.from_numpy(col_major(A[:, :max(k, 1)], lda)).cuda(), lda,
            torch.from_numpy(col_major(B, ldb)).cuda(), ldb,
            col_major(C0, ldc), ldc)


def _problem(g2, m, n, k, A, lda, B, ldb, C, ldc, alpha, beta):
    return g2.make_problems([dict(m=m, n=n, k=k, A=A.data_ptr(), lda=lda, B=B.data_ptr(), ldb=ldb,
                                  C=C.data_ptr(), ldc=ldc, alpha=alpha, beta=beta)])


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _via_grouped(g2, shape, A, lda, B, ldb, C0, ldc, alpha, beta, N=0, repair=0):
    m, n, k = shape
    C = torch.from_numpy(C0.copy()).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    with g2.Handle(1, m * k + 1, k * n + 1, m * n, stream=stream) as h:
        rc, st = h.grouped_dgemm(g2.PATH_EMU_GROUPED, g2.config(N, 1e-15, 0, repair),
                                 _problem(g2, m, n, k, A, lda, B, ldb, C, ldc, alpha, beta), 1)
        torch.cuda.synchronize()
        assert rc == 0
    return C.cpu().numpy()


def _via_noalloc(g2, shape, A, lda, B, ldb, C0, ldc, alpha, beta, N=0, repair=0):
    m, n, k = shape
    C = torch.from_numpy(C0.copy()).cuda()
    rc = g2.lib.ggemm_dgemm_noalloc(_problem(g2, m, n, k, A, lda, B, ldb, C, ldc, alpha, beta),
                                    N, repair, _stream())
    assert rc == 0
    assert g2.lib.ggemm_dgemm_noalloc_status(_stream()) == 0
    return C.cpu().numpy()


# (m, n, k), phi, alpha, beta, pad, N, repair mode, C fill
CASES = [
    ((200, 150, 300), 2.0, 1.5, 0.5, 3, 0, 0, None),       # digit layout, adaptive N
    ((96, 257, 1000), 1.0, 1.0, 0.0, 0, 0, 0, None),       # beta = 0
    ((64, 5, 300), 1.0, 1.0, 0.5, 1, 0, 0, None),          # int32 product layout (n < 10)
    ((130, 70, 640), 2.0, -0.75, 0.25, 0, 16, 0, None),    # fixed N = 16 (accumulator bias)
    ((77, 90, 333), 4.0, 2.0, -1.0, 2, 0, 3, None),        # repair ON, wide exponent range
    ((50, 60, 128), 1.0, 1.0, 0.0, 0, 14, 1, float("nan")),  # beta = 0: NaN in C never read
    ((40, 33, 64), 1.0, 0.0, 0.5, 0, 0, 0, None),          # alpha = 0: C = beta C
    ((40, 33, 64), 1.0, 0.0, 0.0, 0, 0, 0, float("nan")),  # alpha = 0, beta = 0: C = 0
    ((40, 33, 0), 1.0, 1.5, 0.5, 0, 0, 0, None),           # k = 0: C = beta C
    ((40, 33, 0), 1.0, -1.5, 0.0, 0, 0, 0, float("nan")),  # k = 0, beta = 0
    ((40, 33, 0), 1.0, 1.0, -2.0, 0, 0, 0, -0.0),          # k = 0: signed zeros of beta C
    ((40, 33, 64), 1.0, 0.0, 3.0, 0, 0, 0, -0.0),          # alpha = 0: signed zeros
]


def test_noalloc_matches_grouped_entry_point_calls_in_a_row(g2, cuda):
    rng = np.random.default_rng(424242)
    for shape, phi, alpha, beta, pad, N, repair, fill in CASES:  # calls in a row, one array
        A, lda, B, ldb, C0, ldc = _inputs(rng, *shape, phi, pad, fill)
        want = _via_grouped(g2, shape, A, lda, B, ldb, C0, ldc, alpha, beta, N, repair)
        got = _via_noalloc(g2, shape, A, lda, B, ldb, C0, ldc, alpha, beta, N, repair)
        if alpha == 0.0 or shape[2] == 0:
            # C = beta C: the grouped call computes it with cuBLAS, whose zeros may carry the
            # other sign (it adds alpha * 0 to beta C); values, NaN positions included, agree
            assert np.array_equal(got, want, equal_nan=True), (shape, alpha, beta)
            continue
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), (shape, alpha, beta, N)


def test_noalloc_two_calls_of_one_problem_identical(g2, cuda):
    rng = np.random.default_rng(99)
    shape = (300, 200, 500)
    A, lda, B, ldb, C0, ldc = _inputs(rng, *shape, 2.0, 0)
    want = _via_grouped(g2, shape, A, lda, B, ldb, C0, ldc, 1.25, 0.5)
    for _ in range(2):
        got = _via_noalloc(g2, shape, A, lda, B, ldb, C0, ldc, 1.25, 0.5)
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64))


def test_noalloc_status_reports_a_wait_that_ran_out(g2, cuda):
    """The status query reads the word the kernels set in the fixed scratch: a bounded-wait probe
    on that counter block gives up after 2 ms and records its code, the query returns it, and the
    next call clears it (a call's status is valid until the next call starts)."""
    rng = np.random.default_rng(5)
    shape = (64, 64, 96)
    A, lda, B, ldb, C0, ldc = _inputs(rng, *shape, 1.0, 0)
    _via_noalloc(g2, shape, A, lda, B, ldb, C0, ldc, 1.0, 0.0)
    assert g2.lib.ggemm_stage_wait_probe(None, 2_000_000, _stream()) == 0
    assert g2.lib.ggemm_dgemm_noalloc_status(_stream()) == PROBE_TIMEOUT
    _via_noalloc(g2, shape, A, lda, B, ldb, C0, ldc, 1.0, 0.0)  # asserts status 0 again


def test_noalloc_rejects_problems_beyond_its_scratch(g2, cuda):
    m = n = k = 2048
    A = torch.zeros(m * k, dtype=torch.float64, device="cuda")
    B = torch.zeros(k * n, dtype=torch.float64, device="cuda")
    C = torch.full((m * n,), 3.0, dtype=torch.float64, device="cuda")
    rc = g2.lib.ggemm_dgemm_noalloc(_problem(g2, m, n, k, A, m, B, k, C, m, 1.0, 0.0), 0, 0,
                                    _stream())
    torch.cuda.synchronize()
    assert rc == ERR_WORKSPACE
    assert bool(torch.all(C == 3.0))
