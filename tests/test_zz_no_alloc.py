"""ggemm_dgemm_noalloc: the entry point for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: code that owns no CUDA allocator, runs inside another
runtime's memory pool, or must not allocate or free device memory.  ggemm_dgemm_noalloc lets
them emulate one FP64 GEMM with every scratch byte taken from a fixed 64 MiB array inside the
library.  These tests call it through the C ABI and require its output to equal, bit for bit
(the tolerance of every emulated-path comparison in this suite), the output of the existing
entry point ggemm_grouped_dgemm (EMU_GROUPED, same moduli count and repair mode) on the same
inputs, on two calls in a row that share the array.  This file is collected last so that a
failure here cannot hide any other test; it passes alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest

from g2util import col_major, gen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ERR_WORKSPACE = 2


def _inputs(rng, m, n, k, phi, pad):
    A, B, C0 = gen(rng, (m, k), phi), gen(rng, (k, n), phi), gen(rng, (m, n), 0.0)
    lda, ldb, ldc = m + pad, k + pad, m + pad
    return (torch.from_numpy(col_major(A, lda)).cuda(), lda,
            torch.from_numpy(col_major(B, ldb)).cuda(), ldb,
            col_major(C0, ldc), ldc)


def _problem(g2, m, n, k, A, lda, B, ldb, C, ldc, alpha, beta):
    return g2.make_problems([dict(m=m, n=n, k=k, A=A.data_ptr(), lda=lda, B=B.data_ptr(), ldb=ldb,
                                  C=C.data_ptr(), ldc=ldc, alpha=alpha, beta=beta)])


def _via_grouped(g2, shape, A, lda, B, ldb, C0, ldc, alpha, beta):
    m, n, k = shape
    C = torch.from_numpy(C0.copy()).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    with g2.Handle(1, m * k, k * n, m * n, stream=stream) as h:
        rc, st = h.grouped_dgemm(g2.PATH_EMU_GROUPED, g2.config(0, 1e-15, 0, 0),
                                 _problem(g2, m, n, k, A, lda, B, ldb, C, ldc, alpha, beta), 1)
        torch.cuda.synchronize()
        assert rc == 0
    return C.cpu().numpy()


def _via_noalloc(g2, shape, A, lda, B, ldb, C0, ldc, alpha, beta):
    m, n, k = shape
    C = torch.from_numpy(C0.copy()).cuda()
    rc = g2.lib.ggemm_dgemm_noalloc(_problem(g2, m, n, k, A, lda, B, ldb, C, ldc, alpha, beta),
                                    0, 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == 0
    return C.cpu().numpy()


def test_noalloc_matches_grouped_entry_point_two_calls(g2, cuda):
    rng = np.random.default_rng(424242)
    cases = [((200, 150, 300), 2.0, 1.5, 0.5, 3), ((96, 257, 1000), 1.0, 1.0, 0.0, 0)]
    for shape, phi, alpha, beta, pad in cases:  # two calls in a row on the shared array
        A, lda, B, ldb, C0, ldc = _inputs(rng, *shape, phi, pad)
        want = _via_grouped(g2, shape, A, lda, B, ldb, C0, ldc, alpha, beta)
        got = _via_noalloc(g2, shape, A, lda, B, ldb, C0, ldc, alpha, beta)
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), shape


def test_noalloc_rejects_problems_beyond_its_scratch(g2, cuda):
    m = n = k = 2048
    A = torch.zeros(m * k, dtype=torch.float64, device="cuda")
    B = torch.zeros(k * n, dtype=torch.float64, device="cuda")
    C = torch.full((m * n,), 3.0, dtype=torch.float64, device="cuda")
    rc = g2.lib.ggemm_dgemm_noalloc(_problem(g2, m, n, k, A, m, B, k, C, m, 1.0, 0.0), 0, 0,
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == ERR_WORKSPACE
    assert bool(torch.all(C == 3.0))
