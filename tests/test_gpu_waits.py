"""Bounded waits end with a status the host reads, without a fault.

Every wait of this library's kernels (GEMM pipeline stages, TMEM accumulators, prep residue-MMA
rounds) gives up at a %globaltimer deadline and records a status word.  The probe seam
(ggemm_stage_wait_probe) runs that same bounded wait on an mbarrier that nothing arrives on, so
the wait runs out on purpose: the test checks the status word, and that the context is still
usable for a full pipeline call afterwards.
"""
import ctypes

import numpy as np
import pytest

from g2util import col_major, gen

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_sets_status_and_context_stays_usable(g2, oracle, cuda):
    cnt = torch.zeros(64, dtype=torch.uint8, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert g2.lib.ggemm_stage_wait_probe(ctypes.c_void_p(cnt.data_ptr()), 3_000_000, s) == 0
    torch.cuda.synchronize()
    words = cnt.cpu().numpy().view(np.uint32)
    assert words[8] == 3  # status word after the four 64-bit counters
    # the same device then runs a full call, bit-exact against the CPU checker
    rng = np.random.default_rng(3)
    m, n, k, N = 96, 80, 160, 15
    A, B, C0 = gen(rng, (m, k), 1.0), gen(rng, (k, n), 1.0), gen(rng, (m, n), 0.0)
    Af, Bf, Cf = col_major(A, m), col_major(B, k), col_major(C0, m)
    want = Cf.copy()
    oracle.emulated(m, n, k, N, 1.0, 0.5, Af, m, Bf, k, want, m, 1)
    dA, dB, dC = (torch.from_numpy(x).cuda() for x in (Af, Bf, Cf.copy()))
    P = g2.make_problems([dict(m=m, n=n, k=k, A=dA.data_ptr(), lda=m, B=dB.data_ptr(), ldb=k,
                               C=dC.data_ptr(), ldc=m, alpha=1.0, beta=0.5)])
    with g2.Handle(1, m * k, k * n, m * n, stream=torch.cuda.current_stream().cuda_stream) as h:
        rc, _ = h.grouped_dgemm(g2.PATH_EMU_GROUPED, g2.config(N, 1e-15, 0, 0), P, 1)
        torch.cuda.synchronize()
        assert rc == 0 and h.device_status() == 0
    assert np.array_equal(dC.cpu().numpy().view(np.uint64), want.view(np.uint64))
