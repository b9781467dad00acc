"""The application callers (coding-basic-hw-2_b200/apps/): an FP64 MoE FFN forward and an FP64
block-sparse times dense product, every GEMM through ggemm_grouped_dgemm, on small instances.
Each emulated path must agree with the same pipeline on NATIVE_LOOP within twice the FP64
a-priori bound of the whole computation (the reference apps' diagnostic, err_over_bound <= 1).
"""
import os
import sys

import pytest

from g2util import PKG_DIR

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
sys.path.insert(0, os.path.join(PKG_DIR, "apps"))


def test_moe_ffn_paths_agree_with_native(g2, cuda):
    import moe_ffn as M

    L = M.MoELayer(512, 8, 2, 128, 256, 1.2, 0.5, 7, torch.device("cuda", 0))
    R = L.T * L.k
    cfg = g2.config(0, 1e-15, 1, 0)
    with g2.Handle(L.E, R * 256 + L.E * L.d * L.f, R * 512, R * 256,
                   stream=torch.cuda.current_stream().cuda_stream) as h:
        Y_ref, Ha_ref = M.forward(g2, L, h, g2.PATH_NATIVE_LOOP, cfg)
        for path in (g2.PATH_EMU_GROUPED, g2.PATH_AUTO, g2.PATH_EMU_LOOP):
            Y, _ = M.forward(g2, L, h, path, cfg)
            torch.cuda.synchronize()
            assert M.error_over_bound(L, Y, Y_ref, Ha_ref) <= 1.0, path
    assert min(L.counts) >= 0 and max(L.counts) > 2 * min(c for c in L.counts if c)  # skewed


def test_block_sparse_paths_agree_with_native(g2, cuda):
    import block_sparse as B

    S = B.BSR(96, 0.1, 5.0, 24, 0.5, 11, torch.device("cuda", 0))
    out = B.run(g2, S, paths=("emu_grouped", "auto", "native_grouped"), reps=1)
    for key, v in out.items():
        if isinstance(v, dict):
            assert v["err_over_bound"] <= 1.0, (key, v)
    assert out["blocks"] > S.atoms  # more than the diagonal blocks
