"""The paired residue GEMM (CTA pairs, tcgen05.mma.cta_group::2, 256 x 256 tiles) against exact
int64 products, and against the single-CTA GEMM through the public call.

GGEMM_GEMM_PAIR=1 forces the paired kernel (stage seam: read at each call; public call: read
when the handle is created).  Shapes cover the pair's edges: rows below, at and past 128 and 256
(the second CTA of a pair with no valid rows), columns whose MMA width rounds to 32 with the
second CTA holding few or no valid B rows, K not a multiple of 32, one K step, and every moduli
count class; both product layouts (CRT digits and int32).
"""
import ctypes
import os

import numpy as np
import pytest

from test_gpu_digits import _exact, _rand_planes, digits_of, run_gemm_digits, tables  # noqa: F401

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PAIR_SHAPES = [(1, 1, 1, 2), (100, 17, 31, 15), (128, 32, 64, 14), (129, 33, 1000, 15),
               (256, 256, 256, 16), (300, 100, 96, 8), (513, 255, 130, 15), (64, 300, 2048, 20),
               (257, 129, 33, 12), (200, 1, 64, 15), (1, 260, 100, 15), (384, 96, 512, 10)]


class pair_mode:
    def __init__(self, v):
        self.v = v

    def __enter__(self):
        os.environ["GGEMM_GEMM_PAIR"] = str(self.v)

    def __exit__(self, *exc):
        os.environ.pop("GGEMM_GEMM_PAIR", None)


def test_pair_gemm_digits_vs_exact(g2, cuda, tables):  # noqa: F811
    rng = np.random.default_rng(2024)
    A8s, B8s, ks, Ns = [], [], [], []
    for m, n, k, N in PAIR_SHAPES:
        A8s.append(_rand_planes(rng, N + 1, m, k))
        B8s.append(_rand_planes(rng, N + 1, n, k))
        ks.append(k)
        Ns.append(N)
    with pair_mode(1):
        outs = run_gemm_digits(g2, A8s, B8s, ks, Ns)
    for (m, n, k, N), A8, B8, (Y, L) in zip(PAIR_SHAPES, A8s, B8s, outs):
        C = _exact(A8, B8)
        assert np.array_equal(Y.astype(np.int64), digits_of(C, N, tables)), (m, n, k, N)
        assert np.array_equal(L.astype(np.int64), C[N]), (m, n, k, N)


def test_pair_gemm_extremes(g2, cuda, tables):  # noqa: F811
    """All operands -128 at a long K: the largest products the digit step sees."""
    shapes = [(256, 256, 8192, 15), (130, 70, 4000, 20)]
    A8s, B8s, ks, Ns = [], [], [], []
    for m, n, k, N in shapes:
        kp = (k + 31) // 32 * 32
        a = np.zeros((N + 1, m, kp), dtype=np.int8)
        b = np.zeros((N + 1, n, kp), dtype=np.int8)
        a[..., :k] = -128
        b[..., :k] = -128
        A8s.append(a)
        B8s.append(b)
        ks.append(k)
        Ns.append(N)
    with pair_mode(1):
        outs = run_gemm_digits(g2, A8s, B8s, ks, Ns)
    for (m, n, k, N), A8, B8, (Y, L) in zip(shapes, A8s, B8s, outs):
        C = _exact(A8, B8)
        assert np.array_equal(Y.astype(np.int64), digits_of(C, N, tables)), (m, n, k, N)
        assert np.array_equal(L.astype(np.int64), C[N]), (m, n, k, N)


def test_pair_gemm_int32_layout_vs_exact(g2, cuda):
    rng = np.random.default_rng(7)
    shapes = [(300, 5, 200, 15), (129, 9, 64, 8), (512, 3, 1000, 16)]
    descs = (g2.GemmDesc * len(shapes))()
    keep, outs = [], []
    for i, (m, n, k, N) in enumerate(shapes):
        P = N + 1
        A8, B8 = _rand_planes(rng, P, m, k), _rand_planes(rng, P, n, k)
        pa = (g2.img_plane_bytes(m, k) + 255) // 256 * 256
        pb = (g2.img_plane_bytes(n, k) + 255) // 256 * 256
        ha, hb = np.zeros(P * pa, dtype=np.int8), np.zeros(P * pb, dtype=np.int8)
        for l in range(P):
            ha[l * pa:l * pa + g2.img_plane_bytes(m, k)] = g2.pack_plane(A8[l], k)
            hb[l * pb:l * pb + g2.img_plane_bytes(n, k)] = g2.pack_plane(B8[l], k)
        da, db = torch.from_numpy(ha).cuda(), torch.from_numpy(hb).cuda()
        cp = (m * n + 63) // 64 * 64
        dc = torch.full((P * cp,), 0x5A5A5A5A, dtype=torch.int32, device="cuda")
        keep += [da, db]
        outs.append((dc, A8, B8, m, n, P, cp))
        descs[i] = g2.GemmDesc(da.data_ptr(), db.data_ptr(), dc.data_ptr(), pa, pb, cp, m, n, k,
                               P, N, g2.PRODUCTS_INT32)
    scr = torch.empty(g2.lib.ggemm_stage_scratch_bytes(len(shapes)), dtype=torch.uint8,
                      device="cuda")
    cnt = torch.zeros(64, dtype=torch.uint8, device="cuda")
    with pair_mode(1):
        assert g2.lib.ggemm_stage_gemm(descs, len(shapes), scr.data_ptr(), scr.numel(),
                                       cnt.data_ptr(),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    assert int(cnt.cpu().numpy()[32:36].view(np.uint32)[0]) == 0
    for dc, A8, B8, m, n, P, cp in outs:
        h = dc.cpu().numpy()
        C = _exact(A8, B8)
        for l in range(P):
            got = h[l * cp:l * cp + m * n].reshape(n, m).T
            assert np.array_equal(got.astype(np.int64), C[l]), (m, n, l)


def test_public_call_pair_equals_single_cta(g2, cuda):
    """A ragged group through ggemm_grouped_dgemm with the paired GEMM forced on and off:
    identical output bytes."""
    import workloads as W

    wl = W.c2(24, seed=77)
    grp = W.DeviceGroup(g2, wl, W.shard_pieces(g2, wl, 1, 0), torch.device("cuda", 0),
                        keep_c0=True)
    cfg = g2.config(0, 1e-15, 1, 0)
    outs = []
    for mode in (0, 1):
        with pair_mode(mode):
            grp.reset()
            with g2.Handle(grp.num, grp.budget[0] + 1, grp.budget[1] + 1, grp.budget[2] + 1,
                           stream=torch.cuda.current_stream().cuda_stream) as h:
                rc, st = h.grouped_dgemm(g2.PATH_EMU_GROUPED, cfg, grp.problems, grp.num)
                torch.cuda.synchronize()
                assert rc == 0 and h.device_status() == 0
        outs.append(grp.C.clone())
    assert torch.equal(outs[0].view(torch.int64), outs[1].view(torch.int64))
