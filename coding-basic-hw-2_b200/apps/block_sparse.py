#!/usr/bin/env python
"""block_sparse.py -- FP64 block-sparse (BSR, variable block sizes) matrix times dense multi-vector
product Y = A X whose GEMMs all go through this library's ggemm_grouped_dgemm (the reference's
application caller bench/app/block_sparse_fp64.cu, same scenario: atom-blocked Kohn-Sham /
density matrices of Gaussian-basis electronic structure codes, one block per atom pair within a
cutoff, block sizes set by each element's basis functions).

Instance (fixed seed): atoms uniform in a periodic cube at number density rho, 50 % H / 35 % C /
15 % O with the cc-pVDZ basis sizes H 5, C 14, O 14; block (I, J) kept iff the minimum-image
distance is within the cutoff; entries (U - 0.5) exp(phi N(0,1)) scaled by exp(-r_IJ / 2);
X (N x nrhs) of the same distribution.  Two formulations, as in the reference app:
  block  one problem per stored block: T_b (r_I x nrhs) = A_IJ (r_I x c_J) X_J (B a row slice of
         X, ldb = N), then Y_I = sum_J T_b in a fixed order (deterministic);
  panel  one problem per block row: the row's blocks, stored consecutively with ld = r_I, form
         the column-major panel A_I (r_I x K_I); the X rows of its block columns are gathered
         into Xp_I (K_I x nrhs) and Y_I = A_I Xp_I.
Correctness: against the same formulation on NATIVE_LOOP, err = max |Y - Y_ref| / (|A| |X|)
over 2 gamma_n, n = max K_I + max blocks per row + 1 (<= 1: FP64 level).

  python coding-basic-hw-2_b200/apps/block_sparse.py [--atoms 1024] [--nrhs 128] [--reps 10]
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from moe_ffn import load_pkg

NBF = {"H": 5, "C": 14, "O": 14}


class BSR:
    def __init__(self, atoms, density, cutoff, nrhs, phi, seed, device):
        import torch

        rng = np.random.default_rng(seed)
        box = (atoms / density) ** (1.0 / 3.0)
        pos = rng.random((atoms, 3)) * box
        elem = rng.choice(["H", "C", "O"], atoms, p=[0.5, 0.35, 0.15])
        self.size = np.array([NBF[e] for e in elem])
        self.start = np.concatenate([[0], np.cumsum(self.size)[:-1]])
        self.N = int(self.size.sum())
        d = pos[:, None, :] - pos[None, :, :]
        d -= box * np.round(d / box)
        r = np.sqrt((d ** 2).sum(-1))
        self.blocks = []  # (I, J, r_IJ) per block row, columns ascending
        for i in range(atoms):
            for j in np.nonzero(r[i] <= cutoff)[0]:
                self.blocks.append((i, int(j), float(r[i, j])))
        # values: each block row's blocks consecutively, each block column-major (ld = r_I)
        vals, self.off, self.row_first = [], [], []
        o = 0
        prev = -1
        for b, (i, j, rij) in enumerate(self.blocks):
            if i != prev:
                self.row_first.append(b)
                prev = i
            ri, cj = int(self.size[i]), int(self.size[j])
            v = (rng.random((cj, ri)) - 0.5) * np.exp(phi * rng.standard_normal((cj, ri)))
            vals.append((v * np.exp(-rij / 2.0)).reshape(-1))
            self.off.append(o)  # Python ints: the offsets become device pointers
            o += ri * cj
        self.row_first.append(len(self.blocks))
        self.A = torch.from_numpy(np.concatenate(vals)).to(device)
        xs = (rng.random((nrhs, self.N)) - 0.5) * np.exp(phi * rng.standard_normal((nrhs, self.N)))
        self.X = torch.from_numpy(xs).to(device)  # column-major N x nrhs (row-major nrhs x N)
        self.nrhs = nrhs
        self.atoms = atoms
        self.Kmax = max(int(sum(self.size[j] for _, j, _ in self.blocks[self.row_first[i]:
                                                                          self.row_first[i + 1]]))
                        for i in range(atoms))
        self.bmax = max(self.row_first[i + 1] - self.row_first[i] for i in range(atoms))


def block_mode(g2, S, handle, path, cfg, T, Y):
    """One problem per block, then the fixed-order reduction over each row's blocks."""
    import torch

    probs = []
    toff = []
    t = 0
    for b, (i, j, _) in enumerate(S.blocks):
        ri, cj = int(S.size[i]), int(S.size[j])
        probs.append(dict(m=ri, n=S.nrhs, k=cj, A=S.A.data_ptr() + 8 * S.off[b], lda=ri,
                          B=S.X.data_ptr() + 8 * int(S.start[j]), ldb=S.N,
                          C=T.data_ptr() + 8 * t, ldc=ri, alpha=1.0, beta=0.0))
        toff.append(t)
        t += ri * S.nrhs
    P = g2.make_problems(probs)
    rc, _ = handle.grouped_dgemm(path, cfg, P, len(probs))
    if rc != 0:
        raise RuntimeError(f"block GEMMs rc={rc}")
    Y.zero_()
    Yv = Y.view(S.nrhs, S.N)
    for i in range(S.atoms):  # blocks of row i in ascending column order
        ri, r0 = int(S.size[i]), int(S.start[i])
        acc = None
        for b in range(S.row_first[i], S.row_first[i + 1]):
            tb = T[toff[b]:toff[b] + ri * S.nrhs].view(S.nrhs, ri)
            acc = tb.clone() if acc is None else acc + tb
        Yv[:, r0:r0 + ri] = acc
    return Y


def panel_mode(g2, S, handle, path, cfg, Xp, Y):
    """One problem per block row over its gathered X panel."""
    probs = []
    p = 0
    for i in range(S.atoms):
        ri, r0 = int(S.size[i]), int(S.start[i])
        cols = [S.blocks[b][1] for b in range(S.row_first[i], S.row_first[i + 1])]
        K = int(sum(S.size[j] for j in cols))
        # gather the X rows of the row's block columns into Xp (K x nrhs, column-major, ld K)
        panel = Xp[p:p + K * S.nrhs].view(S.nrhs, K)
        c = 0
        for j in cols:
            sj, nj = int(S.start[j]), int(S.size[j])
            panel[:, c:c + nj] = S.X.view(S.nrhs, S.N)[:, sj:sj + nj]
            c += nj
        probs.append(dict(m=ri, n=S.nrhs, k=K, A=S.A.data_ptr() + 8 * S.off[S.row_first[i]],
                          lda=ri, B=Xp.data_ptr() + 8 * p, ldb=K,
                          C=Y.data_ptr() + 8 * r0, ldc=S.N, alpha=1.0, beta=0.0))
        p += K * S.nrhs
    P = g2.make_problems(probs)
    rc, _ = handle.grouped_dgemm(path, cfg, P, len(probs))
    if rc != 0:
        raise RuntimeError(f"panel GEMMs rc={rc}")
    return Y


def abs_product(S):
    """|A| |X| (column-major N x nrhs), natively, for the error denominators."""
    import torch

    den = torch.zeros((S.nrhs, S.N), dtype=torch.float64, device=S.X.device)
    Xa = S.X.view(S.nrhs, S.N).abs()
    for b, (i, j, _) in enumerate(S.blocks):
        ri, cj = int(S.size[i]), int(S.size[j])
        Ab = S.A[S.off[b]:S.off[b] + ri * cj].view(cj, ri).abs()  # row-major view of A_IJ^T
        den[:, int(S.start[i]):int(S.start[i]) + ri] += Xa[:, int(S.start[j]):int(S.start[j]) + cj] @ Ab
    return den.reshape(-1)


def err_over_bound(S, Y, Y_ref, den):
    n = S.Kmax + S.bmax + 1
    u = 2.0 ** -53
    return float(((Y - Y_ref).abs() / den.clamp_min(1e-300)).max().item()) / (2 * n * u / (1 - n * u))


def run(g2, S, modes=("block", "panel"), paths=("native_grouped", "emu_grouped", "auto"), reps=5):
    import torch

    dev = S.X.device
    nb = len(S.blocks)
    total_t = int(sum(S.size[i] for i, _, _ in S.blocks)) * S.nrhs
    T = torch.empty(total_t, dtype=torch.float64, device=dev)
    panel_k = sum(int(sum(S.size[S.blocks[b][1]] for b in range(S.row_first[i], S.row_first[i + 1])))
                  for i in range(S.atoms))
    Xp = torch.empty(panel_k * S.nrhs, dtype=torch.float64, device=dev)
    Y = torch.empty(S.N * S.nrhs, dtype=torch.float64, device=dev)
    den = abs_product(S)
    cfg = g2.config(0, 1e-15, 1, 0)
    s = torch.cuda.current_stream()
    flops = 2.0 * sum(int(S.size[i]) * int(S.size[j]) for i, j, _ in S.blocks) * S.nrhs
    out = {"atoms": S.atoms, "N": S.N, "blocks": nb, "nrhs": S.nrhs}
    with g2.Handle(nb, S.A.numel() + 1, Xp.numel() + S.X.numel() + 1,
                   total_t + Y.numel() + 1, stream=s.cuda_stream) as h:
        for mode in modes:
            fn = block_mode if mode == "block" else panel_mode
            arg = T if mode == "block" else Xp
            Y_ref = fn(g2, S, h, g2.PATH_NATIVE_LOOP, cfg, arg, Y).clone()
            for name in paths:
                path = {v: k for k, v in g2.PATH_NAMES.items()}[name]
                fn(g2, S, h, path, cfg, arg, Y)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                for _ in range(reps):
                    fn(g2, S, h, path, cfg, arg, Y)
                e1.record(s)
                e1.synchronize()
                ms = e0.elapsed_time(e1) / reps
                out[f"{mode}/{name}"] = {"ms": ms, "gflops": flops / ms / 1e6,
                                         "err_over_bound": err_over_bound(S, Y, Y_ref, den)}
    return out


def main():
    import torch

    ap = argparse.ArgumentParser()
    ap.add_argument("--atoms", type=int, default=1024)
    ap.add_argument("--density", type=float, default=0.1)
    ap.add_argument("--cutoff", type=float, default=6.0)
    ap.add_argument("--nrhs", type=int, default=128)
    ap.add_argument("--phi", type=float, default=0.5)
    ap.add_argument("--seed", type=int, default=4321)
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    g2 = load_pkg()
    S = BSR(args.atoms, args.density, args.cutoff, args.nrhs, args.phi, args.seed,
            torch.device("cuda", 0))
    print(json.dumps(run(g2, S, reps=args.reps)))


if __name__ == "__main__":
    main()
